"""Expert parallelism for the prefill path: one process per GPU, torch.distributed over NCCL.

The 256 routed experts are split evenly over the W ranks of the group (256/128/64/32 per GPU at
W = 1/2/4/8); router and shared expert are replicated. For one layer, each rank:

1. routes its own tokens (``b200moe_moe_route``: fp16 activations, ids, bf16 weights, gate);
2. dispatch: for every destination rank, picks (ascending token order) the tokens with at least
   one slot among that rank's experts and masks the other slots to -1; counts are exchanged with
   ``all_to_all_single``, then the fp16 rows, ids and weights. A token crosses the link once per
   destination rank, whatever number of its experts live there;
3. runs its experts on what it received (``b200moe_moe_experts`` with its expert range,
   no shared expert) -> one f32 partial row per received token (its slots summed in ascending
   expert id);
4. combine: partials return along the reversed splits and are added per token in ascending
   rank order, i.e. ascending expert ranges; the token's own rank adds sg * shared expert.

The only host synchronisation per layer is the count exchange (split sizes must be host ints).
Deterministic: every addition has a fixed order. Relative to one GPU, only the association of
the routed sum changes (per-rank partial sums, then the ranks in order).

``route_fn`` / ``experts_fn`` can be replaced (the CPU tests run this exact dispatch/combine code
on gloo ranks with oracle-backed stage functions).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _abi
from .geometry import E, H, RMS_EPS, TOPK


def device_route_fn(layer, ws):
    """``b200moe_moe_route`` on this rank's tokens."""
    def route(x, resid=None):
        T = (resid if resid is not None else x).shape[0]
        dev = layer.device
        x16 = torch.empty((T, H), dtype=torch.float16, device=dev)
        ids = torch.empty((T, TOPK), dtype=torch.int32, device=dev)
        wb = torch.empty((T, TOPK), dtype=torch.int16, device=dev)
        sg = torch.empty((T,), dtype=torch.float32, device=dev)
        xd = _abi.BF16 if (x is not None and x.dtype == torch.bfloat16) else _abi.F32
        _abi.moe_route(x, xd, resid, RMS_EPS, T, layer.abi(), x16, ids, wb, sg, ws(T))
        return x16, ids, wb, sg
    return route


def device_experts_fn(layer, ws):
    """``b200moe_moe_experts`` for pre-routed tokens and an expert range."""
    def experts(x16, ids, wb, e_lo, e_hi, sg, out, accumulate=False):
        T = x16.shape[0]
        if T == 0:
            return out
        _abi.moe_experts(x16, T, ids, wb, e_lo, e_hi, sg, layer.abi(), out, accumulate, ws(T))
        return out
    return experts


class ExpertParallelMoE:
    """One MoE layer with its routed experts sharded over a process group."""

    def __init__(self, layer, group=None, route_fn=None, experts_fn=None, device=None):
        self.group = group
        grouped = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if grouped else 0
        self.world = dist.get_world_size(group) if grouped else 1
        if E % self.world:
            raise ValueError("256 experts do not split over %d ranks" % self.world)
        self.per = E // self.world
        self.e_lo, self.e_hi = self.rank * self.per, (self.rank + 1) * self.per
        self.layer = layer
        self.device = device if device is not None else layer.device
        self._ws = {}
        self.route_fn = route_fn or device_route_fn(layer, self._workspace)
        self.experts_fn = experts_fn or device_experts_fn(layer, self._workspace)

    def _workspace(self, T):
        need = _abi.prefill_workspace_size(max(T, 1))
        ws = self._ws.get("ws")
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._ws["ws"] = ws
        return ws

    def forward(self, x=None, resid=None):
        """``x`` [T_local, 2048] (bf16/f32) -> (out [T_local, 2048] f32, ids [T_local, 8]).
        With ``resid`` instead of ``x``: routes rmsnorm(resid) and returns resid + out."""
        x16, ids, wb, sg = self.route_fn(x, resid) if resid is not None else self.route_fn(x)
        T = x16.shape[0]
        W = self.world
        dest = torch.div(ids, self.per, rounding_mode="floor")
        send_tok, send_ids = [], []
        for r in range(W):
            m = dest == r
            tok = m.any(dim=1).nonzero().flatten()
            send_tok.append(tok)
            send_ids.append(torch.where(m[tok], ids[tok], torch.full_like(ids[tok], -1)))
        send_counts = [int(t.numel()) for t in send_tok]
        if W > 1:
            cnt = torch.tensor(send_counts, dtype=torch.int64, device=self.device)
            rcnt = torch.empty_like(cnt)
            dist.all_to_all_single(rcnt, cnt, group=self.group)
            recv_counts = [int(c) for c in rcnt.tolist()]
        else:
            recv_counts = list(send_counts)
        R = sum(recv_counts)
        x_send = torch.cat([x16[t] for t in send_tok]) if T else x16[:0]
        i_send = torch.cat(send_ids) if T else ids[:0]
        w_send = torch.cat([wb[t] for t in send_tok]) if T else wb[:0]
        x_recv = torch.empty((R, H), dtype=x16.dtype, device=self.device)
        i_recv = torch.empty((R, TOPK), dtype=ids.dtype, device=self.device)
        w_recv = torch.empty((R, TOPK), dtype=wb.dtype, device=self.device)
        for dst, src in ((x_recv, x_send), (i_recv, i_send), (w_recv, w_send)):
            # rows travel as raw bytes (every backend moves uint8; not every one moves fp16)
            if W > 1:
                dist.all_to_all_single(dst.view(torch.uint8), src.contiguous().view(torch.uint8), recv_counts,
                                       send_counts, group=self.group)
            else:
                dst.copy_(src)
        partial = torch.zeros((R, H), dtype=torch.float32, device=self.device)
        self.experts_fn(x_recv, i_recv, w_recv, self.e_lo, self.e_hi, None, partial)
        if W > 1:
            back = torch.empty((sum(send_counts), H), dtype=torch.float32, device=self.device)
            dist.all_to_all_single(back, partial, send_counts, recv_counts, group=self.group)
        else:
            back = partial
        acc = torch.zeros((T, H), dtype=torch.float32, device=self.device)
        off = 0
        for r in range(W):            # ascending rank = ascending expert range; indices unique per r
            n = send_counts[r]
            if n:
                acc.index_add_(0, send_tok[r], back[off:off + n])
            off += n
        out = torch.zeros((T, H), dtype=torch.float32, device=self.device)
        self.experts_fn(x16, ids, wb, 0, 0, sg, out)        # sg * shared expert only
        out = acc + out
        if resid is not None:
            resid += out
            return resid, ids
        return out, ids
