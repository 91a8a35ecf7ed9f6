"""Expert parallelism for the prefill path: one process per GPU, torch.distributed over NCCL.

The 256 routed experts are split evenly over the W ranks of the group (256/128/64/32 per GPU at
W = 1/2/4/8); router and shared expert are replicated. Every rank passes the same number of
tokens T. For one layer, each rank:

1. routes its own tokens (``b200moe_moe_route``: fp16 activations, ids, bf16 weights, gate);
2. dispatch: ``all_gather`` of the fp16 rows, ids and weights -- every rank sees all W*T tokens;
3. runs its experts on all of them in one ``b200moe_moe_experts`` call: the slots in its
   expert range for every gathered token, plus the shared expert for its own tokens' rows (one
   set of GEMM launches). The stage keeps only the slots in range, so each token costs GEMM
   work on the ranks that own its experts and nothing elsewhere; one f32 partial row per
   gathered token (its in-range slots summed in ascending expert id, + sg * shared on its own
   rows, zero when it has none);
4. combine: ``all_to_all_single`` with equal splits sends the partial rows of rank r's tokens
   back to rank r, which adds the W partials per token in ascending rank order (ascending
   expert ranges).

No host synchronisation: every size is known from T and W, so the whole layer is a fixed
sequence of kernels and collectives (capturable in a CUDA graph). Deterministic: every
addition has a fixed order. Relative to one GPU, only the association of the routed sum
changes (per-rank partial sums, then the ranks in order).

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
    """``b200moe_moe_experts`` for pre-routed tokens, an expert range and the shared-expert rows
    ``sh_rows`` = (lo, hi) (sg[t - lo] applies to row t; default all rows)."""
    def experts(x16, ids, wb, e_lo, e_hi, sg, out, accumulate=False, sh_rows=None):
        T = x16.shape[0]
        if T == 0:
            return out
        _abi.moe_experts(x16, T, ids, wb, e_lo, e_hi, sg, layer.abi(), out, accumulate, ws(T), sh_rows=sh_rows)
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
        if experts_fn is None and not getattr(layer, "all_q4k", True):
            # refused here, before any collective, on every rank alike (the grouped GEMMs take Q4_K)
            raise ValueError("expert parallelism runs the grouped GEMMs, which take Q4_K layers; this layer "
                             "has down %s, shared %s" % (layer.down_type, layer.sh_type))
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
        """``x`` [T, 2048] (bf16/f32) -> (out [T, 2048] f32, ids [T, 8]); T is the same on every
        rank. With ``resid`` instead of ``x``: routes rmsnorm(resid) and returns resid + out."""
        x16, ids, wb, sg = self.route_fn(x, resid) if resid is not None else self.route_fn(x)
        T = x16.shape[0]
        W = self.world
        out = torch.zeros((T, H), dtype=torch.float32, device=self.device)
        if W == 1:  # every expert is local: routed + shared in one stage call
            self.experts_fn(x16, ids, wb, 0, E, sg, out)
        else:
            # dispatch: all tokens to every rank (rows travel as raw bytes: every backend moves
            # uint8, not every one moves fp16)
            xg = torch.empty((W * T, H), dtype=x16.dtype, device=self.device)
            ig = torch.empty((W * T, TOPK), dtype=ids.dtype, device=self.device)
            wg = torch.empty((W * T, TOPK), dtype=wb.dtype, device=self.device)
            for dst, src in ((xg, x16), (ig, ids), (wg, wb)):
                dist.all_gather_into_tensor(dst.view(torch.uint8), src.contiguous().view(torch.uint8),
                                            group=self.group)
            partial = torch.empty((W * T, H), dtype=torch.float32, device=self.device)
            own = (self.rank * T, (self.rank + 1) * T)  # this rank's rows get sg * shared expert
            self.experts_fn(xg, ig, wg, self.e_lo, self.e_hi, sg, partial, sh_rows=own)
            back = torch.empty((W, T, H), dtype=torch.float32, device=self.device)
            dist.all_to_all_single(back.view(torch.uint8), partial.view(torch.uint8), group=self.group)
            out = back[0].clone()
            for r in range(1, W):  # ascending rank = ascending expert range
                out += back[r]
        if resid is not None:
            resid += out
            return resid, ids
        return out, ids
