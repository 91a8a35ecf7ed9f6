"""Expert parallelism for the prefill / large-batch path: one process per GPU over NCCL.

The 256 routed experts are split evenly over the W ranks of the group (256/128/64/32 per GPU at
W = 1/2/4/8); router and shared expert are replicated. Every rank holds T tokens of its own (the
same T everywhere). The reference runs the whole expert loop in one process
(``engine/m3_forward.py:447-475``); here one layer is, on every rank:

1. route its own tokens (``b200moe_moe_route``: fp16 rows, ids, bf16 weights, shared gate);
2. pack (``b200moe_ep_pack``): for each destination rank d, the tokens with at least one slot in
   d's expert range -- each token once per destination, however many of its slots land there --
   as dispatch rows (x, ids, weights) in ascending token order; every own token goes to the own
   block, where the shared expert runs. ``pos[t][d]`` remembers each row's place;
3. dispatch: the row blocks reach their ranks -- over peer memory (``transport="p2p"``, the
   default on NVLink GPUs: ``b200moe_ep_dispatch_p2p`` stores only the rows that carry work
   straight into each destination's receive buffer, then signals it), or as one equal-split
   ``all_to_all_single`` of the [W][T] blocks (``transport="a2a"``, any backend);
4. experts (``b200moe_ep_experts``): the received rows' slots in this rank's expert range through
   the Q4_K grouped GEMMs (one set of launches for all sources), summed per row in ascending
   expert id, plus the gated shared expert on the own block -> one f32 partial row per received
   row (zero where a row has no work);
5. combine: the partial rows go back to their sources -- stored by the expert stage's own combine
   kernel into each source's return buffer (p2p), or by an equal-split ``all_to_all_single`` --
   and each rank adds, per token, the partial rows from d = 0, 1, ... in that order
   (``b200moe_ep_combine``: ascending expert ranges, a fixed association).

Sizes are fixed by T and W, so a step is a fixed sequence of kernels and collectives with no host
synchronisation: it can be captured in a CUDA graph (buffers are allocated once per T and reused).
Relative to one GPU only the association of the routed sum changes (per-rank partial sums, then
the ranks in order), so the outputs agree to f32 rounding and the routing ids are identical.

The stage functions can be replaced (the CPU tests run this exact sequence of collectives on gloo
ranks with a host restatement of the three device stages).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _abi
from .geometry import E, H, RMS_EPS, TOPK

ROW_BYTES = _abi.EP_ROW_BYTES
MAX_P2P_RANKS = 8


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


def device_pack_fn():
    """``b200moe_ep_pack``: (send rows [W, T, ROW_BYTES] uint8, pos [T, W] int32)."""
    def pack(x16, ids, wb, rank, world, send, pos):
        _abi.ep_pack(x16, ids, wb, x16.shape[0], rank, world, send, pos)
        return send, pos
    return pack


def device_experts_fn(layer, ws):
    """``b200moe_ep_experts`` on the received rows (W > 1): partial [W, T, 2048] f32."""
    def experts(recv, T, rank, world, sg, partial):
        _abi.ep_experts(recv, T, rank, world, sg, layer.abi(), partial, ws(world * T))
        return partial
    return experts


def device_local_fn(layer, ws):
    """W = 1: ``b200moe_moe_experts`` over every expert and the shared expert."""
    def local(x16, ids, wb, sg, out, accumulate):
        T = x16.shape[0]
        _abi.moe_experts(x16, T, ids, wb, 0, E, sg, layer.abi(), out, accumulate, ws(T))
        return out
    return local


def device_combine_fn():
    def combine(ret, pos, T, world, out, accumulate):
        _abi.ep_combine(ret, pos, T, world, out, accumulate)
        return out
    return combine


class ExpertParallelMoE:
    """One MoE layer with its routed experts sharded over a process group."""

    def __init__(self, layer, group=None, route_fn=None, pack_fn=None, experts_fn=None, combine_fn=None,
                 local_fn=None, device=None, transport: str | None = None):
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
        self._bufs = {}
        self.route_fn = route_fn or device_route_fn(layer, self._workspace)
        self.pack_fn = pack_fn or device_pack_fn()
        self.experts_fn = experts_fn or device_experts_fn(layer, self._workspace)
        self.combine_fn = combine_fn or device_combine_fn()
        self.local_fn = local_fn or device_local_fn(layer, self._workspace)
        if transport is None:  # peer memory where the ranks are CUDA devices of one NVLink node
            nccl = grouped and dist.get_backend(group) == "nccl"
            transport = "p2p" if (nccl and 1 < self.world <= MAX_P2P_RANKS and pack_fn is None
                                  and experts_fn is None and combine_fn is None) else "a2a"
        if transport not in ("p2p", "a2a"):
            raise ValueError("transport must be p2p or a2a, got %r" % (transport,))
        self.transport = transport
        self._peers = {}

    def _workspace(self, rows):
        need = _abi.prefill_workspace_size(max(rows, 1))
        ws = self._ws.get("ws")
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._ws["ws"] = ws
        return ws

    def workspace(self, T):
        """The prefill workspace the expert stage uses (its status word: ``prefill_status``)."""
        return self._workspace(self.world * T if self.world > 1 else T)

    def buffers(self, T):
        """The step's fixed-size buffers for T tokens per rank (allocated once, reused)."""
        b = self._bufs.get(T)
        if b is None:
            W, dev = self.world, self.device
            b = dict(send=torch.empty((W, T, ROW_BYTES), dtype=torch.uint8, device=dev),
                     recv=torch.empty((W, T, ROW_BYTES), dtype=torch.uint8, device=dev),
                     pos=torch.empty((T, W), dtype=torch.int32, device=dev),
                     partial=torch.empty((W, T, H), dtype=torch.float32, device=dev),
                     ret=torch.empty((W, T, H), dtype=torch.float32, device=dev))
            self._bufs[T] = b
        return b

    def _p2p(self, T):
        """The peer-memory buffers for T tokens per rank: allocated, shared by CUDA IPC with every
        rank of the group (a collective: every rank calls it for the same T) and mapped."""
        st = self._peers.get(T)
        if st is not None:
            return st
        W, dev, r = self.world, self.device, self.rank
        own = dict(recv=torch.empty((W, T, ROW_BYTES), dtype=torch.uint8, device=dev),
                   ret=torch.empty((W, T, H), dtype=torch.float32, device=dev),
                   fd=torch.zeros((W,), dtype=torch.int32, device=dev),
                   fr=torch.zeros((W,), dtype=torch.int32, device=dev))
        epoch = torch.zeros((4,), dtype=torch.int32, device=dev)  # [0]: epoch, [1]: status
        torch.cuda.synchronize(dev)
        mine = {k: _abi.ipc_handle(t) for k, t in own.items()}
        every = [None] * W
        dist.all_gather_object(every, mine, group=self.group)
        addrs, opened = {}, []
        for k, t in own.items():
            row = []
            for d in range(W):
                if d == r:
                    row.append(t.data_ptr())
                else:
                    h, off = every[d][k]
                    a = _abi.ipc_open(h, off)
                    opened.append((a, off))
                    row.append(a)
            addrs[k] = row
        P = _abi.EpPeers()
        P.world, P.rank = W, r
        for d in range(W):
            P.recv[d], P.ret[d] = addrs["recv"][d], addrs["ret"][d]
            P.flag_dispatch[d], P.flag_return[d] = addrs["fd"][d], addrs["fr"][d]
        P.epoch = epoch.data_ptr()
        P.status = epoch.data_ptr() + 4
        dist.barrier(group=self.group)  # every rank's flags are zero and mapped before any signal
        st = dict(own=own, epoch=epoch, peers=P, opened=opened, pos=torch.empty((T, W), dtype=torch.int32,
                                                                                   device=dev))
        self._peers[T] = st
        return st

    def p2p_status(self, T) -> int:
        """Status word of the peer-memory exchanges for T tokens (bit 8: a peer wait ran out)."""
        st = self._peers.get(T)
        return 0 if st is None else int(st["epoch"][1].item())

    def close(self):
        """Unmap the peers' buffers (call on every rank before the process group is destroyed)."""
        for st in self._peers.values():
            for a, off in st["opened"]:
                _abi.ipc_close(a, off)
        self._peers.clear()

    def forward(self, x=None, resid=None, out=None, mark=None):
        """``x`` [T, 2048] (bf16/f32) -> (out [T, 2048] f32, ids [T, 8]); T is the same on every
        rank. With ``resid`` instead of ``x``: routes rmsnorm(resid) and adds the block output to
        resid in place (returned). ``mark(stage)`` (optional) is called after each stage is
        enqueued: route, dispatch, experts, combine, sum."""
        mark = mark or (lambda stage: None)
        x16, ids, wb, sg = self.route_fn(x, resid) if resid is not None else self.route_fn(x)
        mark("route")
        T = x16.shape[0]
        W = self.world
        dst = resid if resid is not None else (out if out is not None else
                                               torch.empty((T, H), dtype=torch.float32, device=self.device))
        acc = resid is not None
        if W == 1:  # every expert is local: routed + shared in one stage call
            mark("dispatch")
            self.local_fn(x16, ids, wb, sg, dst, acc)
            for st in ("experts", "combine", "sum"):
                mark(st)
            return dst, ids
        if self.transport == "p2p":
            st = self._p2p(T)
            P, pos = st["peers"], st["pos"]
            _abi.ep_dispatch_p2p(x16, ids, wb, T, P, pos)
            mark("dispatch")
            _abi.ep_experts_p2p(T, sg, self.layer.abi(), P, self._workspace(W * T))
            mark("experts")
            mark("combine")
            _abi.ep_combine_p2p(T, pos, P, dst, acc)
            mark("sum")
            return dst, ids
        b = self.buffers(T)
        self.pack_fn(x16, ids, wb, self.rank, W, b["send"], b["pos"])
        dist.all_to_all_single(b["recv"], b["send"], group=self.group)
        mark("dispatch")
        self.experts_fn(b["recv"], T, self.rank, W, sg, b["partial"])
        mark("experts")
        dist.all_to_all_single(b["ret"].view(torch.uint8), b["partial"].view(torch.uint8), group=self.group)
        mark("combine")
        self.combine_fn(b["ret"], b["pos"], T, W, dst, acc)
        mark("sum")
        return dst, ids
