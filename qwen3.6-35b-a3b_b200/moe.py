"""The MoE block behind the reference's own Python call shapes.

* :func:`moe_block` -- drop-in for ``engine/m3_forward.py:430 moe_block(g, E, layer,
  probe_row=None) -> (out [B,T,2048] f32, {"used", "ids"})``.
* :func:`moe_router` -- the router stage set of ``engine/block_forward.py:614``:
  ``router_logits, topk_ids, topk_weights, topk_weights_f32``.
* :func:`moe_shared`, :func:`moe_routed`, :func:`moe_block_stages` -- the stage dictionaries of
  ``engine/block_forward.py:639-670`` (``shared_raw, shared_gate_prob, shared_out``;
  ``expert_raw`` in top-k slot order, ``routed_sum``; all of them plus the router stages and
  ``combined_out``), for stage-level parity gates.
* :func:`moe_stack` -- the config-4 MoE sub-stack (``engine/m3_forward.py:714-737`` with
  the mixer sublayers removed): ``resid <- resid + moe_block(rmsnorm(resid))`` per layer.

Errors follow the reference: shape and dtype problems raise ``Refused`` (a ValueError with
a tag, as ``engine/m3_forward.py:165-170`` does) before any launch; a failing library call
raises :class:`b200moe._abi.B200MoeError`. Everything runs on the caller's current CUDA
stream with no host synchronisation; ``info["used"]`` is computed (one sync) only when read.
"""
from __future__ import annotations

import torch

from . import _abi
from .engine import DeviceEngine, DeviceLayer
from .geometry import E, H, N_LAYERS, RMS_EPS, TOPK


class Refused(ValueError):
    """A call the block refuses, tagged like the reference's ``Refused(tag, msg)``."""

    def __init__(self, tag: str, msg: str):
        super().__init__("[%s] %s" % (tag, msg))
        self.tag = tag


class _Info(dict):
    """``{"used", "ids"}`` where ``used`` (distinct experts hit) is evaluated on first read."""

    def __getitem__(self, k):
        if k == "used" and not dict.__contains__(self, "used"):
            dict.__setitem__(self, "used", int(torch.unique(dict.__getitem__(self, "ids")).numel()))
        return dict.__getitem__(self, k)


_WS = {}


def workspace(T: int, device) -> torch.Tensor:
    """A cached workspace of ``b200moe_decode_workspace_size(T)`` bytes on ``device``."""
    need = _abi.decode_workspace_size(T)
    key = (torch.device(device), torch.cuda.current_stream(device).cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def _layer_of(E_, layer) -> DeviceLayer:
    if isinstance(E_, DeviceLayer):
        return E_
    if isinstance(E_, DeviceEngine):
        return E_.layers[layer]
    raise Refused("engine-kind", "moe_block needs a b200moe DeviceEngine or DeviceLayer, got %s"
                  % type(E_).__name__)


def _tokens(g, device) -> tuple:
    if g.shape[-1] != H:
        raise Refused("shape", "hidden size %d != %d" % (g.shape[-1], H))
    if g.dtype not in (torch.float32, torch.bfloat16):
        raise Refused("dtype", "input dtype %s: f32 or bf16 only" % g.dtype)
    x = g.reshape(-1, H)
    if x.device != device:
        x = x.to(device, non_blocking=True)
    x = x.contiguous()
    return x, (_abi.F32 if x.dtype == torch.float32 else _abi.BF16)


# At and above this many tokens the grouped-GEMM path is used. Measured on the 40-layer stack
# (config 2 routing law, one B200): the grouped decode kernels (each distinct expert read once,
# int8 tensor-core dots) take 1.05 ms at 2 tokens, 1.36 at 4, 2.14 at 8, 2.97 at 12 and 3.66 at
# 16, the grouped GEMMs a nearly flat ~3 ms (2.92 at 2, 3.01 at 4, 3.19 at 8, 3.20 at 12, 3.27 at
# 16, 3.44 at 32): they cross between 12 and 16 tokens.
PREFILL_MIN_TOKENS = 13
# The decode path runs 2..GROUPED_MAX_TOKENS tokens of a Q4_K layer on the grouped kernels
# (csrc/grouped.cu: each distinct expert's rows read once for all its tokens).
GROUPED_MAX_TOKENS = 16


def prefill_workspace(T: int, device) -> torch.Tensor:
    """A cached workspace of ``b200moe_prefill_workspace_size(T)`` bytes on ``device``."""
    need = _abi.prefill_workspace_size(T)
    key = ("prefill", torch.device(device), torch.cuda.current_stream(device).cuda_stream)
    ws = _WS.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _WS[key] = ws
    return ws


def _raise_status(who: str, status: int):
    if status != 0:
        raise _abi.B200MoeError(who, _abi.ECUDA, "device status word %d: a bounded pipeline or exchange wait ran "
                                "out (or an fp16 operand overflowed, prefill bit 4); the outputs of this call are "
                                "incomplete" % status)


def moe_block(g: torch.Tensor, E_, layer: int = 0, probe_row=None, out: torch.Tensor | None = None,
              path: str = "auto", check: bool = False):
    """``engine/m3_forward.py:430`` on the B200 path.

    ``g`` [B, T, 2048] (or [T, 2048]) f32/bf16; returns ``(out, info)`` with ``out`` f32 in
    ``g``'s leading shape, ``info = {"ids": [B,T,8] int32 (device), "used": int}``.
    Routing is R1-R5 with the cast before the multiply; routed outputs are summed in
    ascending expert id; the shared expert is gated by sigmoid(w_sg . x).
    ``path``: "decode" (one token: the persistent kernel; 2..16 tokens of a Q4_K layer: the
    grouped decode kernels; exact-product int8 tensor-core dots; otherwise the f32 gather-GEMV
    kernels), "prefill" (token sort + tcgen05 grouped GEMMs, fp16 operands) or "auto" (prefill
    from ``PREFILL_MIN_TOKENS`` tokens on). A layer
    with Q5_K / Q6_K down or a Q8_0 shared expert (the published Q4_K_M file) runs on the
    decode kernels at every token count; ``path="prefill"`` refuses it. No tokens give empty
    results (as the reference's own loop does), with no device work. ``check=True`` reads the
    call's device status word back (one stream synchronisation) and raises
    :class:`b200moe._abi.B200MoeError` if a bounded wait ran out, as the reference refuses a
    broken state loudly (``engine/m3_forward.py:165-170``).
    """
    if probe_row is not None:
        raise Refused("probe-row", "band-operand probes are a host-oracle feature; not on the device path")
    if path not in ("auto", "decode", "prefill"):
        raise Refused("path", "path must be auto, decode or prefill, got %r" % (path,))
    L = _layer_of(E_, layer)
    x, xd = _tokens(g, L.device)
    T = x.shape[0]
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=L.device)
    ids = torch.empty((T, TOPK), dtype=torch.int32, device=L.device)
    if path == "prefill" and not L.all_q4k:
        raise Refused("format", "the grouped GEMMs take Q4_K experts; this layer has down %s, shared %s"
                      % (L.down_type, L.sh_type))
    if T == 0:
        pass
    elif path == "prefill" or (path == "auto" and T >= PREFILL_MIN_TOKENS and L.all_q4k):
        pws = prefill_workspace(T, L.device)
        _abi.moe_prefill(x, xd, None, RMS_EPS, T, L.abi(), out, ids, pws)
        if check:
            _raise_status("moe_block (prefill)", _abi.prefill_status(pws, T))
    else:
        dws = workspace(T, L.device)
        _abi.moe_decode(x, xd, T, L.abi(), out, ids, None, dws)
        if check:
            _raise_status("moe_block (decode)", _abi.decode_status(dws, T))
    lead = tuple(g.shape[:-1])
    return out.reshape(*lead, H), _Info(ids=ids.reshape(*lead, TOPK))


def moe_router(g_row: torch.Tensor, E_, layer: int = 0) -> dict:
    """Router stages (``engine/block_forward.py:614-636``) for every row of ``g_row``."""
    L = _layer_of(E_, layer)
    x, xd = _tokens(g_row, L.device)
    T = x.shape[0]
    dev = L.device
    logits = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    ids = torch.empty((T, TOPK), dtype=torch.int32, device=dev)
    wf = torch.empty((T, TOPK), dtype=torch.float32, device=dev)
    wb = torch.empty((T, TOPK), dtype=torch.bfloat16, device=dev)
    if T:
        _abi.router(x, xd, T, L.router_w, L.logit_bias, logits, ids, wf, wb, workspace(T, dev))
    return dict(router_logits=logits, topk_ids=ids, topk_weights=wb, topk_weights_f32=wf)


def moe_stack(resid: torch.Tensor, E_: DeviceEngine, n_layers: int | None = None,
              eps: float = RMS_EPS, ids_out: torch.Tensor | None = None,
              ws: torch.Tensor | None = None, check: bool = False) -> torch.Tensor:
    """In place: for each layer, ``resid += moe_block_l(rmsnorm(resid))``. ``resid`` [T, 2048] f32.

    ``ws`` (optional) is a caller-owned workspace of ``stack_workspace_bytes(T)`` bytes; pass
    one when capturing the call into a CUDA graph so nothing is allocated during capture.
    ``check=True`` (not inside a capture: it synchronises) raises if a bounded wait ran out."""
    if resid.dtype != torch.float32 or resid.shape[-1] != H:
        raise Refused("shape", "resid must be f32 [T, %d]" % H)
    n = len(E_.layers) if n_layers is None else int(n_layers)
    if n > len(E_.layers):
        raise Refused("layers", "%d layers requested, engine holds %d" % (n, len(E_.layers)))
    r = resid.reshape(-1, H)
    T = r.shape[0]
    if T == 0:
        return resid
    dev = E_.layers[0].device
    ws = ws if ws is not None else workspace(T, dev)
    _abi.stack_decode(r, T, [L.abi() for L in E_.layers[:n]], eps, ids_out, ws)
    if check:
        _raise_status("moe_stack", _abi.decode_status(ws, T))
    return resid


def stack_workspace_bytes(T: int) -> int:
    return _abi.stack_workspace_size(T, 1)


def moe_stack_prefill(resid: torch.Tensor, E_: DeviceEngine, n_layers: int | None = None,
                      eps: float = RMS_EPS, ids_out: torch.Tensor | None = None,
                      ws: torch.Tensor | None = None) -> torch.Tensor:
    """The config-4 sub-stack on the prefill path: per layer ``resid += moe(rmsnorm(resid))``
    through the tcgen05 grouped GEMMs. ``ids_out`` (optional) is [n_layers, T, 8] int32.
    Layers that are not Q4_K throughout go through the decode kernels (``b200moe_stack_decode``
    of that one layer, on ``ws`` when it is large enough: the prefill workspace is)."""
    if resid.dtype != torch.float32 or resid.shape[-1] != H:
        raise Refused("shape", "resid must be f32 [T, %d]" % H)
    n = len(E_.layers) if n_layers is None else int(n_layers)
    r = resid.reshape(-1, H)
    T = r.shape[0]
    if T == 0:
        return resid
    dev = E_.layers[0].device
    ws = ws if ws is not None else prefill_workspace(T, dev)
    dws = None  # the decode fallback's workspace (stream-ordered after the previous layer's use of ws)
    for l in range(n):
        L = E_.layers[l]
        ids_l = None if ids_out is None else ids_out[l]
        if L.all_q4k:
            _abi.moe_prefill(None, _abi.F32, r, eps, T, L.abi(), None, ids_l, ws)
        else:
            if dws is None:
                dws = ws if ws.numel() * ws.element_size() >= _abi.decode_workspace_size(T) else workspace(T, dev)
            _abi.stack_decode(r, T, [L.abi()], eps, ids_l, dws)
    return resid


def _stage_route(g_row, E_, layer):
    """fp16 rows, ids, bf16 weights and the shared-expert gate of every row of ``g_row``."""
    L = _layer_of(E_, layer)
    x, xd = _tokens(g_row, L.device)
    T = x.shape[0]
    dev = L.device
    x16 = torch.empty((T, H), dtype=torch.float16, device=dev)
    ids = torch.empty((T, TOPK), dtype=torch.int32, device=dev)
    wb = torch.empty((T, TOPK), dtype=torch.int16, device=dev)
    sg = torch.empty((T,), dtype=torch.float32, device=dev)
    if T:
        _abi.moe_route(x, xd, None, RMS_EPS, T, L.abi(), x16, ids, wb, sg, prefill_workspace(T, dev))
    return L, x16, ids, wb, sg


def _stage_experts(L, x16, ids, wb, e_lo, e_hi, sg):
    T = x16.shape[0]
    out = torch.empty((T, H), dtype=torch.float32, device=L.device)
    if T == 0:
        return out
    _abi.moe_experts(x16, T, ids, wb, e_lo, e_hi, sg, L.abi(), out, False, prefill_workspace(T, L.device))
    return out


def moe_shared(g_row: torch.Tensor, E_, layer: int = 0, _routed=None) -> dict:
    """``engine/block_forward.py:639 moe_shared``: ``shared_raw`` = W_ds (silu(W_gs x) * W_us x)
    [T, 2048], ``shared_gate_prob`` = sigmoid(w_sg . x) [T, 1], ``shared_out`` = their product;
    all f32. Computed by the expert stage of the prefill path (fp16 operands, f32 accumulate):
    the shared expert alone with a unit gate gives ``shared_raw`` exactly as the block adds it."""
    L, x16, ids, wb, sg = _routed if _routed is not None else _stage_route(g_row, E_, layer)
    ones = torch.ones_like(sg)
    raw = _stage_experts(L, x16, ids, wb, 0, 0, ones)  # no routed expert in range: 0 + 1 * shared
    prob = sg.reshape(-1, 1)
    return dict(shared_raw=raw, shared_gate_prob=prob, shared_out=prob * raw)


def moe_routed(g_row: torch.Tensor, E_, route: dict | None = None, layer: int = 0, _routed=None) -> dict:
    """``engine/block_forward.py:652 moe_routed``: ``expert_raw`` [T, 8, 2048] (each slot's
    expert output before weighting, in top-k slot order) and ``routed_sum`` [T, 2048] (the
    weighted outputs added in ascending expert id, the f32 form of ``engine/m3_forward.py:452,
    464-465``). The routing is this library's own (``route`` is accepted for call-shape parity
    and must match it: ``topk_ids`` are checked when given)."""
    L, x16, ids, wb, sg = _routed if _routed is not None else _stage_route(g_row, E_, layer)
    if route is not None and "topk_ids" in route:
        if not torch.equal(route["topk_ids"].reshape(ids.shape).to(ids.dtype), ids):
            raise Refused("route", "topk_ids differ from the device routing of these rows")
    T = x16.shape[0]
    unit = torch.full_like(wb, 0x3F80)  # bf16 1.0: y = o * 1
    raw = torch.empty((T, TOPK, H), dtype=torch.float32, device=L.device)
    for k in range(TOPK):  # one slot at a time: the other slots' ids are out of every range
        ids_k = torch.full_like(ids, -1)
        ids_k[:, k] = ids[:, k]
        raw[:, k] = _stage_experts(L, x16, ids_k, unit, 0, E, None)
    return dict(expert_raw=raw, routed_sum=_stage_experts(L, x16, ids, wb, 0, E, None))


def moe_block_stages(g_row: torch.Tensor, E_, layer: int = 0) -> dict:
    """``engine/block_forward.py:670 moe_block`` (stage order of its section 11.1): the shared
    stages, the router stages (:func:`moe_router`), the routed stages, and ``combined_out`` =
    ``routed_sum + shared_out`` -- bit-identical to :func:`moe_block` with ``path="prefill"``."""
    r = _stage_route(g_row, E_, layer)
    st = moe_shared(g_row, E_, layer, _routed=r)
    st.update(moe_router(g_row, E_, layer))
    st.update(moe_routed(g_row, E_, None, layer, _routed=r))
    st["combined_out"] = st["routed_sum"] + st["shared_out"]
    return st


def prefill_status(T: int, device) -> int:
    """Device status word of the cached prefill workspace (0 = every pipeline wait completed)."""
    return _abi.prefill_status(prefill_workspace(T, device), T)


__all__ = ["moe_block", "moe_router", "moe_shared", "moe_routed", "moe_block_stages", "moe_stack", "Refused",
           "N_LAYERS"]
