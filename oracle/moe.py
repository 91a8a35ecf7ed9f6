"""MoE block oracle (test infrastructure only).

* :func:`router`          -- R1..R5 under the declared deterministic order, via the C
                             restatement (``oracle/c/oracle.c``); restates
                             ``engine/m3_forward.py:443-446``.
* :func:`moe_block_f64`   -- f64 restatement of ``engine/m3_forward.py:430-476``
                             (``moe_block``) given the routing: shared expert
                             :436-442, routed experts in ascending id :452-465, sum :475.
* :func:`moe_block_port`  -- torch-f32 port of the same function, structured like the
                             reference (per hit expert: dequant, three F.linear, weighted
                             add in ascending id). This is the CPU path that ``bench.py``
                             times as the reference arm / ``cpu_baseline`` (kind "port").
* :func:`rmsnorm`, :func:`stack_f64` -- the config-4 layer glue
                             (``engine/m3_forward.py:303-307, 731-737``).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import kquants, q4k
from .bf16 import bf16_bits_to_f32

H, E, TOPK, I = 2048, 256, 8, 512
_LIB = None


def lib():
    """Load (building if needed) the C oracle."""
    global _LIB
    if _LIB is None:
        from .build import build
        path = build()
        L = ctypes.CDLL(path)
        f32p, u16p, i32p = (ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_uint16),
                            ctypes.POINTER(ctypes.c_int32))
        L.b2o_expf.restype = ctypes.c_float
        L.b2o_expf.argtypes = [ctypes.c_float]
        L.b2o_q4k_dequant.argtypes = [ctypes.c_void_p, ctypes.c_int64, f32p]
        L.b2o_router.argtypes = [f32p, ctypes.c_int, u16p, f32p, u16p, f32p, i32p, f32p, u16p]
        L.b2o_router_f32w.argtypes = [f32p, ctypes.c_int, f32p, f32p, u16p, f32p, i32p, f32p, u16p]
        L.b2o_rmsnorm.argtypes = [f32p, ctypes.c_int, ctypes.c_float, f32p]
        L.b2o_dot_chunked.restype = ctypes.c_float
        L.b2o_dot_chunked.argtypes = [f32p, u16p]
        _LIB = L
    return _LIB


def _p(a, ct):
    return a.ctypes.data_as(ctypes.POINTER(ct))


def expf(x) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    f = lib().b2o_expf
    return np.array([f(float(v)) for v in x], dtype=np.float32)


def dequant_c(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = blocks.size // q4k.BLOCK_BYTES
    out = np.empty(nb * 256, dtype=np.float32)
    lib().b2o_q4k_dequant(blocks.ctypes.data, nb, _p(out, ctypes.c_float))
    return out


def wvals(w) -> np.ndarray:
    """Router / shared-gate weights as f32 values: bf16 bits (uint16) widen exactly; f32 as is."""
    w = np.asarray(w)
    return w.astype(np.float32) if w.dtype == np.float32 else bf16_bits_to_f32(w.astype(np.uint16))


def router(x_f32: np.ndarray, wg_bits: np.ndarray, bias: np.ndarray | None = None) -> dict:
    """Declared-order R1..R5 for x [T, 2048] (f32 values), W_g [256, 2048] as bf16 bits
    (uint16) or as f32 values (float32: the published file's F32 router)."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32).reshape(-1, H)
    f32w = np.asarray(wg_bits).dtype == np.float32
    wg = np.ascontiguousarray(wg_bits, dtype=np.float32 if f32w else np.uint16).reshape(E, H)
    T = x.shape[0]
    logits = np.empty((T, E), dtype=np.uint16)
    probs = np.empty((T, E), dtype=np.float32)
    ids = np.empty((T, TOPK), dtype=np.int32)
    wf = np.empty((T, TOPK), dtype=np.float32)
    wb = np.empty((T, TOPK), dtype=np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    (lib().b2o_router_f32w if f32w else lib().b2o_router)(
                     _p(x, ctypes.c_float), T, _p(wg, ctypes.c_float if f32w else ctypes.c_uint16),
                     None if b is None else _p(b, ctypes.c_float), _p(logits, ctypes.c_uint16),
                     _p(probs, ctypes.c_float), _p(ids, ctypes.c_int32), _p(wf, ctypes.c_float),
                     _p(wb, ctypes.c_uint16))
    return dict(logits=logits, probs=probs, ids=ids, w_f32=wf, w_bf16=wb)


def rmsnorm(x: np.ndarray, eps: float = 1e-6, w: np.ndarray | None = None) -> np.ndarray:
    """Declared-order RMSNorm (``engine/m3_forward.py:303 rmsnorm_a``): x * r, then * w when a
    Form A weight (as stored: 1 + w) is given -- two f32 roundings, as the reference's torch."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, H)
    y = np.empty_like(x)
    lib().b2o_rmsnorm(_p(x, ctypes.c_float), x.shape[0], eps, _p(y, ctypes.c_float))
    if w is not None:
        y = (y * np.asarray(w, dtype=np.float32).reshape(1, H)).astype(np.float32)
    return y


# ----------------------------------------------------------------------------------------
# layer weights on the host (for the oracle): Q4_K bytes + bf16 router / shared gate
# ----------------------------------------------------------------------------------------
class HostLayer:
    """One layer's weights as the oracle sees them.

    ``gate/up`` are [E, 512, 8, 144] Q4_K bytes, ``down`` [E, 2048, 2, 144]; ``sh_*`` the
    shared expert in the same per-expert shapes; ``wg`` [256, 2048] and ``wsg`` [2048]
    bf16 bits; ``bias`` an optional f32 [256] logit offset. Expert matrices are produced
    lazily (``expert_blocks``) so a test can hold a full 256-expert layer without
    materialising 453 MB. ``types`` (optional) names other block formats per kind, as the
    published Q4_K_M file has them: ``{"down": "Q5_K" | "Q6_K", "sh_gate" / "sh_up" /
    "sh_down": "Q8_0"}`` (kquants.py decodes them); ``block_fn`` then serves those kinds'
    blocks in their own sizes.
    """

    def __init__(self, block_fn, wg, wsg, bias=None, types=None, norm_w=None, bf16_weights=False):
        self._block_fn = block_fn     # (kind, first_block, nblocks) -> uint8 [n, block bytes]
        self.types = dict(types or {})
        # the dense layout: every expert / shared matrix holds the bf16 rounding (RNE) of its decode
        self.bf16_weights = bool(bf16_weights)
        # post-attention RMSNorm weight as stored (Form A: 1 + w), f32 [2048]; None = 1
        self.norm_w = None if norm_w is None else np.asarray(norm_w, dtype=np.float32).reshape(H)
        keep = lambda a: np.asarray(a) if np.asarray(a).dtype == np.float32 else np.asarray(a, np.uint16)  # noqa
        self.wg = np.ascontiguousarray(keep(wg)).reshape(E, H)      # bf16 bits, or f32 values
        self.wsg = np.ascontiguousarray(keep(wsg)).reshape(H)
        self.bias = None if bias is None else np.asarray(bias, dtype=np.float32)

    def matrix(self, kind: str, e: int = 0) -> np.ndarray:
        """Dequantized f32 matrix: gate/up [512, 2048], down [2048, 512] of expert e, or the
        shared ``sh_gate``/``sh_up``/``sh_down``."""
        rows, cols = {"gate": (I, H), "up": (I, H), "down": (H, I),
                      "sh_gate": (I, H), "sh_up": (I, H), "sh_down": (H, I)}[kind]
        tname = self.types.get(kind, "Q4_K")
        per = rows * cols // kquants.BLOCK_ELTS[tname]
        first = 0 if kind.startswith("sh_") else e * per
        blocks = self._block_fn(kind, first, per)
        m = kquants.dequant(np.ascontiguousarray(blocks).tobytes(), tname, per).reshape(rows, cols)
        if self.bf16_weights:
            from .bf16 import round_bf16
            m = round_bf16(m).reshape(rows, cols)
        return m


def silu64(z):
    return z / (1.0 + np.exp(-z))


def moe_block_f64(x_f32: np.ndarray, layer: HostLayer, ids: np.ndarray, w_bf16: np.ndarray) -> dict:
    """f64 restatement of ``engine/m3_forward.py:430-476`` with the routing given.

    ``x_f32`` [T, 2048]; ``ids`` [T, 8]; ``w_bf16`` [T, 8] bf16 bits (the R5-cast weights).
    Returns the block output [T, 2048] (routed + shared) and the stage tensors.
    """
    x = np.asarray(x_f32, dtype=np.float64).reshape(-1, H)
    T = x.shape[0]
    wsg_g = layer.matrix("sh_gate").astype(np.float64)
    wsg_u = layer.matrix("sh_up").astype(np.float64)
    wsg_d = layer.matrix("sh_down").astype(np.float64)
    shared_raw = (silu64(x @ wsg_g.T) * (x @ wsg_u.T)) @ wsg_d.T
    gate_prob = 1.0 / (1.0 + np.exp(-(x @ wvals(layer.wsg).astype(np.float64))))
    shared = gate_prob[:, None] * shared_raw
    w = bf16_bits_to_f32(np.asarray(w_bf16, dtype=np.uint16)).astype(np.float64).reshape(T, TOPK)
    ids = np.asarray(ids).reshape(T, TOPK)
    routed = np.zeros((T, H), dtype=np.float64)
    expert_raw = np.zeros((T, TOPK, H), dtype=np.float64)
    for e in sorted(set(int(v) for v in ids.reshape(-1))):       # ascending expert id
        rows, slots = np.nonzero(ids == e)
        g = layer.matrix("gate", e).astype(np.float64)
        u = layer.matrix("up", e).astype(np.float64)
        d = layer.matrix("down", e).astype(np.float64)
        xs = x[rows]
        o = (silu64(xs @ g.T) * (xs @ u.T)) @ d.T
        expert_raw[rows, slots] = o
        routed[rows] += o * w[rows, slots][:, None]
    return dict(out=routed + shared, routed=routed, shared_raw=shared_raw,
                shared_gate_prob=gate_prob, shared_out=shared, expert_raw=expert_raw)


def moe_block_port(x_f32, layer: HostLayer, threads: int | None = None) -> tuple:
    """torch-f32 port of ``engine/m3_forward.py:430-476`` as written: shared expert
    (:436-442), router R1-R5 with torch ops (:443-446), host-side grouping (:447-451), and
    per hit expert in ascending id a fresh dequant (:452-458, as ``Engine.expert`` does
    through ``gguf_fast_dequant.dequant_np``) then three F.linear and the weighted add
    (:459-465). Returns (out [T,2048] f32, ids [T,8])."""
    import torch
    import torch.nn.functional as F
    if threads:
        torch.set_num_threads(int(threads))
    x = torch.as_tensor(np.asarray(x_f32, dtype=np.float32)).reshape(-1, H)
    wg = torch.from_numpy(layer.matrix("sh_gate"))
    wu = torch.from_numpy(layer.matrix("sh_up"))
    wd = torch.from_numpy(layer.matrix("sh_down"))
    up = F.linear(x, wg)
    shared = F.linear(F.silu(up) * F.linear(x, wu), wd)
    wsg = torch.from_numpy(wvals(layer.wsg).copy()).reshape(1, H)
    shgate = torch.sigmoid(F.linear(x, wsg)).view(x.shape[0], 1)
    shared = shgate * shared
    wr = torch.from_numpy(wvals(layer.wg).copy())
    lf = F.linear(x, wr)
    if layer.bias is not None:
        lf = lf + torch.from_numpy(layer.bias)
    logits = lf.to(torch.bfloat16)
    probs = torch.softmax(logits.float(), dim=-1)
    tw, ids = torch.topk(probs, TOPK, dim=-1)
    wcast = (tw / tw.sum(-1, keepdim=True)).to(logits.dtype)
    routed = torch.zeros_like(x)
    used = {}
    for tok in range(x.shape[0]):
        for slot in range(TOPK):
            used.setdefault(int(ids[tok, slot]), []).append((tok, slot))
    for e in sorted(used):
        gate_w = torch.from_numpy(layer.matrix("gate", e))
        up_w = torch.from_numpy(layer.matrix("up", e))
        down_w = torch.from_numpy(layer.matrix("down", e))
        rows = [t for t, _ in used[e]]
        s = F.silu(F.linear(x[rows], gate_w)) * F.linear(x[rows], up_w)
        out_e = F.linear(s, down_w)
        wts = torch.stack([wcast[t, slot].to(torch.float32) for t, slot in used[e]])
        routed[rows] += out_e * wts[:, None]
    return (routed + shared).numpy(), ids.numpy()


def compare(out: np.ndarray, ref: np.ndarray) -> dict:
    """Parity figures: rel-L2, max-abs, max-abs normalised by max|ref|."""
    a = np.asarray(out, dtype=np.float64)
    b = np.asarray(ref, dtype=np.float64)
    diff = a - b
    rel = float(np.linalg.norm(diff) / max(np.linalg.norm(b), 1e-300))
    mx = float(np.max(np.abs(diff))) if diff.size else 0.0
    scale = float(np.max(np.abs(b))) if b.size else 1.0
    return dict(rel_l2=rel, max_abs=mx, max_abs_norm=mx / max(scale, 1e-300))


def rmsnorm_port(x, eps: float = 1e-6, w=None):
    """``engine/m3_forward.py:303-307`` rmsnorm_a, torch f32 (the reference's CPU op); ``w`` the
    stored weight (Form A: 1 + w) or None for weight 1."""
    import torch
    xf = torch.as_tensor(x).float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y if w is None else y * torch.as_tensor(w).float()


def stack_port(resid, layers, threads: int | None = None, eps: float = 1e-6):
    """The config-4 sub-stack on the CPU, as the reference's driver glues it
    (``engine/m3_forward.py:731-737`` with the mixer sublayer removed): per layer
    ``h = rmsnorm_a(x); x = x + moe_block(h)``. Returns the final residual (numpy f32)."""
    import torch
    x = torch.as_tensor(np.asarray(resid, dtype=np.float32)).reshape(-1, H).clone()
    for L in layers:
        h = rmsnorm_port(x, eps, getattr(L, "norm_w", None))
        out, _ = moe_block_port(h.numpy(), L, threads)
        x = x + torch.from_numpy(out)
    return x.numpy()


class CachedLayer(HostLayer):
    """A HostLayer whose expert bytes are pre-generated (so a timed run measures the
    reference's dequant + math, not the synthetic generator). ``prefetch(e)`` fills it."""

    def __init__(self, block_fn, wg, wsg, bias=None, types=None, norm_w=None):
        super().__init__(self._serve, wg, wsg, bias, types, norm_w)
        self._gen = block_fn
        self._cache = {}

    def _serve(self, kind, first, n):
        key = (kind, first, n)
        if key not in self._cache:
            self._cache[key] = self._gen(kind, first, n)
        return self._cache[key]
