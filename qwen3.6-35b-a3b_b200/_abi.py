"""ctypes binding of ``libb200moe.so`` (declared in ``include/b200moe.h``).

Thin and strict: each wrapper checks the C return code and raises :class:`B200MoeError`
with the library's own message. Tensors are passed as raw device pointers; the caller's
current torch CUDA stream is used unless a stream is given. There is no fallback: if the
library is missing or no CUDA device is present the call raises.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("B200MOE_LIB") or os.path.join(PKG_DIR, "libb200moe.so")

OK, EINVAL, ECUDA, ESIZE = 0, 1, 2, 3
F32, BF16 = 0, 1

# Every exported symbol of include/b200moe.h (checked by tests/test_abi_exports.py).
EXPORTS = ("b200moe_abi_version", "b200moe_last_error", "b200moe_q4k_dequant", "b200moe_dequant",
           "b200moe_synth_q4k", "b200moe_router_workspace_size", "b200moe_router",
           "b200moe_decode_workspace_size",
           "b200moe_moe_decode", "b200moe_moe_decode_stages", "b200moe_moe_decode_noalloc", "b200moe_decode_status",
           "b200moe_decode_noalloc_status", "b200moe_debug_decode_faults", "b200moe_decode_persistent_info",
           "b200moe_decode_persistent_formats",
           "b200moe_stack_workspace_size",
           "b200moe_stack_decode",
           "b200moe_prefill_workspace_size", "b200moe_moe_prefill", "b200moe_moe_route",
           "b200moe_moe_experts", "b200moe_prefill_status", "b200moe_ep_pack", "b200moe_ep_experts",
           "b200moe_ep_combine", "b200moe_ep_dispatch_p2p", "b200moe_ep_experts_p2p", "b200moe_ep_combine_p2p",
           "b200moe_ipc_handle", "b200moe_ipc_open", "b200moe_ipc_close")
IPC_HANDLE_BYTES = 64

EP_ROW_BYTES = 4160   # B200MOE_EP_ROW_BYTES: 2048 fp16 x, 8 int32 ids, 8 bf16 weights, 16 B pad


class B200MoeError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__("%s failed (code %d): %s" % (fn, code, msg))
        self.code = code


class Layer(ctypes.Structure):
    """``struct b200moe_layer``."""
    _fields_ = [("gate", ctypes.c_void_p), ("up", ctypes.c_void_p),
                ("gate_up_expert_stride", ctypes.c_int64),
                ("down", ctypes.c_void_p), ("down_expert_stride", ctypes.c_int64),
                ("sh_gate", ctypes.c_void_p), ("sh_up", ctypes.c_void_p),
                ("sh_down", ctypes.c_void_p), ("router_w", ctypes.c_void_p),
                ("sh_gate_w", ctypes.c_void_p), ("logit_bias", ctypes.c_void_p),
                ("router_f32", ctypes.c_int32), ("norm_w", ctypes.c_void_p),
                ("down_type", ctypes.c_int32), ("sh_type", ctypes.c_int32), ("gate_type", ctypes.c_int32)]


class EpPeers(ctypes.Structure):
    """``struct b200moe_ep_peers``."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("recv", ctypes.c_void_p * 8),
                ("ret", ctypes.c_void_p * 8), ("flag_dispatch", ctypes.c_void_p * 8),
                ("flag_return", ctypes.c_void_p * 8), ("epoch", ctypes.c_void_p), ("status", ctypes.c_void_p)]


class Stages(ctypes.Structure):
    """``struct b200moe_stages``."""
    _fields_ = [("bf16_stages", ctypes.c_int32), ("router_logits", ctypes.c_void_p),
                ("expert_raw", ctypes.c_void_p), ("routed_sum", ctypes.c_void_p),
                ("shared_raw", ctypes.c_void_p), ("shared_gate", ctypes.c_void_p)]


_LIB = None


def lib():
    """Load the shared library (no build here: ``__graft_entry__.build()`` makes it)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise B200MoeError("load", -1, "%s is missing; build it with "
                               "qwen3.6-35b-a3b_b200/build.py" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32, u64, sz = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint64,
                                 ctypes.c_size_t)
        L.b200moe_abi_version.restype = i32
        L.b200moe_abi_version.argtypes = []
        L.b200moe_last_error.restype = ctypes.c_char_p
        L.b200moe_last_error.argtypes = []
        L.b200moe_q4k_dequant.restype = i32
        L.b200moe_q4k_dequant.argtypes = [vp, i64, vp, i32, vp]
        L.b200moe_dequant.restype = i32
        L.b200moe_dequant.argtypes = [vp, i32, i64, vp, i32, vp]
        L.b200moe_synth_q4k.restype = i32
        L.b200moe_synth_q4k.argtypes = [u64, ctypes.c_uint32, i64, i64, vp, vp]
        L.b200moe_router_workspace_size.restype = sz
        L.b200moe_router_workspace_size.argtypes = [i32]
        L.b200moe_router.restype = i32
        L.b200moe_router.argtypes = [vp, i32, i32, vp, i32, vp, vp, vp, vp, vp, vp, sz, vp]
        L.b200moe_decode_workspace_size.restype = sz
        L.b200moe_decode_workspace_size.argtypes = [i32]
        L.b200moe_moe_decode.restype = i32
        L.b200moe_moe_decode.argtypes = [vp, i32, i32, ctypes.POINTER(Layer), vp, vp, vp, vp, sz, vp]
        L.b200moe_moe_decode_stages.restype = i32
        L.b200moe_moe_decode_stages.argtypes = [vp, i32, i32, ctypes.POINTER(Layer), ctypes.POINTER(Stages), vp, vp,
                                                vp, vp, sz, vp]
        L.b200moe_moe_decode_noalloc.restype = i32
        L.b200moe_moe_decode_noalloc.argtypes = [vp, i32, i32, ctypes.POINTER(Layer), vp, vp, vp, vp]
        L.b200moe_decode_status.restype = i32
        L.b200moe_decode_status.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_int), vp]
        L.b200moe_decode_noalloc_status.restype = i32
        L.b200moe_decode_noalloc_status.argtypes = [i32, ctypes.POINTER(ctypes.c_int), vp]
        L.b200moe_debug_decode_faults.restype = i32
        L.b200moe_debug_decode_faults.argtypes = [ctypes.c_longlong, i32]
        L.b200moe_decode_persistent_info.restype = i32
        L.b200moe_decode_persistent_info.argtypes = [ctypes.POINTER(i32), ctypes.POINTER(i32)]
        L.b200moe_decode_persistent_formats.restype = i32
        L.b200moe_decode_persistent_formats.argtypes = [ctypes.POINTER(i32)]
        L.b200moe_stack_workspace_size.restype = sz
        L.b200moe_stack_workspace_size.argtypes = [i32, i32]
        L.b200moe_stack_decode.restype = i32
        L.b200moe_stack_decode.argtypes = [vp, i32, ctypes.POINTER(Layer), i32, ctypes.c_float,
                                           vp, vp, sz, vp]
        L.b200moe_prefill_workspace_size.restype = sz
        L.b200moe_prefill_workspace_size.argtypes = [i32]
        L.b200moe_moe_prefill.restype = i32
        L.b200moe_moe_prefill.argtypes = [vp, i32, vp, ctypes.c_float, i32, ctypes.POINTER(Layer), vp, vp, vp,
                                          sz, vp]
        L.b200moe_moe_route.restype = i32
        L.b200moe_moe_route.argtypes = [vp, i32, vp, ctypes.c_float, i32, ctypes.POINTER(Layer), vp, vp, vp, vp,
                                        vp, sz, vp]
        L.b200moe_moe_experts.restype = i32
        L.b200moe_moe_experts.argtypes = [vp, i32, vp, vp, i32, i32, vp, i32, i32, ctypes.POINTER(Layer), vp, i32,
                                          vp, sz, vp]
        L.b200moe_prefill_status.restype = i32
        L.b200moe_prefill_status.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_int), vp]
        L.b200moe_ep_pack.restype = i32
        L.b200moe_ep_pack.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp]
        L.b200moe_ep_experts.restype = i32
        L.b200moe_ep_experts.argtypes = [vp, i32, i32, i32, vp, ctypes.POINTER(Layer), vp, vp, sz, vp]
        L.b200moe_ep_combine.restype = i32
        L.b200moe_ep_combine.argtypes = [vp, vp, i32, i32, vp, i32, vp]
        L.b200moe_ep_dispatch_p2p.restype = i32
        L.b200moe_ep_dispatch_p2p.argtypes = [vp, vp, vp, i32, ctypes.POINTER(EpPeers), vp, vp]
        L.b200moe_ep_experts_p2p.restype = i32
        L.b200moe_ep_experts_p2p.argtypes = [i32, vp, ctypes.POINTER(Layer), ctypes.POINTER(EpPeers), vp, sz, vp]
        L.b200moe_ep_combine_p2p.restype = i32
        L.b200moe_ep_combine_p2p.argtypes = [i32, vp, ctypes.POINTER(EpPeers), vp, i32, vp]
        L.b200moe_ipc_handle.restype = i32
        L.b200moe_ipc_handle.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]
        L.b200moe_ipc_open.restype = i32
        L.b200moe_ipc_open.argtypes = [ctypes.c_char_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p)]
        L.b200moe_ipc_close.restype = i32
        L.b200moe_ipc_close.argtypes = [vp, ctypes.c_int64]
        _LIB = L
    return _LIB


def _check(fn: str, rc: int):
    if rc != OK:
        msg = lib().b200moe_last_error()
        raise B200MoeError(fn, rc, msg.decode() if msg else "")


def _stream(stream):
    if stream is not None:
        return ctypes.c_void_p(int(stream))
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def ptr(t):
    """Device pointer of a torch tensor (None -> NULL); refuses host tensors."""
    if t is None:
        return None
    if not t.is_cuda:
        raise B200MoeError("ptr", EINVAL, "tensor on %s; the b200moe path needs CUDA tensors" % t.device)
    if not t.is_contiguous():
        raise B200MoeError("ptr", EINVAL, "tensor must be contiguous")
    return ctypes.c_void_p(t.data_ptr())


def abi_version() -> int:
    return int(lib().b200moe_abi_version())


def q4k_dequant(blocks, out, out_dtype: int, stream=None):
    nb = blocks.numel() // 144
    _check("b200moe_q4k_dequant", lib().b200moe_q4k_dequant(ptr(blocks), nb, ptr(out), out_dtype,
                                                             _stream(stream)))


# GGML block type ids accepted by b200moe_dequant, and their block sizes (bytes, elements).
from .geometry import BLOCK_GEOM, TYPE_IDS  # noqa: E402


def dequant(blocks, tname: str, out, out_dtype: int, stream=None):
    """``b200moe_dequant`` of every whole block in the uint8 tensor ``blocks``."""
    nb = blocks.numel() // BLOCK_GEOM[tname][0]
    _check("b200moe_dequant", lib().b200moe_dequant(ptr(blocks), TYPE_IDS[tname], nb, ptr(out), out_dtype,
                                                     _stream(stream)))


def synth_q4k(seed: int, stream_id: int, block0: int, nblocks: int, out, stream=None):
    _check("b200moe_synth_q4k", lib().b200moe_synth_q4k(int(seed), int(stream_id), int(block0),
                                                         int(nblocks), ptr(out), _stream(stream)))


def router_workspace_size(T: int) -> int:
    return int(lib().b200moe_router_workspace_size(T))


def router(x, x_dtype: int, T: int, wg, bias, logits, ids, w_f32, w_bf16, ws=None, stream=None):
    import torch
    if ws is None:
        ws = torch.empty(router_workspace_size(T), dtype=torch.uint8, device=x.device)
    wdt = F32 if wg.dtype == torch.float32 else BF16
    _check("b200moe_router", lib().b200moe_router(ptr(x), x_dtype, T, ptr(wg), wdt, ptr(bias), ptr(logits),
                                                   ptr(ids), ptr(w_f32), ptr(w_bf16), ptr(ws),
                                                   ws.numel() * ws.element_size(), _stream(stream)))


def decode_workspace_size(T: int) -> int:
    return int(lib().b200moe_decode_workspace_size(T))


def moe_decode(x, x_dtype: int, T: int, layer: Layer, out, ids_out, w_out, ws, stream=None):
    _check("b200moe_moe_decode",
           lib().b200moe_moe_decode(ptr(x), x_dtype, T, ctypes.byref(layer), ptr(out), ptr(ids_out),
                                    ptr(w_out), ptr(ws), ws.numel() * ws.element_size(), _stream(stream)))


def moe_decode_stages(x, x_dtype: int, T: int, layer: Layer, bf16_stages: bool, out, ids_out, w_out, ws,
                      router_logits=None, expert_raw=None, routed_sum=None, shared_raw=None, shared_gate=None,
                      stream=None):
    """``b200moe_moe_decode_stages``: the decode path with its stage tensors written out."""
    p = lambda t: None if t is None else ptr(t).value  # noqa: E731
    st = Stages(1 if bf16_stages else 0, p(router_logits), p(expert_raw), p(routed_sum), p(shared_raw),
                p(shared_gate))
    _check("b200moe_moe_decode_stages",
           lib().b200moe_moe_decode_stages(ptr(x), x_dtype, T, ctypes.byref(layer), ctypes.byref(st), ptr(out),
                                           ptr(ids_out), ptr(w_out), ptr(ws), ws.numel() * ws.element_size(),
                                           _stream(stream)))


def decode_persistent_info():
    """(ctas, cluster) of the persistent single-token decode kernel on the current device, or
    (0, 0) when the device runs the three-kernel path."""
    a, c = ctypes.c_int(0), ctypes.c_int(0)
    _check("b200moe_decode_persistent_info", lib().b200moe_decode_persistent_info(ctypes.byref(a), ctypes.byref(c)))
    return a.value, c.value


def decode_persistent_formats() -> bool:
    """Whether single-token layers in the other block formats also run on the persistent kernel."""
    f = ctypes.c_int(0)
    _check("b200moe_decode_persistent_formats", lib().b200moe_decode_persistent_formats(ctypes.byref(f)))
    return bool(f.value)


def moe_decode_noalloc(x, x_dtype: int, T: int, layer: Layer, out, ids_out, w_out, stream=None):
    """b200moe_moe_decode with the library's built-in scratch (no workspace, no allocation)."""
    _check("b200moe_moe_decode_noalloc",
           lib().b200moe_moe_decode_noalloc(ptr(x), x_dtype, T, ctypes.byref(layer), ptr(out), ptr(ids_out),
                                            ptr(w_out), _stream(stream)))


def decode_status(ws, T: int, stream=None) -> int:
    """Status word of the last decode call on workspace ``ws`` with T tokens (0 = complete)."""
    st = ctypes.c_int(-1)
    _check("b200moe_decode_status", lib().b200moe_decode_status(ptr(ws), T, ctypes.byref(st), _stream(stream)))
    return int(st.value)


def decode_noalloc_status(T: int, stream=None) -> int:
    """Status word of the last ``b200moe_moe_decode_noalloc`` call with T tokens (0 = complete)."""
    st = ctypes.c_int(-1)
    _check("b200moe_decode_noalloc_status", lib().b200moe_decode_noalloc_status(T, ctypes.byref(st),
                                                                                 _stream(stream)))
    return int(st.value)


def debug_decode_faults(wait_budget_cycles: int = 0, withhold_cta: int = -1):
    """Test hook of the persistent decode kernel's failure path (reset with the defaults)."""
    _check("b200moe_debug_decode_faults", lib().b200moe_debug_decode_faults(int(wait_budget_cycles),
                                                                             int(withhold_cta)))


def stack_workspace_size(T: int, n_layers: int) -> int:
    return int(lib().b200moe_stack_workspace_size(T, n_layers))


def stack_decode(resid, T: int, layers, eps: float, ids_out, ws, stream=None):
    arr = (Layer * len(layers))(*layers)
    _check("b200moe_stack_decode",
           lib().b200moe_stack_decode(ptr(resid), T, arr, len(layers), eps, ptr(ids_out), ptr(ws),
                                      ws.numel() * ws.element_size(), _stream(stream)))


def prefill_workspace_size(T: int) -> int:
    return int(lib().b200moe_prefill_workspace_size(T))


def moe_prefill(x, x_dtype: int, resid, eps: float, T: int, layer: Layer, out, ids_out, ws, stream=None):
    _check("b200moe_moe_prefill",
           lib().b200moe_moe_prefill(ptr(x), x_dtype, ptr(resid), eps, T, ctypes.byref(layer), ptr(out),
                                     ptr(ids_out), ptr(ws), ws.numel() * ws.element_size(), _stream(stream)))


def prefill_status(ws, T: int, stream=None) -> int:
    st = ctypes.c_int(-1)
    _check("b200moe_prefill_status", lib().b200moe_prefill_status(ptr(ws), T, ctypes.byref(st), _stream(stream)))
    return int(st.value)


def moe_route(x, x_dtype: int, resid, eps: float, T: int, layer: Layer, x16_out, ids_out, w_out, sg_out, ws,
              stream=None):
    _check("b200moe_moe_route",
           lib().b200moe_moe_route(ptr(x), x_dtype, ptr(resid), eps, T, ctypes.byref(layer), ptr(x16_out),
                                   ptr(ids_out), ptr(w_out), ptr(sg_out), ptr(ws), ws.numel() * ws.element_size(),
                                   _stream(stream)))


def moe_experts(x16, T: int, ids, w_bf16, e_lo: int, e_hi: int, sg, layer: Layer, out, accumulate: bool, ws,
                stream=None, sh_rows=None):
    """b200moe_moe_experts; ``sh_rows`` = (lo, hi): the rows that get sg[t - lo] * shared expert
    (default: all T rows when sg is given)."""
    lo, hi = sh_rows if sh_rows is not None else (0, T)
    _check("b200moe_moe_experts",
           lib().b200moe_moe_experts(ptr(x16), T, ptr(ids), ptr(w_bf16), int(e_lo), int(e_hi), ptr(sg), int(lo),
                                     int(hi), ctypes.byref(layer), ptr(out), 1 if accumulate else 0, ptr(ws),
                                     ws.numel() * ws.element_size(), _stream(stream)))


def ep_pack(x16, ids, w_bf16, T: int, rank: int, world: int, send_rows, pos, stream=None):
    """``b200moe_ep_pack``: send_rows [world, T, EP_ROW_BYTES] uint8, pos [T, world] int32."""
    _check("b200moe_ep_pack", lib().b200moe_ep_pack(ptr(x16), ptr(ids), ptr(w_bf16), T, rank, world,
                                                     ptr(send_rows), ptr(pos), _stream(stream)))


def ep_experts(recv_rows, T: int, rank: int, world: int, sg, layer: Layer, partial, ws, stream=None):
    """``b200moe_ep_experts``: partial [world, T, 2048] f32 from recv_rows [world, T, EP_ROW_BYTES]."""
    _check("b200moe_ep_experts",
           lib().b200moe_ep_experts(ptr(recv_rows), T, rank, world, ptr(sg), ctypes.byref(layer), ptr(partial),
                                    ptr(ws), ws.numel() * ws.element_size(), _stream(stream)))


def ep_combine(ret, pos, T: int, world: int, out, accumulate: bool, stream=None):
    """``b200moe_ep_combine``: out [T, 2048] f32 (+)= ascending-rank sum of the returned partial rows."""
    _check("b200moe_ep_combine", lib().b200moe_ep_combine(ptr(ret), ptr(pos), T, world, ptr(out),
                                                           1 if accumulate else 0, _stream(stream)))


def ipc_handle(t):
    """(64-byte handle, offset) of the CUDA allocation holding tensor ``t``."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_int64(0)
    _check("b200moe_ipc_handle", lib().b200moe_ipc_handle(ptr(t), buf, ctypes.byref(off)))
    return buf.raw, int(off.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Map a peer's allocation; returns the device address of its buffer."""
    p = ctypes.c_void_p(0)
    _check("b200moe_ipc_open", lib().b200moe_ipc_open(handle, int(offset), ctypes.byref(p)))
    return int(p.value)


def ipc_close(addr: int, offset: int):
    _check("b200moe_ipc_close", lib().b200moe_ipc_close(ctypes.c_void_p(addr), int(offset)))


def ep_dispatch_p2p(x16, ids, w_bf16, T: int, peers: EpPeers, pos, stream=None):
    _check("b200moe_ep_dispatch_p2p", lib().b200moe_ep_dispatch_p2p(ptr(x16), ptr(ids), ptr(w_bf16), T,
                                                                     ctypes.byref(peers), ptr(pos), _stream(stream)))


def ep_experts_p2p(T: int, sg, layer: Layer, peers: EpPeers, ws, stream=None):
    _check("b200moe_ep_experts_p2p",
           lib().b200moe_ep_experts_p2p(T, ptr(sg), ctypes.byref(layer), ctypes.byref(peers), ptr(ws),
                                        ws.numel() * ws.element_size(), _stream(stream)))


def ep_combine_p2p(T: int, pos, peers: EpPeers, out, accumulate: bool, stream=None):
    _check("b200moe_ep_combine_p2p", lib().b200moe_ep_combine_p2p(T, ptr(pos), ctypes.byref(peers), ptr(out),
                                                                   1 if accumulate else 0, _stream(stream)))
