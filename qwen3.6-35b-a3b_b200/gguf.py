"""GGUF reader for the MoE block's tensors: one layer's expert stacks, shared expert and router
straight from a GGUF file into :class:`DeviceLayer` (no dequantisation, no copy of the Q4_K
bytes on the host: the tensor data is memory-mapped).

Replaces the reference's ``tools/gguf_reader.py:492 Gguf`` (header parse) and the byte ranges
``engine/loader.py`` addresses (``blk.N.ffn_{gate,up,down}_exps.weight``, expert axis slowest,
``engine/README.md:172-190``). The container format is GGUF v2/v3 as llama.cpp writes it:

    magic "GGUF" | u32 version | u64 n_tensors | u64 n_kv
    n_kv x (string key, u32 value type, value)        strings: u64 length + UTF-8 bytes
    n_tensors x (string name, u32 n_dims, u64 dims[n_dims] (fastest first), u32 ggml type,
                 u64 offset from the data section)
    data section at the next multiple of ``general.alignment`` (default 32)

Block types the device paths take, as stored: expert gate / up Q4_K (type 12); expert down
Q4_K, Q5_K (13) or Q6_K (14); the shared expert Q4_K or Q8_0 (8) -- the published Q4_K_M file
has Q5_K down (Q6_K at three layers) and a Q8_0 shared expert, which run on the decode kernels
(the grouped GEMMs take Q4_K layers). The router and shared-expert gate are used as stored,
bf16 (type 30) or F32 (type 0; F16 is widened to f32 exactly). Other types are refused by name.
"""
from __future__ import annotations

import mmap
import struct

import numpy as np

from .geometry import DOWN_TYPES, E, H, I, SHARED_TYPES

GGML_TYPES = {0: "F32", 1: "F16", 2: "Q4_0", 3: "Q4_1", 6: "Q5_0", 7: "Q5_1", 8: "Q8_0", 9: "Q8_1",
              10: "Q2_K", 11: "Q3_K", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 15: "Q8_K", 30: "BF16"}
# (elements, bytes) per block of the types whose sizes the reader needs
BLOCK = {"F32": (1, 4), "F16": (1, 2), "BF16": (1, 2), "Q4_K": (256, 144), "Q5_K": (256, 176),
         "Q6_K": (256, 210), "Q8_0": (32, 34), "Q4_0": (32, 18)}
# struct format and size of each fixed-width GGUF metadata value type (GGUF spec value-type ids)
_VALUE_TYPE_FMT = {0: ("<B", 1), 1: ("<b", 1), 2: ("<H", 2), 3: ("<h", 2), 4: ("<I", 4), 5: ("<i", 4),
                   6: ("<f", 4), 7: ("<?", 1), 10: ("<Q", 8), 11: ("<q", 8), 12: ("<d", 8)}


class GgufError(ValueError):
    """A malformed file, a missing tensor, or a tensor the device path cannot take."""

    def __init__(self, tag: str, msg: str):
        super().__init__("[%s] %s" % (tag, msg))
        self.tag = tag


class TensorInfo:
    __slots__ = ("name", "dims", "type_id", "type_name", "offset", "n_elts", "nbytes")

    def __init__(self, name, dims, type_id, offset):
        self.name = name
        self.dims = tuple(int(d) for d in dims)  # GGUF order: dims[0] is the fastest axis
        self.type_id = int(type_id)
        self.type_name = GGML_TYPES.get(self.type_id, "type_%d" % self.type_id)
        self.offset = int(offset)
        n = 1
        for d in self.dims:
            n *= d
        self.n_elts = n
        be, bb = BLOCK.get(self.type_name, (0, 0))
        self.nbytes = (n // be) * bb if be else None

    def __repr__(self):
        return "TensorInfo(%s, dims=%s, %s, offset=%d)" % (self.name, self.dims, self.type_name, self.offset)


class GgufFile:
    """Header of a GGUF file; tensor bytes on demand from a read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        self._fh = open(path, "rb")
        try:
            self._mm = mmap.mmap(self._fh.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:  # empty file
            self._fh.close()
            raise GgufError("format", "%s: %s" % (path, e))
        self._parse()

    def close(self):
        try:
            self._mm.close()
        except BufferError:  # byte views handed out are still alive: the map goes with the last one
            pass
        self._fh.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ------------------------------------------------------------------ header
    def _parse(self):
        mm, pos = self._mm, [0]

        def take(k):
            if pos[0] + k > len(mm):
                raise GgufError("format", "header truncated at byte %d (wanted %d more)" % (pos[0], k))
            v = mm[pos[0]:pos[0] + k]
            pos[0] += k
            return v

        def u32():
            return struct.unpack("<I", take(4))[0]

        def u64():
            return struct.unpack("<Q", take(8))[0]

        def string():
            return bytes(take(u64())).decode("utf-8", "replace")

        def value(vt):
            if vt == 8:
                return string()
            if vt == 9:
                et, cnt = u32(), u64()
                return [value(et) for _ in range(cnt)]
            if vt in _VALUE_TYPE_FMT:
                f, k = _VALUE_TYPE_FMT[vt]
                return struct.unpack(f, take(k))[0]
            raise GgufError("format", "unknown metadata value type %d at byte %d" % (vt, pos[0]))

        if bytes(take(4)) != b"GGUF":
            raise GgufError("format", "%s is not a GGUF file" % self.path)
        self.version = u32()
        if self.version not in (2, 3):
            raise GgufError("format", "GGUF version %d (this reader knows 2 and 3)" % self.version)
        n_tensors, n_kv = u64(), u64()
        self.meta = {}
        for _ in range(n_kv):
            k = string()
            self.meta[k] = value(u32())
        self.tensors = {}
        for _ in range(n_tensors):
            name = string()
            nd = u32()
            dims = [u64() for _ in range(nd)]
            ti = TensorInfo(name, dims, u32(), u64())
            self.tensors[name] = ti
        align = int(self.meta.get("general.alignment", 32))
        self.data_start = (pos[0] + align - 1) // align * align
        for ti in self.tensors.values():
            if ti.nbytes is not None and self.data_start + ti.offset + ti.nbytes > len(mm):
                raise GgufError("format", "%s runs past the end of the file" % ti.name)

    # ------------------------------------------------------------------ data
    def info(self, name: str) -> TensorInfo:
        ti = self.tensors.get(name)
        if ti is None:
            raise GgufError("missing", "%s has no tensor %r" % (self.path, name))
        return ti

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the file (no copy)."""
        ti = self.info(name)
        if ti.nbytes is None:
            raise GgufError("type", "%s: block size of %s unknown to this reader" % (name, ti.type_name))
        start = self.data_start + ti.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=ti.nbytes, offset=start)


def _want(gf: GgufFile, name: str, types, dims) -> TensorInfo:
    ti = gf.info(name)
    if ti.type_name not in types:
        raise GgufError("type", "%s is %s; the device path takes %s" % (name, ti.type_name, "/".join(types)))
    strip = lambda t: tuple(t[:max([i + 1 for i, d in enumerate(t) if d != 1] or [0])])  # noqa: E731
    if strip(ti.dims) != strip(tuple(dims)):  # trailing unit dims are immaterial
        raise GgufError("shape", "%s has dims %s (GGUF order), expected %s" % (name, ti.dims, tuple(dims)))
    return ti


_TENSORS = (("gate", "ffn_gate_exps", (H, I, E), ("Q4_K",)), ("up", "ffn_up_exps", (H, I, E), ("Q4_K",)),
            ("down", "ffn_down_exps", (I, H, E), DOWN_TYPES), ("sh_gate", "ffn_gate_shexp", (H, I), SHARED_TYPES),
            ("sh_up", "ffn_up_shexp", (H, I), SHARED_TYPES), ("sh_down", "ffn_down_shexp", (I, H), SHARED_TYPES))


def layer_types(gf: GgufFile, layer: int) -> dict:
    """{"down_type": ..., "sh_type": ...} of layer ``layer`` (block type names as stored). The
    three shared tensors must share one type."""
    p = "blk.%d." % layer
    t = {kind: _want(gf, p + nm + ".weight", types, dims).type_name for kind, nm, dims, types in _TENSORS}
    if len({t["sh_gate"], t["sh_up"], t["sh_down"]}) != 1:
        raise GgufError("type", "blk.%d shared expert mixes block types %s / %s / %s" % (
            layer, t["sh_gate"], t["sh_up"], t["sh_down"]))
    return dict(down_type=t["down"], sh_type=t["sh_gate"])


def layer_host(gf: GgufFile, layer: int, round_router: bool = False) -> tuple:
    """(blocks dict, router bf16 bits [256*2048], shared-gate bf16 bits [2048]) of layer
    ``layer``: the block-byte views of ``blk.<layer>.ffn_{gate,up,down}_exps`` and
    ``ffn_{gate,up,down}_shexp`` in their stored formats (:func:`layer_types` names them;
    views into the memory map: valid while ``gf`` is open) and the router / shared-gate
    vectors (copies).

    The router and gate keep their stored type (F32, or F16 widened exactly, as f32 values;
    BF16 as bits). ``round_router``: round F32 / F16 router and gate weights to bf16 (RNE)
    instead -- half the router bytes, but different logits from the stored values'."""
    p = "blk.%d." % layer
    blocks = {}
    for kind, nm, dims, types in _TENSORS:
        _want(gf, p + nm + ".weight", types, dims)
        blocks[kind] = gf.raw(p + nm + ".weight")
    router = _vector_bf16(gf, p + "ffn_gate_inp.weight", (H, E), round_router)
    shgate = _vector_bf16(gf, p + "ffn_gate_inp_shexp.weight", (H,), round_router)
    return blocks, router, shgate


def _vector_bf16(gf: GgufFile, name: str, dims, round_ok: bool) -> np.ndarray:
    """bf16 bits (uint16) of a BF16 tensor; f32 values (float32) of an F32 / F16 one, or their
    bf16 rounding when ``round_ok``."""
    ti = _want(gf, name, ("BF16", "F32", "F16"), dims)
    raw = gf.raw(name)
    if ti.type_name == "BF16":
        return raw.view(np.uint16).copy()
    f = raw.view(np.float32) if ti.type_name == "F32" else raw.view(np.float16).astype(np.float32)
    if not round_ok:
        return f.copy()
    u = f.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)   # round to nearest even
    r[nan] = 0x7FC0
    return r


def layer_norm(gf: GgufFile, layer: int):
    """f32 values of ``blk.<layer>.post_attention_norm.weight`` (Form A: the file holds 1 + w;
    F32 as stored, BF16 / F16 widened exactly), or None when the file has no such tensor."""
    name = "blk.%d.post_attention_norm.weight" % layer
    if name not in gf.tensors:
        return None
    ti = _want(gf, name, ("F32", "BF16", "F16"), (H,))
    raw = gf.raw(name)
    if ti.type_name == "F32":
        return raw.view(np.float32).copy()
    if ti.type_name == "F16":
        return raw.view(np.float16).astype(np.float32)
    return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)


def device_layer(gf: GgufFile, layer: int, device="cuda", round_router: bool = False):
    """:class:`DeviceLayer` of layer ``layer`` read from ``gf`` (block bytes uploaded as stored,
    with their types; the post-attention norm weight when the file has it)."""
    from .engine import DeviceLayer
    types = layer_types(gf, layer)
    blocks, router, shgate = layer_host(gf, layer, round_router)
    return DeviceLayer.from_host(blocks, router, shgate, device=device, norm_w=layer_norm(gf, layer), **types)


def device_engine(path: str, layers=None, device="cuda", round_router: bool = False):
    """:class:`DeviceEngine` of the given layers (default: every ``blk.N`` with MoE tensors)."""
    from .engine import DeviceEngine
    with GgufFile(path) as gf:
        if layers is None:
            layers = sorted({int(n.split(".")[1]) for n in gf.tensors if n.endswith(".ffn_gate_exps.weight")})
        return DeviceEngine([device_layer(gf, l, device, round_router) for l in layers])
