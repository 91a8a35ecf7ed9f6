"""Device-resident Q4_K weights: the B200 replacement for the reference's weight source.

The reference's ``engine/m3_forward.py:173 Engine`` reads GGUF byte ranges and dequantizes
every hit expert on the host per call (``Engine.expert`` :268 ->
``tools/gguf_fast_dequant.py:Artifact.expert`` :218). Here the Q4_K bytes stay in HBM in
GGUF order (expert axis slowest) and the kernels dequantize in registers.

:class:`DeviceEngine` keeps the ``Engine`` surface the MoE block uses (``cfg``,
``read(role, layer)``, ``expert(role, layer, e, shape_hf)``) so a caller written against the
reference can hand it to :func:`b200moe.moe.moe_block`; those two accessors return
dequantized device tensors and exist for inspection, not for the hot path.
"""
from __future__ import annotations

import warnings

import numpy as np
import torch

from . import _abi
from . import synth
from .geometry import (DENSE_GATE_UP_STRIDE, DOWN_TYPES, E, EXPERT_GATE_BYTES, SHARED_TYPES, TYPE_IDS, Geometry, H, I,
                       KIND_BLOCKS, KIND_DOWN, KIND_GATE, KIND_SH_DOWN, KIND_SH_GATE, KIND_SH_UP,
                       KIND_UP, Q4K_BYTES, row_bytes, stream_id)


def _bf16_tensor(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).view(
        torch.bfloat16).to(device)


def _router_tensor(w: np.ndarray, device) -> torch.Tensor:
    """Router / shared-gate weights on the device: uint16 arrays are bf16 bits, float32 arrays
    f32 values (kept exactly; the kernels take either)."""
    w = np.asarray(w)
    if w.dtype == np.float32:
        return torch.from_numpy(np.ascontiguousarray(w)).to(device)
    return _bf16_tensor(w, device)


class DeviceLayer:
    """One MoE layer in HBM. Weight tensors are uint8 block bytes in GGUF order: gate / up
    Q4_K; down Q4_K, Q5_K or Q6_K (``down_type``); the shared expert Q4_K or Q8_0
    (``sh_type``). A layer with a type other than Q4_K runs on the decode kernels only."""

    def __init__(self, gate, up, down, sh_gate, sh_up, sh_down, router_w, sh_gate_w,
                 logit_bias=None, gate_up_stride: int = EXPERT_GATE_BYTES, norm_w=None,
                 down_type: str = "Q4_K", sh_type: str = "Q4_K", gate_type: str = "Q4_K"):
        self.gate, self.up, self.down = gate, up, down
        self.sh_gate, self.sh_up, self.sh_down = sh_gate, sh_up, sh_down
        self.router_w, self.sh_gate_w, self.logit_bias = router_w, sh_gate_w, logit_bias
        if router_w.dtype not in (torch.bfloat16, torch.float32) or sh_gate_w.dtype != router_w.dtype:
            raise ValueError("router and shared-gate weights must both be bf16 or both f32, got %s / %s"
                             % (router_w.dtype, sh_gate_w.dtype))
        self.gate_up_stride = int(gate_up_stride)
        # post-attention RMSNorm weight as stored (Form A: 1 + w), f32 [2048]; None = 1. Used where
        # the library normalises the residual itself (moe_stack, moe_stack_prefill).
        if norm_w is not None and (norm_w.dtype != torch.float32 or norm_w.numel() != H):
            raise ValueError("norm_w must be f32 [%d]" % H)
        self.norm_w = norm_w
        if gate_type == "BF16":  # dense: the Hugging Face layout, every matrix bf16
            if down_type != "BF16" or sh_type != "BF16":
                raise ValueError("a dense (BF16) layer has BF16 down and shared matrices, got %s / %s"
                                 % (down_type, sh_type))
        elif gate_type != "Q4_K" or down_type not in DOWN_TYPES or sh_type not in SHARED_TYPES:
            raise ValueError("gate_type %r / down_type %r / sh_type %r: the kernels take gate Q4_K (or a dense "
                             "BF16 layer), down %s, shared %s" % (gate_type, down_type, sh_type, "/".join(DOWN_TYPES),
                                                                  "/".join(SHARED_TYPES)))
        self.down_type, self.sh_type, self.gate_type = down_type, sh_type, gate_type
        self.down_stride = H * row_bytes(down_type, I)   # bytes per expert of ffn_down_exps
        if down.numel() != E * self.down_stride:
            raise ValueError("down holds %d B; %d experts of %s need %d" % (down.numel(), E, down_type,
                                                                             E * self.down_stride))
        for name, t, n in (("sh_gate", sh_gate, I * row_bytes(sh_type, H)),
                           ("sh_up", sh_up, I * row_bytes(sh_type, H)),
                           ("sh_down", sh_down, H * row_bytes(sh_type, I))):
            if t.numel() != n:
                raise ValueError("%s holds %d B; %s needs %d" % (name, t.numel(), sh_type, n))
        self._abi = None

    @property
    def all_q4k(self) -> bool:
        """Every expert and shared matrix is Q4_K (the grouped-GEMM path takes only such layers)."""
        return self.gate_type == "Q4_K" and self.down_type == "Q4_K" and self.sh_type == "Q4_K"

    @property
    def dense(self) -> bool:
        """Every expert and shared matrix is bf16 as the Hugging Face checkpoint stores it."""
        return self.gate_type == "BF16"

    # ------------------------------------------------------------------ construction
    @classmethod
    def synthetic(cls, seed: int, layer: int, device="cuda", bias: bool = False,
                  fused_gate_up: bool = False) -> "DeviceLayer":
        """Seeded synthetic layer (BASELINE config-0 field law), Q4_K generated on device.

        ``fused_gate_up`` lays gate and up out as one HF-style [E, 2I, H] stack (gate rows
        first per expert) instead of two GGUF tensors; the bytes of each row are the same.
        """
        dev = torch.device(device)

        def gen(kind):
            n = KIND_BLOCKS[kind]
            t = torch.empty(n * Q4K_BYTES, dtype=torch.uint8, device=dev)
            _abi.synth_q4k(seed, stream_id(layer, kind), 0, n, t)
            return t

        if fused_gate_up:
            g, u = gen(KIND_GATE).view(E, -1), gen(KIND_UP).view(E, -1)
            fused = torch.cat([g, u], dim=1).reshape(-1).contiguous()
            gate, up, stride = fused, fused[EXPERT_GATE_BYTES:], 2 * EXPERT_GATE_BYTES
        else:
            gate, up, stride = gen(KIND_GATE), gen(KIND_UP), EXPERT_GATE_BYTES
        lb = (torch.from_numpy(synth.zipf_bias(seed, layer)).to(dev) if bias else None)
        return cls(gate, up, gen(KIND_DOWN), gen(KIND_SH_GATE), gen(KIND_SH_UP), gen(KIND_SH_DOWN),
                   _bf16_tensor(synth.router_w(seed, layer), dev),
                   _bf16_tensor(synth.shared_gate_w(seed, layer), dev), lb, stride)

    @classmethod
    def from_host(cls, blocks: dict, router_w_bits, sh_gate_w_bits, logit_bias=None,
                  device="cuda", norm_w=None, down_type: str = "Q4_K",
                  sh_type: str = "Q4_K") -> "DeviceLayer":
        """From host arrays: ``blocks[kind]`` uint8 block bytes for gate/up/down/sh_gate/sh_up/sh_down
        (GGUF order; down in ``down_type``, the shared expert in ``sh_type``); the router and
        shared gate as bf16 bit patterns (uint16) or f32 values (float32, both the same type)."""
        dev = torch.device(device)
        with warnings.catch_warnings():  # read-only views (e.g. a memory-mapped GGUF): only read, then copied
            warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
            t = {k: torch.from_numpy(np.ascontiguousarray(v, dtype=np.uint8).reshape(-1)).to(dev)
                 for k, v in blocks.items()}
        lb = None if logit_bias is None else torch.as_tensor(np.asarray(logit_bias, np.float32)).to(dev)
        return cls(t["gate"], t["up"], t["down"], t["sh_gate"], t["sh_up"], t["sh_down"],
                   _router_tensor(router_w_bits, dev), _router_tensor(sh_gate_w_bits, dev), lb,
                   norm_w=None if norm_w is None else torch.from_numpy(
                       np.ascontiguousarray(norm_w, dtype=np.float32)).to(dev),
                   down_type=down_type, sh_type=sh_type)

    @classmethod
    def dense(cls, gate_up, down, shared_gate, shared_up, shared_down, router, shared_scalar_gate,
              logit_bias=None) -> "DeviceLayer":
        """A dense layer from the Hugging Face checkpoint's bf16 tensors as stored (the roles of
        ``speccheck/moe_ref.py:184 BlockWeights``): gate_up [256, 1024, 2048] (gate = rows 0..511
        of each expert, up = rows 512..1023), down [256, 2048, 512], shared gate / up [512, 2048],
        shared down [2048, 512], router [256, 2048], shared_scalar_gate [1, 2048]. The tensors
        are used in place (contiguous CUDA bf16), nothing is copied."""
        want = {"gate_up": (E, 2 * I, H), "down": (E, H, I), "shared_gate": (I, H), "shared_up": (I, H),
                "shared_down": (H, I), "router": (E, H), "shared_scalar_gate": (1, H)}
        got = dict(gate_up=gate_up, down=down, shared_gate=shared_gate, shared_up=shared_up,
                   shared_down=shared_down, router=router, shared_scalar_gate=shared_scalar_gate)
        for k, t in got.items():
            if tuple(t.shape) != want[k] or t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise ValueError("%s: %s %s, want contiguous bf16 %s" % (k, tuple(t.shape), t.dtype, want[k]))
        u8 = lambda t: t.view(torch.uint8).reshape(-1)  # noqa: E731
        gu = u8(gate_up)
        return cls(gu, gu[I * H * 2:], u8(down), u8(shared_gate), u8(shared_up), u8(shared_down),
                   router, shared_scalar_gate.reshape(H), logit_bias, gate_up_stride=DENSE_GATE_UP_STRIDE,
                   down_type="BF16", sh_type="BF16", gate_type="BF16")

    @classmethod
    def synthetic_dense(cls, seed: int, layer: int, device="cuda") -> "DeviceLayer":
        """The seeded synthetic layer in the dense Hugging Face layout: its Q4_K matrices
        dequantised to bf16 on the device (b200moe_q4k_dequant, RNE of the exact f32 values) and
        laid out as moe_ref's tensors."""
        q = cls.synthetic(seed, layer, device)
        dev = torch.device(device)
        deq = lambda t, shape: cls._dequant_bf16(t, shape, dev)  # noqa: E731
        g = deq(q.gate, (E, I, H))
        u = deq(q.up, (E, I, H))
        gate_up = torch.cat([g, u], dim=1).contiguous()
        del g, u
        return cls.dense(gate_up, deq(q.down, (E, H, I)), deq(q.sh_gate, (I, H)), deq(q.sh_up, (I, H)),
                         deq(q.sh_down, (H, I)), q.router_w, q.sh_gate_w.reshape(1, H))

    @staticmethod
    def _dequant_bf16(blocks, shape, dev):
        out = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        _abi.q4k_dequant(blocks, out, _abi.BF16)
        return out

    # ------------------------------------------------------------------ ABI view
    def abi(self) -> _abi.Layer:
        if self._abi is None:
            p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
            self._abi = _abi.Layer(p(self.gate), p(self.up), self.gate_up_stride, p(self.down),
                                   self.down_stride, p(self.sh_gate), p(self.sh_up), p(self.sh_down),
                                   p(self.router_w), p(self.sh_gate_w), p(self.logit_bias),
                                   1 if self.router_w.dtype == torch.float32 else 0, p(self.norm_w),
                                   TYPE_IDS[self.down_type], TYPE_IDS[self.sh_type], TYPE_IDS[self.gate_type])
        return self._abi

    @property
    def device(self):
        return self.down.device

    def nbytes(self) -> int:
        ts = [self.down, self.sh_gate, self.sh_up, self.sh_down, self.router_w, self.sh_gate_w]
        n = sum(t.numel() * t.element_size() for t in ts)
        if self.gate_up_stride == 2 * I * row_bytes(self.gate_type, H):  # one fused gate_up stack
            n += self.gate.numel()
        else:
            n += self.gate.numel() + self.up.numel()
        return n

    # ------------------------------------------------------------------ inspection
    def type_of(self, kind: str) -> str:
        """Block format of ``kind`` (gate / up / down / sh_gate / sh_up / sh_down)."""
        return self.gate_type if kind in ("gate", "up") else self.down_type if kind == "down" else self.sh_type

    def expert_blocks(self, kind: str, e: int = 0) -> torch.Tensor:
        """The block bytes (device uint8 view) of one expert matrix or of a shared matrix."""
        if kind == "down":
            return self.down[e * self.down_stride:(e + 1) * self.down_stride]
        if kind in ("gate", "up"):
            base = self.gate if kind == "gate" else self.up
            return base[e * self.gate_up_stride: e * self.gate_up_stride + I * row_bytes(self.gate_type, H)]
        return {"sh_gate": self.sh_gate, "sh_up": self.sh_up, "sh_down": self.sh_down}[kind]

    def dequant(self, kind: str, e: int = 0, dtype=torch.float32) -> torch.Tensor:
        blocks = self.expert_blocks(kind, e)
        shape = (H, I) if kind.endswith("down") else (I, H)
        if self.type_of(kind) == "BF16":  # dense rows as stored
            return blocks.view(torch.bfloat16).reshape(shape).to(dtype)
        out = torch.empty(shape, dtype=dtype, device=blocks.device)
        _abi.dequant(blocks, self.type_of(kind), out, _abi.BF16 if dtype == torch.bfloat16 else _abi.F32)
        return out


class DeviceEngine:
    """``Engine``-shaped holder of device layers (``engine/m3_forward.py:173``)."""

    ROLE = {"ffn_gate_exps": "gate", "ffn_up_exps": "up", "ffn_down_exps": "down",
            "ffn_gate_shexp": "sh_gate", "ffn_up_shexp": "sh_up", "ffn_down_shexp": "sh_down"}

    def __init__(self, layers, geometry: Geometry | None = None):
        self.layers = list(layers)
        self.geometry = geometry or Geometry()
        self.cfg = self.geometry.as_cfg()
        self.fault = None
        self.probe_ops = []
        self.perturb = None

    @classmethod
    def synthetic(cls, seed: int, n_layers: int, device="cuda", bias: bool = False) -> "DeviceEngine":
        return cls([DeviceLayer.synthetic(seed, l, device, bias) for l in range(n_layers)])

    def read(self, role: str, layer: int):
        """(values, None, handle) like ``Engine.read`` :235 -- dequantized on the device."""
        L = self.layers[layer]
        if role == "ffn_gate_inp":
            return L.router_w.float(), None, dict(type_name="F32" if L.router_w.dtype == torch.float32 else "BF16")
        if role == "ffn_gate_inp_shexp":
            return L.sh_gate_w.float().reshape(1, H), None, dict(
                type_name="F32" if L.sh_gate_w.dtype == torch.float32 else "BF16")
        return L.dequant(self.ROLE[role]), None, dict(type_name=L.type_of(self.ROLE[role]))

    def expert(self, role: str, layer: int, idx: int, shape_hf):
        """(values, None, rec) like ``Engine.expert`` :268 -- dequantized on the device."""
        L = self.layers[layer]
        v = L.dequant(self.ROLE[role], idx)
        if tuple(v.shape) != tuple(shape_hf):
            raise ValueError("%s expert %d is %s, caller wants %s" % (role, idx, tuple(v.shape), tuple(shape_hf)))
        return v, None, dict(type_name=L.type_of(self.ROLE[role]))
