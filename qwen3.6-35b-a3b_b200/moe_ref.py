"""The third caller: ``speccheck/moe_ref.py:499 moe_block(x, w: BlockWeights, g: Geometry,
form="ref")`` -- the reference's spec-check block over the dense Hugging Face bf16 weights --
on the B200 path.

The reference runs this on the CPU in torch (``F.linear`` per hit expert, bf16 tensors,
``speccheck/moe_ref.py:318-518``). Here the same call shapes reach the library's gather-GEMV
decode kernels, which read the dense bf16 rows in place (``b200moe_layer.gate_type`` =
BF16: ``gate_up [256, 1024, 2048]`` with gate = rows 0..511 and up = rows 512..1023 of each
expert, ``down [256, 2048, 512]``, the shared expert's three matrices) through
``b200moe_moe_decode_stages``, which writes the stage tensors out and, in the "ref" form, rounds
to bf16 where the reference's form rounds: each F.linear output, F.silu's output, the SwiGLU
product, each expert output, each weighted product and the running routed sum (bf16
accumulate, ascending expert id: ``moe_ref.py:441-475``), the gated shared output and the block
output (``moe_ref.py:516-517``). The router is the library's declared-order R1..R5 (the
reference's route ``moe_ref.py:318-364`` with its F.linear order fixed).

Types keep the reference's names and fields (``Geometry`` ``:62-90``, ``Form`` ``:263-298``,
``BlockWeights`` ``:184-212``). Forms other than ``[REF]`` (``"ref"``) and the injection knobs
(``expert_index_shift``, ``swap_halves``, ``transpose_stack``) are refused with a tag, as the
reference refuses what it does not implement: they exist to measure arithmetic choices and to
plant bugs, which the host oracle does (``tests/test_must_catch.py``), not the device path.
Returned tensors stay on the device.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _abi
from .engine import DeviceLayer
from .geometry import E, H, I, TOPK
from .moe import Refused, workspace


@dataclass(frozen=True)
class Geometry:
    """``speccheck/moe_ref.py:62 Geometry`` with the Qwen3.6-35B-A3B values as defaults."""

    hidden_size: int = H
    num_experts: int = E
    top_k: int = TOPK
    moe_intermediate_size: int = I
    shared_expert_intermediate_size: int = I
    num_hidden_layers: int = 40
    mtp_num_hidden_layers: int = 1
    dtype: torch.dtype = torch.bfloat16
    rms_norm_eps: float = 1e-6
    config_path: str = "checkpoints/Qwen3.6-35B-A3B.config.json"

    @property
    def n_blocks(self) -> int:
        return self.num_hidden_layers + self.mtp_num_hidden_layers

    @property
    def expert_bytes(self) -> int:
        return (self.two_i * self.hidden_size + self.hidden_size * self.moe_intermediate_size) * 2

    @property
    def two_i(self) -> int:
        return 2 * self.moe_intermediate_size


@dataclass(frozen=True)
class Form:
    """``speccheck/moe_ref.py:263 Form``: the switchable arithmetic choices and their named arms
    (the arm names are the reference's vocabulary). The device path runs the ``[REF]`` form."""

    softmax_dtype: str = "f32"
    renorm: bool = True
    weight_cast: str = "before"
    accumulate: str = "bf16"
    order: str = "expert_asc"
    batching: str = "grouped"
    router_dtype: str = "model"

    @staticmethod
    def named(arm: str) -> "Form":
        arms = {
            "ref": Form(),
            "spec": Form(accumulate="f32", order="rank", batching="per_slot", weight_cast="after"),
            "exact": Form(accumulate="f64", order="rank", batching="per_slot", weight_cast="after",
                          router_dtype="f64"),
            "cast_after": Form(weight_cast="after"),
            "softmax_bf16": Form(softmax_dtype="bf16"),
            "no_renorm": Form(renorm=False),
            "accum_f32": Form(accumulate="f32"),
            "accum_f64": Form(accumulate="f64"),
            "rank_order": Form(order="rank"),
            "per_slot": Form(batching="per_slot"),
        }
        if arm not in arms:
            raise Refused("form", "unknown arm %r; known: %s" % (arm, sorted(arms)))
        return arms[arm]


# The roles of one block's weights and the shapes the geometry implies (moe_ref.py:191-203).
ROLES = ("router", "gate_up", "down", "shared_gate", "shared_up", "shared_down", "shared_scalar_gate")


def _shapes(g: Geometry) -> dict:
    return {"router": (g.num_experts, g.hidden_size),
            "gate_up": (g.num_experts, g.two_i, g.hidden_size),
            "down": (g.num_experts, g.hidden_size, g.moe_intermediate_size),
            "shared_gate": (g.shared_expert_intermediate_size, g.hidden_size),
            "shared_up": (g.shared_expert_intermediate_size, g.hidden_size),
            "shared_down": (g.hidden_size, g.shared_expert_intermediate_size),
            "shared_scalar_gate": (1, g.hidden_size)}


@dataclass
class BlockWeights:
    """``speccheck/moe_ref.py:184 BlockWeights``: the seven bf16 tensors of one block as stored.
    CPU tensors are copied to the device once, on the first call that needs them."""

    block: object
    tensors: dict
    source_shards: dict = field(default_factory=dict)

    def shapes_ok(self, g: Geometry, roles=None) -> None:
        want = _shapes(g)
        for role in ROLES:
            if roles is not None and role not in roles:
                continue
            if role not in self.tensors:
                raise Refused("shape", "block %s is missing %s" % (getattr(self.block, "name", self.block), role))
            t = self.tensors[role]
            if tuple(t.shape) != want[role]:
                raise Refused("shape", "%s: stored shape %s != config-derived %s" % (role, tuple(t.shape), want[role]))
            if t.dtype is not torch.bfloat16:
                raise Refused("dtype", "%s: stored dtype %s, expected bf16" % (role, t.dtype))

    def device_layer(self, device=None) -> DeviceLayer:
        """The block as a dense :class:`DeviceLayer` (cached; the device tensors are used in place)."""
        L = getattr(self, "_device_layer", None)
        if L is None:
            dev = torch.device(device) if device is not None else (
                self.tensors["gate_up"].device if self.tensors["gate_up"].is_cuda else torch.device("cuda"))
            t = {k: self.tensors[k].to(dev).contiguous() for k in ROLES}
            L = DeviceLayer.dense(t["gate_up"], t["down"], t["shared_gate"], t["shared_up"], t["shared_down"],
                                  t["router"], t["shared_scalar_gate"])
            object.__setattr__(self, "_device_layer", L)
        return L


def moe_block(x: torch.Tensor, w: BlockWeights, g: Geometry | None = None, form="ref", *,
              expert_index_shift: int = 0, swap_halves: bool = False, transpose_stack: bool = False) -> dict:
    """``speccheck/moe_ref.py:499 moe_block`` on the device: x [T, 2048] (or [1, T, 2048]) bf16 ->
    the stage dictionary (``input, router_logits, router_probs, topk_ids, topk_weights,
    topk_probs_pre_renorm, expert_raw, routed_sum, shared_raw, shared_gate_prob, shared_out,
    combined_out, form``) in the dtypes the reference's ``expected_dtypes(Form())`` names."""
    g = g or Geometry()
    form = Form.named(form) if isinstance(form, str) else form
    if form != Form():
        raise Refused("form", "the device path runs the [REF] form only (bf16 accumulate, cast before, ascending "
                      "expert id); %s measures an arithmetic choice and stays on the host oracle" % (form,))
    if expert_index_shift or swap_halves or transpose_stack:
        raise Refused("injection", "bug-injection knobs are planted in the host oracle, never in a device kernel")
    if (g.hidden_size, g.num_experts, g.top_k, g.moe_intermediate_size,
            g.shared_expert_intermediate_size) != (H, E, TOPK, I, I):
        raise Refused("geometry", "the kernels are built for Qwen3.6-35B-A3B's MoE geometry, got %s" % (g,))
    if x.ndim == 3:
        if x.shape[0] != 1:
            raise Refused("batch", "only batch 1 is implemented; the engine is single-request")
        x = x.reshape(-1, x.shape[-1])
    if x.ndim != 2 or x.shape[1] != H:
        raise Refused("shape", "x must be [T, %d], got %s" % (H, tuple(x.shape)))
    if x.dtype is not torch.bfloat16:
        raise Refused("dtype", "bf16 accumulation requires a bf16 input, got %s" % x.dtype)
    L = w.device_layer()
    dev = L.device
    x = x.to(dev).contiguous()
    T = x.shape[0]
    out = torch.empty((T, H), dtype=torch.float32, device=dev)
    ids = torch.empty((T, TOPK), dtype=torch.int32, device=dev)
    wb = torch.empty((T, TOPK), dtype=torch.bfloat16, device=dev)
    logits = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    raw = torch.empty((T, TOPK, H), dtype=torch.float32, device=dev)
    routed = torch.empty((T, H), dtype=torch.float32, device=dev)
    shraw = torch.empty((T, H), dtype=torch.float32, device=dev)
    sg = torch.empty((T,), dtype=torch.float32, device=dev)
    if T:
        _abi.moe_decode_stages(x, _abi.BF16, T, L.abi(), True, out, ids, wb, workspace(T, dev),
                               router_logits=logits, expert_raw=raw, routed_sum=routed, shared_raw=shraw,
                               shared_gate=sg)
    bf = torch.bfloat16
    probs = torch.softmax(logits.float(), dim=-1)      # f32 softmax of the bf16 logits (moe_ref.py:336)
    ids64 = ids.to(torch.int64)
    sgb = sg.to(bf).reshape(T, 1)
    shared_raw = shraw.to(bf)
    return {
        "input": x,
        "router_logits": logits,
        "router_probs": probs,
        "topk_ids": ids64,
        "topk_weights": wb,
        "topk_probs_pre_renorm": probs.gather(1, ids64),
        "expert_raw": raw.to(bf),
        "routed_sum": routed.to(bf),
        "shared_raw": shared_raw,
        "shared_gate_prob": sgb,
        "shared_out": (sgb.float() * shared_raw.float()).to(bf),   # the kernel's rounding of sg * raw
        "combined_out": out.to(bf),
        "form": form,
    }


__all__ = ["Geometry", "Form", "BlockWeights", "moe_block", "ROLES"]
