"""Geometry of the Qwen3.6-35B-A3B MoE block and the synthetic-weight stream map.

Values from the reference's ``checkpoints/Qwen3.6-35B-A3B.config.json:17,69,73,74,93``
(hidden_size, num_experts, num_experts_per_tok, moe_intermediate_size,
shared_expert_intermediate_size) and ``:num_hidden_layers`` / ``rms_norm_eps``; the same
numbers the reference's ``moe_ref.Geometry`` (``speccheck/moe_ref.py:62-90``) derives.
"""
from dataclasses import dataclass

H = 2048          # hidden_size
E = 256           # num_experts
TOPK = 8          # num_experts_per_tok
I = 512           # moe_intermediate_size (= shared_expert_intermediate_size)
N_LAYERS = 40     # num_hidden_layers
RMS_EPS = 1e-6    # rms_norm_eps
QK_K = 256
Q4K_BYTES = 144

ROW_UP = H // QK_K * Q4K_BYTES          # 1152 B: one gate/up row
ROW_DOWN = I // QK_K * Q4K_BYTES        # 288 B: one down row
EXPERT_GATE_BYTES = I * ROW_UP          # 589,824 B (ffn_gate_exps / ffn_up_exps per expert)
EXPERT_DOWN_BYTES = H * ROW_DOWN        # 589,824 B (ffn_down_exps per expert)
EXPERT_BYTES = 2 * EXPERT_GATE_BYTES + EXPERT_DOWN_BYTES   # 1,769,472 B
ROUTER_BYTES = E * H * 2                # 1,048,576 B bf16

# Block formats the kernels take (GGML type ids as in GGUF): (bytes, elements) per block. The
# published Q4_K_M file stores expert gate/up as Q4_K, expert down as Q5_K (Q6_K at three layers)
# and the shared expert as Q8_0.
TYPE_IDS = {"Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "BF16": 30}
BLOCK_GEOM = {"Q8_0": (34, 32), "Q4_K": (144, 256), "Q5_K": (176, 256), "Q6_K": (210, 256), "BF16": (2, 1)}
DOWN_TYPES = ("Q4_K", "Q5_K", "Q6_K")      # ffn_down_exps
SHARED_TYPES = ("Q4_K", "Q8_0")            # ffn_{gate,up,down}_shexp
# A dense layer (the Hugging Face checkpoint's bf16 tensors, as speccheck/moe_ref.py takes them)
# has every expert and shared matrix in BF16: gate_up [E, 2I, H] fused, down [E, H, I].
DENSE_GATE_UP_STRIDE = 2 * I * H * 2    # 4 MiB per expert of the fused gate_up stack


def row_bytes(tname: str, n: int) -> int:
    """Bytes of one row of ``n`` weights in block format ``tname``."""
    bb, be = BLOCK_GEOM[tname]
    return n // be * bb

# Synthetic Q4_K streams: stream id = 8*layer + kind.
KIND_GATE, KIND_UP, KIND_DOWN, KIND_SH_GATE, KIND_SH_UP, KIND_SH_DOWN = range(6)
KIND_BLOCKS = {KIND_GATE: E * I * 8, KIND_UP: E * I * 8, KIND_DOWN: E * H * 2,
               KIND_SH_GATE: I * 8, KIND_SH_UP: I * 8, KIND_SH_DOWN: H * 2}
KIND_OF = {"gate": KIND_GATE, "up": KIND_UP, "down": KIND_DOWN,
           "sh_gate": KIND_SH_GATE, "sh_up": KIND_SH_UP, "sh_down": KIND_SH_DOWN}


def stream_id(layer: int, kind: int) -> int:
    return 8 * int(layer) + int(kind)


@dataclass(frozen=True)
class Geometry:
    d: int = H
    n_experts: int = E
    top_k: int = TOPK
    i_e: int = I
    i_s: int = I
    n_layers: int = N_LAYERS
    eps_rms: float = RMS_EPS

    def as_cfg(self) -> dict:
        """The ``cfg`` dict shape ``engine/m3_forward.py:load_geometry`` returns (MoE keys)."""
        import torch
        return dict(d=self.d, n_experts=self.n_experts, top_k=self.top_k, i_e=self.i_e,
                    i_s=self.i_s, L=self.n_layers, eps_rms=self.eps_rms, act_dtype=torch.bfloat16)
