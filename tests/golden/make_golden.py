"""Generate the golden fixtures under tests/golden/ by running the REFERENCE's own Python.

Run only where the reference checkout is present (it imports the reference from the directory
``REF_ROOT`` names, read-only); the GPU box never runs this. Outputs are small ``.npz``
files committed beside this script:

* ``q4k_dequant.npz`` -- edge-case, hand-built and seeded-random Q4_K blocks decoded by the
  reference's audited decoder ``tools/gguf_reader.py:dequant`` (and checked identical to
  ``tools/gguf_fast_dequant.py:dequant_np``), plus the reference's known answer
  (d=1, dmin=0, sc[1]=63, nibble 15 at qs[32g+1] -> only element 33 = 945.0,
  ``prototype/q4k_dequant/q4k_dequant_kernels.h:199-203``).
* ``router_t64.npz`` -- R1..R5 of ``engine/m3_forward.py:443-446`` (the reference's own
  torch expressions, evaluated by ``moe_block`` itself for the ids) on 64 seeded tokens.
* ``moe_block_t4.npz`` -- ``engine/m3_forward.py:430 moe_block`` run unchanged on a
  duck-typed weight provider that serves the seeded synthetic Q4_K bytes through the
  reference's ``gguf_fast_dequant.dequant_np`` (4 tokens, config-0 field law, seed 0).
* ``rmsnorm.npz`` -- ``engine/m3_forward.py:303 rmsnorm_a`` (weight 1) on seeded rows.
* ``moe_ref_t4.npz`` -- ``speccheck/moe_ref.py:499 moe_block`` (the reference's bf16 spec-check
  block over dense Hugging Face weights) run unchanged in its "ref" and "exact" forms on 4 tokens,
  with the seeded synthetic layer (seed 0, layer 0) as dense bf16 tensors: the reference's own
  decoder ``gguf_fast_dequant.dequant_np`` of the Q4_K bytes, rounded to bf16 (RNE). Only the
  experts the 4 tokens hit are filled (the others are never read). ``python make_golden.py
  moe_ref`` makes only this.
* ``kquant_dequant.npz`` -- seeded and edge-case Q5_K, Q6_K and Q8_0 blocks decoded by the
  reference's ``tools/gguf_reader.py:dequant`` (checked identical to
  ``tools/gguf_fast_dequant.py:dequant_np``). ``python make_golden.py kquants`` makes only this.

The Q4_K import chain needs ``tools/ggml_block_geom.py``'s un-vendored third-party header
(llama.cpp ``ggml/src/ggml-common.h`` @ d327bf1f0780f87b8c01b367b61853b0c291d7c4); a shim
module supplies the block geometry the reference states in ``tools/gguf_reader.py:20-27``.
"""
from __future__ import annotations

import hashlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF_ROOT = os.environ.get("REF_ROOT")  # the reference checkout (required: no default path)
sys.dont_write_bytecode = True
sys.path.insert(0, REPO)

from oracle import q4k  # noqa: E402
from oracle.bf16 import bf16_bits_to_f32  # noqa: E402


def import_reference():
    if not REF_ROOT or not os.path.isdir(REF_ROOT):
        raise SystemExit("set REF_ROOT to the reference checkout (read only) to regenerate the fixtures")
    for p in (REF_ROOT, os.path.join(REF_ROOT, "tools"), os.path.join(REF_ROOT, "engine")):
        if p not in sys.path:
            sys.path.insert(0, p)
    shim = types.ModuleType("ggml_block_geom")
    geo = {"Q4_K": (256, 144), "Q5_K": (256, 176), "Q6_K": (256, 210), "Q8_0": (32, 34), "F32": (1, 4),
           "F16": (1, 2), "BF16": (1, 2), "Q4_0": (32, 18), "IQ4_NL": (32, 18)}
    shim.geom = lambda require=None, **kw: {t: {"elts": e, "bytes": b} for t, (e, b) in geo.items()}
    sys.modules["ggml_block_geom"] = shim
    import gguf_reader as GR  # noqa: E402
    import gguf_fast_dequant as FD  # noqa: E402
    import m3_forward as M3  # noqa: E402
    return GR, FD, M3


def synth_layer_blocks(seed: int, layer: int, kind: int, first: int, n: int) -> np.ndarray:
    return q4k.synth_blocks(seed, 8 * layer + kind, first, n)


# ---------------------------------------------------------------------------- Q4_K
def dequant_cases():
    zs = [0] * 8
    grid = np.array([(i * 37 + 11) & 0xFF for i in range(128)], dtype=np.uint8)
    cases, labels = [], []

    def add(label, raw):
        cases.append(np.frombuffer(raw, dtype=np.uint8))
        labels.append(label)

    # the reference gate's synthetic population (prototype/q4k_dequant/gate.py:404-440)
    add("zero", q4k.build_block(0, 0, zs, zs, np.zeros(128, np.uint8)))
    add("grid", q4k.build_block(0x3C00, 0x3800, [0, 9, 17, 26, 35, 44, 53, 63], [63, 53, 44, 35, 26, 17, 9, 0], grid))
    add("flat", q4k.build_block(0x3C00, 0x3800, [5] * 8, [3] * 8, grid))
    add("minonly", q4k.build_block(0, 0x3C00, zs, [63] * 8, np.zeros(128, np.uint8)))
    # the known-answer block: only element 33 is non-zero (945.0)
    kat_qs = np.zeros(128, np.uint8)
    for g in range(4):
        kat_qs[32 * g + 1] = 0xF0
    add("kat945", q4k.build_block(0x3C00, 0, [0, 63, 0, 0, 0, 0, 0, 0], zs, kat_qs))
    # f16 edge values for d / dmin: subnormal, negative, max finite, inf, nan, -0
    rng = np.random.default_rng(20261201)
    for lab, d, m in [("d_subnormal", 0x0001, 0x0003), ("d_negative", 0xBC00, 0x3C00), ("d_max", 0x7BFF, 0x7BFF),
                      ("d_inf", 0x7C00, 0x0000), ("dmin_nan", 0x3C00, 0x7E00), ("d_negzero", 0x8000, 0x8000),
                      ("all_max_fields", 0x3C00, 0x3C00)]:
        sc = rng.integers(0, 64, 8) if lab != "all_max_fields" else [63] * 8
        mm = rng.integers(0, 64, 8) if lab != "all_max_fields" else [63] * 8
        qs = rng.integers(0, 256, 128, dtype=np.uint8) if lab != "all_max_fields" else np.full(128, 0xFF, np.uint8)
        add(lab, q4k.build_block(d, m, sc, mm, qs))
    # 64 fully random byte blocks (any f16 pattern) and 64 seeded synthetic blocks
    for i in range(64):
        add("random_bytes_%d" % i, rng.integers(0, 256, 144, dtype=np.uint8).tobytes())
    syn = synth_layer_blocks(0, 0, 0, 1000, 64)
    for i in range(64):
        add("synth_s0_l0_gate_%d" % (1000 + i), syn[i].tobytes())
    return np.stack(cases), labels


def make_dequant(GR, FD):
    blocks, labels = dequant_cases()
    ref = np.array(GR.dequant(blocks.tobytes(), "Q4_K", blocks.shape[0] * 256), dtype=np.float32)
    fast = FD.dequant_np(blocks.tobytes(), "Q4_K", blocks.shape[0] * 256)
    same = (ref.view(np.uint32) == fast.view(np.uint32)) | (np.isnan(ref) & np.isnan(fast))
    assert same.all(), "reference slow and fast decoders disagree"
    kat = ref[labels.index("kat945") * 256:(labels.index("kat945") + 1) * 256]
    assert np.count_nonzero(kat) == 1 and kat[33] == 945.0, "reference KAT"
    # the pack helper round-trips through the reference's own get_scale_min_k4
    for raw in blocks[:5]:
        sc, m = GR.qk_scale_min(bytes(raw[4:16]))
        assert bytes(q4k.pack_scale_min(sc, m)[0]) == bytes(raw[4:16])
    np.savez_compressed(os.path.join(HERE, "q4k_dequant.npz"), blocks=blocks, labels=np.array(labels),
                        ref_f32_bits=ref.view(np.uint32))
    print("q4k_dequant.npz: %d blocks" % blocks.shape[0])


# ---------------------------------------------------------------------------- block
class RefProvider:
    """Duck-typed ``Engine`` for ``m3_forward.moe_block``: serves synthetic Q4_K layer-0
    weights (seed, layer) through the reference's own decoder ``FD.dequant_np``."""

    ROLE_KIND = {"ffn_gate_exps": 0, "ffn_up_exps": 1, "ffn_down_exps": 2, "ffn_gate_shexp": 3,
                 "ffn_up_shexp": 4, "ffn_down_shexp": 5}

    def __init__(self, M3, FD, seed, layer, wg_bits, wsg_bits):
        self.cfg = M3.load_geometry()
        self.FD = FD
        self.seed, self.layer = seed, layer
        self.wg = wg_bits
        self.wsg = wsg_bits
        self.fault = None
        self.probe_ops = []
        self.perturb = None
        self.expert_calls = 0

    def _deq(self, kind, first, n_blocks, shape):
        import torch
        raw = synth_layer_blocks(self.seed, self.layer, kind, first, n_blocks)
        vals = self.FD.dequant_np(raw.tobytes(), "Q4_K", n_blocks * 256)
        return torch.from_numpy(vals.reshape(shape))

    def read(self, role, layer):
        import torch
        if role == "ffn_gate_inp":
            return torch.from_numpy(bf16_bits_to_f32(self.wg).reshape(256, 2048).copy()), None, {}
        if role == "ffn_gate_inp_shexp":
            return torch.from_numpy(bf16_bits_to_f32(self.wsg).reshape(1, 2048).copy()), None, {}
        kind = self.ROLE_KIND[role]
        shape = (2048, 512) if role == "ffn_down_shexp" else (512, 2048)
        return self._deq(kind, 0, 4096, shape), None, {}

    def expert(self, role, layer, idx, shape_hf):
        self.expert_calls += 1
        kind = self.ROLE_KIND[role]
        return self._deq(kind, idx * 4096, 4096, tuple(shape_hf)), None, dict(type_name="Q4_K")


def wg_and_wsg(seed, layer):
    """The package's host-side bf16 generators (router W_g, shared gate w_sg)."""
    import importlib.util
    pkg = os.path.join(REPO, "qwen3.6-35b-a3b_b200")
    if "b200moe" not in sys.modules:
        spec = importlib.util.spec_from_file_location("b200moe", os.path.join(pkg, "__init__.py"),
                                                      submodule_search_locations=[pkg])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["b200moe"] = mod
        spec.loader.exec_module(mod)
    from b200moe import synth
    return synth, synth.router_w(seed, layer), synth.shared_gate_w(seed, layer)


def make_router(M3):
    import torch
    import torch.nn.functional as F
    synth, wg, _ = wg_and_wsg(0, 0)
    x_bits = synth.tokens(0, 64, stream=0)
    x = torch.from_numpy(bf16_bits_to_f32(x_bits).copy())
    w = torch.from_numpy(bf16_bits_to_f32(wg).copy())
    torch.set_num_threads(1)
    # engine/m3_forward.py:443-446, the reference's own four expressions
    logits = F.linear(x, w).to(torch.bfloat16)
    probs = torch.softmax(logits.float(), dim=-1)
    tw, ids = torch.topk(probs, 8, dim=-1)
    wcast = (tw / tw.sum(-1, keepdim=True)).to(logits.dtype)
    np.savez_compressed(os.path.join(HERE, "router_t64.npz"), x_bits=x_bits,
                        wg_sha256=hashlib.sha256(wg.tobytes()).hexdigest(),
                        logits_bits=logits.view(torch.int16).numpy().view(np.uint16),
                        probs=probs.numpy(), ids=ids.numpy().astype(np.int32),
                        wcast_bits=wcast.view(torch.int16).numpy().view(np.uint16))
    print("router_t64.npz")


def make_block(M3, FD):
    import torch
    synth, wg, wsg = wg_and_wsg(0, 0)
    x_bits = synth.tokens(0, 4, stream=1)
    g = torch.from_numpy(bf16_bits_to_f32(x_bits).copy()).reshape(1, 4, 2048)
    E = RefProvider(M3, FD, 0, 0, wg, wsg)
    torch.set_num_threads(8)
    out, info = M3.moe_block(g, E, 0)
    np.savez_compressed(os.path.join(HERE, "moe_block_t4.npz"), x_bits=x_bits, seed=0, layer=0,
                        wg_sha256=hashlib.sha256(wg.tobytes()).hexdigest(),
                        wsg_sha256=hashlib.sha256(wsg.tobytes()).hexdigest(),
                        out=out.reshape(4, 2048).numpy(), ids=info["ids"].reshape(4, 8).numpy().astype(np.int32),
                        used=info["used"], expert_calls=E.expert_calls)
    print("moe_block_t4.npz used=%d" % info["used"])


def make_moe_ref(FD):
    import torch
    if os.path.join(REF_ROOT, "speccheck") not in sys.path:
        sys.path.insert(0, os.path.join(REF_ROOT, "speccheck"))
    import moe_ref as MR  # noqa: E402
    synth, wg, wsg = wg_and_wsg(0, 0)
    x_bits = synth.tokens(0, 4, stream=2)
    x = torch.from_numpy(x_bits.view(np.int16).copy()).view(torch.bfloat16)
    g = MR.Geometry(hidden_size=2048, num_experts=256, top_k=8, moe_intermediate_size=512,
                    shared_expert_intermediate_size=512, num_hidden_layers=40, mtp_num_hidden_layers=1,
                    dtype=torch.bfloat16, rms_norm_eps=1e-6)

    def deq(kind, first, n_blocks, shape):
        raw = synth_layer_blocks(0, 0, kind, first, n_blocks)
        return torch.from_numpy(FD.dequant_np(raw.tobytes(), "Q4_K", n_blocks * 256).reshape(shape)).to(
            torch.bfloat16)

    router = torch.from_numpy(wg.view(np.int16).copy()).view(torch.bfloat16).reshape(256, 2048)
    hit = set()
    for arm in ("ref", "exact"):
        hit |= set(int(v) for v in MR.route(x, router, g, MR.Form.named(arm))["topk_ids"].reshape(-1))
    gate_up = torch.zeros((256, 1024, 2048), dtype=torch.bfloat16)
    down = torch.zeros((256, 2048, 512), dtype=torch.bfloat16)
    for e in sorted(hit):
        gate_up[e, :512] = deq(0, e * 4096, 4096, (512, 2048))
        gate_up[e, 512:] = deq(1, e * 4096, 4096, (512, 2048))
        down[e] = deq(2, e * 4096, 4096, (2048, 512))
    t = {"router": router, "gate_up": gate_up, "down": down, "shared_gate": deq(3, 0, 4096, (512, 2048)),
         "shared_up": deq(4, 0, 4096, (512, 2048)), "shared_down": deq(5, 0, 4096, (2048, 512)),
         "shared_scalar_gate": torch.from_numpy(wsg.view(np.int16).copy()).view(torch.bfloat16).reshape(1, 2048)}
    w = MR.BlockWeights(MR.Block("layer", 0), t)
    w.shapes_ok(g)
    torch.set_num_threads(8)
    ref = MR.moe_block(x, w, g, "ref")
    exact = MR.moe_block(x, w, g, "exact")
    bits = lambda v: v.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    np.savez_compressed(os.path.join(HERE, "moe_ref_t4.npz"), x_bits=x_bits, seed=0, layer=0,
                        wg_sha256=hashlib.sha256(wg.tobytes()).hexdigest(),
                        wsg_sha256=hashlib.sha256(wsg.tobytes()).hexdigest(),
                        hit=np.array(sorted(hit), dtype=np.int32),
                        **{"ref_" + k: bits(ref[k]) for k in ("router_logits", "topk_weights", "expert_raw",
                                                              "routed_sum", "shared_raw", "shared_gate_prob",
                                                              "shared_out", "combined_out")},
                        ref_router_probs=ref["router_probs"].numpy(),
                        ref_topk_ids=ref["topk_ids"].numpy().astype(np.int32),
                        exact_topk_ids=exact["topk_ids"].numpy().astype(np.int32),
                        exact_topk_weights=exact["topk_weights"].numpy(),
                        exact_routed_sum=exact["routed_sum"].numpy(),
                        exact_combined_out=exact["combined_out"].numpy())
    print("moe_ref_t4.npz: %d experts hit" % len(hit))


def make_rmsnorm(M3):
    import torch
    M3.load_geometry()
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((8, 2048)) * np.array([1e-3, 1, 30, 1e3, 1, 1, 1, 1])[:, None]).astype(np.float32)
    y = M3.rmsnorm_a(torch.from_numpy(x), torch.ones(2048)).numpy()
    np.savez_compressed(os.path.join(HERE, "rmsnorm.npz"), x=x, y=y)
    print("rmsnorm.npz")


def kquant_cases(tname):
    from oracle import kquants as KQ
    bb = KQ.BLOCK_BYTES[tname]
    blocks = [KQ.random_blocks(tname, 24, seed={"Q5_K": 51, "Q6_K": 61, "Q8_0": 81}[tname])]
    edge = np.zeros((4, bb), dtype=np.uint8)
    dcol = {"Q8_0": 0, "Q5_K": 0, "Q6_K": 208}[tname]
    one = np.array([1.0], dtype=np.float16).view(np.uint8)
    edge[0, dcol:dcol + 2] = one                     # d = 1, every quant 0 (Q6_K: q - 32 = -32)
    edge[1] = 0xFF                                   # every field saturated (d = NaN bits)
    edge[1, dcol:dcol + 2] = np.array([-2.0], dtype=np.float16).view(np.uint8)
    if tname == "Q5_K":
        edge[1, 2:4] = np.array([0.5], dtype=np.float16).view(np.uint8)
    edge[2] = edge[1]
    edge[2, dcol:dcol + 2] = np.array([6.1e-5], dtype=np.float16).view(np.uint8)   # near-subnormal d
    edge[3, dcol:dcol + 2] = np.array([0.0], dtype=np.float16).view(np.uint8)      # d = 0
    edge[3, dcol + 2:] = 0x5A if dcol == 0 else edge[3, dcol + 2:]
    if tname == "Q6_K":
        edge[3, 192:208] = 0x80                       # scales = -128
        edge[3, 208:210] = np.array([3.0e-3], dtype=np.float16).view(np.uint8)
    blocks.append(edge)
    return np.concatenate(blocks)


def make_kquants(GR, FD):
    out = {}
    for tname in ("Q5_K", "Q6_K", "Q8_0"):
        blocks = kquant_cases(tname)
        n = blocks.shape[0] * (32 if tname == "Q8_0" else 256)
        ref = np.array(GR.dequant(blocks.tobytes(), tname, n), dtype=np.float32)
        fast = FD.dequant_np(blocks.tobytes(), tname, n)
        same = (ref.view(np.uint32) == fast.view(np.uint32)) | (np.isnan(ref) & np.isnan(fast))
        assert same.all(), "reference slow and fast %s decoders disagree" % tname
        out[tname + "_blocks"] = blocks
        out[tname + "_ref_f32_bits"] = ref.view(np.uint32)
    np.savez_compressed(os.path.join(HERE, "kquant_dequant.npz"), **out)
    print("kquant_dequant.npz:", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    GR, FD, M3 = import_reference()
    if sys.argv[1:] == ["kquants"]:
        make_kquants(GR, FD)
        sys.exit(0)
    if sys.argv[1:] == ["moe_ref"]:
        make_moe_ref(FD)
        sys.exit(0)
    make_kquants(GR, FD)
    make_dequant(GR, FD)
    make_router(M3)
    make_block(M3, FD)
    make_rmsnorm(M3)
    make_moe_ref(FD)
