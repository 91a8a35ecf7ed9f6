"""The GGUF reader (qwen3.6-35b-a3b_b200/gguf.py) on files written here by a minimal GGUF v3
writer: header and metadata parse, tensor byte views at the right offsets (checked by marker
bytes at both ends of every tensor), the block-type rules (Q4_K gate/up; Q4_K / Q5_K / Q6_K
down; Q4_K / Q8_0 shared expert, as the published Q4_K_M file mixes them; bf16 / F32 router),
the F32-router rounding switch, and the refusals (wrong type, wrong shape, missing tensor,
truncated file). Full-size
tensors are sparse holes in the file, so the test writes little and reads little."""
import struct

import numpy as np
import pytest

H, I, E = 2048, 512, 256
Q80, Q4K, Q5K, Q6K, F32, F16, BF16 = 8, 12, 13, 14, 0, 1, 30
SIZES = {Q80: (32, 34), Q4K: (256, 144), Q5K: (256, 176), Q6K: (256, 210), F32: (1, 4), F16: (1, 2),
         BF16: (1, 2)}
NAMES = {Q80: "Q8_0", Q4K: "Q4_K", Q5K: "Q5_K", Q6K: "Q6_K"}


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, align=32, truncate=False, version=3):
    """tensors: list of (name, dims (GGUF order), type, {offset_in_tensor: bytes})."""
    kv = [("general.architecture", 8, _s("qwen35moe")), ("general.alignment", 4, struct.pack("<I", align)),
          ("qwen35moe.expert_count", 4, struct.pack("<I", E)),
          ("tokenizer.ggml.tokens", 9, struct.pack("<IQ", 8, 2) + _s("a") + _s("b"))]
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv))
    for k, t, v in kv:
        head += _s(k) + struct.pack("<I", t) + v
    offs, off = [], 0
    for name, dims, typ, _ in tensors:
        n = int(np.prod(dims))
        nbytes = n // SIZES[typ][0] * SIZES[typ][1]
        offs.append((off, nbytes))
        head += _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, off)
        off = (off + nbytes + align - 1) // align * align
    data0 = (len(head) + align - 1) // align * align
    with open(path, "wb") as f:
        f.write(head)
        for (name, dims, typ, marks), (o, nb) in zip(tensors, offs):
            for at, b in marks.items():
                f.seek(data0 + o + (at if at >= 0 else nb + at))
                f.write(b)
        end = data0 + offs[-1][0] + offs[-1][1]
        f.truncate(end - 100 if truncate else end)
    return data0


def layer_tensors(l, down_type=Q4K, router_type=BF16, router_dims=(H, E), sh_type=Q4K, gate_type=Q4K,
                  sh_down_type=None):
    p = "blk.%d." % l
    mk = lambda tag: {0: tag * 16, -16: tag[::-1] * 16}  # noqa: E731
    t = [(p + "ffn_gate_exps.weight", (H, I, E), gate_type, mk(b"G")),
         (p + "ffn_up_exps.weight", (H, I, E), Q4K, mk(b"U")),
         (p + "ffn_down_exps.weight", (I, H, E), down_type, mk(b"D")),
         (p + "ffn_gate_shexp.weight", (H, I), sh_type, mk(b"g")), (p + "ffn_up_shexp.weight", (H, I), sh_type, mk(b"u")),
         (p + "ffn_down_shexp.weight", (I, H), sh_down_type or sh_type, mk(b"d"))]
    rng = np.random.default_rng(l)
    w = rng.normal(0, 0.02, size=E * H).astype(np.float32)
    g = rng.normal(0, 0.02, size=H).astype(np.float32)
    if router_type == BF16:
        from oracle.bf16 import f32_to_bf16_bits
        t.append((p + "ffn_gate_inp.weight", router_dims, BF16, {0: f32_to_bf16_bits(w).tobytes()}))
        t.append((p + "ffn_gate_inp_shexp.weight", (H, 1), BF16, {0: f32_to_bf16_bits(g).tobytes()}))
    elif router_type == F16:
        w, g = w.astype(np.float16).astype(np.float32), g.astype(np.float16).astype(np.float32)
        t.append((p + "ffn_gate_inp.weight", router_dims, F16, {0: w.astype(np.float16).tobytes()}))
        t.append((p + "ffn_gate_inp_shexp.weight", (H,), F16, {0: g.astype(np.float16).tobytes()}))
    else:
        t.append((p + "ffn_gate_inp.weight", router_dims, F32, {0: w.tobytes()}))
        t.append((p + "ffn_gate_inp_shexp.weight", (H,), F32, {0: g.tobytes()}))
    return t, w, g


def _mod():
    import __graft_entry__ as G
    G.load_package()
    from b200moe import gguf
    return gguf


def test_header_and_layer_views(tmp_path):
    gguf = _mod()
    t, w, g = layer_tensors(3)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, t)
    with gguf.GgufFile(path) as gf:
        assert gf.version == 3 and gf.meta["general.architecture"] == "qwen35moe"
        assert gf.meta["tokenizer.ggml.tokens"] == ["a", "b"]
        assert gf.info("blk.3.ffn_down_exps.weight").dims == (I, H, E)
        blocks, router, shgate = gguf.layer_host(gf, 3)
        sizes = {"gate": E * I * 8 * 144, "up": E * I * 8 * 144, "down": E * H * 2 * 144,
                 "sh_gate": I * 8 * 144, "sh_up": I * 8 * 144, "sh_down": H * 2 * 144}
        tags = {"gate": b"G", "up": b"U", "down": b"D", "sh_gate": b"g", "sh_up": b"u", "sh_down": b"d"}
        for k, v in blocks.items():
            assert v.dtype == np.uint8 and v.size == sizes[k], k
            assert bytes(v[:16]) == tags[k] * 16 and bytes(v[-16:]) == tags[k] * 16, k
        from oracle.bf16 import f32_to_bf16_bits
        assert np.array_equal(router, f32_to_bf16_bits(w)) and np.array_equal(shgate, f32_to_bf16_bits(g))
        del blocks


def test_f32_router_kept_exactly_or_rounded_on_request(tmp_path):
    gguf = _mod()
    t, w, g = layer_tensors(0, router_type=F32)
    path = str(tmp_path / "m.gguf")
    write_gguf(path, t)
    with gguf.GgufFile(path) as gf:
        blocks, router, shgate = gguf.layer_host(gf, 0)
        assert router.dtype == np.float32 and np.array_equal(router, w) and np.array_equal(shgate, g)
        blocks, router, shgate = gguf.layer_host(gf, 0, round_router=True)
        from oracle.bf16 import f32_to_bf16_bits
        assert np.array_equal(router, f32_to_bf16_bits(w)) and np.array_equal(shgate, f32_to_bf16_bits(g))
        del blocks


@pytest.mark.parametrize("down", [Q5K, Q6K])
def test_published_formats(tmp_path, down):
    """The published Q4_K_M file's layer formats: Q5_K (or Q6_K) expert down and a Q8_0 shared
    expert are read as stored, with their types named for the device layer."""
    gguf = _mod()
    t, _, _ = layer_tensors(4, down_type=down, sh_type=Q80)
    path = str(tmp_path / "pub.gguf")
    write_gguf(path, t)
    with gguf.GgufFile(path) as gf:
        assert gguf.layer_types(gf, 4) == dict(down_type=NAMES[down], sh_type="Q8_0")
        blocks, _, _ = gguf.layer_host(gf, 4)
        bd, be = SIZES[down][1], SIZES[down][0]
        sizes = {"gate": E * I * 8 * 144, "up": E * I * 8 * 144, "down": E * H * I // be * bd,
                 "sh_gate": I * H // 32 * 34, "sh_up": I * H // 32 * 34, "sh_down": H * I // 32 * 34}
        tags = {"gate": b"G", "up": b"U", "down": b"D", "sh_gate": b"g", "sh_up": b"u", "sh_down": b"d"}
        for k, v in blocks.items():
            assert v.size == sizes[k], k
            assert bytes(v[:16]) == tags[k] * 16 and bytes(v[-16:]) == tags[k] * 16, k
        del blocks


def test_refusals(tmp_path):
    gguf = _mod()
    t, _, _ = layer_tensors(1, gate_type=Q5K)
    p1 = str(tmp_path / "q5.gguf")
    write_gguf(p1, t)
    with gguf.GgufFile(p1) as gf:
        with pytest.raises(gguf.GgufError) as ei:
            gguf.layer_host(gf, 1)
        assert ei.value.tag == "type" and "Q5_K" in str(ei.value) and "ffn_gate_exps" in str(ei.value)
        with pytest.raises(gguf.GgufError) as ei:
            gguf.layer_host(gf, 2)
        assert ei.value.tag == "missing"
    t, _, _ = layer_tensors(1, sh_type=Q80, sh_down_type=Q4K)
    p0 = str(tmp_path / "mixed_shared.gguf")
    write_gguf(p0, t)
    with gguf.GgufFile(p0) as gf:
        with pytest.raises(gguf.GgufError) as ei:
            gguf.layer_types(gf, 1)
        assert ei.value.tag == "type" and "mixes" in str(ei.value)
    t, _, _ = layer_tensors(1, router_dims=(H, 128))
    p2 = str(tmp_path / "shape.gguf")
    write_gguf(p2, t)
    with gguf.GgufFile(p2) as gf:
        with pytest.raises(gguf.GgufError) as ei:
            gguf.layer_host(gf, 1)
        assert ei.value.tag == "shape"
    t, _, _ = layer_tensors(1)
    p3 = str(tmp_path / "short.gguf")
    write_gguf(p3, t, truncate=True)
    with pytest.raises(gguf.GgufError) as ei:
        gguf.GgufFile(p3)
    assert ei.value.tag == "format"
    p4 = str(tmp_path / "bad.gguf")
    open(p4, "wb").write(b"GGML" + b"\0" * 64)
    with pytest.raises(gguf.GgufError):
        gguf.GgufFile(p4)


def test_post_attention_norm_weight(tmp_path):
    """blk.N.post_attention_norm.weight (Form A: the file holds 1 + w) is read as f32 values;
    a file without it gives None (weight 1)."""
    gguf = _mod()
    t, _, _ = layer_tensors(2)
    w = (1.0 + np.random.default_rng(3).normal(0, 0.05, H)).astype(np.float32)
    t.append(("blk.2.post_attention_norm.weight", (H,), F32, {0: w.tobytes()}))
    path = str(tmp_path / "n.gguf")
    write_gguf(path, t)
    with gguf.GgufFile(path) as gf:
        assert np.array_equal(gguf.layer_norm(gf, 2), w)
        assert gguf.layer_norm(gf, 5) is None


@pytest.mark.parametrize("version,align", [(2, 32), (3, 64)])
def test_f16_router_widened_exactly_v2_and_alignment(tmp_path, version, align):
    """An F16 router / shared gate is widened to f32 exactly; a GGUF v2 header and a data
    alignment other than 32 place every tensor where the writer put it."""
    gguf = _mod()
    t, w, g = layer_tensors(6, router_type=F16)
    path = str(tmp_path / "f16.gguf")
    data0 = write_gguf(path, t, align=align, version=version)
    with gguf.GgufFile(path) as gf:
        assert gf.version == version and gf.data_start == data0 and data0 % align == 0
        blocks, router, shgate = gguf.layer_host(gf, 6)
        assert router.dtype == np.float32 and np.array_equal(router, w) and np.array_equal(shgate, g)
        assert bytes(blocks["down"][:16]) == b"D" * 16 and bytes(blocks["sh_down"][-16:]) == b"d" * 16
        del blocks


@pytest.mark.parametrize("typ", [BF16, F16])
def test_norm_weight_other_types(tmp_path, typ):
    """BF16 / F16 post-attention norm weights are widened to f32 exactly."""
    gguf = _mod()
    t, _, _ = layer_tensors(2)
    w = (1.0 + np.random.default_rng(4).normal(0, 0.05, H)).astype(np.float32)
    if typ == BF16:
        from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
        raw, want = f32_to_bf16_bits(w).tobytes(), bf16_bits_to_f32(f32_to_bf16_bits(w))
    else:
        raw, want = w.astype(np.float16).tobytes(), w.astype(np.float16).astype(np.float32)
    t.append(("blk.2.post_attention_norm.weight", (H,), typ, {0: raw}))
    path = str(tmp_path / "n.gguf")
    write_gguf(path, t)
    with gguf.GgufFile(path) as gf:
        got = gguf.layer_norm(gf, 2)
        assert got.dtype == np.float32 and np.array_equal(got, want)
