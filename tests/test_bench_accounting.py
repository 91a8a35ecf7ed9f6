"""bench.py's algorithmic byte counts (the roofline numerator), on CPU: the per-layer bytes of a
Q4_K layer are the BASELINE figures (1,769,472 B per expert, 1 MiB + 4 KB of bf16 router), and a
layer in the published file's layout counts its own row widths (Q5_K / Q6_K down, Q8_0 shared
expert, F32 router). Layers are built from uninitialised CPU tensors: only sizes matter."""
import os
import sys

import pytest

from conftest import ROOT


def _layer(down_type="Q4_K", sh_type="Q4_K", f32=False):
    import torch
    from b200moe.engine import DeviceLayer
    from b200moe.geometry import E, H, I, row_bytes
    u8 = lambda n: torch.empty(n, dtype=torch.uint8)  # noqa: E731
    rdt = torch.float32 if f32 else torch.bfloat16
    return DeviceLayer(u8(E * I * row_bytes("Q4_K", H)), u8(E * I * row_bytes("Q4_K", H)),
                       u8(E * H * row_bytes(down_type, I)), u8(I * row_bytes(sh_type, H)),
                       u8(I * row_bytes(sh_type, H)), u8(H * row_bytes(sh_type, I)),
                       torch.empty(E * H, dtype=rdt), torch.empty(H, dtype=rdt),
                       down_type=down_type, sh_type=sh_type)


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, ROOT)
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_q4k_layer_bytes(bench):
    assert bench.layer_bytes(_layer()) == (bench.EXPERT_BYTES, bench.EXPERT_BYTES,
                                           bench.ROUTER_BYTES + bench.WSG_BYTES)


@pytest.mark.parametrize("down,per_row", [("Q5_K", 352), ("Q6_K", 420)])
def test_published_layer_bytes(bench, down, per_row):
    routed, shared, router = bench.layer_bytes(_layer(down, "Q8_0", f32=True))
    assert routed == 2 * 512 * 1152 + 2048 * per_row
    assert shared == 2 * 512 * 2176 + 2048 * 544
    assert router == 256 * 2048 * 4 + 2048 * 4


def test_layer_size_checks():
    """A down tensor sized for another block type is refused by name."""
    from b200moe.engine import DeviceLayer
    L = _layer()
    with pytest.raises(ValueError, match="Q5_K"):
        DeviceLayer(L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down, L.router_w, L.sh_gate_w,
                    down_type="Q5_K")
    with pytest.raises(ValueError, match="Q8_0"):
        DeviceLayer(L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down, L.router_w, L.sh_gate_w,
                    sh_type="Q8_0")
    with pytest.raises(ValueError):
        DeviceLayer(L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down, L.router_w, L.sh_gate_w,
                    down_type="Q2_K")
    assert L.all_q4k and not _layer("Q6_K").all_q4k
