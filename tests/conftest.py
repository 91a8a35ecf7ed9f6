"""Shared test setup: the ``gpu`` marker, the package alias, oracle helpers."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen3.6-35b-a3b_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_pkg():
    if "b200moe" not in sys.modules:
        spec = importlib.util.spec_from_file_location("b200moe", os.path.join(PKG, "__init__.py"),
                                                      submodule_search_locations=[PKG])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["b200moe"] = mod
        spec.loader.exec_module(mod)
    return sys.modules["b200moe"]


_load_pkg()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libb200moe.so")


def golden(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def host_layer(seed, layer, bias=False, bf16_weights=False):
    """The oracle's view of synthetic layer (seed, layer): Q4_K from the numpy mirror of
    the device generator, bf16 tensors from the package's host generators. ``bf16_weights``:
    the dense layout of the same layer (every matrix the bf16 rounding of its decode)."""
    from oracle import q4k
    from oracle.moe import HostLayer
    from b200moe import synth
    from b200moe.geometry import KIND_OF, stream_id

    def blocks(kind, first, n):
        return q4k.synth_blocks(seed, stream_id(layer, KIND_OF[kind]), first, n)

    return HostLayer(blocks, synth.router_w(seed, layer), synth.shared_gate_w(seed, layer),
                     synth.zipf_bias(seed, layer) if bias else None, bf16_weights=bf16_weights)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from b200moe import _abi
    _abi.lib()          # fails loudly if the library is missing
    return torch.device("cuda:0")
