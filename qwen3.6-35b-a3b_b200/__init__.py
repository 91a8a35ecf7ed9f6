"""B200-native (sm_100a) Qwen3.6-35B-A3B sparse-MoE block.

Import through the alias ``b200moe`` (the directory name is not an identifier)::

    import b200moe                      # after b200moe.load() from a checkout, see load()
    from b200moe import moe             # reference-shaped block API
    from b200moe import engine          # device-resident Q4_K weights

The compute path is ``libb200moe.so`` (hand-written CUDA for sm_100a, C ABI declared in
``include/b200moe.h``), reached through :mod:`b200moe._abi`. There is no CPU fallback:
every op raises if the library or a CUDA device is missing.
"""
from __future__ import annotations

import importlib.util
import os
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_DIR)


def load(alias: str = "b200moe"):
    """Register this directory as the importable package ``alias`` and return it."""
    if alias in sys.modules:
        return sys.modules[alias]
    spec = importlib.util.spec_from_file_location(alias, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[alias] = mod
    spec.loader.exec_module(mod)
    return mod
