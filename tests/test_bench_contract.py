"""The reference arm of bench.py on CPU: one JSON line with the contract's keys (metric, value,
unit, higher_is_better, config, cpu_baseline, and an e2e without host-device copies); under
torchrun only rank 0 prints, the other ranks exit 0 without work."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--ref-layers-per-step", "1"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    return p.returncode, [l for l in p.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_line():
    rc, lines = _run({"RANK": "0", "LOCAL_RANK": "0", "WORLD_SIZE": "1"})
    assert rc == 0 and len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == "moe_stack_decode_tok_per_s" and d["unit"] == "tok/s"
    assert d["higher_is_better"] is True and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "config4_stack_decode_b1"


def test_reference_arm_other_ranks_exit_quietly():
    rc, lines = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert rc == 0 and lines == []
