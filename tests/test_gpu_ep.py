"""Expert parallelism on 2+ GPUs (skipped on a single-GPU box), over peer memory (the default on
NVLink) and over NCCL all-to-all: three steps in a row, then the EP output equals the single-GPU
prefill within rel-L2 1e-5 (only the association of the routed sum differs) with identical routing
ids, and no peer wait ran out."""
import json
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("transport", ["p2p", "a2a"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_matches_single_gpu(cuda, tmp_path, world, transport):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    out = tmp_path / "ep.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "ep_worker.py"), "--tokens", "512", "--out", str(out), "--transport", transport]
    subprocess.run(cmd, check=True, env=env, cwd=ROOT)
    r = json.loads(out.read_text())
    assert r["transport"] == transport and r["p2p_status"] == 0, r
    assert r["ids_equal"] and r["finite"] and r["status"] == 0, r
    assert r["rel_l2"] < 1e-5, r
