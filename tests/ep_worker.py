"""Multi-GPU expert-parallel check, one process per GPU (launched by tests/test_gpu_ep.py via
torch.distributed.run). Every rank shards the config-3 layer's experts, routes its slice of the
tokens, and runs ExpertParallelMoE; rank 0 gathers the outputs and compares them with the
single-GPU prefill on all tokens (same routing ids, rel-L2 on the outputs)."""
import argparse
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=512)
    ap.add_argument("--out", required=True)
    ap.add_argument("--transport", default=None, choices=[None, "p2p", "a2a"])
    a = ap.parse_args()
    import __graft_entry__ as G
    G.load_package()
    from b200moe import moe, synth
    from b200moe.engine import DeviceLayer
    from b200moe.ep import ExpertParallelMoE
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    L = DeviceLayer.synthetic(3, 0, dev)
    xb = synth.tokens(3, a.tokens, stream=7)
    xall = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).to(dev)
    per = a.tokens // world
    ep = ExpertParallelMoE(L, transport=a.transport)
    for _ in range(3):  # repeated steps: the peer form's epochs and buffer reuse
        out, ids = ep.forward(xall[rank * per:(rank + 1) * per])
    torch.cuda.synchronize()
    p2p_status = ep.p2p_status(per)
    from b200moe import _abi
    ep_status = _abi.prefill_status(ep.workspace(per), world * per)
    outs = [torch.empty_like(out) for _ in range(world)]
    idss = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(outs, out)
    dist.all_gather(idss, ids)
    if rank == 0:
        ref, info = moe.moe_block(xall, L, path="prefill")
        torch.cuda.synchronize()
        o = torch.cat(outs)
        res = dict(world=world, tokens=a.tokens, transport=ep.transport, p2p_status=p2p_status,
                   ids_equal=bool(torch.equal(torch.cat(idss), info["ids"])),
                   rel_l2=float(torch.linalg.norm(o - ref) / torch.linalg.norm(ref)),
                   finite=bool(torch.isfinite(o).all()), status=moe.prefill_status(a.tokens, dev) | ep_status)
        with open(a.out, "w") as f:
            json.dump(res, f)
    dist.barrier()
    ep.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
