"""Expert-parallel dispatch / combine host logic on CPU gloo ranks (world sizes 2 and 4).

The ranks run b200moe.ep.ExpertParallelMoE unchanged, with CPU stage functions: the declared
router from the C oracle, host restatements of the dispatch-row pack, the receiver's expert stage
and the ordered combine (the row format of b200moe_ep_pack / b200moe_ep_experts /
b200moe_ep_combine), and a cheap synthetic expert body (o_e(x) = x * (1 + e/256) + e/64,
shared = x / 2), so the test exercises exactly the per-destination token selection, the two
equal-split all_to_all_single exchanges and the ascending-rank combine. The reference runs the same stage
functions on all tokens in one process; only the association of the routed sum differs.
"""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import ROOT

T_PER_RANK = 6


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _stage_fns():
    import sys
    sys.path.insert(0, ROOT)
    from conftest import _load_pkg
    _load_pkg()
    from oracle import moe as OM
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import synth
    wg = synth.router_w(3, 0)
    wsg = bf16_bits_to_f32(synth.shared_gate_w(3, 0)).astype(np.float64)

    def route(x, resid=None):
        xf = x.numpy().astype(np.float32)
        r = OM.router(xf, wg)
        sg = (1.0 / (1.0 + np.exp(-(xf.astype(np.float64) @ wsg)))).astype(np.float32)
        return (torch.from_numpy(xf.astype(np.float16)), torch.from_numpy(r["ids"].astype(np.int32)),
                torch.from_numpy(r["w_bf16"].view(np.int16).copy()), torch.from_numpy(sg))

    def body(x16, ids, wb, e_lo, e_hi, sg, out, accumulate=False, sh_rows=None):
        x = x16.numpy().astype(np.float64)
        idn = ids.numpy()
        w = bf16_bits_to_f32(wb.numpy().view(np.uint16)).astype(np.float64)
        res = np.zeros_like(x)
        lo, hi = sh_rows if sh_rows is not None else (0, x.shape[0])
        for t in range(x.shape[0]):
            for k in np.argsort(idn[t], kind="stable"):
                e = int(idn[t, k])
                if e_lo <= e < e_hi:
                    res[t] += w[t, k] * (x[t] * (1.0 + e / 256.0) + e / 64.0)
            if sg is not None and lo <= t < hi:
                res[t] += float(sg[t - lo]) * (x[t] * 0.5)
        r32 = torch.from_numpy(res.astype(np.float32))
        if accumulate:
            out += r32
        else:
            out.copy_(r32)
        return out

    return route, body


def _ep_stage_fns():
    """Host restatements of the three device stages of expert parallelism over the dispatch row
    format (b200moe_ep_pack / b200moe_ep_experts / b200moe_ep_combine), around the test body."""
    route, body = _stage_fns()
    row = 4160

    def pack(x16, ids, wb, rank, world, send, pos):
        T = x16.shape[0]
        per = 256 // world
        sv, idn = send.numpy(), ids.numpy()
        pos.fill_(-1)
        for d in range(world):
            p = 0
            for t in range(T):
                if d == rank or ((idn[t] >= d * per) & (idn[t] < (d + 1) * per)).any():
                    sv[d, p, :4096] = x16[t].numpy().view(np.uint8)
                    sv[d, p, 4096:4128] = idn[t].astype(np.int32).view(np.uint8)
                    sv[d, p, 4128:4144] = wb[t].numpy().view(np.uint8)
                    pos[t, d] = p
                    p += 1
            for q in range(p, T):
                sv[d, q, 4096:4128] = np.full(8, -1, np.int32).view(np.uint8)
        return send, pos

    def experts(recv, T, rank, world, sg, partial):
        rv = recv.numpy().reshape(world * T, row)
        x16 = torch.from_numpy(rv[:, :4096].copy().view(np.float16))
        ids = torch.from_numpy(rv[:, 4096:4128].copy().view(np.int32))
        wb = torch.from_numpy(rv[:, 4128:4144].copy().view(np.int16))
        per = 256 // world
        out = torch.zeros((world * T, 2048), dtype=torch.float32)
        body(x16, ids, wb, rank * per, (rank + 1) * per, sg, out, sh_rows=(rank * T, rank * T + T))
        partial.copy_(out.reshape(world, T, 2048))
        return partial

    def combine(ret, pos, T, world, out, accumulate):
        res = torch.zeros((T, 2048), dtype=torch.float32)
        for t in range(T):
            for d in range(world):
                p = int(pos[t, d])
                if p >= 0:
                    res[t] += ret[d, p]
        if accumulate:
            out += res
        else:
            out.copy_(res)
        return out

    return route, pack, experts, combine


def _tokens(world):
    from conftest import _load_pkg
    _load_pkg()
    from oracle.bf16 import bf16_bits_to_f32
    from b200moe import synth
    return torch.from_numpy(bf16_bits_to_f32(synth.tokens(3, world * T_PER_RANK, stream=5)).copy())


def _worker(rank, world, port, path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from conftest import _load_pkg
        _load_pkg()
        from b200moe.ep import ExpertParallelMoE
        route, pack, experts, combine = _ep_stage_fns()
        x = _tokens(world)[rank * T_PER_RANK:(rank + 1) * T_PER_RANK]
        ep = ExpertParallelMoE(layer=None, route_fn=route, pack_fn=pack, experts_fn=experts, combine_fn=combine,
                               device=torch.device("cpu"))
        out, ids = ep.forward(x)
        np.savez(path % rank, out=out.numpy(), ids=ids.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_dispatch_combine_matches_single_process(tmp_path, world):
    import torch.multiprocessing as mp
    path = str(tmp_path / "rank%d.npz")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, start_method="spawn", join=True)
    outs = [np.load(path % r) for r in range(world)]
    ep_out = np.concatenate([o["out"] for o in outs])
    ep_ids = np.concatenate([o["ids"] for o in outs])
    route, body = _stage_fns()
    x = _tokens(world)
    x16, ids, wb, sg = route(x)
    ref = torch.zeros((x.shape[0], 2048), dtype=torch.float32)
    body(x16, ids, wb, 0, 256, sg, ref)
    assert (ep_ids == ids.numpy()).all()
    rel = np.linalg.norm(ep_out - ref.numpy()) / np.linalg.norm(ref.numpy())
    assert rel < 1e-6, rel
    # every rank's experts took part (the test would be vacuous otherwise)
    owners = np.unique(ids.numpy() // (256 // world))
    assert len(owners) == world


def test_refuses_non_q4k_layer_before_any_collective():
    """A layer in the published file's other block formats is refused at construction (every rank
    alike, before a collective could leave the others waiting): the grouped GEMMs take Q4_K."""
    import torch
    from b200moe.ep import ExpertParallelMoE
    from test_bench_accounting import _layer
    with pytest.raises(ValueError, match="Q4_K"):
        ExpertParallelMoE(_layer("Q5_K", "Q8_0"), device=torch.device("cpu"))
    assert ExpertParallelMoE(_layer(), device=torch.device("cpu")).e_hi == 256


def _worker_peer_lost(rank, world, port, path):
    """Rank 1 leaves right after joining (between steps, with nothing in flight); rank 0 runs an
    expert-parallel step, whose first collective must end with an error, not wait for good."""
    import datetime
    import json
    import time
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)
    from conftest import _load_pkg
    _load_pkg()
    from b200moe.ep import ExpertParallelMoE
    route, pack, experts, combine = _ep_stage_fns()
    x = _tokens(world)[:T_PER_RANK]
    ep = ExpertParallelMoE(layer=None, route_fn=route, pack_fn=pack, experts_fn=experts, combine_fn=combine,
                           device=torch.device("cpu"))
    t0 = time.monotonic()
    try:
        ep.forward(x)
        res = dict(detected=False)
    except Exception as e:  # the collective's error: the peer's connection closed, or the timeout
        res = dict(detected=True, error=type(e).__name__, msg=str(e)[:200])
    res["seconds"] = time.monotonic() - t0
    with open(path, "w") as f:
        json.dump(res, f)
    os._exit(0)  # no teardown handshake with a peer that is gone


def test_lost_rank_ends_the_collective_with_an_error(tmp_path):
    import json
    import time
    import torch.multiprocessing as mp
    path = str(tmp_path / "rank0.json")
    ctx = mp.start_processes(_worker_peer_lost, args=(2, _free_port(), path), nprocs=2, start_method="spawn",
                             join=False)
    deadline = time.monotonic() + 120
    try:
        while not ctx.join(timeout=1):
            assert time.monotonic() < deadline, "rank 0 did not finish: the lost peer was not detected"
    finally:
        for p in ctx.processes:  # only the processes this test started
            if p.is_alive():
                p.kill()
    res = json.load(open(path))
    assert res["detected"] and res["seconds"] < 60, res
