#!/usr/bin/env python
"""bench.py -- Qwen3.6-35B-A3B MoE block on B200: the headline decode benchmark.

Default workload (decode B=1): one step = one token through the full
40-layer MoE sub-stack (``resid += moe_block_l(rmsnorm(resid))`` per layer, seeded
synthetic Q4_K weights, ~18 GB resident) as one CUDA-graph replay of the C-ABI path.
Every step decodes a DISTINCT token, so each step streams 40 x 9 experts' Q4_K bytes
(637 MB of expert weights per token > the 126 MB L2: no L2 flush needed).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--workload stack_decode|layer_decode|prefill|prefill_ep] [--batch B]

Multi-GPU (torchrun, one rank per GPU): batch-1 decode does not shard (a per-layer
collective would cost more than the layer), so N ranks run N independent replicas on
distinct tokens ("scaling": "weak", value = all ranks' tokens / max-over-ranks time).

The default line also carries nested sub-results, each timed with CUDA events after the
headline's timed region:
  prefill_ep      (every N) BASELINE config 3: 4096 tokens through one layer with the experts
                  sharded over the N ranks (ExpertParallelMoE: route, per-destination pack,
                  all-to-all dispatch, grouped GEMMs, all-to-all return, ordered combine) as
                  one CUDA-graph replay; per-stage times from an eager pass; on rank 0 a parity
                  check against the single-GPU prefill of the same tokens. Also decode_b256:
                  the same path at config 2's largest batch.
  dequant_config1 (N = 1) config 1: the Q4_K -> bf16 dequant of one layer's expert stack.
  decode_config2  (N = 1) config 2: one MoE layer at B in {1, 8, 32, 64, 256} under the Zipf
                  routing law, rotated over 40 layer copies (> L2), with U(B) and the HBM
                  roofline fraction per B.
  config4         (N = 1) config 4's other cells: decode at B = 32 and a prefill of 8192
                  tokens through the 40-layer stack.

``--impl reference`` times the reference's own CPU MoE path (engine/m3_forward.py
moe_block + rmsnorm glue, restated as the torch-f32 port in oracle/moe.py) on the host
cores, rank 0 only: whole 40-layer tokens, as many steps as fit a bounded time budget
(the line's ``steps`` is the count actually timed).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

EXPERT_BYTES = 1_769_472            # one Q4_K expert: gate+up [1024,2048] + down [2048,512]
ROUTER_BYTES = 256 * 2048 * 2
WSG_BYTES = 2048 * 2
N_LAYERS = 40
Q6K_LAYERS = (34, 38, 39)           # the published file's Q6_K expert-down layers


def published_engine(seed, n_layers, dev):
    """A layer stack in the published Q4_K_M file's layout: Q4_K gate / up (the synthetic
    generator), Q5_K expert down (Q6_K at layers 34, 38, 39), a Q8_0 shared expert, F32 router and
    shared-gate weights, a post-attention RMSNorm weight. Block bytes are seeded random with
    finite f16 scales sized so 40 layers stay finite."""
    import torch
    from b200moe.engine import DeviceEngine, DeviceLayer
    from b200moe.geometry import BLOCK_GEOM, E, H, I
    g = torch.Generator(device=dev).manual_seed(seed)

    def blocks(tname, n):
        bb = BLOCK_GEOM[tname][0]
        t = torch.randint(0, 256, (n, bb), dtype=torch.uint8, device=dev, generator=g)
        for col, lo, hi in {"Q5_K": ((0, 5e-4, 5e-3), (2, 0.0, 2.5e-3)), "Q6_K": ((208, 1e-4, 1e-3),),
                            "Q8_0": ((0, 1e-4, 1e-3),)}[tname]:
            v = (torch.rand(n, device=dev, generator=g) * (hi - lo) + lo).to(torch.float16)
            t[:, col:col + 2] = v.view(torch.uint8).view(n, 2)
        return t.reshape(-1)

    layers = []
    for l in range(n_layers):
        base = DeviceLayer.synthetic(seed, l, dev)
        dt = "Q6_K" if l in Q6K_LAYERS else "Q5_K"
        nw = 1.0 + 0.05 * torch.randn(H, device=dev, generator=g)
        layers.append(DeviceLayer(base.gate, base.up, blocks(dt, E * H * I // 256), blocks("Q8_0", I * H // 32),
                                  blocks("Q8_0", I * H // 32), blocks("Q8_0", H * I // 32), base.router_w.float(),
                                  base.sh_gate_w.float(), norm_w=nw, down_type=dt, sh_type="Q8_0"))
    return DeviceEngine(layers)


def layer_bytes(L) -> tuple:
    """(bytes of one routed expert, of the shared expert, of the router + shared gate) of a layer."""
    from b200moe.geometry import H, I, row_bytes
    routed = 2 * I * row_bytes("Q4_K", H) + H * row_bytes(L.down_type, I)
    shared = 2 * I * row_bytes(L.sh_type, H) + H * row_bytes(L.sh_type, I)
    router = L.router_w.numel() * L.router_w.element_size() + L.sh_gate_w.numel() * L.sh_gate_w.element_size()
    return routed, shared, router


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--workload", choices=["stack_decode", "layer_decode", "prefill", "prefill_ep"],
                   default="stack_decode")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--layers", type=int, default=N_LAYERS)
    p.add_argument("--seed", type=int, default=4)
    p.add_argument("--path", choices=["auto", "decode", "prefill"], default="auto",
                   help="stack_decode with T >= 2: the decode kernels or the grouped-GEMM path (auto: the "
                        "block's own choice by token count)")
    p.add_argument("--law", type=int, choices=[1, 2], default=1,
                   help="Q4_K field law of the stack: 1 = BASELINE's; 2 = the same blocks with d * 2^-6 and "
                        "dmin * 2^-2 (centred weights: O(1) residual, diverse routing through the stack)")
    p.add_argument("--zipf", action="store_true",
                   help="config 2's routing law: a per-expert Zipf(1.1) logit bias on every layer")
    p.add_argument("--formats", choices=["q4k", "published"], default="q4k",
                   help="stack_decode weights: Q4_K throughout (the BASELINE configs), or the published "
                        "Q4_K_M file's layout (Q5_K down, Q6_K at layers 34/38/39, Q8_0 shared expert, F32 "
                        "router, RMSNorm weight) with seeded random block bytes")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true", help="only the headline (no nested sub-results)")
    p.add_argument("--ref-layers-per-step", type=int, default=N_LAYERS,
                   help="reference arm: layers of the stack per timed step (default: the whole token)")
    p.add_argument("--ref-seconds", type=float, default=100.0,
                   help="reference arm: time budget of the timed steps (the step count is cut to fit)")
    p.add_argument("--cpu-layers", type=int, default=2,
                   help="the GPU arm's cpu_baseline sample: layers of one token")
    return p.parse_args()


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def committed_traffic(workload):
    """DRAM bytes per step from the committed ncu summary (profiles/<workload>_traffic.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", "%s_traffic.json" % workload)) as f:
            return json.load(f)
    except Exception:
        return None


# ---------------------------------------------------------------------------------- clocks
class ClockSampler(threading.Thread):
    """Polls NVML (SM clock, throttle reasons) every ~2 ms while the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        super().__init__(daemon=True)
        self.index = index
        self.samples = []
        self.reasons = 0
        self.stop_ev = threading.Event()
        self.max_mhz = None
        self.ok = False

    def run(self):
        try:
            import pynvml as N
            N.nvmlInit()
            h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            self.ok = True
            while not self.stop_ev.is_set():
                self.samples.append(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                try:
                    self.reasons |= int(N.nvmlDeviceGetCurrentClocksEventReasons(h))
                except Exception:
                    self.reasons |= int(N.nvmlDeviceGetCurrentClocksThrottleReasons(h))
                time.sleep(0.002)
        except Exception:
            self.ok = False

    def result(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml_unavailable"]}
        rs = [n for b, n in self.REASONS.items() if self.reasons & b and b != 0x1]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": rs,
                "samples": len(self.samples)}


def physical_index(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local_rank])
        except Exception:
            return local_rank
    return local_rank


# ---------------------------------------------------------------------------------- CPU arm
def host_layer_of(L):
    """The oracle's view of a device layer: its block bytes copied to the host, with their types,
    router / shared-gate values and norm weight (for the published-layout sample)."""
    from oracle import moe as OM
    from b200moe.geometry import BLOCK_GEOM
    src = {"gate": L.gate, "up": L.up, "down": L.down, "sh_gate": L.sh_gate, "sh_up": L.sh_up,
           "sh_down": L.sh_down}
    arr = {k: t.cpu().numpy().reshape(-1, BLOCK_GEOM[L.type_of(k)][0]) for k, t in src.items()}
    f32 = lambda t: t.float().cpu().numpy()  # noqa: E731
    return OM.HostLayer(lambda k, f, n: arr[k][f:f + n], f32(L.router_w), f32(L.sh_gate_w),
                        types={k: L.type_of(k) for k in src},
                        norm_w=None if L.norm_w is None else L.norm_w.cpu().numpy())


def cpu_sample(args, n_layers, threads=None, eng=None):
    """Prepare the reference's CPU path (oracle port) on a sample: one token through ``n_layers``
    layers of the stack (the Q4_K synthetic layers, or with ``--formats published`` the device
    engine's own first layers copied to the host), with one untimed pass that fills each layer's
    byte cache. Returns (layers, x0, cores, n_layers, seconds of the untimed pass)."""
    import numpy as np
    import torch
    from oracle import moe as OM
    from oracle import q4k
    import __graft_entry__ as G
    G.load_package()
    from b200moe import synth
    from b200moe.geometry import KIND_OF, stream_id
    cores = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    nl = max(1, min(int(n_layers), args.layers))
    if getattr(args, "formats", "q4k") == "published" and eng is not None:
        layers = [host_layer_of(eng.layers[l]) for l in range(nl)]
    else:
        layers = [OM.CachedLayer(lambda k, f, n, l=l: q4k.synth_blocks(args.seed, stream_id(l, KIND_OF[k]), f, n),
                                 synth.router_w(args.seed, l), synth.shared_gate_w(args.seed, l))
                  for l in range(nl)]
    x0 = synth.bf16_bits_to_f32(synth.tokens(args.seed, args.batch, stream=0))
    t0 = time.perf_counter()
    OM.stack_port(x0, layers, cores)          # untimed pass: fills each layer's byte cache
    return layers, x0, cores, nl, time.perf_counter() - t0


def run_reference(args):
    rank, _, world = env_rank()
    if rank != 0:
        return 0
    from oracle import moe as OM
    layers, x0, cores, nl, t_first = cpu_sample(args, args.ref_layers_per_step)
    # untimed warm-up passes (the first, above, also filled the byte caches), then as many timed
    # steps as fit the time budget
    for _ in range(max(0, min(args.warmup, 1) - 1)):
        OM.stack_port(x0, layers, cores)
    steps = max(1, min(args.steps, int(args.ref_seconds / max(t_first, 1e-3))))
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        OM.stack_port(x0, layers, cores)
        times.append(time.perf_counter() - t0)
    sec_step = sum(times) / len(times)
    sec_tok = sec_step * (args.layers / nl)
    val = args.batch / sec_tok
    whole = nl == args.layers
    sample = ("%d token(s) through %s per step (torch-f32 port of engine/m3_forward.py moe_block + rmsnorm_a; "
              "per-hit-expert Q4_K dequant inside the timed region; bytes pre-generated)%s; %d of the %d requested "
              "steps timed (a %.0f s budget), 1 untimed warm-up"
              % (args.batch, ("all %d layers" % nl) if whole else ("%d of %d layers" % (nl, args.layers)),
                 "" if whole else ", scaled x%g to the 40-layer token" % (args.layers / nl), steps, args.steps,
                 args.ref_seconds))
    line = {"impl": "reference", "metric": "moe_stack_decode_tok_per_s", "value": val, "unit": "tok/s",
            "n_gpus": world, "steps": steps, "warmup": 1, "ms_per_step": 1e3 * sec_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Q4_K, config-0 field law)",
            "config": {"workload": "config4_stack_decode_b%d" % args.batch, "layers": args.layers,
                       "layers_per_step": nl, "batch": args.batch, "seed": args.seed},
            "cpu_baseline": {"value": val, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------- sub-results
def _tf_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except Exception:
        return 1590.0


def _events_time(fn, K, W, dev):
    """fn() W times untimed (at least 3), then K times between two CUDA events on the current
    stream; returns ms per call."""
    import torch
    for _ in range(max(3, W)):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / K


def _graph_of(fn, dev):
    """Capture fn() (after one eager call on a side stream) into a CUDA graph."""
    import torch
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def bench_dequant(dev, K, W, hbm_peak):
    """b200moe_q4k_dequant of one layer's whole expert stack (gate, up, down of
    the 256 experts, fields from seed 1) to bf16: three launches per step."""
    import torch
    from b200moe import _abi
    from b200moe.engine import DeviceLayer
    L = DeviceLayer.synthetic(1, 0, dev)
    srcs = [L.gate, L.up, L.down]
    nel = [t.numel() // 144 * 256 for t in srcs]
    out = torch.empty(sum(nel), dtype=torch.bfloat16, device=dev)
    views, o = [], 0
    for n in nel:
        views.append(out[o:o + n])
        o += n

    def step():
        for src, v in zip(srcs, views):
            _abi.q4k_dequant(src, v, _abi.BF16)

    ms = _events_time(step, max(K, 10), W, dev)
    nblocks = sum(t.numel() for t in srcs) // 144
    rd, wr = nblocks * 144, nblocks * 256 * 2
    gbs = (rd + wr) / (ms / 1e3) / 1e9
    del out, L
    torch.cuda.empty_cache()
    return {"blocks": nblocks, "read_bytes": rd, "write_bytes": wr, "ms_per_step": ms, "launches_per_step": 3,
            "achieved_gbs": gbs, "peak_gbs": hbm_peak, "frac": gbs / hbm_peak,
            "note": "BASELINE quotes 786,432 blocks for these shapes; the shapes [256,1024,2048] + [256,2048,512] "
                    "hold 3,145,728 blocks, which is what runs"}


def bench_config2(eng, dev, K, W, hbm_peak, batches=(1, 8, 32, 64, 256)):
    """one MoE layer at batch B under the Zipf(1.1) routing law (per-expert
    logit bias), one call per layer rotated over the stack's 40 layer copies so the weights
    streamed per step exceed L2; the block's own path choice per B."""
    import numpy as np
    import torch
    from b200moe import moe, synth
    from b200moe.engine import DeviceLayer
    layers = []
    for l, L in enumerate(eng.layers):
        bias = torch.from_numpy(synth.zipf_bias(2, l)).to(dev)
        layers.append(DeviceLayer(L.gate, L.up, L.down, L.sh_gate, L.sh_up, L.sh_down, L.router_w, L.sh_gate_w,
                                  logit_bias=bias, gate_up_stride=L.gate_up_stride))
    nl = len(layers)
    res = {}
    for B in batches:
        x = torch.from_numpy(synth.tokens(2, B, stream=60 + B).view(np.int16)).view(torch.bfloat16).to(dev)
        out = torch.empty((B, 2048), dtype=torch.float32, device=dev)
        uniq = []
        for L in layers:
            _, info = moe.moe_block(x, L, 0, out=out)
            uniq.append(int(torch.unique(info["ids"]).numel()))

        def step():
            for L in layers:
                moe.moe_block(x, L, 0, out=out)

        g = _graph_of(step, dev)
        ms = _events_time(g.replay, max(K, 5), W, dev)
        del g
        per_layer_ms = ms / nl
        u = float(np.mean(uniq))
        byts = u * EXPERT_BYTES + EXPERT_BYTES + ROUTER_BYTES + WSG_BYTES + B * 2048 * (2 + 4)
        gbs = byts / (per_layer_ms / 1e3) / 1e9
        path = ("persistent kernel (one layer per launch)" if B == 1 else
                "grouped GEMMs (10 per layer)" if B >= moe.PREFILL_MIN_TOKENS else
                "grouped decode (5 per layer)" if B <= moe.GROUPED_MAX_TOKENS else "decode kernels (3 per layer)")
        res["b%d" % B] = {"us_per_layer": per_layer_ms * 1e3, "tok_per_s": B / (per_layer_ms / 1e3),
                          "distinct_experts": u, "bytes_per_layer": byts, "achieved_gbs": gbs,
                          "frac": gbs / hbm_peak, "path": path}
    return res


def bench_config4(eng, dev, K, W, tf_peak):
    """BASELINE config 4's other cells: decode at B = 32 and a prefill of 8192 tokens through the
    40-layer stack (``resid += moe(rmsnorm(resid))`` per layer, the block's own path choice)."""
    import numpy as np
    import torch
    from b200moe import moe, synth
    nl = len(eng.layers)
    res = {}
    for name, T in (("decode_b32", 32), ("prefill_t8192", 8192)):
        x0 = torch.from_numpy(synth.bf16_bits_to_f32(synth.tokens(4, T, stream=80)).reshape(T, 2048).copy()).to(dev)
        resid = x0.clone()
        fn = moe.moe_stack_prefill if T >= moe.PREFILL_MIN_TOKENS else moe.moe_stack
        ws = (torch.empty(moe._abi.prefill_workspace_size(T), dtype=torch.uint8, device=dev)
              if fn is moe.moe_stack_prefill else torch.empty(moe.stack_workspace_bytes(T), dtype=torch.uint8,
                                                                device=dev))

        def step():
            resid.copy_(x0)
            fn(resid, eng, ws=ws)

        g = _graph_of(step, dev)
        ms = _events_time(g.replay, max(3, min(K, 10 if T > 64 else 50)), min(W, 3), dev)
        del g
        fin = bool(torch.isfinite(resid).all())
        flops = nl * 2.0 * T * (9 * 3 * 2048 * 512 + 256 * 2048)
        res[name] = {"tokens": T, "layers": nl, "ms_per_step": ms, "tok_per_s": T / (ms / 1e3),
                     "tflops": flops / (ms / 1e3) / 1e12, "frac_of_bf16_peak": flops / (ms / 1e3) / 1e12 / tf_peak,
                     "path": "grouped GEMMs (10 kernels per layer)", "finite": fin}
        del ws, resid, x0
        torch.cuda.empty_cache()
    return res


def bench_prefill_ep(dev, rank, world, K, W, tf_peak, T_total=4096, seed=3, check=True, bias=False):
    """Config 3 under expert parallelism: T_total tokens split over the ranks, 256/world experts per
    rank, one layer per step as one CUDA-graph replay (eager if capture is refused), max over ranks.
    Stage times come from a separate eager pass with events between the stages. On rank 0 the
    gathered outputs are compared with the single-GPU prefill of all tokens."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from b200moe import moe, synth
    from b200moe.engine import DeviceLayer
    from b200moe.ep import ExpertParallelMoE
    T = T_total // world
    L = DeviceLayer.synthetic(seed, 0, dev, bias=bias)
    ep = ExpertParallelMoE(L)
    xb = synth.tokens(seed, T_total, stream=100)
    x_all = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16).reshape(T_total, 2048)
    x_loc = x_all[rank * T:(rank + 1) * T].to(dev)
    out = torch.empty((T, 2048), dtype=torch.float32, device=dev)

    def step():
        ep.forward(x_loc, out=out)

    for _ in range(2):  # eager warm-up: communicators, tensor maps, buffers
        step()
    torch.cuda.synchronize(dev)
    graph, how = None, "cuda_graph"
    try:
        graph = _graph_of(step, dev)
        ok = 1
    except Exception as e:  # noqa: BLE001 -- any capture refusal falls back to eager launches
        ok, how = 0, "eager (graph capture refused: %s)" % type(e).__name__
        graph = None
    if world > 1:
        t = torch.tensor([ok], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        if int(t.item()) == 0 and graph is not None:
            graph, how = None, "eager (graph capture refused on another rank)"
    run = graph.replay if graph is not None else step
    if world > 1:
        dist.barrier()
    ms = _events_time(run, max(K, 10), W, dev)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    # per-stage times: eager steps with an event after each stage
    names = ("route", "dispatch", "experts", "combine", "sum")
    per = {n: [] for n in names}
    reps = 5
    for rep in range(reps + 1):  # the first rep is discarded; the median of the rest is kept
        # (an eager stage interval also holds any host stall before its launch)
        evs = [torch.cuda.Event(enable_timing=True)]
        evs[0].record()

        def mark(stage):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            evs.append(e)

        ep.forward(x_loc, out=out, mark=mark)
        torch.cuda.synchronize(dev)
        if rep:
            for i, n in enumerate(names):
                per[n].append(evs[i].elapsed_time(evs[i + 1]))
    stages = {n: statistics.median(per[n]) for n in names}
    if world > 1:
        tt = torch.tensor([stages[n] for n in names], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        stages = {n: float(v) for n, v in zip(names, tt.tolist())}
    stages["sum_of_stages_eager"] = sum(stages[n] for n in names)
    status = moe._abi.prefill_status(ep.workspace(T), world * T if world > 1 else T) | ep.p2p_status(T)
    flops = 2.0 * T_total * 9 * 3 * 2048 * 512
    res = {"tokens": T_total, "tokens_per_rank": T, "experts_per_rank": 256 // world, "n_gpus": world,
           "ms_per_step": ms, "tok_per_s": T_total / (ms / 1e3), "tflops_per_gpu": flops / world / (ms / 1e3) / 1e12,
           "frac_of_bf16_peak": flops / world / (ms / 1e3) / 1e12 / tf_peak, "timing": how,
           "stages_ms_max_over_ranks": stages, "status": status, "transport": ep.transport}
    if check:
        step()
        ids = torch.empty((T, 8), dtype=torch.int32, device=dev)
        o, i = ep.forward(x_loc)
        ids.copy_(i)
        if world > 1:
            outs = [torch.empty_like(o) for _ in range(world)]
            idss = [torch.empty_like(ids) for _ in range(world)]
            dist.all_gather(outs, o)
            dist.all_gather(idss, ids)
        else:
            outs, idss = [o], [ids]
        if rank == 0:
            ref, info = moe.moe_block(x_all.to(dev), L, path="prefill")
            got = torch.cat(outs)
            res["parity_vs_single_gpu"] = {
                "ids_equal": bool(torch.equal(torch.cat(idss), info["ids"])),
                "rel_l2": float(torch.linalg.norm(got - ref) / torch.linalg.norm(ref)),
                "finite": bool(torch.isfinite(got).all())}
        if world > 1:
            dist.barrier()
    del graph
    if world > 1:
        dist.barrier()
    ep.close()
    del ep, L
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------------- GPU arm
def run_b200(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    import __graft_entry__ as G
    G.load_package()
    from b200moe import _abi, moe, synth
    from b200moe.engine import DeviceEngine, DeviceLayer

    rank, local_rank, world = env_rank()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    T = args.batch
    K, W = args.steps, args.warmup
    hbm_peak, peak_kind = peaks()
    persist_ctas, persist_cluster = 0, 0
    graph = None
    expert_bytes = None

    if args.workload == "stack_decode":
        eng = (published_engine(args.seed, args.layers, dev) if args.formats == "published"
               else DeviceEngine.synthetic(args.seed, args.layers, dev, bias=args.zipf))
        if args.law == 2 and args.formats == "q4k":
            for Lw in eng.layers:
                for t in (Lw.gate, Lw.up, Lw.down, Lw.sh_gate, Lw.sh_up, Lw.sh_down):
                    synth.law2_blocks_(t)
        nl = args.layers
        persist_ctas, persist_cluster = _abi.decode_persistent_info() if T == 1 else (0, 0)
        if args.formats == "published" and not _abi.decode_persistent_formats():
            persist_ctas, persist_cluster = 0, 0  # such layers take the three-kernel path
        # the block's own path choice: grouped GEMMs (10 kernels per layer) from
        # moe.PREFILL_MIN_TOKENS tokens on, else one persistent kernel (T = 1), the grouped
        # small-batch decode (router, plan, gate/up, down, combine: 5 per layer) for 2..16 tokens
        # of Q4_K layers, or the three gather-GEMV kernels per layer
        use_prefill = (T >= moe.PREFILL_MIN_TOKENS) if args.path == "auto" else (args.path == "prefill" and T > 1)
        grouped = 2 <= T <= moe.GROUPED_MAX_TOKENS and args.formats == "q4k"
        launches_per_step = 10 * nl if use_prefill else (1 if persist_ctas else (5 if grouped else 3) * nl)
        stack_fn = moe.moe_stack_prefill if use_prefill else moe.moe_stack
        bytes_per_step = nl * (9 * EXPERT_BYTES * (1 if T == 1 else 0) + ROUTER_BYTES + WSG_BYTES + 2 * T * 2048 * 4)
        ws = (torch.empty(_abi.prefill_workspace_size(T), dtype=torch.uint8, device=dev) if use_prefill
              else torch.empty(moe.stack_workspace_bytes(T), dtype=torch.uint8, device=dev))
        tok_bits = synth.tokens(args.seed, (K + W) * T, stream=100 + rank)
        tok = torch.from_numpy(synth.bf16_bits_to_f32(tok_bits).reshape(K + W, T, 2048).copy())
        tok_dev = tok.to(dev)
        x_in = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        resid = torch.empty_like(x_in)
        ids_all = torch.zeros((K + W, nl, T, 8), dtype=torch.int32, device=dev)
        ids_step = torch.zeros((nl, T, 8), dtype=torch.int32, device=dev)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            x_in.copy_(tok_dev[0])
            resid.copy_(x_in)
            stack_fn(resid, eng, ws=ws, ids_out=ids_step)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            resid.copy_(x_in)
            stack_fn(resid, eng, ws=ws, ids_out=ids_step)

        def step(i):
            x_in.copy_(tok_dev[i], non_blocking=True)
            graph.replay()
            ids_all[i].copy_(ids_step, non_blocking=True)
    elif args.workload == "layer_decode":
        L = DeviceLayer.synthetic(args.seed, 0, dev, bias=(args.seed == 2))
        # one layer, called again every step: after the first step its rows sit in L2, so this
        # workload times latency, not HBM bandwidth (no roofline; decode_config2 rotates layers)
        nl = 1
        persist_ctas, persist_cluster = _abi.decode_persistent_info() if T == 1 else (0, 0)
        launches_per_step = 1 if persist_ctas else 3
        tok_bits = synth.tokens(args.seed, (K + W) * T, stream=100 + rank)
        tok_dev = torch.from_numpy(tok_bits.view(np.int16)).view(torch.bfloat16).reshape(K + W, T, 2048).to(dev)
        out = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        ids_all = torch.zeros((K + W, 1, T, 8), dtype=torch.int32, device=dev)
        bytes_per_step = None

        def step(i):
            moe.moe_block(tok_dev[i], L, 0, out=out)
    elif args.workload == "prefill":
        # config 3: one layer, 4096 tokens through token sort + tcgen05 grouped GEMMs
        T = args.batch if args.batch > 1 else 4096
        L = DeviceLayer.synthetic(3, 0, dev)
        nl = 1
        launches_per_step = 10
        tok_bits = synth.tokens(3, T, stream=100 + rank)
        tok_dev = torch.from_numpy(tok_bits.view(np.int16)).view(torch.bfloat16).reshape(T, 2048).to(dev)
        out = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        ids_all = torch.zeros((K + W, 1, 1, 8), dtype=torch.int32, device=dev)
        pws = moe.prefill_workspace(T, dev)
        flops_per_step = 2.0 * T * 9 * 3 * 2048 * 512   # 8 routed + shared, gate+up+down MACs x 2
        bytes_per_step = None

        def step(i):
            moe.moe_block(tok_dev, L, 0, out=out, path="prefill")
    elif args.workload == "prefill_ep":
        # config 3 with expert parallelism (strong scaling: total work fixed), as the sub-result
        res = bench_prefill_ep(dev, rank, world, K, W, _tf_peak(), T_total=args.batch if args.batch > 1 else 4096)
        if rank == 0:
            print(json.dumps({"metric": "moe_prefill_ep_tok_per_s", "value": res["tok_per_s"], "unit": "tok/s",
                              "n_gpus": world, "steps": max(K, 10), "warmup": max(3, W),
                              "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                              "vs_baseline": None, "dtype": "fp16 operands, f32 accumulate", "data": "synthetic",
                              "config": {"workload": "config3_prefill_ep_t%d" % res["tokens"],
                                         "parallelism": "ep%d" % world}, "prefill_ep": res}), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    else:
        raise SystemExit("unknown workload %s" % args.workload)

    # ---------------- value: device-resident inputs, CUDA events, max over ranks
    for i in range(W):
        step(i)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(physical_index(local_rank))
    sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for i in range(K):
        step(W + i)
    t_end.record()
    torch.cuda.synchronize(dev)
    sampler.stop_ev.set()
    sampler.join()
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
        dist.barrier()
    ms_step = ms / K
    value = world * K * T / (ms / 1e3)
    scaling = "strong" if args.workload == "prefill_ep" else "weak"
    if args.workload in ("prefill", "prefill_ep"):
        st = moe.prefill_status(T, dev) if args.workload == "prefill" else 0
        if st != 0:
            raise SystemExit("prefill status word %d (pipeline timeout or fp16 range)" % st)

    # algorithmic bytes: distinct experts actually touched per layer (+ shared, router, act)
    ids_np = ids_all[W:].cpu().numpy()
    if args.workload == "stack_decode":
        uniq = [[len(np.unique(ids_np[i, l])) for l in range(nl)] for i in range(K)]
        lb = [layer_bytes(eng.layers[l]) for l in range(nl)]  # Q4_K: (EXPERT_BYTES, EXPERT_BYTES, router)
        expert_bytes = float(np.mean([sum(u * lb[l][0] + lb[l][1] for l, u in enumerate(row)) for row in uniq]))
        bytes_per_step = expert_bytes + sum(r for _, _, r in lb) + nl * 2 * T * 2048 * 4
    achieved = bytes_per_step / (ms_step / 1e3) / 1e9 if bytes_per_step else None
    roof_bound, roof_unit, peak = "hbm", "GB/s", hbm_peak
    if args.workload in ("prefill", "prefill_ep"):
        roof_bound, roof_unit = "tensor", "TFLOP/s"
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peak = float(json.load(f)["bf16_tflops"])
        except Exception:
            peak, peak_kind = 1590.0, "fallback"
        achieved = flops_per_step / world / (ms_step / 1e3) / 1e12   # per GPU

    # ---------------- e2e: pinned host input -> graph -> host read of the result, every step
    e2e = None
    if args.workload == "stack_decode":
        host_in = tok.pin_memory()
        host_out = torch.empty((T, 2048), dtype=torch.float32).pin_memory()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(dev)
        for i in range(W):
            x_in.copy_(host_in[i], non_blocking=True)
            graph.replay()
            host_out.copy_(resid, non_blocking=True)
            cur.synchronize()
        if world > 1:
            dist.barrier()
        e0.record()
        chk = 0.0
        for i in range(K):
            x_in.copy_(host_in[W + i], non_blocking=True)
            graph.replay()
            host_out.copy_(resid, non_blocking=True)
            cur.synchronize()
            chk += float(host_out[0, 0])
        e1.record()
        torch.cuda.synchronize(dev)
        ems = e0.elapsed_time(e1)
        if world > 1:
            tt = torch.tensor([ems], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            ems = float(tt.item())
        if not np.isfinite(chk):
            raise SystemExit("non-finite result in e2e run")
        e2e = {"value": world * K * T / (ems / 1e3), "unit": "tok/s", "h2d_bytes_per_step": T * 2048 * 4,
               "d2h_bytes_per_step": T * 2048 * 4, "ms_per_step": ems / K,
               "api": ("b200moe.moe.moe_stack_prefill (C ABI b200moe_moe_prefill per layer)" if use_prefill else
                       "b200moe.moe.moe_stack (C ABI b200moe_stack_decode)") + " in a CUDA graph"}

    # ---------------- CPU baseline (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload == "stack_decode":
        from oracle import moe as OM
        layers, x0, cores, nlp, _ = cpu_sample(args, args.cpu_layers, eng=eng)
        ts = []
        for _ in range(3):
            t0 = time.perf_counter()
            OM.stack_port(x0, layers, cores)
            ts.append(time.perf_counter() - t0)
        sec_tok = statistics.median(ts) * (args.layers / nlp)
        cpu = {"value": T / sec_tok, "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": "1 token through %d of %d layers, median of 3, scaled x%g (torch-f32 port of "
                         "engine/m3_forward.py moe_block + rmsnorm_a, per-hit-expert dequant timed%s)"
                         % (nlp, args.layers, args.layers / nlp,
                            "; the published layout's first layers: Q5_K down, Q8_0 shared, F32 router, "
                            "norm weight" if args.formats == "published" else "")}

    # the committed ncu traffic is the Q4_K workload's (none recorded for the published layout)
    traffic = committed_traffic(args.workload) if args.formats == "q4k" else None
    line = {
        "metric": {"stack_decode": "moe_stack_decode_tok_per_s", "layer_decode": "moe_layer_decode_tok_per_s",
                   "prefill": "moe_prefill_tok_per_s", "prefill_ep": "moe_prefill_ep_tok_per_s"}[args.workload],
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": (("synthetic (seeded Q4_K, config-0 field law; random-init weights)" if args.law == 1 else
                  "synthetic (seeded Q4_K, config-0 blocks with d * 2^-6 and dmin * 2^-2: centred weights)")
                 if args.formats == "q4k" else
                 "synthetic, published-file layout (Q4_K gate/up, Q5_K/Q6_K down, Q8_0 shared, F32 router; "
                 "seeded random block bytes)"),
        "config": {"workload": {"stack_decode": ("published_formats_stack_decode_b%d" if args.formats == "published"
                                                 else "config2_zipf_stack_decode_b%d" if args.zipf
                                                 else "config4_stack_decode_b%d") % T,
                                "layer_decode": "config0_layer_decode_b%d" % T,
                                "prefill": "config3_prefill_t%d" % T,
                                "prefill_ep": "config3_prefill_ep_t%d" % (T * world)}[args.workload],
                   "layers": nl, "batch": T, "seed": args.seed, "law": args.law,
                   "parallelism": ("ep%d" % world) if args.workload == "prefill_ep" else "replicas%d" % world,
                   "l2": "inputs larger than L2: distinct token per step, %.0f MB of weights streamed per step"
                         % ((bytes_per_step or 0) / 1e6)},
        "roofline": {"bound": roof_bound, "achieved": achieved, "peak": peak, "unit": roof_unit,
                     "frac": (achieved / peak) if achieved else None,
                     "traffic": traffic.get("dram_bytes_per_step") if traffic else None,
                     "peak_kind": peak_kind,
                     "kernel": (("one graph replay = 1 persistent kernel over all %d layers (%d CTAs in clusters "
                                 "of %d; router, routing, bulk-copied %s gate/up and down rows, combine)"
                                 % (nl, persist_ctas, persist_cluster,
                                    "Q4_K" if args.formats == "q4k" else "Q4_K / Q5_K / Q6_K / Q8_0"))
                                if persist_ctas
                                else ("one graph replay = %d kernels (10 per layer: the grouped-GEMM path)"
                                      % launches_per_step if args.workload == "stack_decode" and use_prefill else
                                      "one graph replay = %d kernels (router/shared K1, routed gate_up K2, "
                                      "down+combine K3 per layer)" % launches_per_step))
                               if args.workload in ("stack_decode", "layer_decode")
                               else ("one step = %d kernels per layer (prep, router GEMM, route, count, plan, fill, x gather, "
                                     "tcgen05 gate_up GEMM, tcgen05 down GEMM, combine); achieved = expert FLOPs / "
                                     "step time" % (launches_per_step // max(nl, 1)))},
        "gpu_launches": launches_per_step * K,
        "clocks": sampler.result(),
        "e2e": e2e,
        "cpu_baseline": cpu,
    }
    if args.workload == "stack_decode":
        line["north_star"] = {"expert_bytes_per_token": expert_bytes,
                              "frac_of_8TBs": expert_bytes / (ms_step / 1e3) / 8e12,
                              "target_frac": 0.60, "us_per_token": ms_step * 1e3 / T}
        st = _abi.decode_status(ws, T) if not use_prefill else _abi.prefill_status(ws, T)
        if st != 0:
            raise SystemExit("decode status word %d after the timed region" % st)

    # ---------------- nested sub-results (after the headline's timed region)
    if (args.workload == "stack_decode" and args.formats == "q4k" and not args.zipf and T == 1
            and args.layers == N_LAYERS and args.law == 1 and not args.no_extras):
        graph = None
        tf_peak = _tf_peak()
        xs = ClockSampler(physical_index(local_rank))
        xs.start()
        line["prefill_ep"] = bench_prefill_ep(dev, rank, world, K, W, tf_peak)
        line["prefill_ep"]["decode_b256"] = bench_prefill_ep(dev, rank, world, K, W, tf_peak, T_total=256, seed=2,
                                                           bias=True)
        if world == 1:
            line["dequant_config1"] = bench_dequant(dev, K, W, hbm_peak)
            line["decode_config2"] = bench_config2(eng, dev, K, W, hbm_peak)
            line["config4"] = bench_config4(eng, dev, K, W, tf_peak)
        xs.stop_ev.set()
        xs.join()
        line["extras_clocks"] = xs.result()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        graph = None
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
