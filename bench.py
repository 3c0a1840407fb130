"""Benchmark: one MoE layer decode step through the C ABI (libsmoe_cuda.so).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1: BASELINE config 1 - one Qwen3-30B-A3B-shaped layer: router GEMV +
softmax/top-8/renorm + fused 4-bit (AFFINE-Q4) SwiGLU FFN of the 8 routed
experts + weighted combine, batch 1, x bf16[2048] -> y bf16[2048].
N > 1 (torchrun, one rank per GPU): BASELINE config 3's layer - the
Qwen3-235B-A22B shape (d 4096, d_ff 1536) - expert parallel: rank r holds
experts [r*128/N, (r+1)*128/N) of every layer, x and y live on rank 0, and the
exchange runs inside the layer kernel over NVLink (smoe_cuda_moe_layer_ep);
strong scaling, timed as the max over ranks; rank 0 also times the same layer
on its own GPU alone (`single_gpu_same_layer`), and the N = 1 line carries
config 3's 1-GPU point (`config3_layer_1gpu`).

`value`: algorithmic HBM bytes of the layer step (router + x + 8 experts + y;
config 1: 524,288 + 4,096 + 8 x 2,654,208 + 4,096 = 21,762,144 B) / device
time, inputs resident. Exactly K steps are timed, as one CUDA-graph replay of
K layer calls; step i runs resident layer i % L (L = 8 for config 1, 4 for
config 3, each far beyond L2 in total) on x row i % 64, so every step's
experts and x are fresh. `e2e`: the same K steps with each step's x read from
pinned host memory and its y written into pinned host memory by the library.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "s-moe_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

D, DFF, E, K = 2048, 768, 128, 8
N_LAYERS = 8
LAYER_BYTES = 524_288 + 4_096 + 8 * 2_654_208 + 4_096      # 21,762,144
FFN_BYTES = 8 * 2_654_208                                    # 21,233,664
METRIC = "expert-FFN HBM GB/s, Qwen3-30B-A3B MoE layer decode step, batch 1"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks / throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=None)
    return rank, world, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


SHAPES = {
    # config 1: one Qwen3-30B-A3B MoE layer
    "30b": dict(d=2048, dff=768, E=128, k=8, layers=8,
                workload="config1: Qwen3-30B-A3B MoE layer (d 2048, 128 experts, top-8, d_ff 768, "
                         "AFFINE-Q4 g64), batch 1, bf16 in/out"),
    # config 3: one Qwen3-235B-A22B MoE layer, expert parallel over the GPUs
    "235b": dict(d=4096, dff=1536, E=128, k=8, layers=4,
                 workload="config3: Qwen3-235B-A22B MoE layer (d 4096, 128 experts, top-8, d_ff 1536, "
                          "AFFINE-Q4 g64), batch 1, bf16 in/out"),
}


def shape_bytes(sh):
    """(layer step bytes, expert-FFN bytes) of one batch-1 layer step."""
    import smoe_cuda as S
    ffn = sh["k"] * S.expert_bytes(S.FMT_AFFINE_Q4, sh["d"], sh["dff"])
    return sh["E"] * sh["d"] * 2 + 2 * sh["d"] * 2 + ffn, ffn


# ------------------------------------------------------------------ data
def make_inputs(sh=None, n_layers=None, seed=1234):
    """CPU copies of the benchmark layers (all experts) and 64 x rows."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    sh = sh or SHAPES["30b"]
    layers = []
    for l in range(n_layers or sh["layers"]):
        arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, sh["E"], sh["d"], sh["dff"], seed=seed + l)
        rw = O.normal_bf16(seed + l, 6, sh["E"] * sh["d"], 0.0, 0.02)
        layers.append((arena, stride, off, rw))
    xs = np.stack([O.normal_bf16(seed + 7919 + i, 5, sh["d"]) for i in range(64)])
    return layers, xs


# ------------------------------------------------------------ CPU legs
def cpu_layer_time(layers, xs, budget_s, threads, sh=None):
    """Reference router (compiled sampler/top-k/matvec of the reference) +
    the oracle's restated Q4 FFN (there is no reference CPU FFN) + combine."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    used = O.set_threads(threads)
    R = O.ref()
    sh = sh or SHAPES["30b"]
    E, D, DFF, K = sh["E"], sh["d"], sh["dff"], sh["k"]
    n, t0 = 0, time.perf_counter()
    while True:
        arena, stride, off, rw = layers[n % len(layers)]
        x = O.bf16_to_f32(xs[n % len(xs)])
        if R is not None:
            lg = np.empty(E, np.float32)
            ids = np.zeros(K, np.uint32)
            w = np.zeros(K, np.float32)
            R.ref_route(x, rw, E, D, K, 1, lg, ids, w)
            y = np.zeros(D, np.float32)
            for j in range(K):
                y = y + w[j] * O.expert_ffn(O.FMT_AFFINE_Q4, arena[ids[j]], D, DFF, x, precise=False)
        else:
            O.moe_layer(O.FMT_AFFINE_Q4, x, rw, arena, stride, E, D, DFF, K, precise=False)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    kind = "reference" if R is not None else "port"
    return n, el, used, kind


def run_reference(args, rank, world):
    """The reference's own CPU path, timed on this host: its compiled router
    (matvec_bf16 + top_k + renorm, sampler.hpp/scout.cpp/common.hpp built
    unmodified into oracle/_ref) plus the restated Q4 FFN (the reference has
    no CPU FFN), all host threads. One step = one MoE layer step of the
    workload our arm runs at this N (config 1 at N = 1, config 3 at N > 1)."""
    if rank != 0:
        return
    sh = SHAPES["235b" if world > 1 else "30b"]
    layer_bytes, _ = shape_bytes(sh)
    layers, xs = make_inputs(sh, n_layers=2 if world > 1 else None)
    threads = os.cpu_count() or 1
    for i in range(args.warmup):
        cpu_layer_time(layers, xs, 0.0, threads, sh)
    n_total, el_total, used, kind = 0, 0.0, threads, "port"
    for i in range(args.steps):
        n, el, used, kind = cpu_layer_time(layers, xs, 0.0, threads, sh)   # exactly one layer step
        n_total += n
        el_total += el
    gbs = layer_bytes * n_total / el_total / 1e9
    metric = METRIC if world == 1 else METRIC.replace("Qwen3-30B-A3B", "Qwen3-235B-A22B")
    line = {"impl": "reference", "metric": metric, "value": round(gbs, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * el_total / n_total, 3), "higher_is_better": True,
            "scaling": "weak" if world == 1 else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": sh["workload"], "layers_cycled": len(layers)},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": kind,
                             "sample": f"{n_total} layer steps in {el_total:.2f} s: reference "
                                       "router (compiled from the reference) + restated Q4 FFN, "
                                       "OpenMP"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU arm
def load_layers(ctx, sh, base, per, seed=1234):
    """sh["layers"] resident layers (experts [base, base+per) of each) in the
    tiled device layout, with the full router; returns (descs, keep)."""
    import numpy as np
    import torch
    import oracle as O
    import smoe_cuda as S
    descs, keep = [], []
    for l in range(sh["layers"]):
        arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, per, sh["d"], sh["dff"], seed + l, first=base)
        rw = O.normal_bf16(seed + l, 6, sh["E"] * sh["d"], 0.0, 0.02)
        da = torch.from_numpy(arena).cuda()
        dr = torch.from_numpy(rw.view(np.int16)).cuda()
        vault = S.make_layer(da, stride, off, per, sh["d"], sh["dff"], S.FMT_AFFINE_Q4, dr)
        # one-time load-time re-layout into the tiled device format (the
        # vault-layout copy is dropped afterwards)
        tstride = S.tiled_stride(S.FMT_AFFINE_Q4, sh["d"], sh["dff"])
        tb = torch.empty(per * tstride, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()             # the arena was copied on torch's stream
        descs.append(ctx.prepack_layer(vault, tb, tstride))
        ctx.synchronize()
        keep += [tb, dr]
        del da
    return descs, keep


def graph_of(stream, calls):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for c in calls:
            c()
    return g


def timed_replay(graph, stream, world):
    """Device time (ms) of one replay, barrier + synchronize on both sides."""
    import torch
    barrier(world)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        t0.record(stream)
        graph.replay()
        t1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return t0.elapsed_time(t1)


def run_ours(args, rank, world, local):
    """N = 1: config 1 (the 30B layer). N > 1: config 3 (the 235B layer),
    expert parallel - rank r holds experts [r*128/N, (r+1)*128/N) of every
    layer, x and y live on rank 0, the exchange runs inside the layer kernel
    over NVLink; rank 0 also times the same layer on its own GPU alone."""
    import numpy as np
    import torch
    import oracle as O
    import smoe_cuda as S

    torch.cuda.set_device(local)
    ep = world > 1
    sh = SHAPES["235b" if ep else "30b"]
    d, E, K, NL = sh["d"], sh["E"], sh["k"], sh["layers"]
    layer_bytes, ffn_bytes = shape_bytes(sh)
    ctx = S.Context(local)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    base, per = S.ep_partition(E, world, rank) if ep else (0, E)
    descs, keep = load_layers(ctx, sh, base, per)
    if ep:
        import torch.distributed as dist
        grp = dist.new_group(backend="gloo")
        handles = S.ep_exchange_handles(ctx.ep_export(), world, group=grp)
        ctx.ep_attach(rank, world, handles)
        barrier(world)
    xs = np.stack([O.normal_bf16(1234 + 7919 + i, 5, d) for i in range(64)])
    d_x = torch.from_numpy(xs.view(np.int16)).cuda()          # [64, d] bf16: a fresh x each step
    d_y = torch.zeros(d, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(NL, K, dtype=torch.int32, device="cuda")
    wts = torch.zeros(NL, K, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def layer(i, xptr=None, yptr=None):   # router + top-k + expert FFN + combine: one launch
        l = i % NL
        x = d_x[i % 64].data_ptr() if xptr is None else xptr
        y = d_y if yptr is None else yptr
        if ep:
            ctx.moe_layer_ep(descs[l], E, base, x if rank == 0 else None, S.DTYPE_BF16, 1, K, True,
                             y if rank == 0 else None, S.DTYPE_BF16, ids[l], wts[l])
        else:
            ctx.moe_layer(descs[l], x, S.DTYPE_BF16, 1, K, True, y, S.DTYPE_BF16, ids[l], wts[l])

    def ffn(i):                           # the same with the routing already on the device
        l = i % NL
        ctx.moe_ffn(descs[l], d_x[i % 64].data_ptr(), S.DTYPE_BF16, ids[l], wts[l], K, 1, d_y, S.DTYPE_BF16)

    W, steps = max(args.warmup, 3), args.steps
    # eager warm-up (also sets kernel attributes and fills the routing)
    for i in range(max(W, NL)):
        layer(i)
    ctx.synchronize()
    # exactly `steps` layer steps per graph; step i: layer i % NL, x row i % 64
    g_warm = graph_of(stream, [lambda i=i: layer(i) for i in range(W)])
    g_step = graph_of(stream, [lambda i=i: layer(i) for i in range(steps)])
    g_ffn = None if ep else graph_of(stream, [lambda i=i: ffn(i) for i in range(steps)])
    with torch.cuda.stream(stream):
        g_warm.replay()
        g_step.replay()        # untimed: a graph's first launch also uploads it to the device
    torch.cuda.synchronize()
    barrier(world)
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    ms = max_over_ranks(timed_replay(g_step, stream, world), world)
    ffn_ms = None
    if not ep:
        with torch.cuda.stream(stream):
            g_ffn.replay()                     # its own warm-up
        ffn_ms = timed_replay(g_ffn, stream, world)
    ck = clocks.stop()
    per_step = ms / steps
    value = layer_bytes * steps / (ms * 1e-3) / 1e9

    # ---- end to end through the C ABI with host buffers: every step reads its
    # x from pinned host memory and writes y into pinned host memory (the
    # library stages x with a copy kernel and stores y's rows to the host).
    hx = torch.from_numpy(xs.view(np.int16)).pin_memory()
    hy = torch.zeros(NL, d, dtype=torch.bfloat16).pin_memory()
    g_e2e = graph_of(stream, [lambda i=i: layer(i, hx[(2000 + i) % 64].data_ptr(), hy[i % NL].data_ptr())
                              for i in range(steps)])
    with torch.cuda.stream(stream):
        g_e2e.replay()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(timed_replay(g_e2e, stream, world), world)
    e2e = layer_bytes * steps / (e2e_ms * 1e-3) / 1e9

    single = None
    if ep and rank == 0:
        # the same layer on this GPU alone (all 128 experts), for the scaling curve
        ctx1 = S.Context(local)
        ctx1.set_stream(stream.cuda_stream)
        d1, k1 = load_layers(ctx1, sh, 0, E)
        ids1 = torch.zeros(NL, K, dtype=torch.int32, device="cuda")
        w1 = torch.zeros(NL, K, dtype=torch.float32, device="cuda")
        calls = [lambda i=i: ctx1.moe_layer(d1[i % NL], d_x[i % 64].data_ptr(), S.DTYPE_BF16, 1, K, True, d_y,
                                            S.DTYPE_BF16, ids1[i % NL], w1[i % NL]) for i in range(steps)]
        for c in calls[:NL]:
            c()
        ctx1.synchronize()
        g1 = graph_of(stream, calls)
        with torch.cuda.stream(stream):
            g1.replay()
        ms1 = timed_replay(g1, stream, 1)
        single = {"value": round(layer_bytes * steps / (ms1 * 1e-3) / 1e9, 2), "unit": "GB/s",
                  "layer_us": round(ms1 / steps * 1e3, 3)}
        del g1, d1, k1
        ctx1.close()

    b32 = None
    if ep:
        try:
            b32 = config3_b32_ep_leg(ctx, stream, rank, world, args)
        except Exception as ex:  # noqa: BLE001  (the headline line stays intact)
            b32 = {"error": f"{type(ex).__name__}: {ex}"[:300]}

    if rank == 0:
        peak, peak_kind = peaks()
        traffic = profile_traffic()
        if ep:
            ach = ffn_bytes / world / (per_step * 1e-3) / 1e9
            kern = (f"k_moe_layer expert parallel x{world} (layer incl. routing and NVLink exchange), "
                    f"{ffn_bytes // world:,} B of experts per GPU per launch, {per_step * 1e3:.2f} us avg")
        else:
            ach = ffn_bytes / (ffn_ms / steps * 1e-3) / 1e9
            kern = (f"k_moe_layer (expert FFN + combine, routing given), {ffn_bytes:,} B per launch, "
                    f"{ffn_ms / steps * 1e3:.2f} us avg")
        line = {
            "metric": METRIC if not ep else METRIC.replace("Qwen3-30B-A3B", "Qwen3-235B-A22B"),
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_step, 5),
            "higher_is_better": True, "scaling": "strong" if ep else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config distributions)",
            "config": {"workload": sh["workload"], "layers_cycled": NL,
                       "l2": (f"inputs larger than L2 ({NL} resident layers cycled, a fresh x per step from "
                              "64 rows)"),
                       "warm_up": (f"{max(args.warmup, 3)} eager steps, then one untimed replay of the "
                                   "timed graph (its first launch uploads it)"),
                       "parallelism": (f"expert parallel x{world} ({per} experts per GPU, exchange "
                                       "in-kernel over NVLink)") if ep else "single GPU"},
            "layer_us": round(per_step * 1e3, 3),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "traffic": None if ep else traffic,
                         "kernel": kern, "peak_kind": peak_kind},
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": d * 2,
                    "d2h_bytes_per_step": d * 2},
            "gpu_launches": int(steps),
            "clocks": ck,
        }
        if b32:
            line["config3_b32_ep"] = b32
        if single:
            line["single_gpu_same_layer"] = single
        if world == 1 and not args.no_cpu:
            layers_cpu, xs_cpu = make_inputs(n_layers=4)
            cpu = {}
            for label, threads in (("all", os.cpu_count() or 1), ("one", 1)):
                n, el, used, kind = cpu_layer_time(layers_cpu, xs_cpu, args.cpu_seconds / 2, threads)
                cpu[label] = {"value": round(LAYER_BYTES * n / el / 1e9, 4), "unit": "GB/s", "cores": used,
                              "kind": kind, "sample": f"{n} layer steps in {el:.1f} s (reference router + "
                                                      "restated Q4 FFN, OpenMP)"}
            line["cpu_baseline"] = cpu["all"]
            line["cpu_baseline_1core"] = cpu["one"]
        if world == 1 and not args.no_extra:
            for key, fn in (("config3_layer_1gpu", lambda: config3_leg(ctx, stream, args)),
                            ("sampler", lambda: sampler_leg(ctx, stream)),
                            ("decode_30b", lambda: decode_leg(ctx)),
                            ("batch256", lambda: batch_leg(ctx, stream)),
                            ("decode_b256", lambda: batched_decode_leg(ctx, "30b", 256, 45, 128)),
                            ("decode_235b", lambda: decode_235b_leg(ctx)),
                            ("decode_235b_b32", lambda: batched_decode_leg(ctx, "235b", 32, 45, 32))):
                try:                    # a side leg that fails leaves the headline line intact
                    line[key] = fn()
                except Exception as ex:  # noqa: BLE001
                    line[key] = {"error": f"{type(ex).__name__}: {ex}"[:300]}
                    import torch
                    torch.cuda.empty_cache()
        print(json.dumps(line), flush=True)
    ctx.close()


def config3_b32_ep_leg(ctx, stream, rank, world, args, B=32, nl=4, steps=20):
    """BASELINE config 3's batched case at N > 1: the 235B layer for 32
    tokens, experts sharded over the ranks (vault layout, expert-grouped path
    on each rank's slots, smoe_cuda_moe_layer_shard) and the partial sums
    combined by an NCCL reduce to rank 0; nl layers cycled. Max over ranks of
    the device time; rank 0 also times the whole layer on its own GPU."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import oracle as O
    import smoe_cuda as S
    sh = SHAPES["235b"]
    d, E, K, dff = sh["d"], sh["E"], sh["k"], sh["dff"]
    import datetime
    nccl = dist.new_group(backend="nccl", timeout=datetime.timedelta(seconds=120))   # a lost rank ends it
    base, per = S.ep_partition(E, world, rank)
    router = torch.from_numpy(O.normal_bf16(4242, 6, E * d, 0.0, 0.02).view(np.int16)).cuda()
    shards, keep = [], []
    for l in range(nl):
        arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, per, d, dff, 5000 + l, first=base)
        da = torch.from_numpy(arena).cuda()
        keep.append(da)
        shards.append(S.make_layer(da, stride, off, per, d, dff, O.FMT_AFFINE_Q4, router))
    xs = torch.from_numpy(np.stack([O.normal_bf16(77 + i, 5, B * d) for i in range(4)]).view(np.int16)).cuda()
    y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
    ids = torch.zeros(B, K, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()

    def step(i):
        ctx.moe_layer_shard(shards[i % nl], E, base, xs[i % 4], S.DTYPE_BF16, B, K, True, y, ids)
        dist.reduce(y, dst=0, group=nccl)

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            step(i)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), world)
    touched = int((np.bincount(ids.cpu().numpy().reshape(-1), minlength=E) > 0).sum())
    out = {"workload": f"config3 batched: Qwen3-235B-A22B MoE layer, batch {B}, experts over {world} GPUs "
                       "(expert-grouped path per rank) + NCCL reduce to rank 0", "steps": steps,
           "layer_us": round(ms / steps * 1e3, 2), "tokens_per_s_per_layer": round(B * steps / (ms * 1e-3)),
           "experts_touched": touched}
    if rank == 0:                               # the same layer on this GPU alone (2 layers cycled,
        full = []                               # 2.7 GB: beyond L2 all the same)
        for l in range(2):
            arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, E, d, dff, 5000 + l)
            da = torch.from_numpy(arena).cuda()
            keep.append(da)
            full.append(S.make_layer(da, stride, off, E, d, dff, O.FMT_AFFINE_Q4, router))
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(3):
                ctx.moe_layer(full[i % 2], xs[i % 4], S.DTYPE_BF16, B, K, True, y, S.DTYPE_F32)
            torch.cuda.synchronize()
            e0.record(stream)
            for i in range(steps):
                ctx.moe_layer(full[i % 2], xs[i % 4], S.DTYPE_BF16, B, K, True, y, S.DTYPE_F32)
            e1.record(stream)
            torch.cuda.synchronize()
        out["single_gpu_layer_us"] = round(e0.elapsed_time(e1) / steps * 1e3, 2)
    barrier(world)
    del keep
    torch.cuda.empty_cache()
    return out


def config3_leg(ctx, stream, args):
    """Config 3's layer (Qwen3-235B-A22B shape) on this GPU alone, batch 1:
    the 1-GPU point of the expert-parallel scaling curve."""
    import numpy as np
    import torch
    import oracle as O
    import smoe_cuda as S
    sh = SHAPES["235b"]
    layer_bytes, _ = shape_bytes(sh)
    descs, keep = load_layers(ctx, sh, 0, sh["E"])
    xs = np.stack([O.normal_bf16(99 + i, 5, sh["d"]) for i in range(64)])
    d_x = torch.from_numpy(xs.view(np.int16)).cuda()
    d_y = torch.zeros(sh["d"], dtype=torch.bfloat16, device="cuda")
    steps = 100
    calls = [lambda i=i: ctx.moe_layer(descs[i % sh["layers"]], d_x[i % 64].data_ptr(), S.DTYPE_BF16, 1, sh["k"],
                                       True, d_y, S.DTYPE_BF16) for i in range(steps)]
    for c in calls[:sh["layers"]]:
        c()
    ctx.synchronize()
    g = graph_of(stream, calls)
    with torch.cuda.stream(stream):
        g.replay()
    ms = timed_replay(g, stream, 1)
    out = {"workload": sh["workload"], "layer_us": round(ms / steps * 1e3, 3),
           "value": round(layer_bytes * steps / (ms * 1e-3) / 1e9, 2), "unit": "GB/s"}
    del g, descs, keep
    torch.cuda.empty_cache()
    return out


def profile_traffic():
    """dram bytes (read + write) per launch of the layer kernel from the
    committed ncu summary (profiles/k_moe_layer_config1.md, line
    'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(ROOT, "profiles", "k_moe_layer_config1.md")
    try:
        with open(p) as f:
            for line in f:
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":")[1].strip().replace(",", ""))
    except OSError:
        pass
    return None


def sampler_leg(ctx, stream, reps=50):
    """Config 0: one sampler row (T 0.7, top-k 20, top-p 0.8, repetition
    penalty 1.1 over 64 history ids) on fp32[151,936] logits ~ N(0, 2^2)
    resident on the device; graph replays, device time per row."""
    import numpy as np
    import torch
    import smoe_cuda as S
    V = 151_936
    ctx.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(5)
    logits = torch.from_numpy((rng.standard_normal(V) * 2).astype(np.float32)).cuda()
    hist = torch.from_numpy(rng.integers(0, V, 64).astype(np.int32)).cuda()
    row = np.zeros(6, np.float32)
    row[0:2] = (0.7, 0.8)
    row.view(np.uint32)[2] = 20
    row[3:5] = (1.1, 0.37)
    row.view(np.uint32)[5] = 64
    drow = torch.from_numpy(row.view(np.int32)).cuda()
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ctx.sample(logits, V, 1, drow, hist, 64, tok)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            ctx.sample(logits, V, 1, drow, hist, 64, tok)
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps * 1e3
    return {"workload": "config0: sampler, batch 1, vocab 151,936 (T 0.7, top-k 20, top-p 0.8, rep 1.1)",
            "us_per_row": round(us, 2), "logit_bytes_per_row": V * 4,
            "achieved_gbs": round(V * 4 / (us * 1e-6) / 1e9, 1)}


def batch_leg(ctx, stream, B=256, reps=10):
    """Config 4 shape: one 30B MoE layer for 256 tokens (router + expert-
    grouped FFN + combine, vault layout, AFFINE-Q4, bf16 x ~ N(0, 1)), and
    256 sampler rows (T in {0.6, 0.7, 1.0}, top-k in {20, 40}, top-p in
    {0.8, 0.95}, rep 1.1, 128-token histories) - device time per call."""
    import numpy as np
    import torch
    import oracle as O
    import smoe_cuda as S
    arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, E, D, DFF, 4242)
    rw = O.normal_bf16(4242, 6, E * D, 0.0, 0.02)
    da, dr = torch.from_numpy(arena).cuda(), torch.from_numpy(rw.view(np.int16)).cuda()
    L = S.make_layer(da, stride, off, E, D, DFF, S.FMT_AFFINE_Q4, dr)
    x = torch.from_numpy(np.stack([O.normal_bf16(77 + i, 5, D) for i in range(B)]).view(np.int16)).cuda()
    y = torch.zeros(B, D, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(B, K, dtype=torch.int32, device="cuda")
    w = torch.zeros(B, K, dtype=torch.float32, device="cuda")
    V = 151_936
    rng = np.random.default_rng(9)
    logits = torch.from_numpy((rng.standard_normal(B * V) * 2).astype(np.float32)).cuda()
    hist = torch.from_numpy(rng.integers(0, V, B * 128).astype(np.int32)).cuda()
    rows = np.zeros((B, 6), np.float32)
    rows[:, 0] = np.array([0.6, 0.7, 1.0])[np.arange(B) % 3]
    rows[:, 1] = np.array([0.8, 0.95])[np.arange(B) % 2]
    rows.view(np.uint32)[:, 2] = np.array([20, 40])[(np.arange(B) // 2) % 2]
    rows[:, 3] = 1.1
    rows[:, 4] = (rng.integers(0, 1 << 24, B) / (1 << 24)).astype(np.float32)
    rows.view(np.uint32)[:, 5] = 128
    drows = torch.from_numpy(rows.view(np.int32)).cuda()
    toks = torch.zeros(B, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(stream.cuda_stream)        # the events below are recorded on this stream

    def timed(fn):
        with torch.cuda.stream(stream):
            fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps * 1e3
    layer_us = timed(lambda: ctx.moe_layer(L, x, S.DTYPE_BF16, B, K, True, y, S.DTYPE_BF16, ids, w))
    touched = int((np.bincount(ids.cpu().numpy().reshape(-1), minlength=E) > 0).sum())
    samp_us = timed(lambda: ctx.sample(logits, V, B, drows, hist, 128, toks))
    layer_bytes = 524_288 + touched * 2_654_208 + 2 * B * D * 2
    return {"workload": "config4 shape: one 30B MoE layer for 256 tokens + 256 sampler rows",
            "layer_us": round(layer_us, 1), "tokens_per_s_per_layer": round(B / (layer_us * 1e-6)),
            "experts_touched": touched, "layer_bytes": layer_bytes,
            "achieved_gbs": round(layer_bytes / (layer_us * 1e-6) / 1e9, 1),
            "sampler_us_256_rows": round(samp_us, 1)}


def decode_leg(ctx, prompt=45, gen=256):
    """Config 2 shape: Qwen3-30B-A3B decode (48 layers, random weights with
    the benchmark distributions), batch 1, one CUDA graph per token
    (s-moe_b200/decode.py); tokens per second over the generated tokens."""
    import numpy as np
    import torch
    import smoe_cuda as S
    import decode as DEC
    sh = DEC.Shape()
    model = DEC.Model(ctx, sh)
    rng = np.random.default_rng(11)
    dec = DEC.Decoder(model, uniforms=rng.integers(0, 1 << 24, 4096).astype(np.float64) / (1 << 24))
    dec.capture(torch.cuda.Stream())
    pr = rng.integers(0, sh.vocab, prompt).tolist()
    dec.run(pr, 8)
    dec.reset()
    _, t = dec.run(pr, gen)
    ctx.synchronize()
    attn = (2 * sh.q_dim + 2 * sh.kv_dim) * sh.d_model * 2
    per_tok = (sh.layers * (sh.top_k * S.expert_bytes(sh.fmt, sh.d_model, sh.d_ff) + attn
                            + sh.n_experts * sh.d_model * 2) + sh.vocab * sh.d_model * 2)
    out = {"workload": f"config2 shape: Qwen3-30B-A3B decode, 48 layers, batch 1, prompt {prompt}, "
                       f"{gen} generated (random weights)", "tok_per_s": round(gen / t, 2),
           "ms_per_token": round(1e3 * t / gen, 4), "weight_bytes_per_token": per_tok,
           "achieved_gbs": round(per_tok * gen / t / 1e9, 1)}
    out["prefill"] = prefill_timing(dec, pr)
    del dec, model
    torch.cuda.empty_cache()
    return out


def batched_decode_leg(ctx, shape, batch, prompt, gen):
    """Config 4 (30B shape, 256 sequences) or config 3 at batch 32 (235B
    shape, one GPU): every sequence its own random prompt, KV ring (256
    positions), sampler row (config-4 parameters) and history; one CUDA
    graph per step (s-moe_b200/decode.py BatchDecoder); tokens per second
    summed over the sequences, over the generated steps."""
    import decode as DEC
    sh = DEC.Shape.qwen3_235b() if shape == "235b" else DEC.Shape()
    sh.attn_ctx = 256
    out = DEC.run_batched(ctx, sh, batch, prompt, gen)
    name = "Qwen3-235B-A22B" if shape == "235b" else "Qwen3-30B-A3B"
    out["workload"] = (f"{name}-shaped decode, {sh.layers} layers, batch {batch}, prompt {prompt}, {gen} "
                       "generated per sequence (random weights, vault-layout experts, expert-grouped MoE path)")
    return out


def prefill_timing(dec, prompt, gen=8):
    """Time to first token with the layer-major prefill (the prompt's first
    P - 1 tokens in one chunk, MoE by the layer kernel 4 tokens per launch,
    captured as one graph), then the step on the last prompt token; against
    feeding the prompt one token per step-graph replay."""
    dec.run_prefill(prompt, gen)                         # capture + warm
    _, ttft, _ = dec.run_prefill(prompt, gen)
    dec.reset()
    import torch
    with torch.cuda.stream(dec.stream):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(dec.stream)
        for tok in prompt:
            dec.token.fill_(int(tok))
            dec.graph.replay()
        e1.record(dec.stream)
        torch.cuda.synchronize()
    serial = e0.elapsed_time(e1) / 1e3
    dec.reset()
    return {"prompt_tokens": len(prompt), "ttft_ms": round(ttft * 1e3, 3),
            "ttft_token_by_token_ms": round(serial * 1e3, 3),
            "prefill_tok_per_s": round(len(prompt) / ttft, 1)}


def decode_235b_leg(ctx, prompt=45, gen=64):
    """Config 3 at batch 1 on one GPU: the Qwen3-235B-A22B shape (94 layers,
    ~128 GB of tiled Q4 experts resident), one CUDA graph per token."""
    import numpy as np
    import torch
    import decode as DEC
    sh = DEC.Shape.qwen3_235b()
    t0 = time.time()
    model = DEC.Model(ctx, sh)
    load = time.time() - t0
    rng = np.random.default_rng(11)
    dec = DEC.Decoder(model, uniforms=rng.integers(0, 1 << 24, 4096).astype(np.float64) / (1 << 24))
    dec.capture(torch.cuda.Stream())
    pr = rng.integers(0, sh.vocab, prompt).tolist()
    dec.run(pr, 4)
    dec.reset()
    _, t = dec.run(pr, gen)
    ctx.synchronize()
    ptb = DEC.per_token_bytes(sh)
    pf = prefill_timing(dec, pr)
    out = {"workload": f"config3 shape: Qwen3-235B-A22B decode, 94 layers, batch 1, 1 GPU, prompt {prompt}, "
                       f"{gen} generated (random weights)", "tok_per_s": round(gen / t, 2),
           "ms_per_token": round(1e3 * t / gen, 4), "weight_bytes_per_token": ptb,
           "achieved_gbs": round(ptb * gen / t / 1e9, 1), "load_s": round(load, 1), "prefill": pf}
    del dec, model
    torch.cuda.empty_cache()
    return out


def run_leg(name):
    import torch
    import smoe_cuda as S
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    torch.cuda.set_device(0)
    ctx = S.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    out = {"sampler": lambda: sampler_leg(ctx, stream), "decode_30b": lambda: decode_leg(ctx),
           "batch256": lambda: batch_leg(ctx, stream),
           "decode_b256": lambda: batched_decode_leg(ctx, "30b", 256, 45, 128),
           "decode_235b": lambda: decode_235b_leg(ctx),
           "decode_235b_b32": lambda: batched_decode_leg(ctx, "235b", 32, 45, 32)}[name]()
    print(json.dumps({name: out}), flush=True)
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the sampler and decode legs")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--only", choices=["sampler", "decode_30b", "batch256", "decode_b256", "decode_235b",
                                         "decode_235b_b32"],
                    help="run one side leg alone on GPU 0 and print its JSON (profiling)")
    args = ap.parse_args()
    if args.only:
        run_leg(args.only)
        return
    rank, world, local = dist_init(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
