"""Benchmark: one Qwen3-30B-A3B-shaped MoE layer decode step.

A step = router GEMV + softmax/top-8/renorm + fused 4-bit (AFFINE-Q4) SwiGLU
FFN of the 8 routed experts + weighted combine, batch 1, x bf16[2048] ->
y bf16[2048], all through the C ABI (libsmoe_cuda.so).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`value`: algorithmic HBM bytes of the layer step (router 524,288 + x 4,096 +
8 experts x 2,654,208 + y 4,096 = 21,762,144 B) / device time, inputs
resident. L2 is defeated by cycling through 8 distinct resident layers
(8 x 340 MB) with a fresh x per step: each step's experts were last touched
7 steps (>= 150 MB of other traffic) earlier. `e2e`: the same step with x
copied from pinned host memory and y read back to the host inside the timed
region. N > 1 (torchrun, one rank per GPU): the same layer step expert-
parallel - rank r holds experts [r*128/N, (r+1)*128/N) of every layer, x and
y live on rank 0, and the exchange runs inside the layer kernel over NVLink
(smoe_cuda_moe_layer_ep); strong scaling, timed as the max over ranks.
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

D, DFF, E, K = 2048, 768, 128, 8
N_LAYERS = 8
LAYER_BYTES = 524_288 + 4_096 + 8 * 2_654_208 + 4_096      # 21,762,144
FFN_BYTES = 8 * 2_654_208                                    # 21,233,664
# dram__bytes_read.sum + dram__bytes_write.sum of one k_moe_fused launch on
# this workload, measured once with ncu (--set full, one launch)
NCU_TRAFFIC = 21_848_320
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


# ------------------------------------------------------------------ data
def make_inputs(seed=1234):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    layers = []
    for l in range(N_LAYERS):
        arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, E, D, DFF, seed=seed + l)
        rw = O.normal_bf16(seed + l, 6, E * D, 0.0, 0.02)
        layers.append((arena, stride, off, rw))
    xs = np.stack([O.normal_bf16(seed + 7919 + i, 5, D) for i in range(64)])
    return layers, xs


# ------------------------------------------------------------ CPU legs
def cpu_layer_time(layers, xs, budget_s, threads):
    """Reference router (compiled sampler/top-k/matvec of the reference) +
    the oracle's restated Q4 FFN (there is no reference CPU FFN) + combine."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    used = O.set_threads(threads)
    R = O.ref()
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
    no CPU FFN), all host threads. One step = one MoE layer step."""
    if rank != 0:
        return
    layers, xs = make_inputs()
    threads = os.cpu_count() or 1
    for i in range(args.warmup):
        cpu_layer_time(layers, xs, 0.0, threads)
    n_total, el_total, used, kind = 0, 0.0, threads, "port"
    for i in range(args.steps):
        n, el, used, kind = cpu_layer_time(layers, xs, 0.0, threads)   # exactly one layer step
        n_total += n
        el_total += el
    gbs = LAYER_BYTES * n_total / el_total / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * el_total / n_total, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config1: Qwen3-30B-A3B MoE layer (d 2048, 128 experts, top-8, "
                                   "AFFINE-Q4 g64), batch 1", "layers_cycled": N_LAYERS},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": used, "kind": kind,
                             "sample": f"{n_total} layer steps in {el_total:.2f} s: reference "
                                       "router (compiled from the reference) + restated Q4 FFN, "
                                       "OpenMP"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU arm
def run_ours(args, rank, world, local):
    import numpy as np
    import torch
    import smoe_cuda as S

    torch.cuda.set_device(local)
    layers, xs = make_inputs()
    ctx = S.Context(local)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    ep = world > 1
    base, per = S.ep_partition(E, world, rank) if ep else (0, E)
    descs, keep = [], []
    for arena, stride, off, rw in layers:
        da = torch.from_numpy(np.ascontiguousarray(arena[base:base + per])).cuda()
        dr = torch.from_numpy(rw.view(np.int16)).cuda()
        keep += [da, dr]
        vault = S.make_layer(da, stride, off, per, D, DFF, S.FMT_AFFINE_Q4, dr)
        # one-time load-time re-layout into the tiled device format (the
        # vault-layout copy is dropped afterwards)
        tstride = S.tiled_stride(S.FMT_AFFINE_Q4, D, DFF)
        tb = torch.empty(per * tstride, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()             # the arena was copied on torch's stream
        descs.append(ctx.prepack_layer(vault, tb, tstride))
        ctx.synchronize()
        keep[-2] = tb
    if ep:
        import torch.distributed as dist
        grp = dist.new_group(backend="gloo")
        handles = [None] * world
        dist.all_gather_object(handles, ctx.ep_export(), group=grp)
        ctx.ep_attach(rank, world, handles)
        barrier(world)
    d_x = torch.from_numpy(xs.view(np.int16)).cuda()          # [64, D] bf16
    d_y = torch.zeros(D, dtype=torch.bfloat16, device="cuda")
    ids = torch.zeros(N_LAYERS, K, dtype=torch.int32, device="cuda")
    wts = torch.zeros(N_LAYERS, K, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def layer(l):      # router + top-k + expert FFN + combine: one fused launch
        if ep:
            ctx.moe_layer_ep(descs[l], E, base, d_x[l].data_ptr() if rank == 0 else None,
                             S.DTYPE_BF16, 1, K, True, d_y if rank == 0 else None, S.DTYPE_BF16,
                             ids[l], wts[l])
        else:
            ctx.moe_layer(descs[l], d_x[l].data_ptr(), S.DTYPE_BF16, 1, K, True, d_y, S.DTYPE_BF16,
                          ids[l], wts[l])

    def ffn(l):        # the same with the routing already on the device
        ctx.moe_ffn(descs[l], d_x[l].data_ptr(), S.DTYPE_BF16, ids[l], wts[l], K, 1, d_y,
                    S.DTYPE_BF16)

    # eager warm-up (also sets kernel attributes before capture)
    for i in range(max(args.warmup, 3)):
        for l in range(N_LAYERS):
            layer(l)
            if not ep:
                ffn(l)
    ctx.synchronize()
    # One graph = one MoE layer step on each of the 8 resident layers.
    g_step, g_ffn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step, stream=stream):
        for l in range(N_LAYERS):
            layer(l)
    with torch.cuda.graph(g_ffn, stream=stream):
        for l in range(N_LAYERS):
            if ep:
                layer(l)           # routing-given mode is single-GPU: time the layer again
            else:
                ffn(l)
    reps = max(1, args.steps // N_LAYERS)
    steps = reps * N_LAYERS
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            g_step.replay()
            g_ffn.replay()
    torch.cuda.synchronize()
    barrier(world)

    def timed(graph):
        barrier(world)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):      # replay() launches on the current stream
            t0.record(stream)
            for _ in range(reps):
                graph.replay()
            t1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        return t0.elapsed_time(t1)

    # ---- device-resident timing (CUDA graph replays)
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.3)
    d0 = ctx.dispatches()
    ms = timed(g_step)
    ffn_ms_total = timed(g_ffn)
    ck = clocks.stop()
    launches = steps * 1           # one fused MoE-layer kernel per step (graph replays)
    ctx.synchronize()
    ms = max_over_ranks(ms, world)
    per_step = ms / steps
    ffn_ms = ffn_ms_total / steps
    # replicas would be weak scaling; expert parallel splits one layer step
    value = LAYER_BYTES * steps / (ms * 1e-3) / 1e9
    args.steps = steps
    del d0

    # ---- end to end through the C ABI with host buffers: every step copies
    # its x from pinned host memory, runs the layer call and copies y back.
    # Single GPU: the calls of the 8 steps are captured once as a CUDA graph
    # (as a serving loop would drive them) and replayed, so the host's Python
    # launch overhead is not what is timed; expert parallel: issued eagerly.
    hx = torch.from_numpy(xs.view(np.int16)).pin_memory()
    hy = torch.zeros(N_LAYERS, D, dtype=torch.bfloat16).pin_memory()
    stage_x = torch.zeros(D, dtype=torch.bfloat16, device="cuda")

    def e2e_step(i):
        L = descs[i % N_LAYERS]
        if not ep:
            # the step's x read from pinned host memory and its y written back
            # into pinned host memory by the library itself (staging kernel in,
            # direct row stores out; the bytes below cross the host link)
            ctx.moe_layer(L, hx[(2000 + i) % 64].data_ptr(), S.DTYPE_BF16, 1, K, True,
                          hy[i % N_LAYERS].data_ptr(), S.DTYPE_BF16)
        elif rank == 0:
            stage_x.view(torch.int16).copy_(hx[(2000 + i) % 64], non_blocking=True)
            ctx.moe_layer_ep(L, E, base, stage_x, S.DTYPE_BF16, 1, K, True, d_y, S.DTYPE_BF16)
            hy[i % N_LAYERS].copy_(d_y, non_blocking=True)
        else:
            ctx.moe_layer_ep(L, E, base, None, S.DTYPE_BF16, 1, K, True, None, S.DTYPE_BF16)

    if not ep:
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e, stream=stream):
            for i in range(N_LAYERS):
                e2e_step(i)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g_e2e.replay()
        torch.cuda.synchronize()
        e2e_ms = timed(g_e2e)
        e2e_steps = reps * N_LAYERS
    else:
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                e2e_step(i)
        e1.record(stream)
        torch.cuda.synchronize()
        ctx.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        e2e_steps = args.steps
    e2e_ms = max_over_ranks(e2e_ms, world)
    e2e = LAYER_BYTES * e2e_steps / (e2e_ms * 1e-3) / 1e9

    if rank == 0:
        peak, peak_kind = peaks()
        # per GPU: the fused kernel's share of the expert bytes / its time
        ach = FFN_BYTES / world / (ffn_ms * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step, 5),
            "higher_is_better": True, "scaling": "strong" if ep else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded; BASELINE config-1 distributions)",
            "config": {"workload": "config1: Qwen3-30B-A3B MoE layer (d 2048, 128 experts, "
                                   "top-8, d_ff 768, AFFINE-Q4 g64), batch 1, bf16 in/out",
                       "layers_cycled": N_LAYERS, "l2": "inputs larger than L2 (8 resident "
                       "layers x 340 MB cycled, fresh x per step)",
                       "parallelism": (f"expert parallel x{world} ({per} experts per GPU, exchange "
                                       "in-kernel over NVLink)") if ep else "single GPU"},
            "layer_us": round(per_step * 1e3, 3),
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "traffic": None if ep else NCU_TRAFFIC,
                         "kernel": (f"k_moe_fused expert parallel (layer incl. routing and NVLink "
                                    f"exchange), {FFN_BYTES // world:,} B of experts per GPU per launch, "
                                    f"{ffn_ms * 1e3:.2f} us avg") if ep else
                                   ("k_moe_fused (expert FFN + combine, routing given), 21,233,664 B "
                                    f"per launch, {ffn_ms * 1e3:.2f} us avg"), "peak_kind": peak_kind},
            "e2e": {"value": round(e2e, 2), "unit": "GB/s", "h2d_bytes_per_step": D * 2,
                    "d2h_bytes_per_step": D * 2},
            "gpu_launches": int(launches),
            "clocks": ck,
        }
        if world == 1 and not args.no_cpu:
            n, el, used, kind = cpu_layer_time(layers, xs, args.cpu_seconds, os.cpu_count() or 1)
            line["cpu_baseline"] = {
                "value": round(LAYER_BYTES * n / el / 1e9, 4), "unit": "GB/s", "cores": used,
                "kind": kind, "sample": f"{n} layer steps in {el:.1f} s (reference router + "
                                        "restated Q4 FFN, OpenMP)"}
        if world == 1 and not args.no_extra:
            line["sampler"] = sampler_leg(ctx, stream)
            line["decode_30b"] = decode_leg(ctx)
            line["batch256"] = batch_leg(ctx, stream)
        print(json.dumps(line), flush=True)
    ctx.close()


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
           "batch256": lambda: batch_leg(ctx, stream)}[name]()
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
    ap.add_argument("--only", choices=["sampler", "decode_30b", "batch256"],
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
