"""Phase timeline of the sampler kernel (profiling aid; not used by the
library or the tests). One config-0 row (vocab 151,936, logits N(0, 2^2), T
0.7, top-k 20, top-p 0.8, rep 1.1, a 64-token history), with the kernel's
%globaltimer marks switched on through smoe_cuda_debug_trace (a profiling
entry outside the public header). Prints, per phase, the time after the
kernel's first mark (median over rows of several launches):

    python s-moe_b200/trace_sampler.py [--rows 8] [--reps 5]

Marks: load (slice into shared memory), exp (e values), seq: totals,
prefix, summaries, walk (the exact sequential sum), select (4-pass radix
select), collect (candidates into CTA 0), sort, done.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import smoe_cuda as S  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=8)
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    V, B = 151_936, args.rows
    ctx = S.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    lib = S.lib()
    lib.smoe_cuda_debug_trace.argtypes = [C.c_void_p, C.c_void_p]
    rng = np.random.default_rng(5)
    rows = np.zeros((B, 6), np.float32)
    rows[:, 0], rows[:, 1], rows[:, 3] = 0.7, 0.8, 1.1
    rows.view(np.uint32)[:, 2] = 20
    rows[:, 4] = (rng.integers(0, 1 << 24, B) / (1 << 24)).astype(np.float32)
    rows.view(np.uint32)[:, 5] = 64
    drows = torch.from_numpy(rows.view(np.int32)).cuda()
    hist = torch.from_numpy(rng.integers(0, V, B * 64).astype(np.int32)).cuda()
    toks = torch.zeros(B, dtype=torch.int32, device="cuda")
    trace = torch.zeros(128, dtype=torch.int64, device="cuda")
    names = ["load", "exp", "seq:totals", "seq:prefix", "seq:summaries", "seq:walk", "select", "collect",
             "sort", "done"]
    samples = {n: [] for n in names}
    for rep in range(args.reps + 1):
        logits = torch.from_numpy((rng.standard_normal(B * V) * 2).astype(np.float32)).cuda()
        torch.cuda.synchronize()
        trace.zero_()
        lib.smoe_cuda_debug_trace(ctx.h, trace.data_ptr())
        with torch.cuda.stream(stream):
            ctx.sample(logits, V, B, drows, hist, 64, toks)     # row 0 is traced
        ctx.synchronize()
        lib.smoe_cuda_debug_trace(ctx.h, None)
        if rep == 0:
            continue                                            # first launch: attribute set-up
        t = trace.cpu().numpy().astype(np.int64)
        samp, seq = t[:64].reshape(8, 8), t[64:128].reshape(8, 8)
        t0 = samp[0, 0]
        marks = [samp[0, 1], samp[0, 2], seq[0, 0], seq[0, 1], seq[0, 2], seq[0, 3], samp[0, 4], samp[0, 5],
                 samp[0, 6], samp[0, 7]]
        for n, m in zip(names, marks):
            samples[n].append((m - t0) / 1e3 if m else float("nan"))
    print(json.dumps({n: round(float(np.median(v)), 2) for n, v in samples.items()}))
    ctx.close()


if __name__ == "__main__":
    main()
