"""Phase timeline of the MoE-layer kernel (k_moe_layer) on BASELINE config 1.

    python s-moe_b200/trace_layer.py [LAYERS] [given,routing] [product]

Runs on the trace build of the library (libsmoe_cuda_trace.so, built by
`build.py --trace`; the marks cost about 1 us of the kernel's time, so the
product library has none). Loads LAYERS (default 8) resident config-1
layers, runs warm back-to-back launches and records, for one launch, per-CTA
%globaltimer and SM-cycle marks of the kernel's phases
(smoe_cuda_debug_trace, a profiling aid outside the public header); prints
min / median / max over CTAs relative to the moment griddepcontrol.wait
returned, and the eager time per launch (of the trace build). With
`product` it runs the same launches on the product library and prints the
time per launch only (the command the committed ncu captures profile).
"""
import os, sys, ctypes as C
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.join(os.path.dirname(HERE), 'oracle')]
import build as B
PRODUCT = 'product' in sys.argv[3:]          # the product library: the same launches, no marks (for ncu)
if not PRODUCT:
    os.environ['SMOE_CUDA_LIB'] = B.LIB_TRACE if os.path.exists(B.LIB_TRACE) else B.build(trace=True)
import numpy as np, torch
import smoe_cuda as S, oracle as O
E, D, DFF, K = 128, 2048, 768, 8
ctx = S.Context(0)
st = torch.cuda.Stream(); ctx.set_stream(st.cuda_stream)
NL = int(sys.argv[1]) if len(sys.argv) > 1 else 8
Ls, keep = [], []
for l in range(NL):
    arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, E, D, DFF, 1234 + l)
    rw = O.normal_bf16(1234 + l, 6, E * D, 0.0, 0.02)
    da = torch.from_numpy(arena).cuda(); dr = torch.from_numpy(rw.view(np.int16)).cuda()
    vault = S.make_layer(da, stride, off, E, D, DFF, S.FMT_AFFINE_Q4, dr)
    ts = S.tiled_stride(S.FMT_AFFINE_Q4, D, DFF)
    tb = torch.empty(E * ts, dtype=torch.uint8, device='cuda')
    torch.cuda.synchronize()
    Ls.append(ctx.prepack_layer(vault, tb, ts)); ctx.synchronize(); keep += [tb, dr]
    del da
x = torch.from_numpy(O.normal_bf16(5, 5, D).view(np.int16)).cuda()
y = torch.zeros(D, dtype=torch.bfloat16, device='cuda')
ids = torch.from_numpy(np.arange(0, 128, 16, dtype=np.int32)).cuda(); w = torch.full((K,), 0.125, device='cuda')
trace = torch.zeros(148 * 128, dtype=torch.int64, device='cuda')
torch.cuda.synchronize()
lib = ctx.L
lib.smoe_cuda_debug_trace.argtypes = [C.c_void_p, C.c_void_p]
names = {0: 'start', 1: 'router rows done', 2: 'routed (prod/h)', 3: 'x table built', 4: 'first A chunk in smem',
         5: 'phase A consumers done', 6: 'grid wait passed', 7: 'phase B done', 8: 'h warp arrived', 9: 'end',
         10: 'griddep wait returned', 11: 'producer starts', 12: 'producer issued all', 13: 'first B wave in smem',
         14: 'last A chunk in smem', 15: 'first B unit reduced', 16: 'h records loaded',
         17: 'last D: h ready', 18: 'routing: row count seen / last D: data', 19: 'routing: logits read / last D: done', 20: 'routing: top-k done / A done, last D starts', 21: 'setup: seq loaded', 22: 'setup: barriers init', 23: 'setup: fence', **{25 + i: f'A chunk {i} in smem' for i in range(3)}, 28: 'prod: ids loaded', 29: 'prod: routing state built', 30: 'cons: xtab starts', 31: 'after first syncthreads'}
modes = sys.argv[2].split(',') if len(sys.argv) > 2 else ['given', 'routing']
for mode in modes:
    def call(l):
        if mode == 'given':
            ctx.moe_ffn(Ls[l], x, S.DTYPE_BF16, ids, w, K, 1, y, S.DTYPE_BF16)
        else:
            ctx.moe_layer(Ls[l], x, S.DTYPE_BF16, 1, K, True, y, S.DTYPE_BF16)
    trace.zero_()
    with torch.cuda.stream(st):
        for i in range(20): call((i * 3) % NL)
        lib.smoe_cuda_debug_trace(ctx.h, trace.data_ptr())
        call(3 % NL)
        lib.smoe_cuda_debug_trace(ctx.h, None)
        for i in range(3): call(i % NL)
        torch.cuda.synchronize(); ctx.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(200): call(i % NL)
        e1.record(st)
        torch.cuda.synchronize()
    print(f'== {mode}: {e0.elapsed_time(e1) / 200 * 1e3:.2f} us per launch (eager)')
    if PRODUCT: continue
    t = trace.cpu().numpy()[:148 * 32].reshape(148, 32).astype(np.int64)
    cy = trace.cpu().numpy()[148 * 32:148 * 64].reshape(148, 32).astype(np.int64)
    tw = t[:, 10][t[:, 10] > 0].min()
    for i in range(32):
        sel = t[:, i] > 0
        col = t[sel, i]
        if len(col) == 0: continue
        r = (col - tw) / 1000.0
        dc = (cy[sel, i] - cy[sel, 10]) / 1965.0          # per-CTA cycles since its own wait return, in us at 1965 MHz
        print(f'mark {i:2d} {names.get(i, ""):26s} n={len(col):3d} min {r.min():6.2f} med {np.median(r):6.2f} max {r.max():6.2f} us | cycles-since-wait med {np.median(dc):6.2f} us')
