"""GPU: the allocation-free expert FFN entry point.

smoe_cuda_moe_ffn_noalloc exists for callers that cannot call cudaMalloc
(engines that reserve all device memory in their own pool, code running in
callbacks where allocation is forbidden). It must give the same result as the
context-based smoe_cuda_moe_ffn and as the CPU oracle, call after call, even
though every call reuses the same fixed scratch array inside the library, and
its companion smoe_cuda_noalloc_check must report a device error raised by a
call. This file is named so that pytest collects it last; it also runs alone
in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
import smoe_cuda as S
from gpu_util import Layer, dev, rel_err

pytestmark = pytest.mark.gpu
TIGHT = 1e-4     # same bound the other FFN parity tests use


def noalloc(layer, x, x_dtype, ids, w, k, batch, y, y_dtype):
    L = S.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.smoe_cuda_moe_ffn_noalloc(ctypes.byref(layer), S.ptr(x), x_dtype, S.ptr(ids), S.ptr(w),
                                     k, batch, S.ptr(y), y_dtype, stream)
    return rc, L.smoe_cuda_noalloc_last_error().decode()


def check():
    L = S.lib()
    rc = L.smoe_cuda_noalloc_check(torch.cuda.current_stream().cuda_stream, 10000)
    return rc, L.smoe_cuda_noalloc_last_error().decode()


def oracle_y(L, fmt, X, ids, w, d, dff):
    out = []
    for t in range(X.shape[0]):
        ref = np.zeros(d, np.float32)
        for j in range(ids.shape[1]):
            ref = ref + w[t, j] * O.expert_ffn(fmt, L.arena[ids[t, j]], d, dff, X[t])
        out.append(ref)
    return out


@pytest.mark.parametrize("fmt", [O.FMT_AFFINE_Q4, O.FMT_SMOE_Q4])
def test_noalloc_matches_context_entry_two_calls(fmt):
    ctx = S.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    d, dff, E, k = 2048, 768, 32, 8
    L = Layer(fmt, E, d, dff, seed=91 + fmt)
    for call in range(2):   # the second call reuses the scratch the first one left behind
        B = 1 + call
        Xb = O.normal_bf16(91 + call, 5, B * d)
        ids = np.stack([np.random.default_rng(10 * call + t).permutation(E)[:k]
                        for t in range(B)]).astype(np.uint32)
        w = np.random.default_rng(call).random((B, k)).astype(np.float32)
        dx, di, dw = dev(Xb), dev(ids), dev(w)
        y_ref = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        y_na = torch.full((B, d), float("nan"), dtype=torch.float32, device="cuda")
        ctx.moe_ffn(L.desc, dx, S.DTYPE_BF16, di, dw, k, B, y_ref, S.DTYPE_F32)
        rc, msg = noalloc(L.desc, dx, S.DTYPE_BF16, di, dw, k, B, y_na, S.DTYPE_F32)
        assert rc == S.SMOE_OK, msg
        rc, msg = check()
        assert rc == S.SMOE_OK, msg
        torch.cuda.synchronize()
        ref, got = y_ref.cpu().numpy(), y_na.cpu().numpy()
        assert np.isfinite(got).all()
        orc = oracle_y(L, fmt, O.bf16_to_f32(Xb).reshape(B, d), ids, w, d, dff)
        for t in range(B):
            assert rel_err(got[t], ref[t]) < TIGHT
            assert rel_err(got[t], orc[t]) < TIGHT
    ctx.close()


def test_noalloc_at_the_scratch_limit():
    """batch * k * d_ff == 65536 exactly (the largest call the array serves)."""
    d, dff, E, k, B = 256, 1024, 16, 16, 4
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=93)
    X = O.normal_f32(93, 9, B * d).reshape(B, d)
    ids = np.stack([np.random.default_rng(93 + t).permutation(E)[:k] for t in range(B)]).astype(np.uint32)
    w = np.random.default_rng(94).random((B, k)).astype(np.float32)
    y = torch.full((B, d), float("nan"), dtype=torch.float32, device="cuda")
    rc, msg = noalloc(L.desc, dev(X), S.DTYPE_F32, dev(ids), dev(w), k, B, y, S.DTYPE_F32)
    assert rc == S.SMOE_OK, msg
    rc, msg = check()
    assert rc == S.SMOE_OK, msg
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = oracle_y(L, O.FMT_AFFINE_Q4, X, ids, w, d, dff)
    for t in range(B):
        assert rel_err(got[t], ref[t]) < TIGHT


def test_noalloc_reports_device_error_then_recovers():
    """An expert id past the layer raises the library's error word; the
    companion check reports it once (SMOE_ERR_DEVICE) and clears it."""
    d, dff, E, k = 512, 256, 4, 2
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=95)
    x = dev(O.normal_f32(95, 9, d))
    w = dev(np.array([0.5, 0.5], np.float32))
    y = torch.zeros(d, dtype=torch.float32, device="cuda")
    rc, msg = noalloc(L.desc, x, S.DTYPE_F32, dev(np.array([1, E], np.uint32)), w, k, 1, y, S.DTYPE_F32)
    assert rc == S.SMOE_OK, msg
    rc, msg = check()
    assert rc == S.SMOE_ERR_DEVICE, msg
    rc, msg = noalloc(L.desc, x, S.DTYPE_F32, dev(np.array([1, 0], np.uint32)), w, k, 1, y, S.DTYPE_F32)
    assert rc == S.SMOE_OK, msg
    rc, msg = check()
    assert rc == S.SMOE_OK, msg


def test_noalloc_rejects_oversize():
    d, dff, E = 256, 4096, 16
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=92)
    k, B = 16, 2                     # 2 * 16 * 4096 = 131072 > 65536
    x = torch.zeros(B, d, device="cuda")
    ids = torch.zeros(B * k, dtype=torch.int32, device="cuda")
    w = torch.zeros(B * k, device="cuda")
    y = torch.zeros(B, d, device="cuda")
    rc, msg = noalloc(L.desc, x, S.DTYPE_F32, ids, w, k, B, y, S.DTYPE_F32)
    assert rc == 1 and "65536" in msg
