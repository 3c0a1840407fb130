"""GPU parity: fused 4-bit SwiGLU expert FFN + combine vs the CPU oracle.

Tolerance (BASELINE): max_i |y_i - r_i| / max_j |r_j| <= 1e-2 against the
fp64 oracle; the kernels are expected far below (fp32 accumulate)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import smoe_cuda as S
from gpu_util import Layer, bf16_dev_to_f32, dev, rel_err, tiled

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-2          # BASELINE bar
TIGHT = 1e-4        # what the fp32-accumulate kernels actually reach


def test_group_mirror_on_reference_quantised_blob(ctx):
    """smoe_cuda_fused_ffn_group on a blob made by shatter_moe.py (SMOE-Q4)."""
    g = np.load(os.path.join(GOLD, "q4_expert.npz"))
    d, dff = int(g["d"]), int(g["dff"])
    blob = dev(g["blob"])
    base = blob.data_ptr()
    o = g["offsets"]
    b = S.ExpertBlob(base + int(o[0][0]), base + int(o[0][2]), base + int(o[1][0]),
                     base + int(o[1][2]), base + int(o[2][0]), base + int(o[2][2]), 3)
    for x, y in zip(g["x"], g["y"]):
        h = ctx.fused_ffn_group([b], x.astype(np.float32), dff, d)   # host input
        out = np.zeros(d, np.float32)
        ctx.wait(h, out, 3, d)
        assert rel_err(out, y) < TIGHT


def test_single_and_two_experts_mirror(ctx):
    d, dff = 512, 256
    L = Layer(O.FMT_SMOE_Q4, 4, d, dff, seed=11, router=False)
    x = O.normal_f32(11, 9, d)
    base = L.d_arena.data_ptr()
    blobs = []
    for j, e in enumerate([2, 0]):
        p = base + e * L.stride
        f = L.off
        blobs.append(S.ExpertBlob(p + f[0], p + f[1], p + f[3], p + f[4], p + f[6], p + f[7], j))
    h = ctx.fused_ffn_group(blobs, dev(x), dff, d)            # device input
    for j, e in enumerate([2, 0]):
        out = np.zeros(d, np.float32)
        ctx.wait(h, out, j, d)
        ref = O.expert_ffn(O.FMT_SMOE_Q4, L.arena[e], d, dff, x)
        assert rel_err(out, ref) < TIGHT
    p = base + 1 * L.stride
    f = L.off
    h = ctx.fused_ffn(p + f[0], p + f[1], p + f[3], p + f[4], p + f[6], p + f[7], x, dff, d, 5)
    out = np.zeros(d, np.float32)
    ctx.wait(h, out, 5, d)
    assert rel_err(out, O.expert_ffn(O.FMT_SMOE_Q4, L.arena[1], d, dff, x)) < TIGHT


def test_token_batch_mirror(ctx):
    d, dff, B = 256, 512, 5
    L = Layer(O.FMT_SMOE_Q4, 2, d, dff, seed=12, router=False)
    X = O.normal_f32(12, 9, B * d).reshape(B, d)
    p = L.d_arena.data_ptr() + L.stride
    f = L.off
    h = ctx.fused_ffn_batch(p + f[0], p + f[1], p + f[3], p + f[4], p + f[6], p + f[7], X, B, dff, d)
    out = np.zeros((B, d), np.float32)
    ctx.wait_ffn_batch(h, out, B, d)
    for t in range(B):
        assert rel_err(out[t], O.expert_ffn(O.FMT_SMOE_Q4, L.arena[1], d, dff, X[t])) < TIGHT


@pytest.mark.parametrize("layout", ["vault", "tiled"])
@pytest.mark.parametrize("fmt", [O.FMT_AFFINE_Q4, O.FMT_SMOE_Q4])
def test_moe_layer_config1(ctx, fmt, layout):
    """Config 1: Qwen3-30B-A3B MoE layer, x bf16[2048], 128 experts, top-8.
    vault layout -> two-kernel path; tiled layout -> single persistent launch."""
    d, dff, E, k = 2048, 768, 128, 8
    L = Layer(fmt, E, d, dff, seed=21 + fmt)
    if layout == "tiled":
        L.desc, L._tiled_buf = tiled(ctx, L)
    for s in range(3):
        xb = O.normal_bf16(100 + s, 5, d)
        x = O.bf16_to_f32(xb)
        y = torch.zeros(d, dtype=torch.bfloat16, device="cuda")
        ids = torch.zeros(k, dtype=torch.int32, device="cuda")
        w = torch.zeros(k, dtype=torch.float32, device="cuda")
        ctx.moe_layer(L.desc, dev(xb), S.DTYPE_BF16, 1, k, True, y, S.DTYPE_BF16, ids, w)
        ctx.synchronize()
        ref, rids, rw = O.moe_layer(fmt, x, L.router_w, L.arena, L.stride, E, d, dff, k)
        assert (ids.cpu().numpy().view(np.uint32) == rids).all()
        np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=1e-5, atol=1e-7)
        got = bf16_dev_to_f32(y)
        assert rel_err(got, ref) < TOL
        # fp32 output: the accumulation quality itself
        y32 = torch.zeros(d, dtype=torch.float32, device="cuda")
        ctx.moe_layer(L.desc, dev(xb), S.DTYPE_BF16, 1, k, True, y32, S.DTYPE_F32)
        ctx.synchronize()
        assert rel_err(y32.cpu().numpy(), ref) < TIGHT


def test_moe_ffn_batch_tokens_fp32_in(ctx):
    d, dff, E, k, B = 1024, 512, 32, 8, 6
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=31)
    X = O.normal_f32(31, 9, B * d).reshape(B, d)
    ids = np.stack([O.random_ids(31 + t, 3, 64, E)[:k] for t in range(B)]).astype(np.uint32)
    for t in range(B):   # distinct experts per token
        ids[t] = np.random.default_rng(t).permutation(E)[:k]
    w = np.random.default_rng(5).random((B, k)).astype(np.float32)
    y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
    ctx.moe_ffn(L.desc, dev(X), S.DTYPE_F32, dev(ids), dev(w), k, B, y, S.DTYPE_F32)
    ctx.synchronize()
    got = y.cpu().numpy()
    for t in range(B):
        ref = np.zeros(d, np.float32)
        for j in range(k):
            ref = ref + w[t, j] * O.expert_ffn(O.FMT_AFFINE_Q4, L.arena[ids[t, j]], d, dff, X[t])
        assert rel_err(got[t], ref) < TIGHT


def test_shape_235b_expert(ctx):
    """Qwen3-235B-A22B expert shape (d 4096, d_ff 1536)."""
    d, dff, E, k = 4096, 1536, 8, 8
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=41)
    x = O.normal_f32(41, 9, d)
    ids = np.arange(k, dtype=np.uint32)[::-1].copy()
    w = np.full(k, 1.0 / k, np.float32)
    y = torch.zeros(d, dtype=torch.float32, device="cuda")
    ctx.moe_ffn(L.desc, dev(x), S.DTYPE_F32, dev(ids), dev(w), k, 1, y, S.DTYPE_F32)
    ctx.synchronize()
    ref = np.zeros(d, np.float32)
    for j in range(k):
        ref = ref + w[j] * O.expert_ffn(O.FMT_AFFINE_Q4, L.arena[ids[j]], d, dff, x)
    assert rel_err(y.cpu().numpy(), ref) < TIGHT


def test_bad_arguments_rejected(ctx):
    L = Layer(O.FMT_AFFINE_Q4, 2, 256, 256, seed=1)
    x = torch.zeros(256, device="cuda")
    y = torch.zeros(256, device="cuda")
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    w = torch.ones(1, device="cuda")
    with pytest.raises(S.SmoeCudaError):
        ctx.moe_ffn(L.desc, x, S.DTYPE_F32, ids, w, 0, 1, y, S.DTYPE_F32)     # k = 0
    bad = S.make_layer(L.d_arena, L.stride, L.off, 2, 250, 256, O.FMT_AFFINE_Q4, L.d_router)
    with pytest.raises(S.SmoeCudaError):
        ctx.moe_ffn(bad, x, S.DTYPE_F32, ids, w, 1, 1, y, S.DTYPE_F32)        # d % 64
    ctx.synchronize()


@pytest.mark.parametrize("B,k,fmt", [(2, 8, O.FMT_AFFINE_Q4), (4, 16, O.FMT_SMOE_Q4), (3, 6, O.FMT_AFFINE_Q4)])
def test_moe_layer_fused_small_batch(ctx, B, k, fmt):
    """The persistent single-launch path (batch <= 4), called twice in a row so
    the in-kernel counters must have been reset by the previous launch."""
    d, dff, E = 1024, 512, 64
    L = Layer(fmt, E, d, dff, seed=60 + B)
    L.desc, L._tiled_buf = tiled(ctx, L)
    for call in range(2):
        X = O.normal_bf16(70 + 10 * B + call, 5, B * d)
        y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
        w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
        ctx.moe_layer(L.desc, dev(X), S.DTYPE_BF16, B, k, True, y, S.DTYPE_F32, ids, w)
        ctx.synchronize()
        got = y.cpu().numpy()
        gid = ids.cpu().numpy().view(np.uint32)
        for t in range(B):
            x = O.bf16_to_f32(X[t * d:(t + 1) * d])
            ref, rids, rw = O.moe_layer(fmt, x, L.router_w, L.arena, L.stride, E, d, dff, k)
            assert (gid[t] == rids).all()
            assert rel_err(got[t], ref) < TIGHT


def test_tiled_moe_ffn_given_routing(ctx):
    """moe_ffn on the tiled layout (routing supplied), two fp32 tokens."""
    d, dff, E, k, B = 2048, 1024, 16, 8, 2
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=33)
    desc, buf = tiled(ctx, L)
    X = O.normal_f32(33, 9, B * d).reshape(B, d)
    ids = np.stack([np.random.default_rng(t).permutation(E)[:k] for t in range(B)]).astype(np.uint32)
    w = np.random.default_rng(9).random((B, k)).astype(np.float32)
    y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
    ctx.moe_ffn(desc, dev(X), S.DTYPE_F32, dev(ids), dev(w), k, B, y, S.DTYPE_F32)
    ctx.synchronize()
    got = y.cpu().numpy()
    for t in range(B):
        ref = np.zeros(d, np.float32)
        for j in range(k):
            ref = ref + w[t, j] * O.expert_ffn(O.FMT_AFFINE_Q4, L.arena[ids[t, j]], d, dff, X[t])
        assert rel_err(got[t], ref) < TIGHT


@pytest.mark.parametrize("fmt,x_dtype,d,dff", [(O.FMT_AFFINE_Q4, S.DTYPE_BF16, 2048, 768),
                                                (O.FMT_SMOE_Q4, S.DTYPE_F32, 2048, 768),
                                                (O.FMT_AFFINE_Q4, S.DTYPE_BF16, 1024, 512),
                                                (O.FMT_SMOE_Q4, S.DTYPE_BF16, 1536, 256)])
def test_moe_layer_token_batch_grouped(ctx, fmt, x_dtype, d, dff):
    """Token batches (> 4 tokens) on the vault layout run the expert-grouped
    path: router + grouped FFN + rank-order combine vs the oracle per token,
    and the same result on a second call (deterministic order). The 30B
    shape runs the compile-time-K kernels, the others the generic ones."""
    B, E, k = 48, 32, 8
    L = Layer(fmt, E, d, dff, seed=80 + fmt)
    Xb = O.normal_bf16(90 + fmt, 5, B * d)
    Xf = O.bf16_to_f32(Xb).reshape(B, d)
    xin = dev(Xb) if x_dtype == S.DTYPE_BF16 else dev(np.ascontiguousarray(Xf))
    outs = []
    for call in range(2):
        y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
        w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
        ctx.moe_layer(L.desc, xin, x_dtype, B, k, True, y, S.DTYPE_F32, ids, w)
        ctx.synchronize()
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    gid = ids.cpu().numpy().view(np.uint32)
    for t in range(B):
        ref, rids, rw = O.moe_layer(fmt, Xf[t], L.router_w, L.arena, L.stride, E, d, dff, k)
        assert (gid[t] == rids).all()
        assert rel_err(outs[0][t], ref) < TIGHT
