"""GPU parity of batched decode (sequences at one shared position, each with
its own KV ring): the batched matvec, the batched attention layer, the
expert-grouped MoE layer at the Qwen3-235B-A22B shape for 32 tokens, and
whole teacher-forced steps of a small Qwen3-MoE-shaped model for several
sequences, each sequence's logits against the CPU restatement
(oracle/decode_ref.py) run for that sequence alone. Bars as the batch-1
decode tests: single kernels 5e-5 of max|ref| (the batched matvec carries
the activations as two bf16 planes, ~2^-17 relative), logits 1e-3, the MoE
layer 1e-4 (the other FFN tests' bar; BASELINE bar 1e-2)."""
import math

import numpy as np
import pytest
import torch

import oracle as O
import smoe_cuda as S
from decode_ref import RefDecoder, bf16, make_weights
from gpu_util import Layer, dev, rel_err

pytestmark = pytest.mark.gpu
KERNEL_TOL = 5e-5
LOGIT_TOL = 1e-3


def small_shape(ctx_len=64, heads="30b"):
    from decode import Shape
    if heads == "235b":                  # 64 query heads over 4 KV heads, d_model 4096
        return Shape.qwen3_235b(layers=1, n_experts=16, top_k=4, vocab=512, attn_ctx=ctx_len)
    return Shape(layers=2, n_experts=16, top_k=4, vocab=512, attn_ctx=ctx_len)


@pytest.mark.parametrize("batch,rows,cols", [(7, 300, 2048), (32, 1024, 4096), (256, 520, 2048), (2, 64, 8192)])
def test_gemm_bf16_batch(ctx, batch, rows, cols):
    rng = np.random.default_rng(batch + rows)
    W = (rng.standard_normal(rows * cols).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    X = rng.standard_normal((batch, cols)).astype(np.float32)
    y = torch.zeros(batch, rows, device="cuda")
    dW, dX = dev(W), dev(X)
    torch.cuda.synchronize()
    ctx.gemm_bf16(dW, dX, y, rows, cols, batch)
    ctx.synchronize()
    ref = X.astype(np.float64) @ bf16(W).reshape(rows, cols).T
    got = y.cpu().numpy()
    for b in range(batch):
        assert rel_err(got[b], ref[b]) < KERNEL_TOL


@pytest.mark.parametrize("ctx_len,pos,heads", [(64, 5, "30b"), (64, 100, "30b"), (256, 200, "30b"), (4096, 300, "30b"),
                                               (4096, 2500, "30b"), (64, 100, "235b"), (4096, 1500, "235b")])
def test_attention_batch(ctx, ctx_len, pos, heads):
    """Three sequences with different pre-filled rings at one position (with
    and without the ring wrapping), 8 and 16 query heads per KV head (the
    kernel reads each KV head's ring once for its group), windows of one and
    of several 1024-position score blocks: each sequence against the
    restatement alone."""
    B = 3
    sh = small_shape(ctx_len, heads)
    W = make_weights(sh, 5)
    ref = RefDecoder(W, sh)
    rng = np.random.default_rng(pos)
    rings = [rng.standard_normal(ref.kv[0].shape) for _ in range(B)]
    normed = rng.standard_normal((B, sh.d_model))
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    t = {n: dev(W[n][0]) for n in ("w_q", "w_k", "w_v", "w_o", "q_norm", "k_norm")}
    kv = f(np.stack([r for r in rings], axis=1))            # [2, B, ctx, kv_dim]
    kc, vc = kv[0].contiguous(), kv[1].contiguous()
    bufs = {n: torch.zeros(B, c, device="cuda") for n, c in (("q", sh.q_dim), ("k", sh.kv_dim), ("v", sh.kv_dim),
                                                              ("a", sh.q_dim), ("o", sh.d_model))}
    ang = (np.float32(pos) * ref.inv_freq).astype(np.float32).astype(np.float64)
    cs_d, sn_d, x_d = f(np.cos(ang)), f(np.sin(ang)), f(normed)
    dpos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    a = S.AttnLayerArgs()
    a.w_q, a.w_k, a.w_v, a.w_o = (t[n].data_ptr() for n in ("w_q", "w_k", "w_v", "w_o"))
    a.q_norm_w, a.k_norm_w = t["q_norm"].data_ptr(), t["k_norm"].data_ptr()
    a.rope_cos, a.rope_sin, a.normed_in = cs_d.data_ptr(), sn_d.data_ptr(), x_d.data_ptr()
    a.qbuf, a.kbuf, a.vbuf = bufs["q"].data_ptr(), bufs["k"].data_ptr(), bufs["v"].data_ptr()
    a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
    a.attn_out, a.o_out = bufs["a"].data_ptr(), bufs["o"].data_ptr()
    a.d_model, a.q_dim, a.kv_dim, a.head_dim = sh.d_model, sh.q_dim, sh.kv_dim, sh.head_dim
    a.num_heads, a.num_kv_heads, a.attn_ctx = sh.num_heads, sh.num_kv_heads, sh.attn_ctx
    a.attn_scale = 1.0 / math.sqrt(sh.head_dim)
    ctx.attention_batch(a, B, sh.attn_ctx * sh.kv_dim, dpos)
    ctx.synchronize()
    slot = pos % sh.attn_ctx
    for b in range(B):
        ref.kv[0] = rings[b].copy()
        o_ref, q_ref, k_ref = ref.attention(0, normed[b], pos)
        assert rel_err(bufs["o"][b].cpu().numpy(), o_ref) < KERNEL_TOL
        assert rel_err(bufs["q"][b].cpu().numpy(), q_ref.reshape(-1)) < KERNEL_TOL
        assert rel_err(kc[b, slot].cpu().numpy(), k_ref.reshape(-1)) < KERNEL_TOL
        assert rel_err(vc[b, slot].cpu().numpy(), ref.kv[0, 1, slot]) < KERNEL_TOL


@pytest.mark.parametrize("fmt", [O.FMT_AFFINE_Q4, O.FMT_SMOE_Q4])
def test_moe_layer_235b_shape_batch32(ctx, fmt):
    """BASELINE config 3 at batch 32: the Qwen3-235B-A22B expert shape (d
    4096, d_ff 1536) through the expert-grouped path (vault layout), routing
    on the device, every token against the oracle."""
    B, E, d, dff, k = 32, 16, 4096, 1536, 8
    L = Layer(fmt, E, d, dff, seed=171 + fmt)
    X = O.normal_bf16(172 + fmt, 5, B * d)
    y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
    ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
    w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
    ctx.moe_layer(L.desc, dev(X), S.DTYPE_BF16, B, k, True, y, S.DTYPE_F32, ids, w)
    ctx.synchronize()
    got = y.cpu().numpy()
    gid = ids.cpu().numpy().view(np.uint32)
    for t in range(B):
        x = O.bf16_to_f32(X[t * d:(t + 1) * d])
        ref, rids, _ = O.moe_layer(fmt, x, L.router_w, L.arena, L.stride, E, d, dff, k)
        assert (gid[t] == rids).all()
        assert rel_err(got[t], ref) < 1e-4


def test_batch_decode_teacher_forced(ctx):
    """Five sequences (more than the layer kernel's 4, so the MoE layer runs
    the expert-grouped path) stepped together with teacher forcing: every
    sequence's logits at every step against the restatement of that sequence
    alone; greedy rows, so each sampled token is its logits' argmax; the
    position and every row's history advance."""
    from decode import BatchDecoder, Model
    B = 5
    sh = small_shape()
    W = make_weights(sh, 9)
    model = Model(ctx, sh, weights=W, layout="vault")
    rows = np.zeros((B, 6), np.float32)
    rows[:, 0], rows[:, 1], rows[:, 3] = 0.0, 1.0, 1.0
    rows.view(np.uint32)[:, 2] = 1
    dec = BatchDecoder(model, B, rows=rows)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    ref = RefDecoder(W, sh)
    rings = [np.zeros_like(ref.kv) for _ in range(B)]
    rng = np.random.default_rng(12)
    steps = rng.integers(0, sh.vocab, (6, B))
    for pos in range(steps.shape[0]):
        dec.tokens.copy_(torch.from_numpy(steps[pos].astype(np.int32)))
        dec._step()
        torch.cuda.synchronize()
        ctx.synchronize()
        got = dec.logits.cpu().numpy()
        toks = dec.tokens.cpu().numpy()
        for b in range(B):
            ref.kv = rings[b]
            r = ref.step(int(steps[pos, b]), pos)
            e = rel_err(got[b], r)
            assert e < LOGIT_TOL, f"pos {pos} seq {b}: rel err {e:.2e}"
            assert int(toks[b]) == int(np.argmax(got[b]))
        assert int(dec.pos.item()) == pos + 1
    hist = dec.history.cpu().numpy()
    assert (dec.rows.cpu().numpy().view(np.uint32)[:, 5] == steps.shape[0]).all()
    assert (hist[:, steps.shape[0] - 1] == toks).all()


@pytest.mark.parametrize("heads,ctx_len,pos0,n", [("30b", 64, 0, 7), ("30b", 4096, 1500, 5), ("235b", 4096, 1200, 6)])
def test_attention_prefill_chunk(ctx, heads, ctx_len, pos0, n):
    """smoe_cuda_attention_prefill_async: n tokens of one sequence at
    positions pos0.. (prefill.cpp:131-268) against the restatement stepping
    them one at a time: outputs, normed + roped Q, and the ring rows the
    chunk appended."""
    sh = small_shape(ctx_len, heads)
    W = make_weights(sh, 6)
    ref = RefDecoder(W, sh)
    rng = np.random.default_rng(pos0 + n)
    ring0 = rng.standard_normal(ref.kv[0].shape)
    ref.kv[0] = ring0.copy()
    normed = rng.standard_normal((n, sh.d_model))
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    t = {k: dev(W[k][0]) for k in ("w_q", "w_k", "w_v", "w_o", "q_norm", "k_norm")}
    kc, vc = f(ring0[0]), f(ring0[1])
    bufs = {k: torch.zeros(n, c, device="cuda") for k, c in (("q", sh.q_dim), ("k", sh.kv_dim), ("v", sh.kv_dim),
                                                              ("a", sh.q_dim), ("o", sh.d_model))}
    ang = np.stack([(np.float32(pos0 + i) * ref.inv_freq).astype(np.float32) for i in range(n)]).astype(np.float64)
    cs_d, sn_d, x_d = f(np.cos(ang)), f(np.sin(ang)), f(normed)
    dpos = torch.tensor([pos0], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    a = S.AttnLayerArgs()
    a.w_q, a.w_k, a.w_v, a.w_o = (t[k].data_ptr() for k in ("w_q", "w_k", "w_v", "w_o"))
    a.q_norm_w, a.k_norm_w = t["q_norm"].data_ptr(), t["k_norm"].data_ptr()
    a.rope_cos, a.rope_sin, a.normed_in = cs_d.data_ptr(), sn_d.data_ptr(), x_d.data_ptr()
    a.qbuf, a.kbuf, a.vbuf = bufs["q"].data_ptr(), bufs["k"].data_ptr(), bufs["v"].data_ptr()
    a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
    a.attn_out, a.o_out = bufs["a"].data_ptr(), bufs["o"].data_ptr()
    a.d_model, a.q_dim, a.kv_dim, a.head_dim = sh.d_model, sh.q_dim, sh.kv_dim, sh.head_dim
    a.num_heads, a.num_kv_heads, a.attn_ctx = sh.num_heads, sh.num_kv_heads, sh.attn_ctx
    a.attn_scale = 1.0 / math.sqrt(sh.head_dim)
    ctx.attention_prefill(a, n, dpos)
    ctx.synchronize()
    for i in range(n):
        o_ref, q_ref, k_ref = ref.attention(0, normed[i], pos0 + i)
        slot = (pos0 + i) % sh.attn_ctx
        assert rel_err(bufs["o"][i].cpu().numpy(), o_ref) < KERNEL_TOL
        assert rel_err(bufs["q"][i].cpu().numpy(), q_ref.reshape(-1)) < KERNEL_TOL
        assert rel_err(kc[slot].cpu().numpy(), k_ref.reshape(-1)) < KERNEL_TOL
        assert rel_err(vc[slot].cpu().numpy(), ref.kv[0, 1, slot]) < KERNEL_TOL


@pytest.mark.parametrize("G,fmt", [(2, O.FMT_AFFINE_Q4), (4, O.FMT_SMOE_Q4)])
def test_moe_layer_shards_sum_to_layer(ctx, G, fmt):
    """smoe_cuda_moe_layer_shard on one GPU, once per shard of a 235B-shaped
    layer (16 experts split over G shards), batch 32: the shards' partial
    sums add up to the layer (what the ranks' NCCL reduce computes), routing
    identical in every shard; against the oracle."""
    B, E, d, dff, k = 32, 16, 4096, 1536, 8
    arena, stride, off = O.make_experts(fmt, E, d, dff, 181)
    router = O.normal_bf16(181, 6, E * d, 0.0, 0.02)
    drouter = dev(router)
    X = O.normal_bf16(182, 5, B * d)
    dx = dev(X)
    total = np.zeros((B, d), np.float64)
    per = E // G
    ids0 = None
    for g in range(G):
        da = dev(np.ascontiguousarray(arena[g * per:(g + 1) * per]))
        shard = S.make_layer(da, stride, off, per, d, dff, fmt, drouter)
        y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        ctx.moe_layer_shard(shard, E, g * per, dx, S.DTYPE_BF16, B, k, True, y, ids)
        ctx.synchronize()
        total += y.cpu().numpy()
        gid = ids.cpu().numpy()
        if ids0 is None:
            ids0 = gid
        assert np.array_equal(gid, ids0)
    for t in range(0, B, 3):
        x = O.bf16_to_f32(X[t * d:(t + 1) * d])
        ref, rids, _ = O.moe_layer(fmt, x, router, arena, stride, E, d, dff, k)
        assert (ids0[t].view(np.uint32) == rids).all()
        assert rel_err(total[t], ref) < 1e-4
