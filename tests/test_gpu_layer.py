"""GPU: the MoE layer at the benchmark shapes, expert-id bounds, and the
bounded waits (a device wait that runs out, a host wait that runs out).

Parity is against the CPU oracle (fp64 restatement of the reference's Q4
FFN, its compiled router); tolerance as the other FFN tests: 1e-4 of
max|ref| (BASELINE bar 1e-2)."""
import numpy as np
import pytest
import torch

import oracle as O
import smoe_cuda as S
from gpu_util import Layer, dev, rel_err, tiled

pytestmark = pytest.mark.gpu
TIGHT = 1e-4


@pytest.mark.parametrize("fmt,B", [(O.FMT_AFFINE_Q4, 1), (O.FMT_SMOE_Q4, 2)])
def test_layer_235b_shape_tiled(ctx, fmt, B):
    """Qwen3-235B-A22B expert shape (d 4096, d_ff 1536) through the single-
    launch layer kernel (A units in two chunks), routing on the device."""
    d, dff, E, k = 4096, 1536, 16, 8
    L = Layer(fmt, E, d, dff, seed=141 + fmt)
    desc, buf = tiled(ctx, L)
    for call in range(2):
        X = O.normal_bf16(150 + call + 10 * B, 5, B * d)
        y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
        w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
        ctx.moe_layer(desc, dev(X), S.DTYPE_BF16, B, k, True, y, S.DTYPE_F32, ids, w)
        ctx.synchronize()
        got = y.cpu().numpy()
        gid = ids.cpu().numpy().view(np.uint32)
        for t in range(B):
            x = O.bf16_to_f32(X[t * d:(t + 1) * d])
            ref, rids, rw = O.moe_layer(fmt, x, L.router_w, L.arena, L.stride, E, d, dff, k)
            assert (gid[t] == rids).all()
            assert rel_err(got[t], ref) < TIGHT


def test_layer_repeatable_bitwise(ctx):
    """Every output row has one owner and fixed-order sums: repeated calls
    give identical bits."""
    d, dff, E, k = 2048, 768, 32, 8
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=171)
    desc, buf = tiled(ctx, L)
    xb = dev(O.normal_bf16(171, 5, d))
    outs = []
    for _ in range(3):
        y = torch.zeros(d, dtype=torch.float32, device="cuda")
        ctx.moe_layer(desc, xb, S.DTYPE_BF16, 1, k, True, y, S.DTYPE_F32)
        ctx.synchronize()
        outs.append(y.cpu().numpy())
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


@pytest.mark.parametrize("fmt", [O.FMT_AFFINE_Q4, O.FMT_SMOE_Q4])
def test_config4_shape_grouped(ctx, fmt):
    """BASELINE config 4's layer shape itself: 256 tokens, 128 experts, d 2048,
    d_ff 768, top-8 (each expert ~16 tokens), bf16 x. Ids of every token
    exact; y of every 4th token against the oracle."""
    d, dff, E, k, B = 2048, 768, 128, 8, 256
    L = Layer(fmt, E, d, dff, seed=4242 + fmt)
    Xb = np.concatenate([O.normal_bf16(77 + i, 5, d) for i in range(B)])
    y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
    ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
    w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
    ctx.moe_layer(L.desc, dev(Xb), S.DTYPE_BF16, B, k, True, y, S.DTYPE_F32, ids, w)
    ctx.synchronize()
    got = y.cpu().numpy()
    gid = ids.cpu().numpy().view(np.uint32)
    counts = np.bincount(gid.reshape(-1), minlength=E)
    assert counts.max() <= 64 and counts.sum() == B * k
    for t in range(B):
        x = O.bf16_to_f32(Xb[t * d:(t + 1) * d])
        rids, rw, _ = O.route(x, L.router_w, E, d, k)
        assert (gid[t] == rids).all(), t
        if t % 4 == 0:
            ref, _, _ = O.moe_layer(fmt, x, L.router_w, L.arena, L.stride, E, d, dff, k)
            assert rel_err(got[t], ref) < TIGHT, t


@pytest.mark.parametrize("layout", ["vault", "tiled"])
def test_expert_id_out_of_range_is_reported(ctx, layout):
    """An expert id >= n_experts must not index past the arena: the call
    raises the device error word (SMOE_ERR_DEVICE at synchronize) and the
    next call with good ids works."""
    d, dff, E, k = 1024, 512, 8, 4
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=181)
    desc = L.desc
    if layout == "tiled":
        desc, buf = tiled(ctx, L)
    x = O.normal_f32(181, 9, d)
    w = np.full(k, 0.25, np.float32)
    bad = np.array([1, E, 3, 2], np.uint32)
    y = torch.zeros(d, dtype=torch.float32, device="cuda")
    ctx.moe_ffn(desc, dev(x), S.DTYPE_F32, dev(bad), dev(w), k, 1, y, S.DTYPE_F32)
    with pytest.raises(S.SmoeCudaError) as ei:
        ctx.synchronize()
    assert "device error" in str(ei.value)
    good = np.array([1, 0, 3, 2], np.uint32)
    ctx.moe_ffn(desc, dev(x), S.DTYPE_F32, dev(good), dev(w), k, 1, y, S.DTYPE_F32)
    ctx.synchronize()
    ref = np.zeros(d, np.float32)
    for j in range(k):
        ref = ref + w[j] * O.expert_ffn(O.FMT_AFFINE_Q4, L.arena[good[j]], d, dff, x)
    assert rel_err(y.cpu().numpy(), ref) < TIGHT


def test_device_wait_runs_out_and_context_recovers():
    """A rank > 0 of an expert-parallel layer waits for rank 0's x flag. Here
    nothing ever sets it (this process attaches as rank 1 of 2 to its own
    window, and no rank 0 runs): the bounded wait (2 ms) must run out, the
    call report SMOE_ERR_DEVICE, and a following single-GPU layer call on the
    same context work and match the oracle. No GPU fault is involved."""
    ctx = S.Context(0, device_wait_us=2000)
    s = torch.cuda.Stream()
    ctx.set_stream(s.cuda_stream)
    with torch.cuda.stream(s):
        d, dff, E, k = 1024, 512, 16, 4
        L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=191)
        desc, buf = tiled(ctx, L)
        h = ctx.ep_export()
        ctx.ep_attach(1, 2, [h, h])
        shard = S.make_layer(desc.base + (E // 2) * desc.expert_stride, desc.expert_stride,
                             list(desc.off), E // 2, d, dff, desc.fmt, L.d_router)
        ctx.moe_layer_ep(shard, E, E // 2, None, S.DTYPE_BF16, 1, k, True, None, S.DTYPE_BF16)
        with pytest.raises(S.SmoeCudaError) as ei:
            ctx.synchronize()
        assert "device error" in str(ei.value)
        xb = O.normal_bf16(191, 5, d)
        y = torch.zeros(d, dtype=torch.float32, device="cuda")
        ctx.moe_layer(desc, dev(xb), S.DTYPE_BF16, 1, k, True, y, S.DTYPE_F32)
        ctx.synchronize()
        ref, _, _ = O.moe_layer(O.FMT_AFFINE_Q4, O.bf16_to_f32(xb), L.router_w, L.arena, L.stride, E, d, dff, k)
        assert rel_err(y.cpu().numpy(), ref) < TIGHT
    ctx.close()


def test_host_wait_runs_out():
    """smoe_cuda_synchronize is bounded by timeout_ms: a stream kept busy for
    ~0.5 s (torch's bounded sleep kernel) makes it return SMOE_ERR_TIMEOUT;
    once the stream drains the next synchronize succeeds."""
    ctx = S.Context(0, timeout_ms=50)
    s = torch.cuda.Stream()
    ctx.set_stream(s.cuda_stream)
    with torch.cuda.stream(s):
        torch.cuda._sleep(int(1.0e9))          # ~0.5 s at 1.9 GHz, then it returns
        with pytest.raises(S.SmoeCudaError) as ei:
            ctx.synchronize()
        assert "timed out" in str(ei.value)
    s.synchronize()
    ctx.synchronize()
    ctx.close()


def test_layer_with_pinned_host_x_and_y(ctx):
    """x and y in pinned host memory (the reference engine's buffers): the
    library stages x with a copy kernel and stores y's rows into host memory;
    the result equals the device-buffer call bit for bit. Pageable host
    memory is refused."""
    d, dff, E, k = 2048, 768, 32, 8
    L = Layer(O.FMT_AFFINE_Q4, E, d, dff, seed=211)
    desc, buf = tiled(ctx, L)
    xb = O.normal_bf16(211, 5, d)
    y_dev = torch.zeros(d, dtype=torch.bfloat16, device="cuda")
    ctx.moe_layer(desc, dev(xb), S.DTYPE_BF16, 1, k, True, y_dev, S.DTYPE_BF16)
    hx = torch.from_numpy(xb.view(np.int16)).pin_memory()
    hy = torch.zeros(d, dtype=torch.bfloat16).pin_memory()
    ctx.moe_layer(desc, hx.data_ptr(), S.DTYPE_BF16, 1, k, True, hy.data_ptr(), S.DTYPE_BF16)
    ctx.synchronize()
    assert torch.equal(hy.view(torch.int16), y_dev.cpu().view(torch.int16))
    ref, _, _ = O.moe_layer(O.FMT_AFFINE_Q4, O.bf16_to_f32(xb), L.router_w, L.arena, L.stride, E, d, dff, k)
    got = hy.view(torch.int16).numpy().view(np.uint16).astype(np.uint32).__lshift__(16).view(np.float32)
    assert rel_err(got, ref) < 1e-2
    pageable = np.zeros(d, np.uint16)
    with pytest.raises(S.SmoeCudaError):
        ctx.moe_layer(desc, pageable.ctypes.data, S.DTYPE_BF16, 1, k, True, hy.data_ptr(), S.DTYPE_BF16)
