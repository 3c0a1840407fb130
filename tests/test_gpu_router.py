"""GPU parity: router gate + softmax + top-k + renorm vs the reference
(scout.cpp:77-123 + decode.cpp:280-303 compiled / restated). Expert ids must
match bit-exactly; weights within fp32 rounding."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import smoe_cuda as S
from gpu_util import dev

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def run_router(ctx, W, x, E, d, k, norm=True, x_dtype=S.DTYPE_F32, batch=1):
    ids = torch.zeros(batch * k, dtype=torch.int32, device="cuda")
    w = torch.zeros(batch * k, dtype=torch.float32, device="cuda")
    lg = torch.zeros(batch * E, dtype=torch.float32, device="cuda")
    ctx.router_topk(dev(W), dev(x), x_dtype, E, d, batch, k, norm, ids, w, lg)
    ctx.synchronize()
    return (ids.cpu().numpy().view(np.uint32).reshape(batch, k), w.cpu().numpy().reshape(batch, k),
            lg.cpu().numpy().reshape(batch, E))


def test_router_golden(ctx):
    r = np.load(os.path.join(GOLD, "router.npz"))
    for s in range(len(r["seed"])):
        W = O.normal_bf16(s, 6, 128 * 2048, 0.0, 0.02)
        ids, w, lg = run_router(ctx, W, r["x"][s], 128, 2048, 8)
        assert (ids[0] == r["ids"][s]).all(), s
        np.testing.assert_allclose(w[0], r["weights"][s], rtol=2e-5, atol=1e-8)
        np.testing.assert_allclose(lg[0], r["logits"][s], rtol=1e-4, atol=1e-5)


def test_router_many_seeds_bf16_input_batched(ctx):
    E, d, k, B = 128, 2048, 8, 32
    mism = 0
    for rep in range(4):
        xb = np.concatenate([O.normal_bf16(1000 + rep * B + t, 5, d) for t in range(B)])
        W = O.normal_bf16(500 + rep, 6, E * d, 0.0, 0.02)
        ids, w, _ = run_router(ctx, W, xb, E, d, k, x_dtype=S.DTYPE_BF16, batch=B)
        for t in range(B):
            rids, rw, lg = O.route(O.bf16_to_f32(xb[t * d:(t + 1) * d]), W, E, d, k)
            srt = np.sort(lg)[::-1]
            near_tie = (srt[k - 1] - srt[k]) < 1e-5
            if not (ids[t] == rids).all():
                assert near_tie, (rep, t)
                mism += 1
            else:
                np.testing.assert_allclose(w[t], rw, rtol=2e-5, atol=1e-8)
    assert mism == 0


def test_router_shapes_and_no_norm(ctx):
    for (E, d, k) in [(64, 512, 4), (128, 4096, 8), (256, 1024, 16)]:
        W = O.normal_bf16(E, 6, E * d, 0.0, 0.02)
        x = O.normal_f32(E, 5, d)
        for norm in (True, False):
            ids, w, _ = run_router(ctx, W, x, E, d, k, norm=norm)
            rids, rw, _ = O.route(x, W, E, d, k, norm=norm)
            assert (ids[0] == rids).all()
            np.testing.assert_allclose(w[0], rw, rtol=2e-5, atol=1e-8)


def test_router_ties_lowest_index(ctx):
    E, d, k = 64, 256, 8
    W = np.zeros(E * d, np.uint16)          # all logits 0: every prob ties
    x = O.normal_f32(3, 5, d)
    ids, w, _ = run_router(ctx, W, x, E, d, k)
    assert (ids[0] == np.arange(k)).all()
    np.testing.assert_allclose(w[0], np.full(k, 1.0 / k), rtol=1e-6)
