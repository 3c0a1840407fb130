"""CPU: the C restatement against the reference's own compiled code and the
committed golden fixtures (which come from the reference's quantiser,
sampler.hpp and scout.cpp)."""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")
V = 151936


def test_generators_pinned():
    g = np.load(os.path.join(GOLD, "sampler.npz"))
    for seed, ref_sum in zip(g["seed"][:4], g["logit_sum"][:4]):
        s = O.normal_f32(int(seed), 1, V, 0.0, 2.0)
        assert s.astype(np.float64).sum() == ref_sum
    r = np.load(os.path.join(GOLD, "router.npz"))
    W = O.normal_bf16(0, 6, 128 * 2048, 0.0, 0.02)
    assert O.bf16_to_f32(W).astype(np.float64).sum() == r["w_sum"][0]


def test_sampler_golden():
    g = np.load(os.path.join(GOLD, "sampler.npz"))
    for i, seed in enumerate(g["seed"]):
        T, p, k, rep = (float(v) for v in g["params"][i])
        hl = int(g["hist_len"][i])
        s = O.normal_f32(int(seed), 1, V, 0.0, 2.0)
        u = O.canonical_from_word(int(g["word"][i]))
        tok = O.sample_token(s, T, p, int(k), rep, g["hist"][i][:hl], u)
        assert tok == int(g["token"][i]), (i, seed)


@pytest.mark.skipif(not O.ref_available(), reason="reference not compiled here")
def test_sampler_vs_reference_many():
    for seed in range(1000, 1060):
        s = O.normal_f32(seed, 1, V, 0.0, 2.0)
        h = O.random_ids(seed, 2, 64, V)
        w = int(O.random_ids(seed, 3, 1, 1 << 24)[0]) << 8
        a = O.sample_token(s.copy(), 0.7, 0.8, 20, 1.1, h, O.canonical_from_word(w))
        b = O.ref_sample_token(s.copy(), 0.7, 0.8, 20, 1.1, h, w)
        assert a == b


@pytest.mark.skipif(not O.ref_available(), reason="reference not compiled here")
def test_canonical_and_state_injection():
    R = O.ref()
    for w in [0, 1, 255, 256, 0x80000000, 0xFFFFFF00, 0xFFFFFFFF, 0xDEADBEEF]:
        assert R.ref_mt_next_after_inject(w) == w
        assert np.float32(R.ref_canonical_from_word(w)) == np.float32(O.canonical_from_word(w))


def test_router_golden():
    r = np.load(os.path.join(GOLD, "router.npz"))
    for s in range(len(r["seed"])):
        W = O.normal_bf16(s, 6, 128 * 2048, 0.0, 0.02)
        ids, w, lg = O.route(r["x"][s], W, 128, 2048, 8)
        assert (ids == r["ids"][s]).all()
        assert (w == r["weights"][s]).all()
        assert (lg == r["logits"][s]).all()


def test_q4_format_golden():
    """The restated SMOE-Q4 dequant equals shatter_moe.py's on its own blob."""
    g = np.load(os.path.join(GOLD, "q4_expert.npz"))
    d, dff = int(g["d"]), int(g["dff"])
    blob = g["blob"]
    off, tot = O.blob_layout(O.FMT_SMOE_Q4, d, dff)
    assert tot == blob.size
    for m, (po, ps, so, ss) in enumerate(g["offsets"]):
        assert off[3 * m] == po and off[3 * m + 1] == so
    np.testing.assert_array_equal(O.dequant(O.FMT_SMOE_Q4, blob, d, dff, 0), g["gate"])
    np.testing.assert_array_equal(O.dequant(O.FMT_SMOE_Q4, blob, d, dff, 1), g["up"])
    np.testing.assert_array_equal(O.dequant(O.FMT_SMOE_Q4, blob, d, dff, 2), g["down"])
    for x, y in zip(g["x"], g["y"]):
        y64 = O.expert_ffn(O.FMT_SMOE_Q4, blob, d, dff, x, precise=True)
        y32 = O.expert_ffn(O.FMT_SMOE_Q4, blob, d, dff, x, precise=False)
        scale = np.abs(y).max()
        assert np.abs(y64 - y).max() / scale < 1e-6
        assert np.abs(y32 - y).max() / scale < 1e-4


def test_affine_ffn_matches_dense():
    d, dff = 256, 256
    arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, 2, d, dff, seed=7)
    x = O.normal_f32(7, 9, d)
    blob = arena[1]
    G, U, D = (O.dequant(O.FMT_AFFINE_Q4, blob, d, dff, m).astype(np.float64) for m in range(3))
    g, u = G @ x, U @ x
    y = D @ (g / (1 + np.exp(-g)) * u)
    y64 = O.expert_ffn(O.FMT_AFFINE_Q4, blob, d, dff, x)
    assert np.abs(y64 - y).max() / np.abs(y).max() < 1e-6


def test_moe_layer_combine_order():
    d, dff, E, k = 256, 256, 16, 4
    arena, stride, off = O.make_experts(O.FMT_AFFINE_Q4, E, d, dff, seed=3)
    W = O.normal_bf16(3, 6, E * d, 0.0, 0.02)
    x = O.bf16_to_f32(O.normal_bf16(3, 5, d))
    out, ids, w = O.moe_layer(O.FMT_AFFINE_Q4, x, W, arena, stride, E, d, dff, k)
    ref = np.zeros(d, np.float32)
    for j in range(k):
        ye = O.expert_ffn(O.FMT_AFFINE_Q4, arena[ids[j]], d, dff, x)
        ref = ref + np.float32(w[j]) * ye
    np.testing.assert_allclose(out, ref, rtol=0, atol=0)


def test_expf_restatement_equals_host_libm_everywhere():
    """The sampler's e = expf(x) (sampler.hpp:116): the restated glibc
    algorithm equals this host's libm expf on every float in [-104, 88]
    (2.2e9 inputs; below -103.97 both give +0). The CUDA sampler performs the
    same IEEE operations, so its e values are the reference's."""
    neg_lo, neg_hi = 0x80000000, 0xC2D00000          # -0 .. -104
    pos_lo, pos_hi = 0x00000000, 0x42B00000          # +0 .. 88
    assert O.expf_mismatches(neg_lo, neg_hi) == 0
    assert O.expf_mismatches(pos_lo, pos_hi) == 0
