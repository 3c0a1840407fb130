"""CPU restatement of one decode step of the reference (TEST INFRASTRUCTURE:
imported only by tests/ as the checker, never by the product).

Follows decode.cpp:103-231 (embedding, input RMSNorm, Q/K/V matvecs, per-head
QK RMSNorm, half-split RoPE, KV ring append, softmax attention over the
`valid` newest positions, O projection, residual), the MoE block (router +
top-k + renorm + experts + combine, the C oracle's moe_layer in fp64) and
main.cpp:621-641 (final RMSNorm, LM head). Arithmetic in float64 except the
RoPE angle, which is float32 as in decode.cpp:116 (float(pos) * inv_freq).
rms_norm_bf16: common.hpp:245-256.
"""
from __future__ import annotations

import numpy as np

import oracle as O


def bf16(a) -> np.ndarray:
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def rms_norm_bf16(x: np.ndarray, w_bf16) -> np.ndarray:
    ss = np.mean(x * x) + 1e-6
    return (x * (1.0 / np.sqrt(ss))) * bf16(w_bf16)


class RefDecoder:
    def __init__(self, W: dict, shape):
        self.W, self.sh = W, shape
        sh = shape
        self.kv = np.zeros((sh.layers, 2, sh.attn_ctx, sh.kv_dim))
        half = sh.head_dim // 2
        self.inv_freq = np.array([1.0 / np.power(np.float64(sh.rope_theta), float(2 * d) / float(sh.head_dim))
                                  for d in range(half)], np.float32)
        self.mats = []
        for l in range(sh.layers):
            self.mats.append({k: bf16(W[k][l]).reshape(r, c) for k, r, c in (
                ("w_q", sh.q_dim, sh.d_model), ("w_k", sh.kv_dim, sh.d_model), ("w_v", sh.kv_dim, sh.d_model),
                ("w_o", sh.d_model, sh.q_dim))})
        self.embed = bf16(W["embed"]).reshape(sh.vocab, sh.d_model)
        self.lm_head = bf16(W["lm_head"]).reshape(sh.vocab, sh.d_model)

    def rope(self, x, pos):
        half = self.sh.head_dim // 2
        ang = (np.float32(pos) * self.inv_freq).astype(np.float32).astype(np.float64)
        cs, sn = np.cos(ang), np.sin(ang)
        a, b = x[:, :half], x[:, half:]
        return np.concatenate([a * cs - b * sn, a * sn + b * cs], axis=1)

    def attention(self, l, normed, pos):
        """decode.cpp:159-231 for layer l: returns o_proj output, updates the ring."""
        sh, W, m = self.sh, self.W, self.mats[l]
        hd = sh.head_dim
        q = (m["w_q"] @ normed).reshape(sh.num_heads, hd)
        k = (m["w_k"] @ normed).reshape(sh.num_kv_heads, hd)
        v = m["w_v"] @ normed
        q = self.rope(np.stack([rms_norm_bf16(x, W["q_norm"][l]) for x in q]), pos)
        k = self.rope(np.stack([rms_norm_bf16(x, W["k_norm"][l]) for x in k]), pos)
        slot, valid = pos % sh.attn_ctx, min(pos + 1, sh.attn_ctx)
        self.kv[l, 0, slot] = k.reshape(-1)
        self.kv[l, 1, slot] = v
        out = np.zeros((sh.num_heads, hd))
        per = sh.num_heads // sh.num_kv_heads
        idx = [(slot - i) % sh.attn_ctx for i in range(valid)]
        for h in range(sh.num_heads):
            kvh = h // per
            K = self.kv[l, 0, idx, kvh * hd:(kvh + 1) * hd]
            V = self.kv[l, 1, idx, kvh * hd:(kvh + 1) * hd]
            s = K @ q[h] / np.sqrt(hd)
            p = np.exp(s - s.max())
            out[h] = (p / p.sum()) @ V
        return m["w_o"] @ out.reshape(-1), q, k

    def step(self, token: int, pos: int) -> np.ndarray:
        sh, W = self.sh, self.W
        hidden = self.embed[token].copy()
        for l in range(sh.layers):
            o, _, _ = self.attention(l, rms_norm_bf16(hidden, W["in_norm"][l]), pos)
            hidden = hidden + o
            normed = rms_norm_bf16(hidden, W["post_norm"][l])
            arena, stride, off = W["experts"][l]
            y, _, _ = O.moe_layer(sh.fmt, normed.astype(np.float32), W["router"][l], arena, stride,
                                  sh.n_experts, sh.d_model, sh.d_ff, sh.top_k, norm=sh.norm_topk)
            hidden = hidden + y.astype(np.float64)
        return self.lm_head @ rms_norm_bf16(hidden, W["model_norm"])


def make_weights(shape, seed: int) -> dict:
    """Seeded synthetic weights (numpy): bf16 matrices ~ N(0, 0.02^2),
    embeddings ~ N(0, 0.5^2), norm weights ~ 1 + N(0, 0.1^2), experts as
    O.make_experts (the benchmark distributions)."""
    sh = shape
    rng = np.random.default_rng(seed)

    def bf(n, mean, std):
        f = (rng.standard_normal(n) * std + mean).astype(np.float32)
        return (f.view(np.uint32) >> 16).astype(np.uint16)   # truncate to bf16
    W = {"embed": bf(sh.vocab * sh.d_model, 0, 0.5), "lm_head": bf(sh.vocab * sh.d_model, 0, 0.02),
         "model_norm": bf(sh.d_model, 1, 0.1)}
    for k in ("w_q", "w_k", "w_v", "w_o", "router", "in_norm", "post_norm", "q_norm", "k_norm", "experts"):
        W[k] = []
    for l in range(sh.layers):
        W["w_q"].append(bf(sh.q_dim * sh.d_model, 0, 0.02))
        W["w_k"].append(bf(sh.kv_dim * sh.d_model, 0, 0.02))
        W["w_v"].append(bf(sh.kv_dim * sh.d_model, 0, 0.02))
        W["w_o"].append(bf(sh.d_model * sh.q_dim, 0, 0.02))
        W["router"].append(bf(sh.n_experts * sh.d_model, 0, 0.02))
        W["in_norm"].append(bf(sh.d_model, 1, 0.1))
        W["post_norm"].append(bf(sh.d_model, 1, 0.1))
        W["q_norm"].append(bf(sh.head_dim, 1, 0.1))
        W["k_norm"].append(bf(sh.head_dim, 1, 0.1))
        W["experts"].append(O.make_experts(sh.fmt, sh.n_experts, sh.d_model, sh.d_ff, seed * 100 + l))
    return W
