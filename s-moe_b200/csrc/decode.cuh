// decode.cuh - the dense-trunk kernels of a decode step around the MoE layer:
// embedding, residual add + RMSNorm, bf16 GEMV (several matrices per launch),
// per-head QK-RMSNorm + RoPE + KV-ring append, GQA decode attention, and the
// per-step bookkeeping that lets a whole step be one CUDA graph (position,
// token history, uniform draw live on the device).
//
// Reference math: decode.cpp:103-231 (embedding, input norm, QKV, QK norm,
// half-split RoPE, KV ring, softmax attention over `valid` positions newest
// first, O projection, residual), common.hpp:245-256 (rms_norm_bf16, eps
// 1e-6), engine.cpp:351-356 (inv_freq), main.cpp:621-641 (final norm, LM
// head, sampler). Like the reference's own GPU attention
// (metal_bridge.h:163-169) these kernels are not bit-exact with the CPU
// loops: reductions are trees, exp/cos/sin are CUDA's.
#pragma once
#include "router.cuh"
#include "smoe_common.cuh"

namespace smoe {

constexpr int kAttnThreads = 256;
constexpr int kAttnMaxCtx = 8192;      // scores of one head held in shared memory

// Block-wide sum (blockDim.x a multiple of 32, <= 1024); result in every thread.
SMOE_DEVINL float block_sum(float v, float* red32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red32[warp] = v;
    __syncthreads();
    v = lane < nw ? red32[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
SMOE_DEVINL float block_max(float v, float* red32) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red32[warp] = v;
    __syncthreads();
    v = lane < nw ? red32[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// out[t*d + i] = embedding row token[t] (decode.cpp:103-107). grid (ceil(d/256), ntok).
__global__ void k_embed(const uint16_t* table, const uint32_t* token, uint32_t d, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (i < d) out[size_t(t) * d + i] = bf16_bits_to_f32(table[size_t(token[t]) * d + i]);
}

// hidden += delta (when delta), then normed = rms_norm_bf16(hidden, w)
// (common.hpp:245-256: x * (1/sqrt(mean(x^2) + 1e-6)) * w). One CTA per row.
__global__ void k_add_rms_norm(float* hidden, const float* delta, const uint16_t* w, float* normed,
                               uint32_t n) {
    __shared__ float red32[32];
    float* h = hidden + size_t(blockIdx.x) * n;
    const float* dl = delta ? delta + size_t(blockIdx.x) * n : nullptr;
    float* o = normed + size_t(blockIdx.x) * n;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        float v = h[i];
        if (dl) {
            v += dl[i];
            h[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red32);
    const float inv = 1.0f / sqrtf(ss / float(n) + 1e-6f);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) o[i] = (h[i] * inv) * bf16_bits_to_f32(w[i]);
}

// Up to 3 bf16 GEMVs over the same fp32 input, one warp per output row:
// y_m[r] = sum_j W_m[r, j] x[j] (matvec_bf16, common.hpp:293-306).
struct GemvSet {
    const uint16_t* w[3];
    float* y[3];
    uint32_t rows[3];
    uint32_t nmat, cols;
    const float* x;
};
constexpr int kGemvRowsPerCta = 8;
__global__ void __launch_bounds__(256) k_gemv_set(GemvSet a) {
    extern __shared__ __align__(16) float xs[];
    for (uint32_t i = threadIdx.x; i < a.cols; i += blockDim.x) xs[i] = a.x[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t r = blockIdx.x * kGemvRowsPerCta + warp;
    for (uint32_t m = 0; m < a.nmat; ++m) {
        if (r < a.rows[m]) {
            const float v = warp_row_dot_bf16(a.w[m] + size_t(r) * a.cols, xs, a.cols, lane);
            if (lane == 0) a.y[m][r] = v;
            return;
        }
        r -= a.rows[m];
    }
}

// cos/sin of this step's RoPE angles: angle = float(pos) * inv_freq[i]
// (decode.cpp:113-118), pos read from the device.
__global__ void k_rope_table(const uint32_t* pos, const float* inv_freq, float* cs, float* sn, uint32_t half) {
    const uint32_t i = threadIdx.x + blockIdx.x * blockDim.x;
    if (i < half) {
        const float a = float(*pos) * inv_freq[i];
        cs[i] = cosf(a);
        sn[i] = sinf(a);
    }
}

struct AttnArgs {
    const float *q, *k, *v;              // projections [q_dim], [kv_dim], [kv_dim]
    const uint16_t *q_norm_w, *k_norm_w; // [head_dim] bf16 or null
    const float *rope_cos, *rope_sin;    // [head_dim/2]
    float *qbuf, *kbuf, *vbuf;           // normed + roped copies (outputs)
    float *k_cache, *v_cache;            // ring [attn_ctx x kv_dim]
    float* attn_out;                     // [q_dim]
    uint32_t q_dim, kv_dim, head_dim, num_heads, num_kv_heads;
    uint32_t slot, valid, attn_ctx;
    const uint32_t* pos;                 // when set: slot = pos % ctx, valid = min(pos + 1, ctx)
    float scale;
};

SMOE_DEVINL void attn_slot_valid(const AttnArgs& a, uint32_t& slot, uint32_t& valid) {
    if (a.pos) {
        const uint32_t p = *a.pos;
        slot = p % a.attn_ctx;
        valid = p + 1 < a.attn_ctx ? p + 1 : a.attn_ctx;
    } else {
        slot = a.slot;
        valid = a.valid;
    }
}

// One CTA per head: Q heads (QK norm + RoPE -> qbuf), K heads (QK norm +
// RoPE -> kbuf and the ring slot), V heads (-> vbuf and the ring slot)
// (decode.cpp:159-195). blockDim = head_dim (<= 1024, multiple of 32). Each
// thread reads and writes only its own element of q/k/v, so they may alias
// qbuf/kbuf/vbuf.
__global__ void k_qk_rope_append(AttnArgs a) {
    __shared__ float red32[32];
    __shared__ float row[1024];
    const uint32_t b = blockIdx.x, t = threadIdx.x, hd = a.head_dim, half = hd / 2;
    uint32_t slot, valid;
    attn_slot_valid(a, slot, valid);
    const bool isq = b < a.num_heads, isk = !isq && b < a.num_heads + a.num_kv_heads;
    const uint32_t h = isq ? b : isk ? b - a.num_heads : b - a.num_heads - a.num_kv_heads;
    const float* src = (isq ? a.q : isk ? a.k : a.v) + size_t(h) * hd;
    float v = src[t];
    if (isq || isk) {
        const uint16_t* nw = isq ? a.q_norm_w : a.k_norm_w;
        if (nw) {
            const float ss = block_sum(v * v, red32);
            const float inv = 1.0f / sqrtf(ss / float(hd) + 1e-6f);
            v = (v * inv) * bf16_bits_to_f32(nw[t]);
        }
        row[t] = v;
        __syncthreads();
        const uint32_t d = t < half ? t : t - half;
        const float c = a.rope_cos[d], s = a.rope_sin[d];
        v = t < half ? row[t] * c - row[t + half] * s : row[t - half] * s + row[t] * c;
    }
    if (isq) {
        a.qbuf[size_t(h) * hd + t] = v;
    } else {
        (isk ? a.kbuf : a.vbuf)[size_t(h) * hd + t] = v;
        (isk ? a.k_cache : a.v_cache)[size_t(slot) * a.kv_dim + size_t(h) * hd + t] = v;
    }
}

// GQA decode attention, one CTA per query head: scores against the `valid`
// newest ring entries (i = 0 is this step's slot), softmax, weighted sum of
// V (decode.cpp:197-226). head_dim <= 256.
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnArgs a) {
    __shared__ float red32[32];
    __shared__ float qs[256];
    __shared__ float sc[kAttnMaxCtx];
    __shared__ float part[kAttnThreads];
    const uint32_t h = blockIdx.x, hd = a.head_dim, kvh = h / (a.num_heads / a.num_kv_heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = kAttnThreads / 32;
    uint32_t slot, valid;
    attn_slot_valid(a, slot, valid);
    for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) qs[i] = a.qbuf[size_t(h) * hd + i];
    __syncthreads();
    for (uint32_t i = warp; i < valid; i += nw) {               // one warp per position
        const uint32_t ki = (slot + a.attn_ctx - i) % a.attn_ctx;
        const float* kr = a.k_cache + size_t(ki) * a.kv_dim + size_t(kvh) * hd;
        float s = 0.f;
        for (uint32_t j = lane; j < hd; j += 32) s = fmaf(qs[j], kr[j], s);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sc[i] = s * a.scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (uint32_t i = threadIdx.x; i < valid; i += blockDim.x) m = fmaxf(m, sc[i]);
    m = block_max(m, red32);
    float sum = 0.f;
    for (uint32_t i = threadIdx.x; i < valid; i += blockDim.x) {
        const float e = expf(sc[i] - m);
        sc[i] = e;
        sum += e;
    }
    sum = block_sum(sum, red32);
    const float inv = sum > 0.f ? 1.0f / sum : 0.f;
    __syncthreads();
    // thread t handles dim t % hd over positions t / hd, t / hd + g, ...
    const uint32_t g = kAttnThreads / hd, dim = threadIdx.x % hd, grp = threadIdx.x / hd;
    float acc = 0.f;
    if (grp < g)
        for (uint32_t i = grp; i < valid; i += g) {
            const uint32_t vi = (slot + a.attn_ctx - i) % a.attn_ctx;
            acc = fmaf(sc[i] * inv, a.v_cache[size_t(vi) * a.kv_dim + size_t(kvh) * hd + dim], acc);
        }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < hd) {
        float o = 0.f;
        for (uint32_t q = 0; q < g; ++q) o += part[q * hd + threadIdx.x];
        a.attn_out[size_t(h) * hd + threadIdx.x] = o;
    }
}

// End of a decode step on the device: append this step's token to the
// history of sampler row 0, advance the position, and set the next uniform
// draw (u_seq[pos % u_len], when given). One thread.
struct SamplerRowDevMut {
    float temperature, top_p;
    uint32_t top_k;
    float rep_penalty, u;
    uint32_t history_len;
};
__global__ void k_decode_advance(SamplerRowDevMut* row, uint32_t* history, uint32_t hcap,
                                 const uint32_t* token, uint32_t* pos, const float* u_seq, uint32_t u_len) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    const uint32_t n = row->history_len;
    if (n < hcap) {
        history[n] = *token;
        row->history_len = n + 1;
    }
    const uint32_t p = *pos + 1;
    *pos = p;
    if (u_seq && u_len) row->u = u_seq[p % u_len];
}

}  // namespace smoe
