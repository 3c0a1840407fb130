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

// Programmatic dependent launch: every trunk kernel lets the next kernel in
// the stream launch at once (its CTAs then wait in pdl_wait, which returns
// only when this whole grid has completed and its writes are visible), and
// waits for its own predecessor before reading anything that one wrote.
SMOE_DEVINL void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
SMOE_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

constexpr int kAttnThreads = 256;
constexpr int kAttnMaxCtx = 8192;      // scores of one head held in shared memory
constexpr int kAttnSplits = 8;         // position splits per head (flash-decoding)
constexpr int kAttnMaxHeads = 128;

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
    pdl_trigger();
    pdl_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (i < d) out[size_t(t) * d + i] = bf16_bits_to_f32(table[size_t(token[t]) * d + i]);
}

// hidden += delta (when delta), then normed = rms_norm_bf16(hidden, w)
// (common.hpp:245-256: x * (1/sqrt(mean(x^2) + 1e-6)) * w). One CTA per row.
__global__ void k_add_rms_norm(float* hidden, const float* delta, const uint16_t* w, float* normed,
                               uint32_t n) {
    __shared__ float red32[32];
    pdl_trigger();
    pdl_wait();
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
// Grid-stride over row pairs: a lane keeps 2 x 8 16-byte weight loads in
// flight (both rows' chunks, issued before any use) and reads x through L1
// (the same few KB for every warp), so no staging barrier sits in front of
// the weight stream. cols % 8 == 0.
struct GemvSet {
    const uint16_t* w[3];
    float* y[3];
    uint32_t rows[3];
    uint32_t nmat, cols;
    const float* x;
};
constexpr int kGemvThreads = 256;

SMOE_DEVINL void gemv_locate(const GemvSet& a, uint32_t r, const uint16_t*& w, float*& y) {
    for (uint32_t m = 0; m < a.nmat; ++m) {
        if (r < a.rows[m]) {
            w = a.w[m] + size_t(r) * a.cols;
            y = a.y[m] + r;
            return;
        }
        r -= a.rows[m];
    }
    w = nullptr;
    y = nullptr;
}

SMOE_DEVINL float dot8_bf16(uint4 v, const float4* xp) {
    const float4 a = __ldg(xp), b = __ldg(xp + 1);
    float s = __uint_as_float(v.x << 16) * a.x;
    s = fmaf(__uint_as_float(v.x & 0xffff0000u), a.y, s);
    s = fmaf(__uint_as_float(v.y << 16), a.z, s);
    s = fmaf(__uint_as_float(v.y & 0xffff0000u), a.w, s);
    s = fmaf(__uint_as_float(v.z << 16), b.x, s);
    s = fmaf(__uint_as_float(v.z & 0xffff0000u), b.y, s);
    s = fmaf(__uint_as_float(v.w << 16), b.z, s);
    s = fmaf(__uint_as_float(v.w & 0xffff0000u), b.w, s);
    return s;
}

// RPW rows per warp (1 for small matrices, so the grid covers the SMs; 2
// for large ones). The first chunk of weight loads is issued before waiting
// for the kernel that produced x (weights do not depend on it).
// CH: 16-byte chunks per lane per row in flight at once (8: rows of up to
// 2048 bf16 in one round trip; 16 for rows up to 4096).
template <int RPW, int CH = 8>
__global__ void __launch_bounds__(kGemvThreads) k_gemv_set(GemvSet a, uint32_t total) {
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    const uint32_t nwarp = gridDim.x * (kGemvThreads / 32);
    const uint32_t n = a.cols / 8;                                   // 16-byte chunks per row
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    bool waited = false;
    for (uint32_t r0 = (blockIdx.x * (kGemvThreads / 32) + (threadIdx.x >> 5)) * RPW; r0 < total;
         r0 += nwarp * RPW) {
        const uint4* p[RPW];
        float* y[RPW];
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            const uint16_t* w;
            gemv_locate(a, r0 + q < total ? r0 + q : r0, w, y[q]);
            if (r0 + q >= total) y[q] = nullptr;
            p[q] = reinterpret_cast<const uint4*>(w);
        }
        float sacc[RPW];
#pragma unroll
        for (int q = 0; q < RPW; ++q) sacc[q] = 0.f;
        for (uint32_t c0 = lane; c0 < n; c0 += 32 * CH) {
            uint4 v[RPW][CH];
#pragma unroll
            for (int j = 0; j < CH; ++j) {
                const uint32_t c = c0 + j * 32;
#pragma unroll
                for (int q = 0; q < RPW; ++q)
                    if (c < n) v[q][j] = __ldcs(p[q] + c);           // streamed once: do not keep in L2
            }
            if (!waited) {
                pdl_wait();
                waited = true;
            }
#pragma unroll
            for (int j = 0; j < CH; ++j) {
                const uint32_t c = c0 + j * 32;
#pragma unroll
                for (int q = 0; q < RPW; ++q)
                    if (c < n) sacc[q] += dot8_bf16(v[q][j], x4 + 2 * c);
            }
        }
#pragma unroll
        for (int q = 0; q < RPW; ++q) {
            float sv = sacc[q];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, o);
            if (lane == 0 && y[q]) *y[q] = sv;
        }
    }
    if (!waited) pdl_wait();
}

// cos/sin of this step's RoPE angles: angle = float(pos) * inv_freq[i]
// (decode.cpp:113-118), pos read from the device.
__global__ void k_rope_table(const uint32_t* pos, const float* inv_freq, float* cs, float* sn, uint32_t half) {
    pdl_trigger();
    pdl_wait();
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
    float* part;                         // split partials [num_heads][gridDim.y][head_dim + 2]
    uint32_t* cnt;                       // [num_heads] splits done (zero between launches)
    size_t kv_seq_stride;                // batched decode (gridDim.z sequences): floats between the
                                         // rings of consecutive sequences; q/k/v/qbuf/attn_out are
                                         // [sequences][q_dim or kv_dim] (one split per head then)
    uint32_t blk;                        // k_attn_batch_gqa: positions per score block (shared memory)
    uint32_t prefill;                    // k_attn_batch_gqa: row z is token z of one sequence at
                                         // position *pos + z, its K/V already in the ring
                                         // (k_prefill_kv), RoPE tables [tokens][head_dim/2]
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

// QK RMSNorm (when w) + half-split RoPE of one head held in x[0..hd) of
// shared memory, in place; every thread of the CTA calls it (decode.cpp:159-195).
SMOE_DEVINL void head_norm_rope(float* x, const uint16_t* w, const float* cs, const float* sn, uint32_t hd,
                                float* red32) {
    const uint32_t t = threadIdx.x, half = hd / 2;
    float v = t < hd ? x[t] : 0.f;
    if (w) {
        const float ss = block_sum(v * v, red32);
        const float inv = 1.0f / sqrtf(ss / float(hd) + 1e-6f);
        if (t < hd) v = (v * inv) * bf16_bits_to_f32(w[t]);
    }
    __syncthreads();
    if (t < hd) x[t] = v;
    __syncthreads();
    float r = 0.f;
    if (t < hd) {
        const uint32_t d = t < half ? t : t - half;
        r = t < half ? x[t] * cs[d] - x[t + half] * sn[d] : x[t - half] * sn[d] + x[t] * cs[d];
    }
    __syncthreads();
    if (t < hd) x[t] = r;
    __syncthreads();
}

// Grid (query head h, split s) (decode.cpp:159-226, split-K over the
// positions as in flash-decoding): QK norm + RoPE of head h's Q (-> qbuf,
// split 0) and of its KV head's K; split 0 of the first Q head of each KV
// group appends K and V to the ring slot. Split s takes positions
// [s P, (s+1) P) of the `valid` newest (i = 0: this step, from shared
// memory; the others from the ring, written by earlier steps), P =
// ceil(valid / splits): scores, its own max m, l = sum exp(score - m) and
// o = sum exp(score - m) v, stored as a partial; the head's last split to
// finish adds the partials in split order (weights exp(m_s - M)) and writes
// attn_out. Scores: a warp takes 8 positions per round, 4 lanes per position
// with all their loads issued before the reduction. head_dim % 16 == 0,
// <= 256.
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(AttnArgs a) {
    // (a is this CTA's own copy: the batched offsets below rebase it)
    __shared__ float red32[32];
    __shared__ __align__(16) float qs[256];
    __shared__ __align__(16) float ks[256];
    __shared__ __align__(16) float vs[256];
    __shared__ float sc[kAttnMaxCtx];
    __shared__ float part[kAttnThreads];
    __shared__ uint32_t last;
    const uint32_t h = blockIdx.x, hd = a.head_dim, per = a.num_heads / a.num_kv_heads, kvh = h / per;
    const uint32_t split = blockIdx.y, nsplit = gridDim.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = kAttnThreads / 32;
    pdl_trigger();
    pdl_wait();
    uint32_t slot, valid;
    attn_slot_valid(a, slot, valid);
    if (blockIdx.z) {                    // sequence z of a batch: its rows and its own ring
        const size_t z = blockIdx.z;
        a.q += z * a.q_dim;
        a.k += z * a.kv_dim;
        a.v += z * a.kv_dim;
        a.qbuf += z * a.q_dim;
        a.attn_out += z * a.q_dim;
        a.k_cache += z * a.kv_seq_stride;
        a.v_cache += z * a.kv_seq_stride;
    }
    for (uint32_t i = tid; i < hd; i += blockDim.x) {
        qs[i] = a.q[size_t(h) * hd + i];
        ks[i] = a.k[size_t(kvh) * hd + i];
        vs[i] = a.v[size_t(kvh) * hd + i];
    }
    __syncthreads();
    head_norm_rope(qs, a.q_norm_w, a.rope_cos, a.rope_sin, hd, red32);
    head_norm_rope(ks, a.k_norm_w, a.rope_cos, a.rope_sin, hd, red32);
    if (split == 0)
        for (uint32_t i = tid; i < hd; i += blockDim.x) {
            a.qbuf[size_t(h) * hd + i] = qs[i];
            if (h % per == 0) {
                a.k_cache[size_t(slot) * a.kv_dim + size_t(kvh) * hd + i] = ks[i];
                a.v_cache[size_t(slot) * a.kv_dim + size_t(kvh) * hd + i] = vs[i];
            }
        }
    const uint32_t P = (valid + nsplit - 1) / nsplit;
    const uint32_t i0 = min(valid, split * P), i1 = min(valid, i0 + P);
    // scores of positions [i0, i1), at sc[i - i0]
    const uint32_t sub = lane & 3, q4 = hd / 16;                  // float4s per lane and position
    const float4* qv = reinterpret_cast<const float4*>(qs) + sub * q4;
    for (uint32_t base = i0 + warp * 8; base < i1; base += nw * 8) {
        const uint32_t i = base + (lane >> 2);
        float s = 0.f;
        if (i < i1) {
            const float4* kr = i == 0 ? reinterpret_cast<const float4*>(ks) + sub * q4
                                      : reinterpret_cast<const float4*>(
                                            a.k_cache + size_t((slot + a.attn_ctx - i) % a.attn_ctx) * a.kv_dim +
                                            size_t(kvh) * hd) + sub * q4;
            float4 kk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < int(q4)) kk[j] = kr[j];
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < int(q4)) {
                    const float4 qq = qv[j];
                    s = fmaf(qq.x, kk[j].x, s);
                    s = fmaf(qq.y, kk[j].y, s);
                    s = fmaf(qq.z, kk[j].z, s);
                    s = fmaf(qq.w, kk[j].w, s);
                }
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (sub == 0 && i < i1) sc[i - i0] = s * a.scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (uint32_t i = i0 + tid; i < i1; i += blockDim.x) m = fmaxf(m, sc[i - i0]);
    m = block_max(m, red32);
    float sum = 0.f;
    for (uint32_t i = i0 + tid; i < i1; i += blockDim.x) {
        const float e = expf(sc[i - i0] - m);
        sc[i - i0] = e;
        sum += e;
    }
    sum = block_sum(sum, red32);
    __syncthreads();
    // thread t: dim t % hd over positions i0 + t / hd + g k; 4 loads in flight
    const uint32_t g = kAttnThreads / hd, dim = tid % hd, grp = tid / hd;
    float acc = 0.f;
    if (grp < g) {
        const float* vb = a.v_cache + size_t(kvh) * hd + dim;
        uint32_t i = i0 + grp;
        if (i == 0 && i < i1) {
            acc = sc[0] * vs[dim];
            i += g;
        }
        for (; i + 3 * g < i1; i += 4 * g) {
            float vv[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) vv[q] = vb[size_t((slot + a.attn_ctx - (i + q * g)) % a.attn_ctx) * a.kv_dim];
#pragma unroll
            for (int q = 0; q < 4; ++q) acc = fmaf(sc[i - i0 + q * g], vv[q], acc);
        }
        for (; i < i1; i += g)
            acc = fmaf(sc[i - i0], vb[size_t((slot + a.attn_ctx - i) % a.attn_ctx) * a.kv_dim], acc);
    }
    part[tid] = acc;
    __syncthreads();
    float o = 0.f;
    if (uint32_t(tid) < hd)
        for (uint32_t q = 0; q < g; ++q) o += part[q * hd + tid];
    if (nsplit == 1) {
        if (uint32_t(tid) < hd) a.attn_out[size_t(h) * hd + tid] = o * (sum > 0.f ? 1.0f / sum : 0.f);
        return;
    }
    // this split's partial; the head's last split combines them
    float* pp = a.part + (size_t(h) * nsplit + split) * (hd + 2);
    if (uint32_t(tid) < hd) pp[2 + tid] = o;
    if (tid == 0) {
        pp[0] = m;
        pp[1] = sum;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.cnt + h, 1u) == nsplit - 1 ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    float M = -INFINITY;
    for (uint32_t q = 0; q < nsplit; ++q) M = fmaxf(M, __ldcg(a.part + (size_t(h) * nsplit + q) * (hd + 2)));
    float L = 0.f, out = 0.f;
    for (uint32_t q = 0; q < nsplit; ++q) {
        const float* pq = a.part + (size_t(h) * nsplit + q) * (hd + 2);
        const float mq = __ldcg(pq);
        const float wq = mq == -INFINITY ? 0.f : expf(mq - M);
        L = fmaf(__ldcg(pq + 1), wq, L);
        if (uint32_t(tid) < hd) out = fmaf(__ldcg(pq + 2 + tid), wq, out);
    }
    if (uint32_t(tid) < hd) a.attn_out[size_t(h) * hd + tid] = out * (L > 0.f ? 1.0f / L : 0.f);
    if (tid == 0) a.cnt[h] = 0u;                  // ready for the next launch
}

// Batched decode attention, one CTA per (KV head, sequence): the ring of a
// KV head is read once for all G = num_heads / num_kv_heads query heads of
// its group (the per-query-head kernel above reads it G times). Same math
// as k_attn_decode (decode.cpp:159-226), one split per head:
//  1. warp w takes heads w, w + 8, ... (and the KV head's K last): QK
//     RMSNorm + half-split RoPE with a lane holding dims lane + 32 j (a RoPE
//     pair d, d + hd/2 stays in one lane: hd % 64 == 0); normed + roped Q
//     to qbuf, K and V to the ring slot;
//  2. scores: 4 lanes per position (hd / 4 dims each, all loads issued
//     before the dots), G dot products per K row, reduced over the 4 lanes;
//  3. softmax per head (warp per head): max, exp, sum;
//  steps 2-4 run over blocks of `blk` positions with the softmax carried
//  from block to block (running max, sum and accumulators rescaled), so the
//  scores held in shared memory are bounded whatever the ring size;
//  4. out[g][d] = sum_i p[g][i] V[i][d] / sum_g: a warp takes every 8th
//     position, a lane 4 dims of the row (one float4), G float4
//     accumulators, 4 rows in flight; the warps' partials added through
//     shared memory.
// head_dim == 128. Dynamic shared memory (floats): q [G hd], k [hd], v [hd],
// scores [G blk], warp partials [8][G hd].
constexpr int kAttnGqaMaxG = 16;
template <int GM>      // query heads per KV head, at most (8 or 16): sizes the accumulators
__global__ void __launch_bounds__(kAttnThreads, 2) k_attn_batch_gqa(AttnArgs a) {
    extern __shared__ __align__(16) float gqa_sm[];
    const uint32_t hd = a.head_dim, G = a.num_heads / a.num_kv_heads, kvh = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = kAttnThreads / 32;
    float* qs = gqa_sm;
    float* ks = qs + G * hd;
    float* vs = ks + hd;
    float* sc = vs + hd;
    float* gp = sc + size_t(G) * a.blk;
    pdl_trigger();
    pdl_wait();
    const size_t z = blockIdx.y;
    const bool pf = a.prefill != 0;
    uint32_t slot, valid;
    if (pf) {                            // token z of the chunk (prefill.cpp:216-220)
        const uint32_t p = *a.pos + uint32_t(z);
        slot = p % a.attn_ctx;
        valid = p + 1 < a.attn_ctx ? p + 1 : a.attn_ctx;
        a.rope_cos += z * (hd / 2);
        a.rope_sin += z * (hd / 2);
    } else {
        attn_slot_valid(a, slot, valid);
    }
    const float* q = a.q + z * a.q_dim + size_t(kvh) * G * hd;
    float* k_cache = a.k_cache + z * a.kv_seq_stride;
    float* v_cache = a.v_cache + z * a.kv_seq_stride;
    // 1. norm + RoPE: rows 0..G-1 are the query heads, row G the K head
    const uint32_t per_lane = hd / 32, half = hd / 2;
    for (uint32_t r = warp; r < G + (pf ? 0u : 1u); r += nw) {
        const float* src = r < G ? q + size_t(r) * hd : a.k + z * a.kv_dim + size_t(kvh) * hd;
        const uint16_t* nw_ = r < G ? a.q_norm_w : a.k_norm_w;
        float v[8];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (uint32_t(j) < per_lane) {
                v[j] = src[lane + 32 * j];
                ss = fmaf(v[j], v[j], ss);
            }
        if (nw_) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.0f / sqrtf(ss / float(hd) + 1e-6f);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (uint32_t(j) < per_lane) v[j] = (v[j] * inv) * bf16_bits_to_f32(nw_[lane + 32 * j]);
        }
        const uint32_t jh = per_lane / 2;                   // dims lane + 32 j, j < jh, are the first half
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (uint32_t(j) < per_lane) {
                const uint32_t t = lane + 32 * j;
                const uint32_t d = t < half ? t : t - half;
                o[j] = uint32_t(j) < jh ? v[j] * a.rope_cos[d] - v[j + jh] * a.rope_sin[d]
                                        : v[j - jh] * a.rope_sin[d] + v[j] * a.rope_cos[d];
            }
        float* dst = r < G ? qs + size_t(r) * hd : ks;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (uint32_t(j) < per_lane) dst[lane + 32 * j] = o[j];
        if (r < G) {
            float* qb = a.qbuf + z * a.q_dim + (size_t(kvh) * G + r) * hd;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (uint32_t(j) < per_lane) qb[lane + 32 * j] = o[j];
        }
    }
    if (!pf)
        for (uint32_t i = tid; i < hd; i += blockDim.x) vs[i] = a.v[z * a.kv_dim + size_t(kvh) * hd + i];
    __syncthreads();
    if (!pf)
        for (uint32_t i = tid; i < hd; i += blockDim.x) {
            k_cache[size_t(slot) * a.kv_dim + size_t(kvh) * hd + i] = ks[i];
            v_cache[size_t(slot) * a.kv_dim + size_t(kvh) * hd + i] = vs[i];
        }
    // 2-4 over blocks of a.blk positions, the softmax carried across blocks
    // (running max per head; the sum and the accumulators rescaled by
    // exp(old max - new max) when it grows)
    __shared__ float sums[GM], mx[GM], alpha[GM];
    if (uint32_t(tid) < G) {
        sums[tid] = 0.f;
        mx[tid] = -INFINITY;
    }
    float4 acc[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t sub = lane & 3, q4 = hd / 16;                  // float4s per lane and position
    const float4* vb = reinterpret_cast<const float4*>(v_cache + size_t(kvh) * hd) + lane;
    const float4 vnew = pf ? make_float4(0.f, 0.f, 0.f, 0.f) : reinterpret_cast<const float4*>(vs)[lane];
    const uint32_t BL = a.blk;
    for (uint32_t b0 = 0; b0 < valid; b0 += BL) {
        const uint32_t b1 = min(valid, b0 + BL), nb = b1 - b0;
        // 2. scores of positions [b0, b1) (0 = this step; from the ring in
        //    prefill) at sc[g * BL + i - b0]
        for (uint32_t base = b0 + warp * 8; base < b1; base += nw * 8) {
            const uint32_t i = base + (lane >> 2);
            float4 kk[8];                                 // hd == 128: 8 float4 per lane
            if (i < b1) {
                const float4* kr = i == 0 && !pf ? reinterpret_cast<const float4*>(ks) + sub * q4
                                                 : reinterpret_cast<const float4*>(
                                                       k_cache + size_t((slot + a.attn_ctx - i) % a.attn_ctx) *
                                                                     a.kv_dim + size_t(kvh) * hd) + sub * q4;
#pragma unroll
                for (int j = 0; j < 8; ++j) kk[j] = kr[j];
            }
            for (uint32_t g = 0; g < G; ++g) {
                const float4* qv = reinterpret_cast<const float4*>(qs + size_t(g) * hd) + sub * q4;
                float s = 0.f;
                if (i < b1) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                            const float4 qq = qv[j];
                            s = fmaf(qq.x, kk[j].x, s);
                            s = fmaf(qq.y, kk[j].y, s);
                            s = fmaf(qq.z, kk[j].z, s);
                            s = fmaf(qq.w, kk[j].w, s);
                        }
                }
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                if (sub == 0 && i < b1) sc[size_t(g) * BL + (i - b0)] = s * a.scale;
            }
        }
        __syncthreads();
        // 3. softmax terms per head (a warp per head)
        for (uint32_t g = warp; g < G; g += nw) {
            float* sg = sc + size_t(g) * BL;
            float m = -INFINITY;
            for (uint32_t i = lane; i < nb; i += 32) m = fmaxf(m, sg[i]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const float m_old = mx[g], M = fmaxf(m_old, m);
            float sum = 0.f;
            for (uint32_t i = lane; i < nb; i += 32) {
                const float e = expf(sg[i] - M);
                sg[i] = e;
                sum += e;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            if (lane == 0) {
                const float al = m_old == -INFINITY ? 0.f : expf(m_old - M);
                alpha[g] = al;
                sums[g] = fmaf(sums[g], al, sum);
                mx[g] = M;
            }
        }
        __syncthreads();
        // 4. weighted V sum: warp w takes positions b0 + w, + 8, ..., a lane
        //    the float4 of dims 4 lane.. of each V row (hd == 128), 4 rows in
        //    flight
#pragma unroll
        for (int g = 0; g < GM; ++g)
            if (uint32_t(g) < G) {
                const float al = alpha[g];
                acc[g].x *= al; acc[g].y *= al; acc[g].z *= al; acc[g].w *= al;
            }
        for (uint32_t i = b0 + warp; i < b1; i += 4 * nw) {
            float4 vv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t p = i + u * nw;
                vv[u] = p == 0 && !pf ? vnew
                      : p < b1 ? vb[size_t((slot + a.attn_ctx - p) % a.attn_ctx) * (a.kv_dim / 4)]
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t p = i + u * nw;
                if (p < b1)
#pragma unroll
                    for (int g = 0; g < GM; ++g)
                        if (uint32_t(g) < G) {
                            const float w = sc[size_t(g) * BL + (p - b0)];
                            acc[g].x = fmaf(w, vv[u].x, acc[g].x);
                            acc[g].y = fmaf(w, vv[u].y, acc[g].y);
                            acc[g].z = fmaf(w, vv[u].z, acc[g].z);
                            acc[g].w = fmaf(w, vv[u].w, acc[g].w);
                        }
            }
        }
        __syncthreads();                 // the next block's scores overwrite sc
    }
    float4* gp4 = reinterpret_cast<float4*>(gp);                 // [8 warps][G][32 float4]
#pragma unroll
    for (int g = 0; g < GM; ++g)
        if (uint32_t(g) < G) gp4[(size_t(warp) * G + g) * 32 + lane] = acc[g];
    __syncthreads();
    for (uint32_t o = tid; o < G * 32; o += blockDim.x) {
        const uint32_t g = o / 32;
        float4 r = gp4[o];
        for (int w = 1; w < nw; ++w) {
            const float4 q = gp4[size_t(w) * G * 32 + o];
            r.x += q.x; r.y += q.y; r.z += q.z; r.w += q.w;
        }
        const float sum = sums[g];
        const float inv = sum > 0.f ? 1.0f / sum : 0.f;
        r.x *= inv; r.y *= inv; r.z *= inv; r.w *= inv;
        reinterpret_cast<float4*>(a.attn_out + z * a.q_dim + size_t(kvh) * G * hd)[o] = r;
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
    pdl_trigger();
    pdl_wait();
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

// Prefill (prefill.cpp:165-203): token t of a chunk at position *pos + t:
// K RMSNorm + half-split RoPE (table row t) of every KV head, K and V to the
// ring slot (*pos + t) % ctx, before any token of the chunk attends (so
// token t sees tokens 0..t of the chunk through the ring, as the reference's
// causal loop does). Grid (num_kv_heads, tokens), one warp; head_dim % 64 ==
// 0, <= 256.
__global__ void k_prefill_kv(const float* k, const float* v, const uint16_t* k_norm_w, const float* rope_cos,
                             const float* rope_sin, float* k_cache, float* v_cache, uint32_t kv_dim,
                             uint32_t hd, uint32_t attn_ctx, const uint32_t* pos) {
    pdl_trigger();
    pdl_wait();
    const uint32_t kvh = blockIdx.x, t = blockIdx.y, lane = threadIdx.x;
    const uint32_t slot = (*pos + t) % attn_ctx, per_lane = hd / 32, jh = per_lane / 2, half = hd / 2;
    const float* src = k + size_t(t) * kv_dim + size_t(kvh) * hd;
    const float* cs = rope_cos + size_t(t) * half;
    const float* sn = rope_sin + size_t(t) * half;
    float x[8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (uint32_t(j) < per_lane) {
            x[j] = src[lane + 32 * j];
            ss = fmaf(x[j], x[j], ss);
        }
    if (k_norm_w) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / float(hd) + 1e-6f);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (uint32_t(j) < per_lane) x[j] = (x[j] * inv) * bf16_bits_to_f32(k_norm_w[lane + 32 * j]);
    }
    float* kd = k_cache + size_t(slot) * kv_dim + size_t(kvh) * hd;
    float* vd = v_cache + size_t(slot) * kv_dim + size_t(kvh) * hd;
    const float* vs = v + size_t(t) * kv_dim + size_t(kvh) * hd;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (uint32_t(j) < per_lane) {
            const uint32_t i = lane + 32 * j, d = i < half ? i : i - half;
            kd[i] = uint32_t(j) < jh ? x[j] * cs[d] - x[j + jh] * sn[d] : x[j - jh] * sn[d] + x[j] * cs[d];
            vd[i] = vs[i];
        }
}

// RoPE tables of `n` consecutive positions *pos + t (decode.cpp:113-118 per
// token): cs / sn [n][half]. Grid (ceil(half / 128), n).
__global__ void k_rope_tables(const uint32_t* pos, const float* inv_freq, float* cs, float* sn, uint32_t half) {
    pdl_trigger();
    pdl_wait();
    const uint32_t i = threadIdx.x + blockIdx.x * blockDim.x, t = blockIdx.y;
    if (i < half) {
        const float a = float(*pos + t) * inv_freq[i];
        cs[size_t(t) * half + i] = cosf(a);
        sn[size_t(t) * half + i] = sinf(a);
    }
}

// Batched decode (one position shared by `batch` sequences): sequence b's
// token joins its sampler row's history, its next uniform is u_seq[(p *
// batch + b) % u_len] for the new position p, and the position advances once.
// One CTA, batch <= 1024 threads.
__global__ void k_decode_advance_batch(SamplerRowDevMut* rows, uint32_t* history, uint32_t hcap,
                                       const uint32_t* tokens, uint32_t batch, uint32_t* pos,
                                       const float* u_seq, uint32_t u_len) {
    pdl_trigger();
    pdl_wait();
    const uint32_t b = threadIdx.x;
    const uint32_t p = *pos + 1;
    __syncthreads();                     // every thread has read the position
    if (b < batch) {
        SamplerRowDevMut* r = rows + b;
        const uint32_t n = r->history_len;
        if (n < hcap) {
            history[size_t(b) * hcap + n] = tokens[b];
            r->history_len = n + 1;
        }
        if (u_seq && u_len) r->u = u_seq[(size_t(p) * batch + b) % u_len];
    }
    if (b == 0) *pos = p;
}

// fp32 rows -> two bf16 planes, hi = bf16(x) and lo = bf16(x - hi), so that a
// bf16 tensor-core GEMM over both planes (fp32 accumulation) reproduces an
// fp32-activation matvec to ~2^-17 relative per element. out: [2][n].
__global__ void k_split_bf16(const float* x, uint16_t* out, size_t n) {
    pdl_trigger();
    pdl_wait();
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        out[i] = __bfloat16_as_ushort(hi);
        out[n + i] = __bfloat16_as_ushort(lo);
    }
}

}  // namespace smoe
