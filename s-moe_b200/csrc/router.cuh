// router.cuh - exact router gate + softmax + top-k + renorm, and the plain
// bf16 GEMV of metal_bridge.h:157 (sm_100a).
//
// Router (decode.cpp:280-303 -> common.hpp:294-306, scout.cpp:77-123):
//   logits[e] = sum_j bf16(W[e,j]) * x[j]           fp32 accumulate
//   p = softmax(logits)  (max-subtracted exp, * 1/sum)
//   top-k by p, descending, lowest expert index wins ties
//   w_j = p_j * (1 / sum_{rank order} p)   when norm_topk
// One warp per expert row; the last CTA of a token (atomic ticket) finishes
// the softmax/selection in one warp, so there is no second launch.
#pragma once
#include "smoe_common.cuh"

namespace smoe {

struct RouterArgs {
    const uint16_t* w;        // [E x d] bf16
    const void*     x;        // [batch x d]
    int             x_dtype;
    uint32_t        E, d, k;
    int             norm;
    float*          logits;   // [batch x E] (scratch or caller's)
    uint32_t*       ids;      // [batch x k]
    float*          wts;      // [batch x k]
    uint32_t*       ticket;   // [batch] zero on entry, left zero on exit
    uint32_t*       err;
};

constexpr int kRouterRowsPerCta = 8;
constexpr int kRouterMaxE = 512;

// Warp dot of one bf16 row with the smem fp32 vector (16-byte loads).
SMOE_DEVINL float warp_row_dot_bf16(const uint16_t* row, const float* xs, int d, int lane) {
    float acc = 0.f;
    const uint4* rp = reinterpret_cast<const uint4*>(row);
    const int n = d / 8;
    for (int c0 = lane; c0 < n; c0 += 32 * 8) {
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)              // all loads in flight before any use
            if (c0 + q * 32 < n) v[q] = __ldg(rp + c0 + q * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (c0 + q * 32 >= n) break;
            const float* xv = xs + (c0 + q * 32) * 8;
            const uint32_t u[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                acc = fmaf(__uint_as_float(u[r] << 16), xv[2 * r], acc);
                acc = fmaf(__uint_as_float(u[r] & 0xffff0000u), xv[2 * r + 1], acc);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

// Two rows at once: both rows' loads are in flight together; each row's
// accumulator sees exactly warp_row_dot_bf16's operation sequence.
SMOE_DEVINL void warp_row_dot_bf16_x2(const uint16_t* row0, const uint16_t* row1, const float* xs, int d,
                                      int lane, float& o0, float& o1) {
    float acc[2] = {0.f, 0.f};
    const uint4* rp[2] = {reinterpret_cast<const uint4*>(row0), reinterpret_cast<const uint4*>(row1)};
    const int n = d / 8;
    for (int c0 = lane; c0 < n; c0 += 32 * 8) {
        uint4 v[2][8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
            for (int m = 0; m < 2; ++m)
                if (c0 + q * 32 < n) v[m][q] = __ldg(rp[m] + c0 + q * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (c0 + q * 32 >= n) break;
            const float* xv = xs + (c0 + q * 32) * 8;
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const uint32_t u[4] = {v[m][q].x, v[m][q].y, v[m][q].z, v[m][q].w};
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    acc[m] = fmaf(__uint_as_float(u[r] << 16), xv[2 * r], acc[m]);
                    acc[m] = fmaf(__uint_as_float(u[r] & 0xffff0000u), xv[2 * r + 1], acc[m]);
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
        acc[1] += __shfl_xor_sync(0xffffffffu, acc[1], o);
    }
    o0 = acc[0];
    o1 = acc[1];
}

template <typename T>
SMOE_DEVINL void stage_vec(const void* src, int x_dtype, size_t off, int d, float* xs) {
    if (x_dtype == 0) {
        const float* s = static_cast<const float*>(src) + off;
        for (int i = threadIdx.x; i < d; i += blockDim.x) xs[i] = s[i];
    } else {
        const uint16_t* s = static_cast<const uint16_t*>(src) + off;
        for (int i = threadIdx.x; i < d; i += blockDim.x) xs[i] = bf16_bits_to_f32(s[i]);
    }
}

// One warp: softmax over E logits (read from global, bypassing L1), top-k
// by probability with the lowest index winning ties, renormalised over the k
// in rank order when `norm` (scout.cpp:77-123, decode.cpp:296-303). The
// denominator is a warp tree sum; expert ids do not depend on it.
// ids/wts: k outputs (global or shared).
template <int NV>
SMOE_DEVINL void warp_topk_regs(float (&p)[NV], int E, uint32_t k, int norm, uint32_t* ids, float* wts,
                                int lane) {
    // Lane l holds logits l + 32j in p[j] (-inf past E). Selection keys:
    // bits(p) + 1 for a live probability (p >= 0, so the order of the keys is
    // the order of p), 0 for removed or absent entries. Each round is two warp
    // reductions: the largest key, then the lowest index among the lanes
    // holding it.
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < NV; ++j) mx = fmaxf(mx, p[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        if (lane + 32 * j < E) {
            p[j] = expf(p[j] - mx);
            se += p[j];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const float inv = se > 0.f ? 1.0f / se : 0.f;
    uint32_t key[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) key[j] = lane + 32 * j < E ? __float_as_uint(p[j] * inv) + 1u : 0u;
    float wsel = 0.f;
    uint32_t idsel = 0;
#pragma unroll 1
    for (uint32_t s = 0; s < k; ++s) {
        uint32_t lb = 0u;
        int lj = 0;
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (key[j] > lb) { lb = key[j]; lj = j; }               // ascending index: first max per lane
        const uint32_t gm = __reduce_max_sync(0xffffffffu, lb);
        const uint32_t win = __reduce_min_sync(0xffffffffu, lb == gm ? uint32_t(lane + 32 * lj) : 0xffffffffu);
        if (lane == (int)s) { wsel = __uint_as_float(gm - 1u); idsel = win; }
#pragma unroll
        for (int j = 0; j < NV; ++j)                                // remove the winner
            if (win == uint32_t(lane + 32 * j)) key[j] = 0u;
    }
    float ws = 0.f;                                   // rank-order sum (decode.cpp:296-303)
#pragma unroll 1
    for (uint32_t s = 0; s < k; ++s) ws += __shfl_sync(0xffffffffu, wsel, s);
    const float winv = (norm && ws > 0.f) ? 1.0f / ws : 1.0f;
    if (lane < (int)k) {
        ids[lane] = idsel;
        wts[lane] = wsel * winv;
    }
}

template <int NV>
SMOE_DEVINL void warp_topk_n(const float* lg, int E, uint32_t k, int norm, uint32_t* ids, float* wts,
                             int lane) {
    float p[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const int i = lane + 32 * j;
        p[j] = i < E ? __ldcg(lg + i) : -INFINITY;
    }
    warp_topk_regs<NV>(p, E, k, norm, ids, wts, lane);
}

SMOE_DEVINL void warp_topk(const float* lg, uint32_t E_, uint32_t k_, int norm, uint32_t* ids, float* wts,
                           int lane) {
    const uint32_t k = k_ < E_ ? k_ : E_;
    if (E_ <= 128) warp_topk_n<4>(lg, (int)E_, k, norm, ids, wts, lane);
    else warp_topk_n<kRouterMaxE / 32>(lg, (int)E_, k, norm, ids, wts, lane);
}

// grid (ceil(E/8), batch), 256 threads, smem d floats + selection scratch.
__global__ void __launch_bounds__(256) k_router(RouterArgs a) {
    extern __shared__ __align__(16) float xs[];
    __shared__ uint32_t last_flag;
    const int tok = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    stage_vec<float>(a.x, a.x_dtype, size_t(tok) * a.d, a.d, xs);
    __syncthreads();
    const int e = blockIdx.x * kRouterRowsPerCta + warp;
    float* lg = a.logits + size_t(tok) * a.E;
    if (e < (int)a.E) {
        const float v = warp_row_dot_bf16(a.w + size_t(e) * a.d, xs, a.d, lane);
        if (lane == 0) lg[e] = v;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t old = atomicAdd(a.ticket + tok, 1u);
        last_flag = (old == gridDim.x - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    if (warp != 0) return;
    warp_topk(lg, a.E, a.k, a.norm, a.ids + size_t(tok) * a.k, a.wts + size_t(tok) * a.k, lane);
    if (lane == 0) a.ticket[tok] = 0;                 // ready for the next call
}

// Token batches: one CTA per token computes all its logit rows (x staged
// once, 16 warps over the rows), then warp 0 selects. Same arithmetic per
// row and the same selection as k_router. grid (batch), 512 threads.
__global__ void __launch_bounds__(512) k_router_tok(RouterArgs a) {
    extern __shared__ __align__(16) float xs[];
    const int tok = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    stage_vec<float>(a.x, a.x_dtype, size_t(tok) * a.d, a.d, xs);
    __syncthreads();
    float* lg = a.logits + size_t(tok) * a.E;
    int e = warp;
    for (; e + 16 < int(a.E); e += 32) {             // rows e and e + 16 together
        float v0, v1;
        warp_row_dot_bf16_x2(a.w + size_t(e) * a.d, a.w + size_t(e + 16) * a.d, xs, a.d, lane, v0, v1);
        if (lane == 0) {
            lg[e] = v0;
            lg[e + 16] = v1;
        }
    }
    if (e < int(a.E)) {
        const float v = warp_row_dot_bf16(a.w + size_t(e) * a.d, xs, a.d, lane);
        if (lane == 0) lg[e] = v;
    }
    __threadfence_block();
    __syncthreads();
    if (warp == 0) warp_topk(lg, a.E, a.k, a.norm, a.ids + size_t(tok) * a.k, a.wts + size_t(tok) * a.k, lane);
}

// Plain bf16 GEMV y = W . x (metal_bridge.h:157), one warp per row.
__global__ void __launch_bounds__(256) k_gemv_bf16(const uint16_t* w, const float* x, float* y,
                                                   uint32_t rows, uint32_t cols) {
    extern __shared__ __align__(16) float xs[];
    for (uint32_t i = threadIdx.x; i < cols; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
        const float v = warp_row_dot_bf16(w + size_t(r) * cols, xs, cols, lane);
        if (lane == 0) y[r] = v;
    }
}

}  // namespace smoe
