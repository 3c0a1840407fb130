// ffn_q4.cuh - fused 4-bit SwiGLU expert FFN for decode (sm_100a).
//
// Computes, per (token, routed expert) "slot":
//   h = silu(W_gate . x) * (W_up . x)            (kernels.metal:240-337)
//   y = W_down . h                                (kernels.metal:159-235, 340-365)
// and combines y over the k slots of a token in rank order,
//   out = sum_j w_j * y_j                          (decode.cpp:485-499)
//
// Arithmetic. A 4-bit code q is turned into an fp16 operand by one LOP3
// that ORs it into the mantissa of 1024.0 (0x6400): codes at bits 0-3 of a
// half word become 1024+q, codes at bits 4-7 become 1024+16q; one packed
// fp16 subtraction of 1024 leaves the exact q or 16q, so no large offset is
// left to cancel inside the fp32 accumulator. The matching activation slots
// of the B operand carry x or x/16, so the tensor core sums q.x. The activation is split
// into two fp16 halves x = hi + lo held in two B columns, so the product is
// accumulated at ~fp32 quality in fp32. Per 64-element group g:
//     sum_k w_k x_k = scale_g * D_g + bias_g * sum_g(x)
// with (scale, bias) = (bf16 scale, bf16 bias) for AFFINE-Q4 and
// (s/7.5, -s) for SMOE-Q4 (the same identity kernels.metal:136-143 uses).
//
// Within each 16-wide MMA k-step the 16 K positions may be permuted freely
// as long as A and B agree; lane (g = lane/4, c = lane%4) reads 8 bytes of a
// group (bytes 8c..8c+7 of its 32) from rows g and g+8, and the B table is
// laid out in the same permuted order (see build_btab).
#pragma once
#include "smoe_common.cuh"

namespace smoe {

constexpr int kFmtSmoe = 0;
constexpr int kFmtAffine = 1;
constexpr int kMaxSlotsPtr = 16;

struct FfnArgs {
    // Weights, table mode: expert e = ids[slot] at base + e * stride + off[].
    const uint8_t*  base;
    uint64_t        stride;
    uint64_t        off[9];
    const uint32_t* ids;                   // device [ntok * k]; null -> pointer mode
    // Weights, pointer mode: per "expert column" j = slot % k.
    const uint8_t*  p_nib[kMaxSlotsPtr][3];
    const uint16_t* p_sc[kMaxSlotsPtr][3];
    const uint16_t* p_bi[kMaxSlotsPtr][3];
    const float*    wts;                   // device [ntok * k] combine weights
    const void*     x;                     // [ntok x d_model]
    int             x_dtype;               // 0 f32, 1 bf16
    float*          hidden;                // scratch [ntok * k x d_ff]
    void*           y;                     // combine: [ntok x d_model]; per-slot: [ntok*k x d_model] f32
    int             y_dtype;
    int             per_slot;              // 1 -> write each slot's y (mirror API)
    uint32_t        d_model, d_ff, k, ntok;
    uint32_t        n_experts;             // table mode: ids >= n_experts are rejected
    uint32_t*       err;
};

struct SlotW {
    const uint8_t* nib[3];
    const uint16_t* sc[3];
    const uint16_t* bi[3];
};

SMOE_DEVINL SlotW slot_weights(const FfnArgs& a, uint32_t slot) {
    SlotW w;
    if (a.ids) {
        uint32_t e = a.ids[slot];
        if (e >= a.n_experts) {           // never index past the arena: flag it, read expert 0
            atomicCAS(a.err, 0u, uint32_t(SMOE_DEVERR_BAD_EXPERT));
            e = 0;
        }
        const uint8_t* b = a.base + uint64_t(e) * a.stride;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
            w.nib[m] = b + a.off[3 * m];
            w.sc[m] = reinterpret_cast<const uint16_t*>(b + a.off[3 * m + 1]);
            w.bi[m] = reinterpret_cast<const uint16_t*>(b + a.off[3 * m + 2]);
        }
    } else {
        uint32_t j = slot % a.k;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
            w.nib[m] = a.p_nib[j][m];
            w.sc[m] = a.p_sc[j][m];
            w.bi[m] = a.p_bi[j][m];
        }
    }
    return w;
}

// ---------------------------------------------------------------- B table
// For a K-vector v: btab[(grp*4 + s)*8 + lane8] (uint2 = the two B regs of
// lanes 0..7 of the MMA at k-step s of group grp; lanes 0-3 hold the hi
// column, 4-7 the lo column), and gsum[grp] = (1/scale, sum of scale*x over
// the group as the MMA sees it, hi + lo). The vector is multiplied by a power
// of two `scale` first; the epilogue multiplies the group result by 1/scale.
// `part` scratch: K/4 float2. Must be followed by __syncthreads() (inside).
// Power-of-two factor that brings max|v| to [2^13, 2^14): keeps the fp16
// halves of small vectors (e.g. SiLU outputs ~1e-3) out of the subnormals.
SMOE_DEVINL float pow2_scale_for(float amax) {
    if (!(amax > 0.0f) || !isfinite(amax)) return 1.0f;
    int e;
    frexpf(amax, &e);                        // amax in [2^(e-1), 2^e)
    return ldexpf(1.0f, 14 - e);
}

// Table layouts. kTabSlot: the per-slot kernels' [g][k-step][hi 4 c, lo 4 c]
// uint2 entries. kTabMma: the grouped mma.sync kernel's - per (group,
// k-step, c) one 16-byte entry {hi.x, hi.y, lo.x, lo.y}; the hi pair alone
// is the A-fragment pair of one token in a 16-token MMA. kTabTc: the
// tensor-core kernel's - per (group g, 8-column chunk kc) a hi and a lo
// 16-byte row of fp16, [g][kc][hi, lo][8], each in the order in which one
// 32-bit word of 4-bit codes dequantises (columns 0, 4, 1/16, 5/16, 2, 6,
// 3/16, 7/16 of the chunk, the odd ones pre-divided by 16 as their codes
// come out as 16 q): B-operand rows of a tcgen05 MMA against codes
// dequantised that way. lo_flag (grouped layouts) gets a nonzero word if
// any lo half of this vector is nonzero.
constexpr int kTabSlot = 0, kTabMma = 1, kTabTc = 2;
template <int LAYOUT = kTabSlot, typename Load>
SMOE_DEVINL void build_btab(Load ld, int K, uint2* btab, float2* gsum, float2* part,
                            uint32_t* lo_flag = nullptr) {
    // Tuple t (4 columns: base + {0, 4, 1, 5}) of a 64-group; the tuples
    // cover every column once. Up to kCache tuples per thread are read once
    // and kept in registers for both passes (max, then the split).
    const int ntup = K / 4;
    auto tbase = [](int t) {
        const int grp = t >> 4, r = t & 15, s = r >> 2, c = r & 3;
        return grp * 64 + c * 16 + (s >> 1) * 8 + (s & 1) * 2;
    };
    constexpr int kCache = 4;
    const bool cached = ntup <= kCache * int(blockDim.x);
    float cv[kCache][4];
    float amax = 0.0f;
    if (cached) {
#pragma unroll
        for (int j = 0; j < kCache; ++j) {
            const int t = threadIdx.x + j * blockDim.x;
            if (t < ntup) {
                const int base = tbase(t);
                cv[j][0] = ld(base); cv[j][1] = ld(base + 4); cv[j][2] = ld(base + 1); cv[j][3] = ld(base + 5);
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(cv[j][0]), fabsf(cv[j][1])), fmaxf(fabsf(cv[j][2]), fabsf(cv[j][3]))));
            }
        }
    } else {
        for (int i = threadIdx.x; i < K; i += blockDim.x) amax = fmaxf(amax, fabsf(ld(i)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5].x = amax;
    __syncthreads();
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) amax = fmaxf(amax, part[w].x);
    __syncthreads();
    const float sc = pow2_scale_for(amax), inv = 1.0f / sc;
    auto emit = [&](int t, float v0, float v4, float v1, float v5) {
        const int grp = t >> 4, r = t & 15, s = r >> 2, c = r & 3;
        float e0 = v0 * sc, e4 = v4 * sc;
        float o1 = v1 * (sc * 0.0625f), o5 = v5 * (sc * 0.0625f);
        __half he0 = __float2half_rn(e0), he4 = __float2half_rn(e4);
        __half le0 = __float2half_rn(e0 - __half2float(he0));
        __half le4 = __float2half_rn(e4 - __half2float(he4));
        __half ho1 = __float2half_rn(o1), ho5 = __float2half_rn(o5);
        __half lo1 = __float2half_rn(o1 - __half2float(ho1));
        __half lo5 = __float2half_rn(o5 - __half2float(ho5));
        const int row = (grp * 4 + s) * 8;
        if (LAYOUT == kTabMma) {
            const uint32_t l0 = pack_half2(le0, le4), l1 = pack_half2(lo1, lo5);
            reinterpret_cast<uint4*>(btab)[row / 2 + c] = make_uint4(pack_half2(he0, he4), pack_half2(ho1, ho5), l0, l1);
            if (lo_flag && ((l0 | l1) & 0x7fff7fffu)) atomicOr(lo_flag, 1u);
        } else if (LAYOUT == kTabTc) {
            // tuple (s, c) holds columns base + {0, 4, 1, 5}: 8 bytes of chunk
            // kc = 2c + s/2, at byte 8 (s & 1)
            const uint32_t l0 = pack_half2(le0, le4), l1 = pack_half2(lo1, lo5);
            uint2* ch = btab + (size_t(grp * 8 + 2 * c + (s >> 1)) * 2) * 2 + (s & 1);
            ch[0] = make_uint2(pack_half2(he0, he4), pack_half2(ho1, ho5));
            ch[2] = make_uint2(l0, l1);
            if (lo_flag && ((l0 | l1) & 0x7fff7fffu)) atomicOr(lo_flag, 1u);
        } else {
            btab[row + c] = make_uint2(pack_half2(he0, he4), pack_half2(ho1, ho5));
            btab[row + 4 + c] = make_uint2(pack_half2(le0, le4), pack_half2(lo1, lo5));
        }
        float x0 = __half2float(he0) + __half2float(le0);
        float x4 = __half2float(he4) + __half2float(le4);
        float x1 = 16.0f * (__half2float(ho1) + __half2float(lo1));
        float x5 = 16.0f * (__half2float(ho5) + __half2float(lo5));
        part[t] = make_float2(0.0f, (x0 + x4) + (x1 + x5));
    };
    if (cached) {
#pragma unroll
        for (int j = 0; j < kCache; ++j) {
            const int t = threadIdx.x + j * blockDim.x;
            if (t < ntup) emit(t, cv[j][0], cv[j][1], cv[j][2], cv[j][3]);
        }
    } else {
        for (int t = threadIdx.x; t < ntup; t += blockDim.x) {
            const int base = tbase(t);
            emit(t, ld(base), ld(base + 4), ld(base + 1), ld(base + 5));
        }
    }
    __syncthreads();
    for (int grp = threadIdx.x; grp < K / 64; grp += blockDim.x) {
        float cs = 0.f, xs = 0.f;
        for (int i = 0; i < 16; ++i) {
            float2 p = part[grp * 16 + i];
            cs += p.x;
            xs += p.y;
        }
        gsum[grp] = make_float2(inv, xs);
    }
    __syncthreads();
}

// One 64-wide group of one 16-row tile: 4 MMAs, returns the group sums of
// rows (lane/4) and (lane/4 + 8) for the token held in column pair 0/1
// (valid in lanes with lane%4 == 0).
//   rowp: shared-memory tile, row stride rs bytes; grp: group index.
SMOE_DEVINL void group_mma(const uint8_t* rowp, int rs, int grp, const uint2* btab,
                           int lane, float& r0, float& r8) {
    const int gr = lane >> 2, c = lane & 3;
    const uint2 w = *reinterpret_cast<const uint2*>(rowp + gr * rs + grp * 32 + c * 8);
    const uint2 v = *reinterpret_cast<const uint2*>(rowp + (gr + 8) * rs + grp * 32 + c * 8);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u, OR = 0x64006400u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t wg = i ? w.y : w.x, wh = i ? v.y : v.x;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t g8 = h ? (wg >> 8) : wg, h8 = h ? (wh >> 8) : wh;
            uint32_t a[4];
            a[0] = hsub_1024(lop3_and_or(g8, M0, OR));
            a[1] = hsub_1024(lop3_and_or(h8, M0, OR));
            a[2] = hsub_1024(lop3_and_or(g8, M1, OR));
            a[3] = hsub_1024(lop3_and_or(h8, M1, OR));
            uint2 b = make_uint2(0u, 0u);
            if (lane < 8) b = btab[(grp * 4 + i * 2 + h) * 8 + lane];
            uint32_t bb[2] = {b.x, b.y};
            mma_f16_16816(d, a, bb);
        }
    }
    r0 = d[0] + d[1];
    r8 = d[2] + d[3];
}

template <int FMT>
SMOE_DEVINL float group_epilogue(float dsum, float2 gs, const uint16_t* sc, const uint16_t* bi,
                                 int idx) {
    if (FMT == kFmtAffine) {
        const float s = bf16_bits_to_f32(sc[idx]), b = bf16_bits_to_f32(bi[idx]);
        return (s * dsum + b * gs.y) * gs.x;
    } else {
        const float s = f16_bits_to_f32(sc[idx]);
        return s * (dsum * (1.0f / 7.5f) - gs.y) * gs.x;
    }
}

// --------------------------------------------------------- gate+up kernel
// grid (d_ff/16, ntok*k), 256 threads. One CTA = 16 hidden rows of one slot.
template <int FMT>
__global__ void __launch_bounds__(256) k_gate_up(FfnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int d = a.d_model, tile = blockIdx.x, slot = blockIdx.y;
    const int rs = d / 2 + 32, G = d / 64, nsb = 16 * G;
    uint8_t* wt = smem;                                              // [2][16][rs]
    uint16_t* sb = reinterpret_cast<uint16_t*>(wt + 2 * 16 * rs);    // [2][2][nsb]
    uint2* btab = reinterpret_cast<uint2*>(sb + 4 * nsb);            // [d/16][8]
    float2* gsum = reinterpret_cast<float2*>(btab + (d / 16) * 8);   // [G]
    float2* part = gsum + G;                                         // [d/4]
    float* red = reinterpret_cast<float*>(part + d / 4);             // [8][2][16]
    uint64_t* bar = reinterpret_cast<uint64_t*>(red + 256);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const SlotW W = slot_weights(a, slot);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t sbytes = nsb * 2;
        const uint32_t total = 2 * 16 * (d / 2) + (FMT == kFmtAffine ? 4 : 2) * sbytes;
        if (lane == 0) mbar_arrive_expect_tx(bar, total);
        __syncwarp();
        const int m = lane >> 4, r = lane & 15;
        bulk_g2s(wt + (m * 16 + r) * rs, W.nib[m] + size_t(tile * 16 + r) * (d / 2), d / 2, bar);
        if (lane < 2)
            bulk_g2s(sb + (lane * 2) * nsb, W.sc[lane] + size_t(tile) * nsb, sbytes, bar);
        if (FMT == kFmtAffine && lane >= 2 && lane < 4)
            bulk_g2s(sb + ((lane - 2) * 2 + 1) * nsb, W.bi[lane - 2] + size_t(tile) * nsb, sbytes, bar);
    }
    // Activation table, overlapped with the copies.
    const uint32_t tok = slot / a.k;
    if (a.x_dtype == 0) {
        const float* xv = static_cast<const float*>(a.x) + size_t(tok) * d;
        build_btab([&](int i) { return xv[i]; }, d, btab, gsum, part);
    } else {
        const uint16_t* xv = static_cast<const uint16_t*>(a.x) + size_t(tok) * d;
        build_btab([&](int i) { return bf16_bits_to_f32(xv[i]); }, d, btab, gsum, part);
    }
    if (!mbar_wait_bounded(bar, 0)) {
        if (tid == 0) atomicExch(a.err, SMOE_DEVERR_MBAR_TIMEOUT);
        return;
    }
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};   // [mat][row g / g+8]
    const int gr = lane >> 2;
    for (int grp = warp; grp < G; grp += 8) {
        const float2 gs = gsum[grp];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            float r0, r8;
            group_mma(wt + m * 16 * rs, rs, grp, btab, lane, r0, r8);
            const uint16_t* sc = sb + (m * 2) * nsb;
            const uint16_t* bi = sb + (m * 2 + 1) * nsb;
            acc[m][0] += group_epilogue<FMT>(r0, gs, sc, bi, gr * G + grp);
            acc[m][1] += group_epilogue<FMT>(r8, gs, sc, bi, (gr + 8) * G + grp);
        }
    }
    if ((lane & 3) == 0) {
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            red[(warp * 2 + m) * 16 + gr] = acc[m][0];
            red[(warp * 2 + m) * 16 + gr + 8] = acc[m][1];
        }
    }
    __syncthreads();
    if (tid < 16) {
        float g = 0.f, u = 0.f;
        for (int w = 0; w < 8; ++w) {
            g += red[(w * 2 + 0) * 16 + tid];
            u += red[(w * 2 + 1) * 16 + tid];
        }
        const float hval = g * (1.0f / (1.0f + expf(-g))) * u;     // kernels.metal:61-63
        a.hidden[size_t(slot) * a.d_ff + tile * 16 + tid] = hval;
    }
}

inline size_t gate_up_smem_bytes(int d) {
    const int rs = d / 2 + 32, G = d / 64;
    return size_t(2 * 16 * rs) + 4 * 16 * G * 2 + (d / 16) * 8 * 8 + G * 8 + (d / 4) * 8 + 256 * 4 + 16;
}

// ------------------------------------------------- down + combine kernel
// grid (d_model/16, ntok), 256 threads. One CTA = 16 output rows of one
// token, all k slots (in chunks of 8), combined in rank order.
constexpr int kDownChunk = 8;

template <int FMT>
__global__ void __launch_bounds__(256) k_down_combine(FfnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int dff = a.d_ff, tile = blockIdx.x, tok = blockIdx.y;
    const int rs = dff / 2 + 32, G = dff / 64, nsb = 16 * G, S = dff / 16;
    uint8_t* wt = smem;                                                       // [8][16][rs]
    uint16_t* sb = reinterpret_cast<uint16_t*>(wt + kDownChunk * 16 * rs);     // [8][2][nsb]
    uint2* btab = reinterpret_cast<uint2*>(sb + kDownChunk * 2 * nsb);         // [8][S][8]
    float2* gsum = reinterpret_cast<float2*>(btab + kDownChunk * S * 8);       // [8][G]
    float2* part = gsum + kDownChunk * G;                                      // [dff/4]
    float* ys = reinterpret_cast<float*>(part + dff / 4);                      // [8][16]
    uint64_t* bar = reinterpret_cast<uint64_t*>(ys + kDownChunk * 16);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gr = lane >> 2;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    float outacc = 0.f;
    const uint32_t k = a.k;
    uint32_t phase = 0;
    for (uint32_t j0 = 0; j0 < k; j0 += kDownChunk, phase ^= 1) {
        const int nj = min(kDownChunk, int(k - j0));
        if (warp == 0) {
            const uint32_t sbytes = nsb * 2;
            const uint32_t total = nj * (16 * (dff / 2) + (FMT == kFmtAffine ? 2 : 1) * sbytes);
            if (lane == 0) mbar_arrive_expect_tx(bar, total);
            __syncwarp();
            for (int jj = 0; jj < nj; ++jj) {
                const SlotW W = slot_weights(a, tok * k + j0 + jj);
                if (lane < 16)
                    bulk_g2s(wt + (jj * 16 + lane) * rs,
                             W.nib[2] + size_t(tile * 16 + lane) * (dff / 2), dff / 2, bar);
                else if (lane == 16)
                    bulk_g2s(sb + (jj * 2) * nsb, W.sc[2] + size_t(tile) * nsb, sbytes, bar);
                else if (FMT == kFmtAffine && lane == 17)
                    bulk_g2s(sb + (jj * 2 + 1) * nsb, W.bi[2] + size_t(tile) * nsb, sbytes, bar);
            }
        }
        for (int jj = 0; jj < nj; ++jj) {
            const float* hv = a.hidden + size_t(tok * k + j0 + jj) * dff;
            build_btab([&](int i) { return hv[i]; }, dff, btab + jj * S * 8, gsum + jj * G, part);
        }
        if (!mbar_wait_bounded(bar, phase)) {
            if (tid == 0) atomicExch(a.err, SMOE_DEVERR_MBAR_TIMEOUT);
            return;
        }
        if (warp < nj) {
            const int jj = warp;
            float y0 = 0.f, y8 = 0.f;
            const uint16_t* sc = sb + (jj * 2) * nsb;
            const uint16_t* bi = sb + (jj * 2 + 1) * nsb;
            for (int grp = 0; grp < G; ++grp) {
                float r0, r8;
                group_mma(wt + jj * 16 * rs, rs, grp, btab + jj * S * 8, lane, r0, r8);
                const float2 gs = gsum[jj * G + grp];
                y0 += group_epilogue<FMT>(r0, gs, sc, bi, gr * G + grp);
                y8 += group_epilogue<FMT>(r8, gs, sc, bi, (gr + 8) * G + grp);
            }
            if ((lane & 3) == 0) {
                ys[jj * 16 + gr] = y0;
                ys[jj * 16 + gr + 8] = y8;
            }
        }
        __syncthreads();
        if (tid < 16) {
            const int row = tile * 16 + tid;
            for (int jj = 0; jj < nj; ++jj) {
                const uint32_t slot = tok * k + j0 + jj;
                const float yv = ys[jj * 16 + tid];
                if (a.per_slot) {
                    static_cast<float*>(a.y)[size_t(slot) * a.d_model + row] = yv;
                } else {
                    // routed[i] += w * y[i]: a product then a sum, no FMA (axpy_f32)
                    outacc = __fadd_rn(outacc, __fmul_rn(a.wts[slot], yv));
                }
            }
        }
        __syncthreads();   // smem reuse by the next chunk
    }
    if (!a.per_slot && tid < 16) {
        const size_t o = size_t(tok) * a.d_model + tile * 16 + tid;
        if (a.y_dtype == 0) static_cast<float*>(a.y)[o] = outacc;
        else static_cast<__nv_bfloat16*>(a.y)[o] = __float2bfloat16_rn(outacc);
    }
}

inline size_t down_smem_bytes(int dff) {
    const int rs = dff / 2 + 32, G = dff / 64, S = dff / 16;
    return size_t(kDownChunk) * 16 * rs + kDownChunk * 2 * 16 * G * 2 + kDownChunk * S * 64 +
           kDownChunk * G * 8 + (dff / 4) * 8 + kDownChunk * 16 * 4 + 16;
}

}  // namespace smoe
