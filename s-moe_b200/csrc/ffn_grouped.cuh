// ffn_grouped.cuh - expert-grouped 4-bit SwiGLU FFN for token batches (the
// batched-decode shape: hundreds of tokens, each expert routed ~16 of them).
//
// The per-slot path (ffn_q4.cuh) streams an expert's weights once per
// (token, expert) slot. Here the work is grouped by expert: a CTA owns 32
// (gate/up) or 64 (down) rows of one expert's matrices, loads that weight
// tile once and applies it to every token routed to the expert, four tokens
// per MMA (B columns 2t,
// 2t+1 = hi and lo halves of token t). The arithmetic is that of
// ffn_q4.cuh (exact fp16 operands q / 16q, activations split hi + lo with a
// per-vector power-of-two scale, per-group scale/bias epilogue), so results
// match the per-slot path to fp32 rounding. Launch sequence per layer:
//   k_group_slots   ids -> per-expert slot lists in slot order
//   k_build_tabs    x rows -> B-operand tables (once per token)
//   k_ffn_grouped<2> h[slot] = silu(g) * u for the expert's slots
//   k_build_tabs    h rows -> tables (once per slot)
//   k_ffn_grouped<1> y_slot = W_down . h[slot]
//   k_combine_slots y[t] = sum_j w[t,j] * y_slot[t*k+j] in rank order
//                   (product then sum, as axpy_f32 in decode.cpp:485-499)
#pragma once
#include "ffn_q4.cuh"

namespace smoe {

struct GroupedArgs {
    const uint8_t* base;          // vault-layout arena, expert e at base + e * stride
    uint64_t stride;
    uint64_t off[9];
    const uint32_t* list;         // [E][lcap] slots of each expert, slot order
    const uint32_t* count;        // [E]
    uint32_t lcap;                // list capacity per expert
    const uint2* tab;             // B tables of the input vectors [nvec][K/16][8]
    const float2* gs;             // their group sums [nvec][K/64]
    uint32_t tab_div;             // input vector of a slot = slot / tab_div (k for x, 1 for h)
    float* out;                   // gate/up: h [nslots][d_ff]; down: y_slot [nslots][d_model]
    uint32_t d_model, d_ff;
    uint32_t* err;
};

// B registers of group grp (4 k-steps) for this lane: column g (lane / 4)
// comes from vector g / 2, hi (g even) or lo (g odd) half.
SMOE_DEVINL void load_b4(const uint2* tabg, int grp, int lane, uint2* bs) {
    const int gr = lane >> 2, c = lane & 3;
#pragma unroll
    for (int s = 0; s < 4; ++s) bs[s] = tabg ? __ldg(tabg + (grp * 4 + s) * 8 + (gr & 1) * 4 + c) : make_uint2(0u, 0u);
}

// One 64-group of a 16-row tile against 4 vectors (B registers bs from
// load_b4): returns the group sums of rows lane/4 and lane/4 + 8 for vector
// lane % 4.
SMOE_DEVINL void group_mma4(const uint8_t* rowp, int rs, int grp, const uint2* bs, int lane, float& r0,
                            float& r8) {
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
            const uint32_t bb[2] = {bs[i * 2 + h].x, bs[i * 2 + h].y};
            mma_f16_16816(d, a, bb);
        }
    }
    r0 = d[0] + d[1];
    r8 = d[2] + d[3];
}

// Per-expert slot lists: one CTA (one warp) per expert, ballot compaction
// over the slots in order (deterministic); ids are read 16 per lane ahead of
// the ballots so the scan is not a chain of dependent loads.
__global__ void k_group_slots(const uint32_t* ids, uint32_t nslots, uint32_t* list, uint32_t* count,
                              uint32_t lcap) {
    const uint32_t e = blockIdx.x, lane = threadIdx.x;
    uint32_t n = 0;
    for (uint32_t b0 = 0; b0 < nslots; b0 += 32 * 16) {
        uint32_t v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            const uint32_t s = b0 + q * 32 + lane;
            v[q] = s < nslots ? __ldg(ids + s) : 0xffffffffu;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            const uint32_t s = b0 + q * 32 + lane;
            const bool mine = v[q] == e;
            const uint32_t m = __ballot_sync(0xffffffffu, mine);
            const uint32_t pos = n + __popc(m & ((1u << lane) - 1u));
            if (mine && pos < lcap) list[size_t(e) * lcap + pos] = s;
            n += __popc(m);
        }
    }
    if (lane == 0) count[e] = n < lcap ? n : lcap;
}

// B tables of n vectors (one CTA each): f32 or bf16 rows of K, row stride K.
__global__ void __launch_bounds__(256) k_build_tabs(const void* src, int bf16, uint32_t K, uint2* tab,
                                                    float2* gs) {
    extern __shared__ __align__(16) float2 part[];            // [K/4]
    const size_t v = blockIdx.x;
    uint2* t = tab + v * (K / 16) * 8;
    float2* g = gs + v * (K / 64);
    if (bf16) {
        const uint16_t* xv = static_cast<const uint16_t*>(src) + v * K;
        build_btab([&](int i) { return bf16_bits_to_f32(xv[i]); }, int(K), t, g, part);
    } else {
        const float* xv = static_cast<const float*>(src) + v * K;
        build_btab([&](int i) { return xv[i]; }, int(K), t, g, part);
    }
}

// Shared layout of a grouped CTA: tile [mats][rb][rs] nibbles (rows padded
// by 32 B: conflict-free fragment loads), scales/biases [mats][2][rb * G].
inline size_t grouped_smem_bytes(int K, int mats, int rb) {
    const int rs = K / 2 + 32, G = K / 64;
    return size_t(mats * rb * rs) + size_t(mats) * 2 * rb * G * 2 + 16;
}

// MATS = 2: gate + up rows (K = d_model) -> h; MATS = 1: down rows (K = d_ff)
// -> y_slot. grid (rows / RB, E), 256 threads. A warp task is (16-row tile,
// chunk of 4 of the expert's vectors) over all K groups, so results are
// complete inside the warp: no CTA barrier and no cross-warp reduction in
// the token loop.
template <int FMT, int MATS, int RB>
__global__ void __launch_bounds__(256) k_ffn_grouped(GroupedArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t e = blockIdx.y, T = a.count[e];
    if (T == 0) return;
    const int K = MATS == 2 ? a.d_model : a.d_ff, R = MATS == 2 ? a.d_ff : a.d_model;
    const int blk = blockIdx.x, rs = K / 2 + 32, G = K / 64, nsb = RB * G;
    uint8_t* wt = smem;                                                 // [MATS][RB][rs]
    uint16_t* sb = reinterpret_cast<uint16_t*>(wt + MATS * RB * rs);    // [MATS][2][nsb]
    uint64_t* bar = reinterpret_cast<uint64_t*>(sb + MATS * 2 * nsb);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gr = lane >> 2, c = lane & 3;
    const uint8_t* eb = a.base + uint64_t(e) * a.stride;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t sbytes = nsb * 2;
        const uint32_t total = MATS * RB * (K / 2) + MATS * (FMT == kFmtAffine ? 2 : 1) * sbytes;
        if (lane == 0) mbar_arrive_expect_tx(bar, total);
        __syncwarp();
        const int m0 = MATS == 2 ? 0 : 2;
        for (int i = lane; i < MATS * RB; i += 32) {
            const int m = i / RB, r = i % RB;
            bulk_g2s(wt + (m * RB + r) * rs, eb + a.off[3 * (m0 + m)] + size_t(blk * RB + r) * (K / 2), K / 2, bar);
        }
        if (lane < MATS)
            bulk_g2s(sb + (lane * 2) * nsb, eb + a.off[3 * (m0 + lane) + 1] + size_t(blk) * sbytes, sbytes, bar);
        if (FMT == kFmtAffine && lane >= 2 && lane < 2 + MATS)
            bulk_g2s(sb + ((lane - 2) * 2 + 1) * nsb, eb + a.off[3 * (m0 + lane - 2) + 2] + size_t(blk) * sbytes,
                     sbytes, bar);
    }
    if (!mbar_wait_bounded(bar, 0)) {
        if (tid == 0) atomicExch(a.err, SMOE_DEVERR_MBAR_TIMEOUT);
        return;
    }
    const uint32_t* lst = a.list + size_t(e) * a.lcap;
    const int nchunk = int((T + 3) / 4), ntask = (RB / 16) * nchunk;
    for (int task = warp; task < ntask; task += 8) {
        const int tile = task % (RB / 16), c0 = (task / (RB / 16)) * 4;
        const uint32_t tb = c0 + (gr >> 1), tc = c0 + c;
        const uint2* tabg = tb < T ? a.tab + size_t(lst[tb] / a.tab_div) * (K / 16) * 8 : nullptr;
        const float2* gsv = tc < T ? a.gs + size_t(lst[tc] / a.tab_div) * G : nullptr;
        float acc[MATS][2];
#pragma unroll
        for (int m = 0; m < MATS; ++m) acc[m][0] = acc[m][1] = 0.f;
        // four groups at a time: their 16 B loads and 4 group sums are in
        // flight together (the tables come from L2), then their MMAs
        for (int g0 = 0; g0 < G; g0 += 4) {
            uint2 bs[4][4];
            float2 gsum[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int grp = min(g0 + q, G - 1);
                load_b4(tabg, grp, lane, bs[q]);
                gsum[q] = gsv ? __ldg(gsv + grp) : make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int grp = g0 + q;
                if (grp < G) {
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        float r0, r8;
                        group_mma4(wt + (m * RB + tile * 16) * rs, rs, grp, bs[q], lane, r0, r8);
                        const uint16_t* sc = sb + (m * 2) * nsb;
                        const uint16_t* bi = sb + (m * 2 + 1) * nsb;
                        acc[m][0] += group_epilogue<FMT>(r0, gsum[q], sc, bi, (tile * 16 + gr) * G + grp);
                        acc[m][1] += group_epilogue<FMT>(r8, gsum[q], sc, bi, (tile * 16 + gr + 8) * G + grp);
                    }
                }
            }
        }
        if (tc < T) {
            float* o = a.out + size_t(lst[tc]) * R + blk * RB + tile * 16 + gr;
            if (MATS == 2) {
                o[0] = acc[0][0] * (1.0f / (1.0f + expf(-acc[0][0]))) * acc[1][0];   // kernels.metal:61-63
                o[8] = acc[0][1] * (1.0f / (1.0f + expf(-acc[0][1]))) * acc[MATS - 1][1];
            } else {
                o[0] = acc[0][0];
                o[8] = acc[0][1];
            }
        }
    }
}

// y[t] = sum_j w[t*k+j] * ys[t*k+j] in rank order j (axpy_f32: product, then
// sum). grid (ceil(d/256), ntok).
__global__ void k_combine_slots(const float* ys, const float* wts, uint32_t k, uint32_t d, void* y,
                                int y_dtype) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (i >= d) return;
    float acc = 0.f;
    for (uint32_t j = 0; j < k; ++j)
        acc = __fadd_rn(acc, __fmul_rn(wts[t * k + j], ys[size_t(t * k + j) * d + i]));
    if (y_dtype == 0) static_cast<float*>(y)[size_t(t) * d + i] = acc;
    else static_cast<__nv_bfloat16*>(y)[size_t(t) * d + i] = __float2bfloat16_rn(acc);
}

}  // namespace smoe
