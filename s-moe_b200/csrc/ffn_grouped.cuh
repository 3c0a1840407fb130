// ffn_grouped.cuh - expert-grouped 4-bit SwiGLU FFN for token batches (the
// batched-decode shape: hundreds of tokens, each expert routed ~16 of them).
//
// The per-slot path (ffn_q4.cuh) streams an expert's weights once per
// (token, expert) slot. Here the work is grouped by expert: a CTA owns a
// block of rows of one expert's matrices, loads that weight tile once and
// applies it to every token routed to the expert. The arithmetic is that of
// ffn_q4.cuh (exact fp16 operands q / 16 q, activations split hi + lo with a
// per-vector power-of-two scale, per-group scale/bias epilogue), so results
// match the per-slot path to fp32 rounding. Launch sequence per layer:
//   k_group_slots        ids -> per-expert slot lists in slot order
//   k_build_tabs<Mma>    x rows -> B-operand tables (once per token)
//   k_ffn_grouped<.., 2> gate/up with mma.sync, token-major:
//                        h[slot] = silu(g) * u for the expert's slots
//   k_build_tabs<Tc>     h rows -> tables (once per slot)
//   k_ffn_down_tc        down with tcgen05: y_slot = W_down . h[slot]
//   k_combine_slots      y[t] = sum_j w[t,j] * y_slot[t*k+j] in rank order
//                        (product then sum, as axpy_f32 in decode.cpp:485-499)
#pragma once
#include <type_traits>
#include "ffn_q4.cuh"
#include "tc05.cuh"

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
    const uint32_t* lo_flag;      // 0: every table's lo halves are zero (16-token MMAs); null: 8
    float* out;                   // gate/up: h [nslots][d_ff]; down: y_slot [nslots][d_model]
    uint32_t d_model, d_ff;
    uint32_t* err;
};

// Per-expert slot lists: one CTA (one warp) per expert, ballot compaction
// over the slots in order (deterministic); ids are read 16 per lane, one
// 512-slot round ahead of the ballots, so the scan is not a chain of loads.
// Also clears the lo flag that the following k_build_tabs of x sets.
// Expert-parallel shard (base > 0 or e_total > gridDim.x): the lists hold
// the slots of experts [base, base + gridDim.x); other slots belong to
// other ranks and are left out; ids >= e_total are errors.
__global__ void k_group_slots(const uint32_t* ids, uint32_t nslots, uint32_t* list, uint32_t* count,
                              uint32_t lcap, uint32_t* lo_flag, uint32_t* err, uint32_t base, uint32_t e_total) {
    const uint32_t e = blockIdx.x, lane = threadIdx.x;
    if (e == 0 && lane == 0 && lo_flag) *lo_flag = 0u;
    uint32_t n = 0;
    uint32_t nx[16];                                   // ids of the next round, loaded ahead
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        const uint32_t s = q * 32 + lane;
        nx[q] = s < nslots ? __ldg(ids + s) : 0xffffffffu;
    }
    for (uint32_t b0 = 0; b0 < nslots; b0 += 32 * 16) {
        uint32_t v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            v[q] = nx[q];
            const uint32_t s = b0 + 512 + q * 32 + lane;
            nx[q] = s < nslots ? __ldg(ids + s) : 0xffffffffu;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            const uint32_t s = b0 + q * 32 + lane;
            const bool mine = v[q] - base == e;             // (unsigned: ids below base wrap past the shard)
            if (e == 0 && s < nslots && v[q] >= e_total)      // an id past the layer's experts: no list takes it
                atomicCAS(err, 0u, uint32_t(SMOE_DEVERR_BAD_EXPERT));
            const uint32_t m = __ballot_sync(0xffffffffu, mine);
            const uint32_t pos = n + __popc(m & ((1u << lane) - 1u));
            if (mine && pos < lcap) list[size_t(e) * lcap + pos] = s;
            n += __popc(m);
        }
    }
    if (lane == 0) count[e] = n < lcap ? n : lcap;
}

// B tables of n vectors (one CTA each): f32 or bf16 rows of K, row stride K.
// LAYOUT: kTabMma for the x tables the gate/up kernel reads, kTabTc for
// the hidden-vector tables of the tensor-core down kernel.
template <int LAYOUT>
__global__ void __launch_bounds__(256) k_build_tabs(const void* src, int bf16, uint32_t K, uint2* tab,
                                                    float2* gs, uint32_t* lo_flag) {
    extern __shared__ __align__(16) float2 part[];            // [K/4]
    const size_t v = blockIdx.x;
    uint2* t = tab + v * (K / 16) * 8;
    float2* g = gs + v * (K / 64);
    if (bf16) {
        const uint16_t* xv = static_cast<const uint16_t*>(src) + v * K;
        build_btab<LAYOUT>([&](int i) { return bf16_bits_to_f32(xv[i]); }, int(K), t, g, part, lo_flag);
    } else {
        const float* xv = static_cast<const float*>(src) + v * K;
        build_btab<LAYOUT>([&](int i) { return xv[i]; }, int(K), t, g, part, lo_flag);
    }
}

// Shared layout of a grouped CTA: weight tile [MATS][RB][rs] nibbles (rows
// padded by 32 B: conflict-free fragment loads), the scales/biases in the
// lanes' order [MATS][2][G][WN][c][NTW][2], one region holding first the
// scales/biases as copied [MATS][2][RB][G] and afterwards the split-K
// partial sums [8 warps][accumulators][32 lanes] of one token chunk, and
// the first kSlotCache entries of the expert's slot list.
constexpr int kSlotCache = 256;
__host__ __device__ inline size_t grouped_union_bytes(int K, int mats, int rb, int wn) {
    const size_t sbb = size_t(mats) * 2 * rb * (K / 64) * 2;
    const size_t redb = size_t(8) * mats * (rb / 8 / wn) * 4 * 32 * 4;      // 16-token chunks
    return sbb > redb ? sbb : redb;
}
inline size_t grouped_smem_bytes(int K, int mats, int rb, int wn) {
    const int rs = K / 2 + 32, G = K / 64;
    return size_t(mats * rb * rs) + size_t(mats) * 2 * rb * G * 2 + grouped_union_bytes(K, mats, rb, wn) +
           kSlotCache * 4 + 16;
}

// MATS = 2: gate + up rows (K = d_model) -> h; MATS = 1: down rows (K = d_ff)
// -> y_slot. grid (rows / RB, E), 256 threads = WK k-slices x WN row slices.
// Token-major MMAs: M rows = tokens, N columns = 8 weight rows, so one
// dequantised weight fragment (2 registers; one 8-byte shared load covers
// 4 k-steps) serves every token of the MMA. Two row modes:
//   16 tokens (rows g and g+8 = two tokens) when every input vector of the
//     batch is exact in fp16 after its power-of-two scale (lo halves all
//     zero, flagged by k_build_tabs: any bf16 input with a dynamic range
//     below 2^27);
//   8 tokens (rows g = hi halves, g+8 = lo halves of the same tokens;
//     d0 + d2, d1 + d3 add them) otherwise - the fp32 hidden vectors.
// Lane (g, c) holds weight rows 2c, 2c+1 of each of its NTW n-tiles. Each
// warp runs its 64-groups for all NTW n-tiles of every matrix, so an x
// fragment is loaded once per CTA and feeds MATS * NTW MMAs; a warp's
// (chunk, group) items form one software pipeline whose loads run ahead
// across chunk boundaries; the WK partial sums are added in shared memory in
// k-slice order (fixed order: deterministic), with SiLU(gate) * up or the
// down output written there. Group epilogue as group_epilogue, the
// per-vector scale gs.x applied once at the end.
// KC: K when known at compile time (0: read from the arguments), which makes
// every shared-memory offset of the inner loop an immediate.
template <int FMT, int MATS, int RB, int WN, int KC>
__global__ void __launch_bounds__(256, 2) k_ffn_grouped(GroupedArgs a) {
    constexpr int WK = 8 / WN, NTW = RB / 8 / WN;
    static_assert(NTW % 4 == 0, "scale rows are read 8 at a time");
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t e = blockIdx.y, T = a.count[e];
    if (T == 0) return;
    const int K = KC ? KC : (MATS == 2 ? int(a.d_model) : int(a.d_ff)), R = MATS == 2 ? a.d_ff : a.d_model;
    const int blk = blockIdx.x, rs = K / 2 + 32, G = K / 64, nsb = RB * G;
    uint8_t* wt = smem;                                                 // [MATS][RB][rs]
    uint16_t* st = reinterpret_cast<uint16_t*>(wt + MATS * RB * rs);    // [MATS][2][G][WN][4][NTW][2]
    uint16_t* sb = st + MATS * 2 * nsb;                                 // [MATS][2][RB][G], then:
    float* red = reinterpret_cast<float*>(sb);                          // [8][acc][32]
    uint32_t* sl = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(sb) + grouped_union_bytes(K, MATS, RB, WN));
    uint64_t* bar = reinterpret_cast<uint64_t*>(sl + kSlotCache);
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
    const uint32_t* lst = a.list + size_t(e) * a.lcap;
    for (uint32_t i = tid; i < T && i < uint32_t(kSlotCache); i += 256) sl[i] = lst[i];
    const bool hi_only = a.lo_flag && *a.lo_flag == 0u;
    if (!mbar_wait_bounded(bar, 0)) {
        if (tid == 0) atomicExch(a.err, SMOE_DEVERR_MBAR_TIMEOUT);
        return;
    }
    // scales/biases into the lanes' order: lane c of row slice wn reads its
    // 2 * NTW values of a group with NTW / 4 16-byte loads
    for (int i = tid; i < MATS * 2 * nsb; i += 256) {
        const int q = i & 1, nt = (i >> 1) % NTW, c4 = (i / (2 * NTW)) & 3, wn = (i / (8 * NTW)) % WN;
        const int grp = (i / RB) % G, mk = i / (RB * G);
        st[i] = sb[mk * nsb + (wn * NTW * 8 + nt * 8 + 2 * c4 + q) * G + grp];
    }
    __syncthreads();                      // sb is dead from here: red may overwrite it
    auto slot_of = [&](uint32_t i) { return i < uint32_t(kSlotCache) ? sl[i] : lst[i]; };
    const int wk = warp / WN, wn = warp % WN;
    const int gpw = (G + WK - 1) / WK, g0 = wk * gpw, g1 = min(G, g0 + gpw), ng = max(g1 - g0, 0);
    const uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u, OR = 0x64006400u;

    auto body = [&](auto tpc_tag) {
        constexpr int TPC = decltype(tpc_tag)::value;       // tokens per chunk: 8 or 16
        constexpr int TT = TPC / 8;                          // tokens per lane
        constexpr int NAC = MATS * NTW * TT * 2;             // accumulators per lane
        const int nchunk = int((T + TPC - 1) / TPC);
        // load cursor (chunk ich, group igrp), running NB - 1 items ahead of
        // the MMAs: A registers x[s][0..3] of the 4 k-steps and the group
        // sums of the lane's tokens; per-chunk table pointers ip / gp
        int ich = ng > 0 ? 0 : nchunk, igrp = g0;
        const uint4* ip[TT];
        const float* gp[TT];
        auto set_chunk = [&]() {
#pragma unroll
            for (int tt = 0; tt < TT; ++tt) {
                const uint32_t tk = ich * TPC + tt * 8 + gr;
                const uint32_t vec = slot_of(tk < T ? tk : 0) / a.tab_div;
                ip[tt] = reinterpret_cast<const uint4*>(a.tab) + size_t(vec) * (K / 16) * 4 + c;
                gp[tt] = &a.gs[size_t(vec) * G].y;
            }
        };
        if (ich < nchunk) set_chunk();
        auto issue = [&](uint32_t (&x)[4][4], float (&y)[TT]) {
            if (ich >= nchunk) return;
#pragma unroll
            for (int tt = 0; tt < TT; ++tt) {
                const uint4* q4 = ip[tt] + igrp * 16;
                if (TT == 1) {
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint4 q = __ldg(q4 + s * 4);
                        x[s][0] = q.x; x[s][1] = q.z; x[s][2] = q.y; x[s][3] = q.w;   // hi.x lo.x hi.y lo.y
                    }
                } else {
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        const uint2 h = __ldg(reinterpret_cast<const uint2*>(q4 + s * 4));
                        x[s][tt] = h.x;
                        x[s][2 + tt] = h.y;
                    }
                }
                y[tt] = __ldg(gp[tt] + igrp * 2);
            }
            if (++igrp == g1) {
                igrp = g0;
                if (++ich < nchunk) set_chunk();
            }
        };
        constexpr int NB = TT == 1 ? 3 : 2;                  // load buffers (pipeline depth NB - 1)
        uint32_t xb[NB][4][4];
        float yb[NB][TT];
#pragma unroll
        for (int p = 0; p < NB - 1; ++p) issue(xb[p], yb[p]);
        for (int ch = 0; ch < nchunk; ++ch) {
            float acc[NAC];
#pragma unroll
            for (int i = 0; i < NAC; ++i) acc[i] = 0.f;
            for (int grp = g0; grp < g1; ++grp) {
                issue(xb[NB - 1], yb[NB - 1]);
                const uint8_t* wl = wt + (wn * NTW * 8 + gr) * rs + grp * 32 + c * 8;   // this lane's rows
#pragma unroll
                for (int m = 0; m < MATS; ++m) {
                    uint32_t scw[NTW], biw[NTW];
                    const uint16_t* sp = st + ((((m * 2) * G + grp) * WN + wn) * 4 + c) * NTW * 2;
#pragma unroll
                    for (int v = 0; v < NTW / 4; ++v) {
                        const uint4 s4 = *reinterpret_cast<const uint4*>(sp + v * 8);
                        scw[v * 4 + 0] = s4.x; scw[v * 4 + 1] = s4.y; scw[v * 4 + 2] = s4.z; scw[v * 4 + 3] = s4.w;
                        if (FMT == kFmtAffine) {
                            const uint4 b4 = *reinterpret_cast<const uint4*>(sp + G * WN * 4 * NTW * 2 + v * 8);
                            biw[v * 4 + 0] = b4.x; biw[v * 4 + 1] = b4.y; biw[v * 4 + 2] = b4.z; biw[v * 4 + 3] = b4.w;
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < NTW; ++nt) {
                        const uint2 w = *reinterpret_cast<const uint2*>(wl + (m * RB + nt * 8) * rs);
                        float d[4];
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            const uint32_t wi = (s >> 1) ? w.y : w.x;
                            const uint32_t g8 = (s & 1) ? (wi >> 8) : wi;
                            const uint32_t b[2] = {hsub_1024(lop3_and_or(g8, M0, OR)),
                                                   hsub_1024(lop3_and_or(g8, M1, OR))};
                            if (s == 0) mma_f16_16816_z(d, xb[0][s], b);
                            else mma_f16_16816(d, xb[0][s], b);
                        }
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            float* ac = acc + (m * NTW + nt) * TT * 2;
                            if (FMT == kFmtAffine) {
                                const float sv = __uint_as_float(q ? (scw[nt] & 0xffff0000u) : (scw[nt] << 16));
                                const float bv = __uint_as_float(q ? (biw[nt] & 0xffff0000u) : (biw[nt] << 16));
                                if (TT == 1) {
                                    ac[q] = fmaf(sv, d[q] + d[2 + q], fmaf(bv, yb[0][0], ac[q]));
                                } else {
#pragma unroll
                                    for (int tt = 0; tt < TT; ++tt)
                                        ac[tt * 2 + q] = fmaf(sv, d[tt * 2 + q], fmaf(bv, yb[0][tt], ac[tt * 2 + q]));
                                }
                            } else {
                                const float sv = f16_bits_to_f32(uint16_t(q ? (scw[nt] >> 16) : (scw[nt] & 0xffffu)));
                                if (TT == 1) {
                                    ac[q] = fmaf(sv, fmaf(d[q] + d[2 + q], 1.0f / 7.5f, -yb[0][0]), ac[q]);
                                } else {
#pragma unroll
                                    for (int tt = 0; tt < TT; ++tt)
                                        ac[tt * 2 + q] = fmaf(sv, fmaf(d[tt * 2 + q], 1.0f / 7.5f, -yb[0][tt]),
                                                              ac[tt * 2 + q]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int p = 0; p < NB - 1; ++p) {
#pragma unroll
                    for (int s = 0; s < 4; ++s)
#pragma unroll
                        for (int r = 0; r < 4; ++r) xb[p][s][r] = xb[p + 1][s][r];
#pragma unroll
                    for (int tt = 0; tt < TT; ++tt) yb[p][tt] = yb[p + 1][tt];
                }
            }
            float* rw = red + warp * NAC * 32 + lane;
#pragma unroll
            for (int i = 0; i < NAC; ++i) rw[i * 32] = acc[i];
            __syncthreads();
            for (int o = tid; o < TPC * RB; o += 256) {
                const int t = o / RB, r = o % RB;
                const uint32_t tk2 = ch * TPC + t;
                if (tk2 < T) {
                    const int wn2 = r / (NTW * 8), nt = (r / 8) % NTW, q = r & 1;
                    const int ln = (t & 7) * 4 + ((r & 7) >> 1), tt = t >> 3;
                    float v[MATS];
#pragma unroll
                    for (int m = 0; m < MATS; ++m) {
                        float sum = 0.f;
#pragma unroll
                        for (int k2 = 0; k2 < WK; ++k2)
                            sum += red[((k2 * WN + wn2) * NAC + ((m * NTW + nt) * TT + tt) * 2 + q) * 32 + ln];
                        v[m] = sum;
                    }
                    const uint32_t slot = slot_of(tk2);
                    const float inv = __ldg(&a.gs[size_t(slot / a.tab_div) * G].x);
                    float outv;
                    if (MATS == 2) {
                        const float g = v[0] * inv, u = v[MATS - 1] * inv;
                        outv = g * (1.0f / (1.0f + expf(-g))) * u;                  // kernels.metal:61-63
                    } else {
                        outv = v[0] * inv;
                    }
                    a.out[size_t(slot) * R + blk * RB + r] = outv;
                }
            }
            __syncthreads();
        }
    };
    if (MATS == 2 && hi_only) body(std::integral_constant<int, 16>{});     // down inputs are fp32
    else body(std::integral_constant<int, 8>{});
}

// ------------------------------------------------------------------------
// tcgen05 down projection of the grouped path. CTA = (128 rows of W_down,
// expert), 256 threads: thread (r, h) = (tid & 127, tid >> 7) serves weight
// row r, which is tensor-memory lane r (warps w and w + 4 share lanes
// 32 (w % 4)..). The expert's slots are taken 32 at a time (a pass); per
// pass the K = d_ff dimension runs in slabs of one 64-column group:
//   each thread cp.asyncs 16 bytes of its row's codes 4 slabs ahead and
//     dequantises them into A (fp16 q or 16 q, exact) in the no-swizzle
//     K-major core-matrix layout; the B rows (slot t: rows 2t and 2t+1 =
//     hi and lo half of its scaled hidden vector, from the table k_build_tabs
//     wrote in the same column order) come from registers loaded two slabs
//     ahead;
//   one thread issues the 4 k-steps of D[slab] = A B^T (M 128, N = 2 x
//     slots rounded up to 16) into one of two tensor-memory column buffers
//     and commits them to that buffer's mbarrier;
//   meanwhile every thread reads the previous slab's D for its row and its
//     8-slot blocks (h = block parity) and adds the group epilogue
//     (group_epilogue's arithmetic) to its accumulators: the MMAs of one slab
//     overlap the epilogue of the last and the dequantisation of the next.
// The hidden vectors are fp32, so two B rows per slot keep the products
// exact (the gate/up kernel above takes its bf16 x as one fp16 row).
constexpr int kTcPass = 32;        // slots per pass
constexpr int kTcNib = 5;          // code stages (prefetch depth 4)
struct TcSmem {
    static constexpr int A = 16384, B = 8192, NIB = 4096;
    __host__ __device__ static size_t scales(int G) { return size_t(2) * G * 128 * 2; }
    __host__ __device__ static size_t bytes(int G) {
        return 2 * A + 2 * B + kTcNib * NIB + scales(G) + (3 + 1 + 1 + 1) * kTcPass * 4 + 64;
    }
};

SMOE_DEVINL void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
SMOE_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SMOE_DEVINL void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

template <int FMT>
__global__ void __launch_bounds__(256, 2) k_ffn_down_tc(GroupedArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t e = blockIdx.y, T = a.count[e];
    if (T == 0) return;
    const int K = int(a.d_ff), R = int(a.d_model), G = K / 64;
    const int tid = threadIdx.x, warp = tid >> 5, row = tid & 127, hh = tid >> 7;
    uint8_t* sA = smem;                                                  // [2][128 rows x 64 cols fp16]
    uint8_t* sB = sA + 2 * TcSmem::A;                                    // [2][64 rows x 64 cols fp16]
    uint8_t* sN = sB + 2 * TcSmem::B;                                    // [kTcNib][2][128][16 B]
    uint16_t* sS = reinterpret_cast<uint16_t*>(sN + kTcNib * TcSmem::NIB);   // [2][G][128]
    float* gsm = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(sS) + TcSmem::scales(G));   // [3][32]
    float* sinv = gsm + 3 * kTcPass;                                     // [32]
    uint32_t* sslot = reinterpret_cast<uint32_t*>(sinv + kTcPass);      // [32]
    uint32_t* svec = sslot + kTcPass;                                    // [32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(svec + kTcPass);       // [2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);
    uint32_t* sfail = tslot + 1;

    // this thread's weight row (matrix 2 = down)
    const int mrow = blockIdx.x * 128 + row;
    const uint8_t* eb = a.base + uint64_t(e) * a.stride;
    const uint8_t* nsrc = eb + a.off[6] + size_t(mrow) * (K / 2) + hh * 16;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        *sfail = 0u;
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, 128);
    // code prefetch: one commit group per slab; slabs run over the groups
    // of every pass in order
    const int npass = int((T + kTcPass - 1) / kTcPass);
    uint8_t* nst = sN + hh * 2048 + row * 16;                            // this thread's 16 B of a stage
    int is_stage = 0, is_g = 0, is_left = npass * G, rd_stage = 0;
    auto nib_issue = [&]() {
        if (is_left > 0) cp_async16(nst + is_stage * TcSmem::NIB, nsrc + is_g * 32);
        cp_async_commit();
        is_stage = is_stage + 1 == kTcNib ? 0 : is_stage + 1;
        is_g = is_g + 1 == G ? 0 : is_g + 1;
        --is_left;
    };
#pragma unroll
    for (int i = 0; i < kTcNib - 1; ++i) nib_issue();
    // this row's scales (hh = 0) or biases (hh = 1): all loads first (G <= 64
    // in 8-byte pieces), then the transposed shared-memory stores
    if (hh == 0 || FMT == kFmtAffine) {
        const uint2* sc = reinterpret_cast<const uint2*>(eb + a.off[7 + hh] + size_t(mrow) * G * 2);
        uint2 v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = j * 4 < G ? __ldg(sc + j) : make_uint2(0u, 0u);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (j * 4 < G) {
                uint16_t* d = sS + (hh * G + j * 4) * 128 + row;
                d[0] = uint16_t(v[j].x); d[128] = uint16_t(v[j].x >> 16);
                d[256] = uint16_t(v[j].y); d[384] = uint16_t(v[j].y >> 16);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tslot;
    const uint32_t lane_base = taddr + (uint32_t((warp & 3) * 32) << 16);
    const uint32_t* lst = a.list + size_t(e) * a.lcap;
    // descriptors of k-step 0 of buffer 0 (the start address field is in
    // the low bits: k-step ks adds 256 bytes >> 4)
    const uint64_t adesc0 = tc_desc(smem_u32(sA), 128, 1024), bdesc0 = tc_desc(smem_u32(sB), 128, 1024);

    // slab pipeline state (identical in every thread): buffer of the slab
    // being prepared (cb, its group-sum buffer c3) and of the previous one
    // (pb, p3), and each MMA buffer's next mbarrier parity
    int cb = 0, c3 = 0, pb = 0, p3 = 0;
    uint32_t par0 = 0, par1 = 0;
    // B rows: 64 rows (slot n / 2, half n & 1) x 8 chunks; thread -> row
    // tid & 63, chunks (tid >> 6) and (tid >> 6) + 4
    const int bn = tid & 63, bkc0 = tid >> 6, bt = bn >> 1, bpart = bn & 1;
    uint8_t* bdst0 = sB + (bn >> 3) * 1024 + (bn & 7) * 16 + bkc0 * 128;
    uint8_t* arow0 = sA + (row >> 3) * 1024 + hh * 512 + (row & 7) * 16;
    for (int pass = 0; pass < npass; ++pass) {
        const int p0 = pass * kTcPass, TP = min(int(T) - p0, kTcPass);
        const int N = (2 * TP + 15) & ~15;
        const uint32_t idesc = tc_idesc_f16(128, N);
        if (tid < TP) {
            const uint32_t slot = lst[p0 + tid], vec = slot / a.tab_div;
            sslot[tid] = slot;
            svec[tid] = vec;
            sinv[tid] = __ldg(&a.gs[size_t(vec) * G].x);
        }
        __syncthreads();
        const bool bvalid = bt < TP;
        const uint4* btab = reinterpret_cast<const uint4*>(a.tab) + (bvalid ? size_t(svec[bt]) * G * 16 : 0) +
                            bkc0 * 2 + bpart;
        const float* gsrc = tid < TP ? &a.gs[size_t(svec[tid]) * G].y : nullptr;
        uint4 bq0[2], bq1[2];                   // B chunks of groups g and g + 1
        float gq0 = 0.f, gq1 = 0.f;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            bq0[j] = bvalid ? __ldg(btab + 8 * j) : make_uint4(0u, 0u, 0u, 0u);
            bq1[j] = (bvalid && G > 1) ? __ldg(btab + 16 + 8 * j) : make_uint4(0u, 0u, 0u, 0u);
        }
        if (gsrc) {
            gq0 = __ldg(gsrc);
            if (G > 1) gq1 = __ldg(gsrc + 2);
        }
        float acc[2][8];                        // slots 8 (2 i + hh) + k
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[i][k] = 0.f;

        for (int g = 0; g <= G; ++g) {
            if (g < G) {
                // 1. this thread's 32 codes of the slab (and the next prefetch)
                cp_async_wait<kTcNib - 2>();
                const uint4 w = *reinterpret_cast<const uint4*>(nst + rd_stage * TcSmem::NIB);
                rd_stage = rd_stage + 1 == kTcNib ? 0 : rd_stage + 1;
                nib_issue();
                // 2. dequantise: word i (8 codes) -> core-matrix row chunk 4 hh + i
                {
                    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
                    const uint32_t M0 = 0x000F000Fu, M1 = 0x00F000F0u, OR = 0x64006400u;
                    uint8_t* arow = arow0 + cb * TcSmem::A;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t x = wv[i], x8 = x >> 8;
                        uint4 o;
                        o.x = hsub_1024(lop3_and_or(x, M0, OR));
                        o.y = hsub_1024(lop3_and_or(x, M1, OR));
                        o.z = hsub_1024(lop3_and_or(x8, M0, OR));
                        o.w = hsub_1024(lop3_and_or(x8, M1, OR));
                        *reinterpret_cast<uint4*>(arow + i * 128) = o;
                    }
                }
                // 3. B rows of group g (rows of absent slots are zero), group sums
                {
                    uint8_t* bdst = bdst0 + cb * TcSmem::B;
#pragma unroll
                    for (int j = 0; j < 2; ++j) *reinterpret_cast<uint4*>(bdst + j * 512) = bq0[j];
                    if (tid < TP) gsm[c3 * kTcPass + tid] = gq0;
#pragma unroll
                    for (int j = 0; j < 2; ++j) bq0[j] = bq1[j];
                    gq0 = gq1;
                    btab += 16;                             // now group g + 1
                    if (g + 2 < G) {
#pragma unroll
                        for (int j = 0; j < 2; ++j) bq1[j] = bvalid ? __ldg(btab + 16 + 8 * j) : make_uint4(0u, 0u, 0u, 0u);
                        if (gsrc) gq1 = __ldg(gsrc + 2 * (g + 2));
                    }
                }
                fence_proxy_async();
                tc_fence_before();
                __syncthreads();
                // 4. one thread issues the slab's MMAs
                if (tid == 0) {
                    tc_fence_after();
                    const uint64_t ad = adesc0 + uint64_t(cb * (TcSmem::A >> 4)), bd = bdesc0 + uint64_t(cb * (TcSmem::B >> 4));
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) tc_mma_f16(taddr + cb * 64, ad + ks * 16, bd + ks * 16, idesc, ks > 0);
                    tc_commit(&bars[cb]);
                }
            }
            // 5. epilogue of the previous slab (buffers pb, p3, group g - 1):
            //    this row's dots for the thread's slot blocks 2 i + hh
            if (g > 0) {
                const int gv = g - 1;
                const uint32_t par = pb ? par1 : par0;
                if (!mbar_try_wait(&bars[pb], par)) {
                    if (!*reinterpret_cast<volatile uint32_t*>(sfail) && !mbar_wait_slow(&bars[pb], par)) {
                        *reinterpret_cast<volatile uint32_t*>(sfail) = 1u;
                        atomicExch(a.err, SMOE_DEVERR_MBAR_TIMEOUT);
                    }
                }
                if (pb) par1 ^= 1u; else par0 ^= 1u;
                tc_fence_after();
                const float* gs3 = gsm + p3 * kTcPass;
                const float sv = FMT == kFmtAffine ? bf16_bits_to_f32(sS[gv * 128 + row])
                                                   : f16_bits_to_f32(sS[gv * 128 + row]);
                const float bv = bf16_bits_to_f32(sS[(G + gv) * 128 + row]);
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const int t0 = (2 * i + hh) * 8;
                    if (t0 < TP) {
                        float d[16];
                        tmem_ld16(lane_base + pb * 64 + t0 * 2, d);
                        const float4 ga = *reinterpret_cast<const float4*>(gs3 + t0);
                        const float4 gb = *reinterpret_cast<const float4*>(gs3 + t0 + 4);
                        const float gsv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
                        tmem_ld_wait();
#pragma unroll
                        for (int k = 0; k < 8; ++k) {
                            const float dsum = d[2 * k] + d[2 * k + 1];
                            if (FMT == kFmtAffine) acc[i][k] = fmaf(sv, dsum, fmaf(bv, gsv[k], acc[i][k]));
                            else acc[i][k] = fmaf(sv, fmaf(dsum, 1.0f / 7.5f, -gsv[k]), acc[i][k]);
                        }
                    }
                }
                tc_fence_before();
            }
            if (g < G) {
                pb = cb;
                p3 = c3;
                cb ^= 1;
                c3 = c3 == 2 ? 0 : c3 + 1;
            }
        }
        // output: this thread's slots 8 (2 i + hh) + k
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int t = (2 * i + hh) * 8 + k;
                if (t < TP) a.out[size_t(sslot[t]) * R + mrow] = acc[i][k] * sinv[t];
            }
        __syncthreads();                       // sslot / svec / sinv reused by the next pass
    }
    cp_async_wait<0>();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(taddr, 128);
}

// y[t] = sum_j w[t*k+j] * ys[t*k+j] in rank order j (axpy_f32: product, then
// sum). grid (ceil(d/256), ntok).
// ids (shard mode, else null): only slots of experts [base, base + e_local)
// are added (this rank's partial sum; the ranks' partials are summed by the
// caller's reduction).
__global__ void k_combine_slots(const float* ys, const float* wts, uint32_t k, uint32_t d, void* y,
                                int y_dtype, const uint32_t* ids, uint32_t base, uint32_t e_local) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (i >= d) return;
    float acc = 0.f;
    for (uint32_t j = 0; j < k; ++j) {
        if (ids && ids[t * k + j] - base >= e_local) continue;
        acc = __fadd_rn(acc, __fmul_rn(wts[t * k + j], ys[size_t(t * k + j) * d + i]));
    }
    if (y_dtype == 0) static_cast<float*>(y)[size_t(t) * d + i] = acc;
    else static_cast<__nv_bfloat16*>(y)[size_t(t) * d + i] = __float2bfloat16_rn(acc);
}

}  // namespace smoe
