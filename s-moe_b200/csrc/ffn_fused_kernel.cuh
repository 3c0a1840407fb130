// ffn_fused_kernel.cuh - the persistent fused MoE-layer kernel (sm_100a).
//
// One launch, one CTA per SM, does a whole MoE layer of a decode
// step for up to kFusedMaxTok tokens:
//   routing (optional): router logit rows spread over the grid, then every
//     CTA runs the softmax / top-k / renorm of router.cuh on all logits;
//   units (slot j, hidden rows 16t..16t+15) split evenly over the CTAs, each
//     computing  h = silu(Wg.x) * (Wu.x) * w_j  for its 16 rows and at once
//     its share of the down projection, W_down[:, 16t..16t+15] . h, into a
//     per-CTA fp32 partial output in shared memory (split-K down: no unit
//     waits for another CTA);
//   each CTA adds its partial outputs to a global fp32 accumulator with
//   vector reductions; the last CTA to finish writes y and clears the
//   accumulator, so consecutive launches need no host work.
// Warp 17 (producer) streams every byte the CTA will use - each unit is one
// contiguous block of the tiled layout (tiled.cuh), plus the down scales of
// a 64-row group when the unit starts one - into a ring of shared-memory
// stages with 1-D bulk copies, the first ones before the CTA's first barrier;
// sixteen consumer warps run the gate/up dots as integer MMAs on the raw
// codes and the down slice as bf16 MMAs (arithmetic in ffn_fused.cuh); warp
// 16 turns each unit's partial sums into h.
// Note: the fp32 reductions make the sum over units order-dependent in its
// last bits (results within 1e-6 relative of each other run to run).
#pragma once
#include "ffn_fused.cuh"

// cycle counters of the phases, for profiling builds only (-DSMOE_FUSED_PROFILE)
#ifdef SMOE_FUSED_PROFILE
#define SMOE_PROF(...) __VA_ARGS__
#else
#define SMOE_PROF(...)
#endif

namespace smoe {

// Phase R: logit row r = (token, expert) by all consumer warps of this CTA.
SMOE_DEVINL float router_row(const FusedArgs& A, const void* xsrc, uint32_t t, uint32_t e, int ctid) {
    const FfnArgs& f = A.f;
    const int d = A.g.d;
    float acc = 0.f;
    const uint4* wp = reinterpret_cast<const uint4*>(A.rw + size_t(e) * d);
    for (int c = ctid; c < d / 8; c += kFusedCThreads) {
        const uint4 v = __ldg(wp + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        float xv[8];
        if (f.x_dtype == 0) {
            const float4* xp =
                reinterpret_cast<const float4*>(static_cast<const float*>(xsrc) + size_t(t) * d + c * 8);
            const float4 a0 = xp[0], a1 = xp[1];
            xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
            xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
        } else {
            const uint4 b =
                *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xsrc) + size_t(t) * d + c * 8);
            const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                xv[2 * q] = __uint_as_float(bw[q] << 16);
                xv[2 * q + 1] = __uint_as_float(bw[q] & 0xffff0000u);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            acc = fmaf(__uint_as_float(u[q] << 16), xv[2 * q], acc);
            acc = fmaf(__uint_as_float(u[q] & 0xffff0000u), xv[2 * q + 1], acc);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

SMOE_DEVINL void red_add_v4(float* p, float4 v) {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

// GW: 64-groups of the gate/up rows per consumer warp, ceil(d_model / 1024)
template <int FMT, int GW>
__global__ void __launch_bounds__(kFusedThreads, 1) k_moe_fused(FusedArgs A) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const FusedGeom& g = A.g;
    const FfnArgs& f = A.f;
    const TiledGeom& tg = g.tg;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool consumer = warp < kFusedConsumers;
    uint8_t* ring = sm + g.o_ring;
    uint4* xtab = reinterpret_cast<uint4*>(sm + g.o_xtab);
    float2* xg = reinterpret_cast<float2*>(sm + g.o_xg);
    float* ysum = reinterpret_cast<float*>(sm + g.o_ysum);     // [ntok][d]; earlier x staging / softmax scratch
    uint16_t* sbc0 = reinterpret_cast<uint16_t*>(sm + g.o_sbc); // [2][down sc[d] (+ bias[d])] by group parity
    float* red0 = reinterpret_cast<float*>(sm + g.o_red);       // [2][16 warps][32]
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + g.o_bar);
    uint64_t* empty = full + 16;
    uint64_t* redF = full + 32;                                 // [2] partial sums written (16 arrivals)
    uint64_t* hR = full + 34;                                   // [2] h ready (1 arrival)
    uint64_t* routedB = full + 36;                              // routing in s_ids / s_w (1 arrival)
    uint32_t* s_ids = reinterpret_cast<uint32_t*>(sm + g.o_ids);
    float* s_w = reinterpret_cast<float*>(sm + g.o_w);
    float* red = red0;                                          // routing uses buffer 0
    const int NS = g.nstages, k = g.k, d = g.d;
    const uint32_t nslots = uint32_t(g.ntok * k);
    __shared__ uint32_t last_cta;

    trace_mark(A.trace, 0);
    SMOE_PROF(if (A.trace && tid == 0) A.trace[gridDim.x * 32 + blockIdx.x * 8 + 4] = clock64();)
    // inputs (x, routing) may come from the previous kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const FusedEp& ep = A.ep;
    const bool epm = ep.world > 1;
    const uint32_t epoch = epm ? A.st->epoch + 1u : 0u;            // written by the previous launch only
    uint32_t* s_loc = reinterpret_cast<uint32_t*>(sm + g.o_loc);     // expert parallel: local slots, count
    // this CTA's units [u0, u1) of nU: every unit of every slot, or (expert
    // parallel) of the slots whose expert this rank holds, known after routing
    int u0 = 0, u1 = 0;
    auto set_range = [&](int nU) {
        u0 = int(blockIdx.x * uint32_t(nU) / gridDim.x);                 // nU * grid < 2^31
        u1 = int((blockIdx.x + 1) * uint32_t(nU) / gridDim.x);
    };
    if (!epm) set_range(g.nU);
    auto slot_of = [&](int u) { return epm ? int(s_loc[u / g.tilesU]) : u / g.tilesU; };
    auto needs_sb = [&](int u) { return u == u0 || (u % g.tilesU) % 4 == 0; };
    // x: the caller's, or on ranks > 0 rank 0's published copy (peer memory)
    const void* xsrc = f.x;
    if (epm) {
        const size_t xbytes = size_t(g.ntok) * d * (f.x_dtype == 0 ? 4 : 2);
        if (ep.rank == 0 && blockIdx.x == 0) {
            for (size_t i = tid; i < xbytes / 16; i += blockDim.x)
                reinterpret_cast<uint4*>(ep.x0)[i] = reinterpret_cast<const uint4*>(f.x)[i];
        } else if (ep.rank > 0) {
            if (tid == 0 && !spin_sys_until_geq(ep.flag0, epoch)) atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT);
            xsrc = ep.x0;
        }
    }
    // copy of unit u (the n-th of this CTA) into its stage: one bulk copy, plus
    // the down scales of the 64-row group it starts (producer lane 0)
    auto issue = [&](int u, int n) {
        const int st = n % NS, slot = slot_of(u), t = u % g.tilesU;
        const bool sb = needs_sb(u);
        const uint8_t* ex = f.base + uint64_t(s_ids[slot] - (epm ? ep.base : 0u)) * f.stride;
        mbar_arrive_expect_tx(full + st, tg.unit + (sb ? tg.dgroup : 0));
        bulk_g2s(ring + size_t(st) * g.stage, ex + tg.unit_off(t), tg.unit, full + st);
        if (sb) bulk_g2s(sbc0 + ((u / 4) & 1) * (tg.dgroup / 2), ex + tg.group_off(t / 4), tg.dgroup, full + st);
        if (n < 3) trace_mark(A.trace, 25 + n, true);
    };
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kFusedConsumers);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(redF + b, kFusedConsumers);
            mbar_init(hR + b, 1);
        }
        mbar_init(routedB, 1);
        fence_mbar_init();
    }
    __syncthreads();              // (ranks > 0: rank 0's x is published; rank 0 CTA 0: x0 is written)
    if (epm && ep.rank == 0 && blockIdx.x == 0 && tid == 0) {
        __threadfence_system();
        st_release_sys(ep.flag0, epoch);
    }
    int pre = 0;                                                // units issued ahead of the main loop
    if (!A.rw && warp == kFusedProdWarp) {
        // routing given: read it and start the weight stream at once
        for (uint32_t i = lane; i < nslots; i += 32) s_ids[i] = f.ids[i];
        __syncwarp();
        pre = min(NS, u1 - u0);
        if (lane == 0)
            for (int n = 0; n < pre; ++n) issue(u0 + n, n);
        __syncwarp();
    } else if (!A.rw && warp == kFusedHWarp) {
        for (uint32_t i = lane; i < nslots; i += 32) s_w[i] = f.wts[i];
        __syncwarp();
    }
    trace_mark(A.trace, 8);

    // ---------------------------------------------------------- routing
    if (A.rw) {
        const uint32_t rows = A.E * g.ntok;
        for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
            float v = 0.f;
            if (consumer) v = router_row(A, xsrc, r / A.E, r % A.E, tid);
            if (consumer && lane == 0) red[warp] = v;
            __syncthreads();
            if (tid == 0) {
                float sum = 0.f;
                for (int w = 0; w < kFusedConsumers; ++w) sum += red[w];
                A.logits[r] = sum;
                asm volatile("red.release.gpu.global.add.u32 [%0], 1;" :: "l"(&A.st->rdone) : "memory");
            }
            __syncthreads();
        }
        trace_mark(A.trace, 11);
    }
    // x table (consumers): one round of wide loads, then the table in shared memory
    if (consumer) {
        if (f.x_dtype == 0) stage_vec_smem<false>(xsrc, g.ntok * d, ysum, tid);
        else stage_vec_smem<true>(xsrc, g.ntok * d, ysum, tid);
        consumer_sync();
        trace_mark(A.trace, 9);
        build_xplanes<FMT>(ysum, g.ntok, d, xtab, xg, tid);

        consumer_sync();
        trace_mark(A.trace, 10);                             // x staging (ysum) is reused below
    }
    if (A.rw && warp == kFusedHWarp) {
        // routing (h warp, while the consumers build the x table): wait for
        // every logit row of the grid, then softmax / top-k / renorm per token
        if (lane == 0 && !spin_until_geq(&A.st->rdone, A.E * g.ntok)) atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT);
        __syncwarp();
        trace_mark(A.trace, 13, lane == 0);
        SMOE_PROF(long long c0 = clock64();)
        for (int t = 0; t < g.ntok; ++t) {
            warp_topk(A.logits + size_t(t) * A.E, A.E, k, A.norm, s_ids + t * k, s_w + t * k, lane);
            SMOE_PROF(if (A.trace && lane == 0 && t == 0) reinterpret_cast<long long*>(A.trace)[gridDim.x * 56 + blockIdx.x * 8 + 1] = clock64() - c0;)
            __syncwarp();
            if (blockIdx.x == 0 && lane < k) {
                const_cast<uint32_t*>(f.ids)[t * k + lane] = s_ids[t * k + lane];
                const_cast<float*>(f.wts)[t * k + lane] = s_w[t * k + lane];
            }
        }
        __syncwarp();
        if (epm) {                                   // slots whose expert this rank holds, in slot order
            uint32_t cnt = 0;
            for (uint32_t s0 = 0; s0 < nslots; s0 += 32) {
                const uint32_t sl = s0 + lane;
                const bool loc = sl < nslots && s_ids[sl] - ep.base < ep.nlocal;
                const uint32_t m = __ballot_sync(0xffffffffu, loc);
                if (loc) s_loc[cnt + __popc(m & ((1u << lane) - 1u))] = sl;
                cnt += __popc(m);
            }
            if (lane == 0) s_loc[kFusedMaxTok * kFusedMaxK] = cnt;
            __syncwarp();
            set_range(int(cnt) * g.tilesU);
        }
        // start the weight stream from here: no hand-off to the producer,
        // which takes over from unit `pre` once routedB completes
        pre = min(NS, u1 - u0);
        if (lane == 0) {
            for (int n = 0; n < pre; ++n) issue(u0 + n, n);
            mbar_arrive(routedB);
        }
        SMOE_PROF(if (A.trace && lane == 0) reinterpret_cast<long long*>(A.trace)[gridDim.x * 56 + blockIdx.x * 8 + 2] = clock64() - c0;)
        trace_mark(A.trace, 1, lane == 0);
    }

    if (warp == kFusedProdWarp) {
        // ------------------------------------------------------ producer
        if (A.rw) {                                  // expert ids (and the first units) come from the h warp
            if (lane == 0 && !mbar_wait_bounded(routedB, 0)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            __syncwarp();
            if (epm) set_range(int(s_loc[kFusedMaxTok * kFusedMaxK]) * g.tilesU);
            pre = min(NS, u1 - u0);
        }
        for (int u = u0 + pre, n = pre; u < u1; ++u, ++n) {
            const int st = n % NS, round = n / NS;
            if (round > 0 && lane == 0 && !mbar_wait_bounded(empty + st, (round - 1) & 1))
                atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            if (lane == 0) issue(u, n);
            __syncwarp();
        }
    } else if (warp == kFusedHWarp) {
        // ---------------------------------------------------------- h warp
        SMOE_PROF(if (A.trace) for (int n = 0; n < 3 && n < u1 - u0; ++n) { mbar_wait_bounded(full + n, 0); trace_mark(A.trace, 28 + n, lane == 0); })
        for (int u = u0, n = 0; u < u1; ++u, ++n) {
            const int b = n & 1, slot = slot_of(u);
            if (!mbar_wait_bounded(redF + b, (n >> 1) & 1)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            const float* rb = red0 + b * kFusedConsumers * 32;
            float* hq = reinterpret_cast<float*>(sm + g.o_hq + b * 256);
            uint2* dB = reinterpret_cast<uint2*>(sm + g.o_hq + b * 256 + 64);
            float* hsum = reinterpret_cast<float*>(sm + g.o_hq + b * 256 + 128);
            float v = 0.f;                                        // lane = (matrix, row)
#pragma unroll
            for (int w = 0; w < kFusedConsumers; ++w) v += rb[w * 32 + lane];
            const float up = __shfl_down_sync(0xffffffffu, v, 16);
            if (lane < 16) hq[lane] = v * (1.0f / (1.0f + expf(-v))) * up * s_w[slot];   // kernels.metal:61-63
            __syncwarp();
            float part = 0.f;
            if (lane < 16) {
                const float hv = hq[lane];
                const float hi = __bfloat162float(__float2bfloat16_rn(hv));
                part = hi + __bfloat162float(__float2bfloat16_rn(hv - hi));
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (lane == 0) *hsum = part;
            if (lane < 8) {                                       // standard B layout: k 2c,2c+1 / 2c+8,2c+9
                const int c = lane & 3, col = lane >> 2;
                float e[4] = {hq[2 * c], hq[2 * c + 1], hq[2 * c + 8], hq[2 * c + 9]};
                if (col) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) e[q] -= __bfloat162float(__float2bfloat16_rn(e[q]));
                }
                dB[lane] = make_uint2(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]));
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(hR + b);
            if (n == 0) trace_mark(A.trace, 12, lane == 0);
        }
    } else {
        // ----------------------------------------------------- consumers
        // step n: gate/up of unit n, then the down slice of unit n-1 (whose h
        // the h warp computed meanwhile)
        const int gr = lane >> 2;
        for (int i = tid; i < g.ntok * d; i += kFusedCThreads) ysum[i] = 0.f;
        consumer_sync();
        if (epm) {                                   // the unit list depends on the routing
            if (!mbar_wait_bounded(routedB, 0)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            set_range(int(s_loc[kFusedMaxTok * kFusedMaxK]) * g.tilesU);
        }
        trace_mark(A.trace, 2);
        const int cq = lane & 3;                         // token whose results this lane holds
        // Down projection, split-K: this CTA's units are consecutive (slot,
        // 16 hidden rows) blocks, so four of them in a row share one 64-column
        // quantisation group of W_down. Warp w owns output tiles w + 16q; for
        // q < kDownRegTiles the raw MMA sums stay in registers for the whole
        // group (the epilogue is linear in the dot and the h sum) and are
        // scaled into the token's shared-memory partial output once per
        // group. Tiles beyond those (d_model > 2048) take the scale per unit.
        float dacc[kDownRegTiles][4], hsg = 0.f;
#pragma unroll
        for (int q = 0; q < kDownRegTiles; ++q) dacc[q][0] = dacc[q][1] = dacc[q][2] = dacc[q][3] = 0.f;
        const uint32_t M = 0x000F000Fu, OR = 0x43004300u;
        SMOE_PROF(long long cy_wait = 0, cy_gu = 0, cy_hw = 0, cy_dn = 0, cy_t = 0;)
        auto down = [&](int u, int n) {
            const int b = n & 1, st = n % NS, tok = slot_of(u) / k, t = u % g.tilesU;
            SMOE_PROF(cy_t = clock64();)
            if (!mbar_wait_bounded(hR + b, (n >> 1) & 1)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            SMOE_PROF(cy_hw += clock64() - cy_t; cy_t = clock64();)
            const uint8_t* sp = ring + size_t(st) * g.stage;
            const uint32_t* sl = reinterpret_cast<const uint32_t*>(sp + tg.gateup);
            const uint2* dB = reinterpret_cast<const uint2*>(sm + g.o_hq + b * 256 + 64);
            const uint2 bv = lane < 8 ? dB[lane] : make_uint2(0u, 0u);
            const uint32_t bb[2] = {bv.x, bv.y};
            const float hs = *reinterpret_cast<const float*>(sm + g.o_hq + b * 256 + 128);
            const uint16_t* dsc = sbc0 + ((u / 4) & 1) * (tg.dgroup / 2);
            const uint16_t* dbi = dsc + d;
            float* yt = ysum + tok * d;
#pragma unroll
            for (int q = 0; q < kDownRegTiles; ++q) {
                const int o = warp + q * kFusedConsumers;
#ifdef SMOE_EXP_NODOWN
                if (false) {
#else
                if (o < g.outTiles) {
#endif
                    const uint32_t w = sl[o * 32 + lane];
                    uint32_t a[4];
                    a[0] = lop3_and_or(w, M, OR);
                    a[1] = lop3_and_or(w >> 4, M, OR);
                    a[2] = lop3_and_or(w >> 8, M, OR);
                    a[3] = lop3_and_or(w >> 12, M, OR);
                    mma_bf16_16816(dacc[q], a, bb);
                }
            }
            for (int o = warp + kDownRegTiles * kFusedConsumers; o < g.outTiles; o += kFusedConsumers) {
                float dd[4] = {0.f, 0.f, 0.f, 0.f};
                const uint32_t w = sl[o * 32 + lane];
                uint32_t a[4];
                a[0] = lop3_and_or(w, M, OR);
                a[1] = lop3_and_or(w >> 4, M, OR);
                a[2] = lop3_and_or(w >> 8, M, OR);
                a[3] = lop3_and_or(w >> 12, M, OR);
                mma_bf16_16816(dd, a, bb);
                if ((lane & 3) == 0) {
                    const int r0 = o * 16 + gr, r8 = r0 + 8;
                    yt[r0] += group_epi<FMT>(dd[0] + dd[1], hs, dsc, dbi, r0);
                    yt[r8] += group_epi<FMT>(dd[2] + dd[3], hs, dsc, dbi, r8);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + st);           // stage of unit n fully consumed
            if (n < 3) trace_mark(A.trace, 22 + n);
            hsg += hs;
            SMOE_PROF(cy_dn += clock64() - cy_t; if (n < 3 && A.trace && lane == 0 && warp == 0) reinterpret_cast<long long*>(A.trace)[gridDim.x * 48 + blockIdx.x * 8 + 4 + n] = clock64() - cy_t;)
            const bool last = (u + 1 == u1);
            if (last || (t & 3) == 3) {
                // group ends: scale once per group and add into the token's
                // partial output. All shared-memory loads of the flush are
                // issued before any store (the compiler cannot prove that the
                // stores to yt do not alias the scale loads).
                if ((lane & 3) == 0) {
#pragma unroll
                    for (int q0 = 0; q0 < kDownRegTiles; q0 += 4) {      // 4 tiles: 24 loads in flight
                        float sv[4][2], bi[4][2], yv[4][2];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int o = min(warp + (q0 + q) * kFusedConsumers, g.outTiles - 1);
                            const int r0 = o * 16 + gr;
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                if (FMT == kFmtAffine) {
                                    sv[q][h] = bf16_bits_to_f32(dsc[r0 + 8 * h]);
                                    bi[q][h] = bf16_bits_to_f32(dbi[r0 + 8 * h]);
                                } else {
                                    sv[q][h] = f16_bits_to_f32(dsc[r0 + 8 * h]);
                                    bi[q][h] = 0.f;
                                }
                                yv[q][h] = yt[r0 + 8 * h];
                            }
                        }
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int o = warp + (q0 + q) * kFusedConsumers;
                            if (o < g.outTiles) {
#pragma unroll
                                for (int h = 0; h < 2; ++h) {
                                    const float dsum = dacc[q0 + q][2 * h] + dacc[q0 + q][2 * h + 1];
                                    const float qv = fmaf(-128.0f, hsg, dsum);
                                    const float v = (FMT == kFmtAffine) ? sv[q][h] * qv + bi[q][h] * hsg
                                                                        : sv[q][h] * (qv * (1.0f / 7.5f) - hsg);
                                    yt[o * 16 + gr + 8 * h] = yv[q][h] + v;
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < kDownRegTiles; ++q) dacc[q][0] = dacc[q][1] = dacc[q][2] = dacc[q][3] = 0.f;
                hsg = 0.f;
            }
        };
        // step n: gate/up of unit n (if any), then the down slice of unit n-1;
        // one call site each keeps the loop body small (instruction cache)
        const int nun = u1 - u0;
        for (int n = 0; n <= nun; ++n) {
          if (n < nun) {
            const int u = u0 + n;
            const int st = n % NS, b = n & 1;
            const int slot = slot_of(u), tok = slot / k;
            SMOE_PROF(cy_t = clock64();)
            if (!mbar_wait_bounded(full + st, (n / NS) & 1)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            SMOE_PROF(cy_wait += clock64() - cy_t; cy_t = clock64();)
            if (n < 3) trace_mark(A.trace, 16 + n);
            const uint8_t* sp = ring + size_t(st) * g.stage;
            // -- gate / up dots of the unit's 16 rows: groups warp + 16j
            const uint8_t* sbp = sp + 2 * tg.fragA;              // [gate sb][up sb]
            float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
            uint4 w[GW][2];
#pragma unroll
            for (int j = 0; j < GW; ++j) {
                const int grp = min(warp + j * kFusedConsumers, g.G - 1);
#pragma unroll
                for (int m = 0; m < 2; ++m)
                    w[j][m] = *reinterpret_cast<const uint4*>(sp + m * tg.fragA + (grp * 32 + lane) * 16);
            }
#pragma unroll
            for (int j = 0; j < GW; ++j) {
                const int grp = warp + j * kFusedConsumers;
                if (grp < g.G) {
                    const float2 xv = xg[grp * 4 + cq];
                    const uint4 bA = xtab[(grp * 2) * 32 + lane], bB = xtab[(grp * 2 + 1) * 32 + lane];
                    const uint32_t be[2] = {bA.x, bA.y}, bo[2] = {bA.z, bA.w};
                    const uint32_t be2[2] = {bB.x, bB.y}, bo2[2] = {bB.z, bB.w};
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const uint32_t ae[4] = {w[j][m].x & 0x0F0F0F0Fu, w[j][m].y & 0x0F0F0F0Fu,
                                                w[j][m].z & 0x0F0F0F0Fu, w[j][m].w & 0x0F0F0F0Fu};
                        const uint32_t ao[4] = {w[j][m].x & 0xF0F0F0F0u, w[j][m].y & 0xF0F0F0F0u,
                                                w[j][m].z & 0xF0F0F0F0u, w[j][m].w & 0xF0F0F0F0u};
                        int de[4] = {0, 0, 0, 0}, dO[4] = {0, 0, 0, 0}, de2[4] = {0, 0, 0, 0}, dO2[4] = {0, 0, 0, 0};
                        mma_u8s8_16832(de, ae, be);
                        mma_u8s8_16832(dO, ao, bo);
                        mma_u8s8_16832(de2, ae, be2);
                        mma_u8s8_16832(dO2, ao, bo2);
                        const float v0 = fmaf(float(16 * de2[0] + dO2[0]), 65536.0f,
                                              float((16 * de[0] + dO[0]) + 256 * (16 * de[1] + dO[1])));
                        const float v8 = fmaf(float(16 * de2[2] + dO2[2]), 65536.0f,
                                              float((16 * de[2] + dO[2]) + 256 * (16 * de[3] + dO[3])));
                        if (FMT == kFmtAffine) {
                            const uint32_t* sbw = reinterpret_cast<const uint32_t*>(sbp + m * tg.sbA) + grp * 16 + gr;
                            const uint32_t s0 = sbw[0], s8 = sbw[8];
                            acc[m][0] += fmaf(bf16_bits_to_f32(uint16_t(s0)), v0 * xv.x,
                                              bf16_bits_to_f32(uint16_t(s0 >> 16)) * xv.y);
                            acc[m][1] += fmaf(bf16_bits_to_f32(uint16_t(s8)), v8 * xv.x,
                                              bf16_bits_to_f32(uint16_t(s8 >> 16)) * xv.y);
                        } else {
                            const uint16_t* sbh = reinterpret_cast<const uint16_t*>(sbp + m * tg.sbA) + grp * 16 + gr;
                            acc[m][0] += f16_bits_to_f32(sbh[0]) * fmaf(v0, xv.x, -xv.y);
                            acc[m][1] += f16_bits_to_f32(sbh[8]) * fmaf(v8, xv.x, -xv.y);
                        }
                    }
                }
            }
            float* rb = red0 + (b * kFusedConsumers + warp) * 32;
            if (cq == tok) {
                rb[gr] = acc[0][0];
                rb[gr + 8] = acc[0][1];
                rb[16 + gr] = acc[1][0];
                rb[16 + gr + 8] = acc[1][1];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(redF + b);
            SMOE_PROF(cy_gu += clock64() - cy_t; if (n < 3 && A.trace && lane == 0 && warp == 0) reinterpret_cast<long long*>(A.trace)[gridDim.x * 48 + blockIdx.x * 8 + n] = clock64() - cy_t;)
            if (n < 3) trace_mark(A.trace, 19 + n);
          }
          if (n > 0) down(u0 + n - 1, n - 1);
        }
        trace_mark(A.trace, 3);
        if (A.trace && lane == 0 && (warp == 0 || warp == 15)) {
            SMOE_PROF(long long* cy = reinterpret_cast<long long*>(A.trace) + gridDim.x * 40 + blockIdx.x * 8 + (warp ? 4 : 0);)
            SMOE_PROF(cy[0] = cy_wait; cy[1] = cy_gu; cy[2] = cy_hw; cy[3] = cy_dn;)
        }
    }

    // the next kernel in the stream may start its launch now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // ---------------- partial outputs: vector reductions into the accumulator
    if (consumer) {
        consumer_sync();                             // every warp's share of ysum is written
        for (int i = tid; i < g.ntok * d / 4; i += kFusedCThreads)
            red_add_v4(A.acc + 4 * i, reinterpret_cast<const float4*>(ysum)[i]);
    }
    trace_mark(A.trace, 6);

    // ------------------------------------- last CTA: write y, clear scratch
    __syncthreads();
    if (tid == 0) {
        trace_mark(A.trace, 14);
        // acq_rel: releases this CTA's reductions (ordered before it by the
        // barrier) and, in the last CTA, acquires every other CTA's
        uint32_t old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&A.st->done) : "memory");
        last_cta = (old == gridDim.x - 1) ? 1u : 0u;
        trace_mark(A.trace, 15);
    }
    __syncthreads();
    if (last_cta) {
        const int n4 = g.ntok * d / 4;                               // d % 64 == 0: whole float4s
        float4* acc4 = reinterpret_cast<float4*>(A.acc);
        if (epm && ep.rank > 0) {
            // this rank's partial output -> rank 0 (peer stores), then count it
            float4* dst = reinterpret_cast<float4*>(ep.part0 + size_t(ep.rank) * ep.part_stride);
            for (int i = tid; i < n4; i += blockDim.x) {
                dst[i] = __ldcg(acc4 + i);
                acc4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            __syncthreads();
            if (tid == 0) {
                __threadfence_system();
                atomicAdd_system(ep.done0, 1u);
            }
        } else {
            if (epm) {                                               // wait for every other rank's partial
                if (tid == 0 && !spin_sys_until_geq(ep.done0, uint32_t(ep.world - 1)))
                    atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT);
                __syncthreads();
            }
            for (int i = tid; i < n4; i += blockDim.x) {
                float4 v = __ldcg(acc4 + i);
                for (int r = 1; r < (epm ? ep.world : 1); ++r) {       // rank order
                    const float4 p = __ldcg(reinterpret_cast<const float4*>(ep.part0 + size_t(r) * ep.part_stride) + i);
                    v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
                }
                acc4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (f.y_dtype == 0) {
                    reinterpret_cast<float4*>(f.y)[i] = v;
                } else {
                    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
                    uint2 o;
                    o.x = *reinterpret_cast<uint32_t*>(&lo);
                    o.y = *reinterpret_cast<uint32_t*>(&hi);
                    reinterpret_cast<uint2*>(f.y)[i] = o;
                }
            }
            // the other ranks' next partials come only after the next x epoch
            if (epm && tid == 0) *ep.done0 = 0u;
        }
        if (tid == 0) {
            A.st->rdone = 0;
            A.st->done = 0;
            if (epm) A.st->epoch = epoch;
        }
        // (no fence: the next launch reads these counters only after this
        // grid has completed - stream order or griddepcontrol.wait)
    }
    trace_mark(A.trace, 7);
    SMOE_PROF(if (A.trace && tid == 0) A.trace[gridDim.x * 32 + blockIdx.x * 8 + 5] = clock64();)
}

}  // namespace smoe
