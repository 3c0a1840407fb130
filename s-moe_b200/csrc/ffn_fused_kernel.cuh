// ffn_fused_kernel.cuh - the persistent MoE-layer kernel (design notes in
// ffn_fused.cuh).
#pragma once
#include "ffn_fused.cuh"

namespace smoe {

// Phase R: logit row r = (token, expert) by all consumer warps of this CTA.
SMOE_DEVINL float router_row(const FusedArgs& A, uint32_t t, uint32_t e, int ctid) {
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
                reinterpret_cast<const float4*>(static_cast<const float*>(f.x) + size_t(t) * d + c * 8);
            const float4 a0 = xp[0], a1 = xp[1];
            xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
            xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
        } else {
            const uint4 b =
                *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(f.x) + size_t(t) * d + c * 8);
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

template <int FMT>
__global__ void __launch_bounds__(kFusedThreads, 1) k_moe_fused(FusedArgs A) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const FusedGeom& g = A.g;
    const FfnArgs& f = A.f;
    const TiledGeom& tg = g.tg;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool consumer = warp < kFusedConsumers;
    uint8_t* ring = sm + g.o_ring;
    uint2* xtab = reinterpret_cast<uint2*>(sm + g.o_xtab);
    float* xg = reinterpret_cast<float*>(sm + g.o_xg);
    uint2* htab = reinterpret_cast<uint2*>(sm + g.o_htab);
    float* hg = reinterpret_cast<float*>(sm + g.o_hg);
    float* red = reinterpret_cast<float*>(sm + g.o_red);       // [kFusedRedBufs][16 warps][32]
    float* redB = reinterpret_cast<float*>(sm + g.o_yslot);    // [4 chunks][16 warps][32]
    float* hq = reinterpret_cast<float*>(sm + g.o_hq);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + g.o_bar);
    uint64_t* empty = full + 16;
    uint64_t* pub_full = full + 32;
    uint64_t* pub_empty = pub_full + kFusedRedBufs;
    uint32_t* s_ids = reinterpret_cast<uint32_t*>(sm + g.o_ids);
    float* s_w = reinterpret_cast<float*>(sm + g.o_w);
    float* ps = reinterpret_cast<float*>(sm + g.o_ps);
    float* vst = reinterpret_cast<float*>(sm + g.o_vst);
    const int NS = g.nstages, k = g.k, d = g.d, dff = g.dff;
    const uint32_t nslots = uint32_t(g.ntok * k);

    trace_mark(A.trace, 0);
    const uint32_t tag = ld_volatile_u32(&A.st->epoch) + 1u;    // this launch's h-table tag
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kFusedConsumers);
        }
        for (int i = 0; i < kFusedRedBufs; ++i) {
            mbar_init(pub_full + i, kFusedConsumers);
            mbar_init(pub_empty + i, 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // ---------------------------------------------------------- routing
    if (A.rw) {
        const uint32_t rows = A.E * g.ntok;
        for (uint32_t r = blockIdx.x; r < rows; r += gridDim.x) {
            float v = 0.f;
            if (consumer) v = router_row(A, r / A.E, r % A.E, tid);
            if (consumer && lane == 0) red[warp] = v;
            __syncthreads();
            if (tid == 0) {
                float sum = 0.f;
                for (int w = 0; w < kFusedConsumers; ++w) sum += red[w];
                A.logits[r] = sum;
                __threadfence();
                atomicAdd(&A.st->rdone, 1u);
            }
            __syncthreads();
        }
    }
    // x: one round of wide loads, finished before any weight copy is issued
    // (loads issued behind this SM's bulk traffic would wait for all of it)
    if (consumer) {
        if (f.x_dtype == 0) stage_vec_smem<false>(f.x, g.ntok * d, vst, tid);
        else stage_vec_smem<true>(f.x, g.ntok * d, vst, tid);
    }
    if (A.rw) {
        if (tid == 0 && !spin_until_geq(&A.st->rdone, A.E * g.ntok)) atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT);
        __syncthreads();
        if (warp < g.ntok) {
            warp_topk(A.logits + size_t(warp) * A.E, A.E, k, A.norm, ps + warp * kRouterMaxE,
                      s_ids + warp * k, s_w + warp * k, lane);
            __syncwarp();
            if (blockIdx.x == 0 && lane < k) {
                const_cast<uint32_t*>(f.ids)[warp * k + lane] = s_ids[warp * k + lane];
                const_cast<float*>(f.wts)[warp * k + lane] = s_w[warp * k + lane];
            }
        }
    } else {
        for (uint32_t i = tid; i < nslots; i += blockDim.x) {
            s_ids[i] = f.ids[i];
            s_w[i] = f.wts[i];
        }
    }
    __syncthreads();
    trace_mark(A.trace, 1);

    const FusedShare sh{A.a_bound[blockIdx.x], A.a_bound[blockIdx.x + 1],
                        int(blockIdx.x * g.nB / gridDim.x), int((blockIdx.x + 1) * g.nB / gridDim.x)};

    if (warp == kFusedProdWarp) {
        // ------------------------------------------------------ producer
        int n = 0;
        auto acquire = [&](int stage_n, uint32_t bytes) -> uint8_t* {
            const int st = stage_n % NS, round = stage_n / NS;
            if (round > 0 && lane == 0 && !mbar_wait_bounded(empty + st, (round - 1) & 1))
                atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            __syncwarp();
            if (lane == 0) mbar_arrive_expect_tx(full + st, bytes);
            __syncwarp();
            return ring + size_t(st) * g.stage;
        };
        for (int u = sh.a0; u < sh.a1; ++u, ++n) {
            const int slot = u / g.tilesA, tile = u % g.tilesA;
            uint8_t* sp = acquire(n, tg.tileA);
            if (lane == 0)
                bulk_g2s(sp, f.base + uint64_t(s_ids[slot]) * f.stride + tg.a_tile(tile), tg.tileA, full + n % NS);
        }
        for (int v = sh.b0; v < sh.b1; ++v) {
            const int tok = v / g.tilesB, tile = v % g.tilesB;
            for (int ch = 0; ch < g.chunksB; ++ch, ++n) {
                const int j0 = ch * kFusedSlotsPerB, nj = min(kFusedSlotsPerB, k - j0);
                uint8_t* sp = acquire(n, nj * tg.tileB);
                if (lane < nj)
                    bulk_g2s(sp + lane * tg.tileB,
                             f.base + uint64_t(s_ids[tok * k + j0 + lane]) * f.stride + tg.b_tile(tile), tg.tileB,
                             full + n % NS);
            }
        }
    } else if (warp == kFusedPubWarp) {
        // ---------------------------------------------------- publisher
        // Reduces each phase-A unit over the 16 consumer warps and writes its
        // 16 h rows as tagged B-table entries + tagged quarter sum. Readers
        // validate the tags, so no fence or counter is needed.
        for (int u = sh.a0; u < sh.a1; ++u) {
            const int i = u - sh.a0, b = i % kFusedRedBufs;
            const int slot = u / g.tilesA, tile = u % g.tilesA;
            if (!mbar_wait_bounded(pub_full + b, (i / kFusedRedBufs) & 1))
                atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            const float* rb = red + b * kFusedConsumers * 32;
            float acc = 0.f;                                          // lane = (matrix, row)
#pragma unroll
            for (int w = 0; w < kFusedConsumers; ++w) acc += rb[w * 32 + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(pub_empty + b);                // red buffer b is free again
            const float up = __shfl_down_sync(0xffffffffu, acc, 16);
            if (lane < 16) hq[lane] = acc * (1.0f / (1.0f + expf(-acc))) * up;   // kernels.metal:61-63
            __syncwarp();
            const int grp = tile >> 2, c = tile & 3;                  // rows = lane quarter c of grp
            if (lane < 8) {
                const int s = lane >> 1, col = lane & 1;
                st_tagged2(A.htab_g + (size_t(slot) * (dff / 16) + grp * 4 + s) * 8 + col * 4 + c,
                           btab_entry(hq, s, col), tag);
            }
            float qs = 0.f;                                           // quarter sum of hi + lo
            if (lane < 16) {
                const float hv = hq[lane];
                const float hi = __bfloat162float(__float2bfloat16_rn(hv));
                qs = hi + __bfloat162float(__float2bfloat16_rn(hv - hi));
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
            if (lane == 0) {
                st_tagged1(A.hsum_g + (size_t(slot) * g.Gd + grp) * 4 + c, qs, tag);
                atomicAdd(&A.st->hcount[slot / k], 1u);   // a hint for readers, no ordering implied
            }
            __syncwarp();
        }
    } else {
        // ----------------------------------------------------- consumers
        const int ctid = tid, gr = lane >> 2;
        build_btab_bf16(vst, g.ntok, d, xtab, xg, ctid);
        consumer_sync();
        int n = 0;
        // phase A: gate/up dots of each unit -> reduction buffer -> publisher
        for (int u = sh.a0; u < sh.a1; ++u, ++n) {
            const int i = u - sh.a0, b = i % kFusedRedBufs;
            const int st = n % NS;
            const int slot = u / g.tilesA, tok = slot / k;
            if (!mbar_wait_bounded(full + st, (n / NS) & 1)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            const uint8_t* sp = ring + size_t(st) * g.stage;
            const uint16_t* sb = reinterpret_cast<const uint16_t*>(sp + 2 * tg.fragA);   // [gsc][usc][gbi][ubi]
            const int nsc = tg.scA / 2;
            const uint2* bt = xtab + tok * (d / 16) * 8;
            float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
            const int ng = (A.dbg_skip == 1) ? 0 : g.G;
            int grp = warp;
            for (; grp + kFusedConsumers < ng; grp += 2 * kFusedConsumers) {      // 4 group-mats at once
                const uint8_t* fr[4] = {sp, sp + tg.fragA, sp, sp + tg.fragA};
                const int gp[4] = {grp, grp, grp + kFusedConsumers, grp + kFusedConsumers};
                const uint2* bts[4] = {bt, bt, bt, bt};
                float r0[4], r8[4];
                group_mma_n<4>(fr, gp, bts, lane, r0, r8);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int m = q & 1, gq = gp[q];
                    const float xs = xg[tok * g.G + gq];
                    acc[m][0] += group_epi<FMT>(r0[q], xs, sb + m * nsc, sb + (2 + m) * nsc, gq * 16 + gr);
                    acc[m][1] += group_epi<FMT>(r8[q], xs, sb + m * nsc, sb + (2 + m) * nsc, gq * 16 + gr + 8);
                }
            }
            for (; grp < ng; grp += kFusedConsumers) {                              // remainder
                const uint8_t* fr[2] = {sp, sp + tg.fragA};
                const int gp[2] = {grp, grp};
                const uint2* bts[2] = {bt, bt};
                float r0[2], r8[2];
                group_mma_n<2>(fr, gp, bts, lane, r0, r8);
                const float xs = xg[tok * g.G + grp];
#pragma unroll
                for (int m = 0; m < 2; ++m) {
                    acc[m][0] += group_epi<FMT>(r0[m], xs, sb + m * nsc, sb + (2 + m) * nsc, grp * 16 + gr);
                    acc[m][1] += group_epi<FMT>(r8[m], xs, sb + m * nsc, sb + (2 + m) * nsc, grp * 16 + gr + 8);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + st);
            if (i >= kFusedRedBufs && !mbar_wait_bounded(pub_empty + b, ((i / kFusedRedBufs) - 1) & 1))
                atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
            float* rb = red + (b * kFusedConsumers + warp) * 32;
            if ((lane & 3) == 0) {
                rb[gr] = acc[0][0];
                rb[gr + 8] = acc[0][1];
                rb[16 + gr] = acc[1][0];
                rb[16 + gr + 8] = acc[1][1];
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(pub_full + b);
        }
        trace_mark(A.trace, 3);
        // phase B: down projection of the token's k slots + combine
        for (int v = sh.b0; v < sh.b1; ++v) {
            const int tok = v / g.tilesB, tile = v % g.tilesB;
            // cheap gate: one thread polls the token's counter; the tags below
            // remain the proof that each entry is this launch's data
            if (ctid == 0 && !spin_until_geq(&A.st->hcount[tok], uint32_t(k * g.tilesA)))
                atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT);
            consumer_sync();
            trace_mark(A.trace, 4);
            {   // h tables of the token's k slots, tag-validated, into shared memory
                const int sl0 = tok * k;
                const uint4* src = A.htab_g + size_t(sl0) * (dff / 16) * 8;
                const int n16 = k * (dff / 16) * 8;
                uint4 t[6];
#pragma unroll
                for (int q = 0; q < 6; ++q) {
                    const int ii = ctid + q * kFusedCThreads;
                    if (ii < n16) t[q] = ld_tagged2(src + ii);
                }
                const int ngs = k * g.Gd * 4;
                uint2 hsv = make_uint2(0u, tag);
                if (ctid < ngs) hsv = ld_tagged1(A.hsum_g + size_t(sl0) * g.Gd * 4 + ctid);
#pragma unroll
                for (int q = 0; q < 6; ++q) {
                    const int ii = ctid + q * kFusedCThreads;
                    if (ii < n16) {
                        for (uint32_t it = 0; (t[q].y != tag || t[q].w != tag); ++it) {
                            if (it > SMOE_SPIN_LIMIT) { atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT); break; }
                            if (it > 32) __nanosleep(32);
                            t[q] = ld_tagged2(src + ii);
                        }
                        htab[ii] = make_uint2(t[q].x, t[q].z);
                    }
                }
                for (int ii = ctid + 6 * kFusedCThreads; ii < n16; ii += kFusedCThreads) {
                    uint4 tt = ld_tagged2(src + ii);
                    for (uint32_t it = 0; (tt.y != tag || tt.w != tag); ++it) {
                        if (it > SMOE_SPIN_LIMIT) { atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT); break; }
                        if (it > 32) __nanosleep(32);
                        tt = ld_tagged2(src + ii);
                    }
                    htab[ii] = make_uint2(tt.x, tt.z);
                }
                for (int ii = ctid; ii < ngs; ii += kFusedCThreads) {
                    if (ii != ctid) hsv = ld_tagged1(A.hsum_g + size_t(sl0) * g.Gd * 4 + ii);
                    for (uint32_t it = 0; hsv.y != tag; ++it) {
                        if (it > SMOE_SPIN_LIMIT) { atomicExch(f.err, SMOE_DEVERR_SPIN_TIMEOUT); break; }
                        if (it > 32) __nanosleep(32);
                        hsv = ld_tagged1(A.hsum_g + size_t(sl0) * g.Gd * 4 + ii);
                    }
                    vst[ii] = __uint_as_float(hsv.x);       // quarter sums (x staging is free now)
                }
            }
            consumer_sync();
            if (ctid < k * g.Gd) hg[ctid] = (vst[4 * ctid] + vst[4 * ctid + 1]) + (vst[4 * ctid + 2] + vst[4 * ctid + 3]);
            consumer_sync();
            trace_mark(A.trace, 5);
            for (int ch = 0; ch < g.chunksB; ++ch, ++n) {
                const int st = n % NS;
                const int j0 = ch * kFusedSlotsPerB, nj = min(kFusedSlotsPerB, k - j0);
                if (!mbar_wait_bounded(full + st, (n / NS) & 1)) atomicExch(f.err, SMOE_DEVERR_MBAR_TIMEOUT);
                if (ch == 0) trace_mark(A.trace, 7);
                const uint8_t* sp = ring + size_t(st) * g.stage;
                const int jj = warp >> 2, quarter = warp & 3;
                float y0 = 0.f, y8 = 0.f;
                if (jj < nj) {
                    const int j = j0 + jj;
                    const uint8_t* tp = sp + jj * tg.tileB;
                    const uint16_t* sc = reinterpret_cast<const uint16_t*>(tp + tg.fragB);
                    const uint16_t* bi = sc + tg.scB / 2;
                    const uint2* hb = htab + j * (dff / 16) * 8;
                    int grp = quarter;
                    for (; grp + 8 < g.Gd; grp += 12) {                     // 3 groups at once
                        const uint8_t* fr[3] = {tp, tp, tp};
                        const int gp[3] = {grp, grp + 4, grp + 8};
                        const uint2* bts[3] = {hb, hb, hb};
                        float r0[3], r8[3];
                        group_mma_n<3>(fr, gp, bts, lane, r0, r8);
#pragma unroll
                        for (int q = 0; q < 3; ++q) {
                            const float hs = hg[j * g.Gd + gp[q]];
                            y0 += group_epi<FMT>(r0[q], hs, sc, bi, gp[q] * 16 + gr);
                            y8 += group_epi<FMT>(r8[q], hs, sc, bi, gp[q] * 16 + gr + 8);
                        }
                    }
                    for (; grp < g.Gd; grp += 4) {
                        const uint8_t* fr[1] = {tp};
                        const int gp[1] = {grp};
                        const uint2* bts[1] = {hb};
                        float r0[1], r8[1];
                        group_mma_n<1>(fr, gp, bts, lane, r0, r8);
                        const float hs = hg[j * g.Gd + grp];
                        y0 += group_epi<FMT>(r0[0], hs, sc, bi, grp * 16 + gr);
                        y8 += group_epi<FMT>(r8[0], hs, sc, bi, grp * 16 + gr + 8);
                    }
                }
                if (ch == 0) trace_mark(A.trace, 2);
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + st);
                if ((lane & 3) == 0) {
                    redB[(ch * kFusedConsumers + warp) * 32 + gr] = y0;
                    redB[(ch * kFusedConsumers + warp) * 32 + gr + 8] = y8;
                }
            }
            consumer_sync();
            if (ctid < 16) {
                float o = 0.f;     // routed[i] += w * y[i]: product then sum, no FMA (axpy_f32)
                for (int j = 0; j < k; ++j) {
                    const float* rj = redB + ((j / kFusedSlotsPerB) * kFusedConsumers + (j % kFusedSlotsPerB) * 4) * 32;
                    const float yj = (rj[ctid] + rj[32 + ctid]) + (rj[64 + ctid] + rj[96 + ctid]);
                    o = __fadd_rn(o, __fmul_rn(s_w[tok * k + j], yj));
                }
                const size_t oi = size_t(tok) * d + tile * 16 + ctid;
                if (f.y_dtype == 0) static_cast<float*>(f.y)[oi] = o;
                else static_cast<__nv_bfloat16*>(f.y)[oi] = __float2bfloat16_rn(o);
            }
        }
    }

    // ------------------------------------------------ finish: reset counters
    trace_mark(A.trace, 6);
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&A.st->done, 1u);
        if (old == gridDim.x - 1) {
            A.st->rdone = 0;
            A.st->done = 0;
            for (int t = 0; t < kFusedMaxTok; ++t) A.st->hcount[t] = 0;
            A.st->epoch = tag;                   // next launch tags with tag + 1
            __threadfence();
        }
    }
}

}  // namespace smoe
