// seqsum.cuh - the reference's sequential fp32 sum, reproduced exactly in
// parallel (for sampler.hpp:113-129: sum_exp += e in index order).
//
// Facts used:
//  * While the running sum s stays in one binade [2^b, 2^(b+1)) its ulp u is
//    fixed and s = S*u for an integer S in [2^23, 2^24). For e >= 0,
//    fl(s + e) = (S + round(e/u)) * u exactly, as long as e/u is not a tie
//    (fractional part 1/2, where rounding to even depends on S) and the
//    result stays below 2^(b+1). So a run of elements with no tie and no
//    binade crossing advances S by an integer that does not depend on S.
//  * With non-negative terms the sequential fp32 sum after i terms deviates
//    from the exact prefix P_i by at most gamma_i * P_i, gamma_i =
//    i*2^-24 / (1 - i*2^-24) (< 1.2% for 196,608 terms), so fp64 prefix sums
//    predict the binade of every chunk, up to chunks within that margin of a
//    binade boundary.
// Layout: element i lives in CTA (i / L) of the cluster, thread-contiguous
// chunks of C elements, warp-chunks of 32*C elements (256 per cluster).
// Each warp summarises its chunk for its predicted binade; one warp of CTA 0
// walks the 256 summaries in order and replays only chunks that straddle a
// binade or contain a tie, element by element with real fp32 additions.
#pragma once
#include <cooperative_groups.h>
#include "smoe_common.cuh"

namespace smoe {

constexpr int kSeqChunks = 256;            // 8 CTAs x 32 warps
constexpr int kSeqMaxC = 24;               // elements per thread (vocab <= 8 * 1024 * 24)
constexpr uint32_t kSeqTie = 1u, kSeqStraddle = 2u, kSeqOver = 4u;

SMOE_DEVINL int f32_expo(float s) { return int((__float_as_uint(s) >> 23) & 0xff); }
SMOE_DEVINL long long f32_units(float s) { return (long long)((__float_as_uint(s) & 0x7fffffu) | 0x800000u); }
SMOE_DEVINL float f32_from(int expo, long long units) {     // units in [2^23, 2^24)
    return __uint_as_float((uint32_t(expo) << 23) | uint32_t(units - 0x800000ll));
}

// round(e / u) with u = 2^(expo - 150) for e >= 0, in integer arithmetic on
// e's bits: e = M * 2^(E - 150) (M with the implicit bit; subnormals E = 1),
// so e/u = M * 2^(E - expo). Returns the increment, sets *tie when the
// fractional part is exactly 1/2. Values that cannot be absorbed without a
// binade crossing return a huge increment.
SMOE_DEVINL long long inc_for(float e, int expo, bool* tie) {
    const uint32_t b = __float_as_uint(e);
    int E = int((b >> 23) & 0xff);
    uint32_t M = b & 0x7fffffu;
    *tie = false;
    if (E == 255) return 1ll << 40;
    if (E) M |= 0x800000u;
    else E = 1;
    const int k = E - expo;
    if (k >= 0) return k > 16 ? (1ll << 40) : ((long long)M << k);
    const int sh = -k;
    if (sh > 25) return 0;                               // e/u < 1/2
    const uint32_t half = 1u << (sh - 1), rem = M & ((half << 1) - 1u);
    *tie = (rem == half);
    return (long long)(M >> sh) + (rem > half ? 1 : 0);
}

struct SeqShared {            // per CTA
    double wtot[32];          // warp-chunk totals (fp64)
    int tinc[2][1024];        // per thread: increment at the chunk's predicted binade and the next
    uint8_t tflag[1024];      // per thread: bit0 tie at binade, bit1 tie at binade+1, bit2/3 overflow
    int binfo[32];            // predicted exponent | (flags << 16) for this CTA's warp-chunks
    // CTA 0 only: summaries of all 256 warp-chunks
    long long sinc[kSeqChunks];
    int sinfo[kSeqChunks];    // exponent | flags << 16
    float result;
};

// Exact sequential fp32 sum of e[0..V) held in the cluster's shared memory
// (e: this CTA's slice, n elements, slice length L, C per thread), part 1:
// chunk totals, predicted binades and chunk summaries. All threads of all
// CTAs call it; seq_walk (below) then produces the sum.
SMOE_DEVINL void seq_mark(unsigned long long* tr, int i) {
    if (tr && threadIdx.x == 0 && blockIdx.y == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        tr[64 + blockIdx.x * 8 + i] = t;
    }
}

SMOE_DEVINL void seq_summarise_cluster(cooperative_groups::cluster_group& cl, const float* e, uint32_t n,
                                 uint32_t L, uint32_t V, uint32_t C, SeqShared* ss,
                                 unsigned long long* tr = nullptr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, rank = (int)cl.block_rank();
    const uint32_t c0 = min(n, tid * C), c1 = min(n, c0 + C);
    // 1. warp-chunk totals
    double t = 0.0;
    for (uint32_t i = c0; i < c1; ++i) t += (double)e[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) ss->wtot[warp] = t;
    cl.sync();
    seq_mark(tr, 0);
    // 2. CTA 0: prefix sums -> predicted binade + straddle flag per chunk
    if (rank == 0 && warp == 0) {
        double tot[8];
        for (int q = 0; q < 8; ++q) {
            const int c = q * 32 + lane;
            tot[q] = cl.map_shared_rank(ss, c >> 5)->wtot[c & 31];
        }
        double base = 0.0;
        const double gam = double(V) * 0x1p-24 / (1.0 - double(V) * 0x1p-24);
        for (int q = 0; q < 8; ++q) {
            double inc = tot[q];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const double y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            const double pend = base + inc, pstart = pend - tot[q];
            base += __shfl_sync(0xffffffffu, inc, 31);
            const float lo = (float)(pstart * (1.0 - gam)), hi = (float)(pend * (1.0 + gam));
            const int elo = f32_expo(lo), ehi = f32_expo(hi);
            uint32_t flags = 0;
            if (elo != ehi || elo == 0 || !(pstart * (1.0 - gam) > 0.0) || ehi == 255) flags |= kSeqStraddle;
            const int c = q * 32 + lane;
            cl.map_shared_rank(ss, c >> 5)->binfo[c & 31] = elo | int(flags << 16);
        }
    }
    cl.sync();
    seq_mark(tr, 1);
    // 3. every thread summarises its elements for the warp-chunk's predicted
    //    binade and the next one; warps reduce to chunk summaries
    {
        const int info = ss->binfo[warp];
        const int expo = info & 0xffff;
        uint32_t flags = uint32_t(info) >> 16;
        long long i0 = 0, i1 = 0;
        bool t0 = false, t1 = false;
        for (uint32_t i = c0; i < c1; ++i) {
            bool ta, tb;
            i0 += inc_for(e[i], expo, &ta);
            i1 += inc_for(e[i], expo + 1, &tb);
            t0 |= ta;
            t1 |= tb;
        }
        const long long cap = 1ll << 30;
        ss->tinc[0][tid] = int(i0 < cap ? i0 : cap);
        ss->tinc[1][tid] = int(i1 < cap ? i1 : cap);
        ss->tflag[tid] = uint8_t((t0 ? 1 : 0) | (t1 ? 2 : 0));
        long long inc = (flags & kSeqStraddle) ? 0 : i0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) inc += __shfl_xor_sync(0xffffffffu, inc, o);
        if (__any_sync(0xffffffffu, t0)) flags |= kSeqTie;
        if (inc >= (1ll << 24)) flags |= kSeqOver;
        if (lane == 0) {
            SeqShared* s0 = cl.map_shared_rank(ss, 0);
            s0->sinc[rank * 32 + warp] = inc;
            s0->sinfo[rank * 32 + warp] = expo | int(flags << 16);
        }
    }
    cl.sync();
    seq_mark(tr, 2);
}

// 4. the walk: one warp (warp 0 of CTA 0) goes through the 256 summaries in
// order, replaying only chunks that straddle a binade or hold a tie; reads
// the other CTAs' e values and thread increments through distributed shared
// memory, so they must stay resident (and leave them unchanged) until it
// returns. The result is in CTA 0's ss->result.
SMOE_DEVINL void seq_walk(cooperative_groups::cluster_group& cl, const float* e, uint32_t L, uint32_t V, uint32_t C,
                          SeqShared* ss, unsigned long long* tr = nullptr) {
    const int lane = threadIdx.x & 31;
    {
        float s = 0.0f;
        // replay of chunk c (predicted binade ce): lane l stands for thread l
        // of the chunk's warp
        auto replay = [&](int c, int ce) {
                const int r = c >> 5, w = c & 31;
                const SeqShared* sr = cl.map_shared_rank(ss, r);
                const float* er = cl.map_shared_rank(e, r);
                const int th = w * 32 + lane;
                const long long ti0 = sr->tinc[0][th], ti1 = sr->tinc[1][th];
                const uint32_t tf = sr->tflag[th];
                const uint32_t nr = min(V - min(V, uint32_t(r) * L), L);
                const uint32_t a0 = min(nr, uint32_t(th) * C), a1 = min(nr, a0 + C);
                const int cnt = int(a1 - a0);
                float my_e[kSeqMaxC];                      // this lane's elements, loaded once per replay
#pragma unroll
                for (int q = 0; q < kSeqMaxC; ++q) my_e[q] = (q < cnt) ? er[a0 + q] : 0.0f;
                int ls = 0;
                while (ls < 32) {
                    const int ex = f32_expo(s);
                    if (ex == 0 || ex == 255 || (ex != ce && ex != ce + 1)) {
                        // no increment applies: the next lane with elements replays them
                        // one by one (what the general step below does here, without its
                        // prefix sum)
                        const unsigned m = __ballot_sync(0xffffffffu, lane >= ls && cnt > 0);
                        if (m == 0) break;
                        const int evl = __ffs(m) - 1;
                        float sv = s;
                        if (lane == evl) {
#pragma unroll
                            for (int q = 0; q < kSeqMaxC; ++q)
                                if (q < cnt) sv = __fadd_rn(sv, my_e[q]);
                        }
                        s = __shfl_sync(0xffffffffu, sv, evl);
                        ls = evl + 1;
                        continue;
                    }
                    long long li = 0;
                    bool ev = false;
                    if (lane >= ls) {
                        if (ex == 0 || ex == 255) ev = (cnt > 0);
                        else if (ex == ce) { li = ti0; ev = (tf & 1) || ti0 >= (1ll << 30); }
                        else if (ex == ce + 1) { li = ti1; ev = (tf & 2) || ti1 >= (1ll << 30); }
                        else ev = (cnt > 0);   // another binade: replay element by element
                    }
                    long long incl = li;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const long long y = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o) incl += y;
                    }
                    const long long su = (ex == 0 || ex == 255) ? 0 : f32_units(s);
                    if (lane >= ls && su + incl >= (1ll << 24)) ev = true;
                    const unsigned evm = __ballot_sync(0xffffffffu, ev && lane >= ls);
                    if (evm == 0) {
                        const long long tot = __shfl_sync(0xffffffffu, incl, 31);
                        if (ex != 0 && ex != 255) s = f32_from(ex, su + tot);
                        break;
                    }
                    const int evl = __ffs(evm) - 1;
                    const long long before = __shfl_sync(0xffffffffu, incl - li, evl);   // lanes ls..evl-1
                    if (evl > ls && ex != 0 && ex != 255) s = f32_from(ex, su + before);
                    float sv = s;
                    if (lane == evl) {
#pragma unroll
                        for (int q = 0; q < kSeqMaxC; ++q)
                            if (q < cnt) sv = __fadd_rn(sv, my_e[q]);
                    }
                    s = __shfl_sync(0xffffffffu, sv, evl);
                    ls = evl + 1;
                }
        };
        // 32 chunks at a time (lane j: chunk cb + j): while the running sum
        // stays in its binade, a clean chunk (no flag, predicted binade = the
        // sum's) adds its increment to the sum's integer units - so the chunks
        // from j0 up to the first one that is not clean or would carry the
        // units to 2^24 are added at once through a prefix sum (increments
        // are >= 0: the units only grow); that chunk is replayed, and the
        // batch continues after it. The same result as chunk by chunk.
        for (int cb = 0; cb < kSeqChunks; cb += 32) {
            const int my_info = ss->sinfo[cb + lane];
            const long long my_inc = ss->sinc[cb + lane];
            const int my_ce = my_info & 0xffff;
            const uint32_t my_cf = uint32_t(my_info) >> 16;
            int j0 = 0;
            while (j0 < 32) {
                const int es = f32_expo(s);
                const long long su = (es == 0 || es == 255) ? 0 : f32_units(s);
                const bool act = lane >= j0;
                long long incl = act ? my_inc : 0;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const long long y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                const bool good = my_cf == 0 && my_ce == es && es != 0 && es != 255 && su + incl < (1ll << 24);
                const unsigned bad = __ballot_sync(0xffffffffu, act && !good);
                if (bad == 0) {
                    s = f32_from(es, su + __shfl_sync(0xffffffffu, incl, 31));
                    break;
                }
                const int fb = __ffs(bad) - 1;
                const long long upto = __shfl_sync(0xffffffffu, incl, fb > 0 ? fb - 1 : 0);
                if (fb > j0) s = f32_from(es, su + upto);
                replay(cb + fb, __shfl_sync(0xffffffffu, my_ce, fb));
                j0 = fb + 1;
            }
        }
        if (lane == 0) ss->result = s;
    }
    seq_mark(tr, 3);
}

}  // namespace smoe
