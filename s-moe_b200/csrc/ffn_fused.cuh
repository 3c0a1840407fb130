// ffn_fused.cuh - persistent fused MoE layer for decode (sm_100a).
//
// One cooperative launch, one CTA per SM, does the whole MoE layer of a
// decode step for up to kFusedMaxTok tokens:
//   phase R (optional) router logits spread over the grid, then every CTA
//           runs the softmax / top-k / renorm of router.cuh on them;
//   phase A units  (slot, 16 hidden rows): h = silu(Wg.x) * (Wu.x)
//   phase B units  (token, 16 output rows): y = sum_j w_j * Wd_j . h_j
// Warp 16 (producer) issues 1-D bulk copies of every weight byte the CTA will
// consume - its A units, then its B units - into a ring of shared-memory
// stages as soon as a stage is free; sixteen consumer warps dequantise in
// registers and run mma.sync. Because the down-projection bytes of phase B do
// not depend on h, they stream in while phase A computes; a B unit only waits
// (bounded spin on a per-token counter in global memory) for the h vectors
// other CTAs publish.
//
// Arithmetic (bf16 variant of ffn_q4.cuh). One LOP3 ORs a code q into the
// mantissa of bf16 128.0 (0x4300), giving the exact operand 128+q; the
// activation v is split into bf16 hi + lo held in two B columns (16
// significant bits, fp32 exponent range, so no scaling). Per 64-group the
// MMA yields D = sum (128+q).v and
//     sum w.v = scale * (D - 128 sum v) + bias * sum v.
//
// Each phase-A unit writes its 16 h rows straight into the B-operand table
// layout in global memory: the 16 rows of a unit are exactly the positions
// one lane quarter (c = row/16 % 4) of a 64-group holds, so a unit owns
// whole table entries, plus the quarter's sum of v. Phase B loads the
// finished tables with one round of wide loads.
//
// Work split: bytes per CTA balanced by a host-computed partition - B units
// round-robin, A units filling each CTA up to the mean byte count. The last
// CTA to finish resets the counters, so consecutive launches (and CUDA-graph
// replays) need no host-side reset.
#pragma once
#include "ffn_q4.cuh"
#include "router.cuh"
#include "tiled.cuh"

namespace smoe {

constexpr int kFusedConsumers = 16;                // consumer warps
constexpr int kFusedCThreads = kFusedConsumers * 32;
constexpr int kFusedPubWarp = kFusedConsumers;     // reduces + publishes phase-A units
constexpr int kFusedProdWarp = kFusedConsumers + 1; // issues the bulk copies
constexpr int kFusedThreads = kFusedCThreads + 64;
constexpr int kFusedRedBufs = 4;                   // phase-A reduction buffers in flight
constexpr int kFusedMaxTok = 4;
constexpr int kFusedSlotsPerB = 4;                 // slots per phase-B stage
constexpr int kFusedMaxK = 16;
constexpr int kFusedMaxGrid = 256;

struct FusedState {          // device scratch, zero at context creation
    uint32_t rdone;                 // router logit rows finished (reset at exit)
    uint32_t done;                  // CTAs finished (reset at exit)
    uint32_t epoch;                 // launches completed: tags this launch's h tables
    uint32_t hcount[kFusedMaxTok];  // phase-A units written, per token (relaxed; reset at exit)
    uint32_t pad[1];
};

struct FusedGeom {           // shared by host (smem sizing) and device
    int d, dff, k, ntok;
    int G, Gd;               // groups per A row / per B row
    TiledGeom tg;            // tiled expert layout (tiled.cuh)
    int stageA, stageB, stage;
    int nstages;
    int nA, nB, tilesA, tilesB, chunksB;
    int o_ring, o_xtab, o_xg, o_htab, o_hg, o_red, o_yslot, o_hq, o_bar, o_ids, o_w, o_ps, o_vst;
    int total;

    __host__ __device__ void init(int fmt, int d_, int dff_, int k_, int ntok_, int max_smem) {
        d = d_; dff = dff_; k = k_; ntok = ntok_;
        G = d / 64; Gd = dff / 64;
        tg.init(fmt, d, dff);
        stageA = int(tg.tileA);
        stageB = kFusedSlotsPerB * int(tg.tileB);
        stage = (stageA > stageB ? stageA : stageB);
        stage = (stage + 127) & ~127;
        tilesA = dff / 16; tilesB = d / 16;
        nA = ntok * k * tilesA;
        nB = ntok * tilesB;
        chunksB = (k + kFusedSlotsPerB - 1) / kFusedSlotsPerB;
        int off = 0;
        auto take = [&](int bytes) { int o = off; off += (bytes + 127) & ~127; return o; };
        o_xtab = take(ntok * (d / 16) * 64);
        o_xg = take(ntok * G * 4);
        o_htab = take(k * (dff / 16) * 64);
        o_hg = take(k * Gd * 4);
        o_red = take(kFusedRedBufs * kFusedConsumers * 32 * 4);
        o_yslot = take(4 * kFusedConsumers * 32 * 4);     // phase-B partials per chunk
        o_hq = take(16 * 4);
        o_bar = take((2 * 16 + 2 * kFusedRedBufs) * 8);
        o_ids = take(ntok * k * 4);
        o_w = take(ntok * k * 4);
        o_ps = take(kFusedMaxTok * kRouterMaxE * 4);
        o_vst = take(4 * (ntok * d > k * dff / 16 ? ntok * d : k * dff / 16));   // staged x / quarter sums
        off = (off + 1023) & ~1023;
        o_ring = off;
        nstages = (max_smem - off) / stage;
        if (nstages > 16) nstages = 16;
        total = off + nstages * stage;
    }
};

// CTA c's share of the grid's work: A units [a0, a1), B units [b0, b1).
struct FusedShare { int a0, a1, b0, b1; };

// Host-side partition (the per-CTA loop is too slow to run on the device).
inline FusedShare fused_share(const FusedGeom& g, int c, int G) {
    const double cA = double(g.tg.tileA), cB = double(g.k) * double(g.tg.tileB);
    const double rho = cB / cA;
    const double T = g.nA + rho * g.nB;
    auto bstart = [&](int i) { return int((long long)i * g.nB / G); };
    auto abound = [&](int i) {
        const double p = double(i) * T / G - rho * bstart(i);
        const int b = int(p + 0.5);
        return b < 0 ? 0 : (b > g.nA ? g.nA : b);
    };
    int run = 0, a0 = 0, a1 = 0;               // running max keeps the partition monotone
    for (int i = 0; i <= c + 1; ++i) {
        const int b = (i == G) ? g.nA : abound(i);
        run = b > run ? b : run;
        if (i == c) a0 = run;
        if (i == c + 1) a1 = run;
    }
    FusedShare s{a0, a1, bstart(c), bstart(c + 1)};
    return s;
}

SMOE_DEVINL void consumer_sync() {
    asm volatile("bar.sync 1, %0;" :: "n"(kFusedCThreads) : "memory");
}
// consumers -> producer: "x loads issued, start streaming" (barrier 2)
SMOE_DEVINL void start_arrive() {
    asm volatile("bar.arrive 2, %0;" :: "n"(kFusedCThreads + 32) : "memory");
}
SMOE_DEVINL void start_wait() {
    asm volatile("bar.sync 2, %0;" :: "n"(kFusedCThreads + 32) : "memory");
}

// One 64-group of a 16-row tile in fragment order (tiled.cuh): rows lane/4
// and lane/4+8 of this lane, bf16 operands, two independent accumulator
// chains. Returns the sums for the token held in B columns 0/1 (valid in
// lanes with lane%4 == 0).
SMOE_DEVINL void group_mma_bf16(const uint8_t* frag, int grp, const uint2* btab, int lane, float& r0,
                                float& r8) {
    const uint2 w = *reinterpret_cast<const uint2*>(frag + grp * 512 + lane * 8);
    const uint2 v = *reinterpret_cast<const uint2*>(frag + grp * 512 + 256 + lane * 8);
    float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t M = 0x000F000Fu, OR = 0x43004300u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t wg = i ? w.y : w.x, wh = i ? v.y : v.x;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t g8 = wg >> (8 * h), h8 = wh >> (8 * h);
            uint32_t a[4];
            a[0] = lop3_and_or(g8, M, OR);                    // 128+q at positions +0, +4
            a[1] = lop3_and_or(h8, M, OR);
            a[2] = lop3_and_or(g8 >> 4, M, OR);               // positions +1, +5
            a[3] = lop3_and_or(h8 >> 4, M, OR);
            uint2 b = make_uint2(0u, 0u);
            if (lane < 8) b = btab[(grp * 4 + i * 2 + h) * 8 + lane];
            const uint32_t bb[2] = {b.x, b.y};
            mma_bf16_16816(h ? d1 : d0, a, bb);
        }
    }
    r0 = (d0[0] + d0[1]) + (d1[0] + d1[1]);
    r8 = (d0[2] + d0[3]) + (d1[2] + d1[3]);
}

// dsum = sum (128+q).v from the MMA, vsum = sum v: sum q.v = dsum - 128 vsum.
// N independent 64-groups at once (same arithmetic as group_mma_bf16): the
// 4N loads are issued first and the 4 k-steps of all N groups interleaved,
// so a warp has 2N accumulator chains in flight instead of 2.
template <int N>
SMOE_DEVINL void group_mma_n(const uint8_t* const* frag, const int* grp, const uint2* const* btab,
                             int lane, float* r0, float* r8) {
    uint2 w[N], v[N];
#pragma unroll
    for (int q = 0; q < N; ++q) {
        w[q] = *reinterpret_cast<const uint2*>(frag[q] + grp[q] * 512 + lane * 8);
        v[q] = *reinterpret_cast<const uint2*>(frag[q] + grp[q] * 512 + 256 + lane * 8);
    }
    float d[N][2][4];
#pragma unroll
    for (int q = 0; q < N; ++q)
#pragma unroll
        for (int z = 0; z < 4; ++z) d[q][0][z] = d[q][1][z] = 0.f;
    const uint32_t M = 0x000F000Fu, OR = 0x43004300u;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int q = 0; q < N; ++q) {
                const uint32_t g8 = (i ? w[q].y : w[q].x) >> (8 * h), h8 = (i ? v[q].y : v[q].x) >> (8 * h);
                uint32_t a[4];
                a[0] = lop3_and_or(g8, M, OR);
                a[1] = lop3_and_or(h8, M, OR);
                a[2] = lop3_and_or(g8 >> 4, M, OR);
                a[3] = lop3_and_or(h8 >> 4, M, OR);
                uint2 b = make_uint2(0u, 0u);
                if (lane < 8) b = btab[q][(grp[q] * 4 + i * 2 + h) * 8 + lane];
                const uint32_t bb[2] = {b.x, b.y};
                mma_bf16_16816(d[q][h], a, bb);
            }
        }
    }
#pragma unroll
    for (int q = 0; q < N; ++q) {
        r0[q] = (d[q][0][0] + d[q][0][1]) + (d[q][1][0] + d[q][1][1]);
        r8[q] = (d[q][0][2] + d[q][0][3]) + (d[q][1][2] + d[q][1][3]);
    }
}

template <int FMT>
SMOE_DEVINL float group_epi(float dsum, float vsum, const uint16_t* sc, const uint16_t* bi, int idx) {
    const float qv = fmaf(-128.0f, vsum, dsum);
    if (FMT == kFmtAffine)
        return bf16_bits_to_f32(sc[idx]) * qv + bf16_bits_to_f32(bi[idx]) * vsum;
    return f16_bits_to_f32(sc[idx]) * (qv * (1.0f / 7.5f) - vsum);
}

// bf16 hi/lo B-table entry of table position (grp, step s, lane c) of a
// vector whose 16-element quarter c of group grp is q[0..15]; col 0 -> hi, 1 -> lo.
SMOE_DEVINL uint2 btab_entry(const float* q, int s, int col) {
    const int base = (s >> 1) * 8 + (s & 1) * 2;
    float e[4] = {q[base], q[base + 4], q[base + 1], q[base + 5]};
    if (col) {
#pragma unroll
        for (int i = 0; i < 4; ++i) e[i] -= __bfloat162float(__float2bfloat16_rn(e[i]));
    }
    return make_uint2(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]));
}

// sum over a quarter of hi + lo as the MMA sees it
SMOE_DEVINL float quarter_sum(const float* q) {
    float s = 0.f;
    for (int i = 0; i < 16; ++i) {
        const float hi = __bfloat162float(__float2bfloat16_rn(q[i]));
        s += hi + __bfloat162float(__float2bfloat16_rn(q[i] - hi));
    }
    return s;
}

// Table of nvec K-vectors held in shared fp32 (v at vs + v*K): entries
// btab[v*(K/16)*8 + (grp*4+s)*8 + col*4 + c], group sums gsum[v*(K/64)+grp].
SMOE_DEVINL void build_btab_bf16(const float* vs, int nvec, int K, uint2* btab, float* gsum, int ctid) {
    const int total = nvec * (K / 4);                  // (v, grp, s, c) tuples
    for (int t = ctid; t < total; t += kFusedCThreads) {
        const int v = t / (K / 4), tl = t - v * (K / 4);
        const int grp = tl >> 4, r = tl & 15, s = r >> 2, c = r & 3;
        const float* q = vs + size_t(v) * K + grp * 64 + c * 16;
        uint2* bt = btab + size_t(v) * (K / 16) * 8 + (grp * 4 + s) * 8;
        bt[c] = btab_entry(q, s, 0);
        bt[4 + c] = btab_entry(q, s, 1);
        float part = 0.f;
        if (s == 0) part = quarter_sum(q);
        const unsigned mask = __activemask();          // whole 16-lane groups are active together
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) part += __shfl_xor_sync(mask, part, o);
        if ((ctid & 15) == 0) gsum[v * (K / 64) + grp] = part;
    }
}

// Copy n contiguous elements (n % 4 == 0) of a global vector into shared fp32
// with all of a thread's loads in flight at once.
template <bool kBf16>
SMOE_DEVINL void stage_vec_smem(const void* src, int n, float* dst, int ctid) {
    constexpr int U = 8;
    for (int base = 0; base < n / 4; base += U * kFusedCThreads) {
        float4 v[U];
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const int i = base + q * kFusedCThreads + ctid;
            if (i < n / 4) {
                if (kBf16) {
                    const uint2 b = reinterpret_cast<const uint2*>(src)[i];
                    v[q] = make_float4(__uint_as_float(b.x << 16), __uint_as_float(b.x & 0xffff0000u),
                                       __uint_as_float(b.y << 16), __uint_as_float(b.y & 0xffff0000u));
                } else {
                    v[q] = reinterpret_cast<const float4*>(src)[i];
                }
            }
        }
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const int i = base + q * kFusedCThreads + ctid;
            if (i < n / 4) reinterpret_cast<float4*>(dst)[i] = v[q];
        }
    }
}

struct FusedArgs {
    FfnArgs f;                 // table mode; f.ids/f.wts: routing (written here if rw)
    FusedState* st;
    FusedGeom g;
    const uint16_t* rw;        // optional router phase: W [E x d] bf16 (null: routing given)
    uint32_t E;
    int norm;
    float* logits;             // scratch [ntok x E]
    uint4* htab_g;             // scratch: tagged h B-tables [ntok*k][dff/16][8] {w0,tag,w1,tag}
    uint2* hsum_g;             // scratch: tagged quarter sums [ntok*k][dff/64][4] {sum,tag}
    unsigned long long* trace; // optional [grid x 8] phase timestamps (ns), null in production
    int dbg_skip;              // profiling experiment: 1 = consumers skip the phase-A math
    int a_bound[kFusedMaxGrid + 1];   // CTA c owns A units [a_bound[c], a_bound[c+1])
};

// Fill FusedArgs::a_bound for a grid of G CTAs (host side, once per launch).
inline void fused_partition(const FusedGeom& g, int G, int* a_bound) {
    for (int c = 0; c < G; ++c) a_bound[c] = fused_share(g, c, G).a0;
    a_bound[G] = g.nA;
}

SMOE_DEVINL void trace_mark(unsigned long long* tr, int i, bool who = threadIdx.x == 0) {
    if (tr && who) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        tr[blockIdx.x * 8 + i] = t;
    }
}

SMOE_DEVINL SlotW expert_ptrs(const FfnArgs& a, uint32_t e) {
    SlotW w;
    const uint8_t* b = a.base + uint64_t(e) * a.stride;
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        w.nib[m] = b + a.off[3 * m];
        w.sc[m] = reinterpret_cast<const uint16_t*>(b + a.off[3 * m + 1]);
        w.bi[m] = reinterpret_cast<const uint16_t*>(b + a.off[3 * m + 2]);
    }
    return w;
}

// Tagged 8-byte stores/loads: each 64-bit word {data, tag} is written and
// read in one single-copy-atomic access, so a reader that sees the current
// tag also sees the data, with no fence on the writer side (the scheme of
// NCCL's LL protocol).
SMOE_DEVINL void st_tagged2(uint4* p, uint2 v, uint32_t tag) {
    asm volatile("st.global.v2.u64 [%0], {%1, %2};" ::"l"(p),
                 "l"((uint64_t(tag) << 32) | v.x), "l"((uint64_t(tag) << 32) | v.y) : "memory");
}
SMOE_DEVINL void st_tagged1(uint2* p, float v, uint32_t tag) {
    asm volatile("st.global.u64 [%0], %1;" ::"l"(p), "l"((uint64_t(tag) << 32) | __float_as_uint(v)) : "memory");
}
SMOE_DEVINL uint4 ld_tagged2(const uint4* p) {
    uint64_t a, b;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p));
    return make_uint4(uint32_t(a), uint32_t(a >> 32), uint32_t(b), uint32_t(b >> 32));
}
SMOE_DEVINL uint2 ld_tagged1(const uint2* p) {
    uint64_t a;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(p));
    return make_uint2(uint32_t(a), uint32_t(a >> 32));
}

SMOE_DEVINL bool spin_until_geq(const uint32_t* p, uint32_t target) {
    for (uint32_t i = 0; i < SMOE_SPIN_LIMIT; ++i) {
        if (ld_volatile_u32(p) >= target) return true;
        if (i > 32) __nanosleep(i > 256 ? 256 : 64);
    }
    return false;
}

}  // namespace smoe
