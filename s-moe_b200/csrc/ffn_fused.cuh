// ffn_fused.cuh - shared pieces of the persistent fused MoE-layer kernel
// (ffn_fused_kernel.cuh): geometry, bf16 fragment MMAs, operand tables.
//
// Gate/up arithmetic: integer tensor-core MMA m16n8k32 (u8 x s8 -> s32).
// A 32-bit word of the tiled fragments holds 8 codes; masking it with
// 0x0F0F0F0F gives the even columns' codes q as u8, with 0xF0F0F0F0 the odd
// columns' 16q - no shifts. The activation of each 64-group is turned into
// fixed point X = round(x * 2^(20-E)) (E = exponent of the group's largest
// |x|, so |X| < 2^21: 21 bits relative to the group maximum) and split into
// signed 8-bit digits X = p0 + 2^8 p1 + 2^16 p2. Two B sets carry them:
// set 0 has (p0, p1) of token t in columns (2t, 2t+1), set 1 has p2 in
// column 2t. Four MMAs per 16 x 64 group (even/odd columns x two sets) give
//     V01 = 16 D1[p0] + D16[p0] + 2^8 (16 D1[p1] + D16[p1])     (exact int32)
//     V2  = 16 D1'[p2] + D16'[p2]                                (exact int32)
//     sum q x = (V01 + 2^16 V2) * 2^(E-24),
// and per (row, group) sum w.x = scale * sum q x + bias * sum x (AFFINE-Q4)
// or scale * (sum q x / 7.5 - sum x) (SMOE-Q4), sum x taken over the same
// fixed-point values. Lane 4g + c receives token c's sums, so one MMA serves
// up to four tokens. The only roundings are the fixed-point step of x and
// the fp32 epilogue.
#pragma once
#include "ffn_q4.cuh"
#include "router.cuh"
#include "tiled.cuh"

namespace smoe {

#ifndef SMOE_FUSED_CONSUMERS
#define SMOE_FUSED_CONSUMERS 16
#endif
constexpr int kFusedConsumers = SMOE_FUSED_CONSUMERS;   // consumer warps
constexpr int kFusedCThreads = kFusedConsumers * 32;
constexpr int kFusedHWarp = kFusedConsumers;        // turns each unit's partial sums into h
constexpr int kFusedProdWarp = kFusedConsumers + 1; // issues the bulk copies
constexpr int kFusedThreads = kFusedCThreads + 64;
constexpr int kFusedMaxTok = 4;
constexpr int kFusedMaxK = 16;
#ifndef SMOE_DOWN_REG_TILES
#define SMOE_DOWN_REG_TILES (128 / SMOE_FUSED_CONSUMERS)
#endif
constexpr int kDownRegTiles = SMOE_DOWN_REG_TILES;       // down output tiles per consumer warp kept in registers (d_model <= 2048)
constexpr int kFusedCluster = 4;                   // CTAs that pre-reduce partial outputs together

struct FusedState {          // device scratch, zero at context creation and on exit
    uint32_t rdone;                 // router logit rows finished
    uint32_t done;                  // CTAs finished
    uint32_t epoch;                 // expert-parallel launches completed (advanced by the last CTA)
    uint32_t pad[5];
};

SMOE_DEVINL void consumer_sync() {
    asm volatile("bar.sync 1, %0;" :: "n"(kFusedCThreads) : "memory");
}


// Down-slice epilogue (bf16 path): dsum = sum (128+q).v from the MMA, vsum =
// sum v, so sum q.v = dsum - 128 vsum.
template <int FMT>
SMOE_DEVINL float group_epi(float dsum, float vsum, const uint16_t* sc, const uint16_t* bi, int idx) {
    const float qv = fmaf(-128.0f, vsum, dsum);
    if (FMT == kFmtAffine)
        return bf16_bits_to_f32(sc[idx]) * qv + bf16_bits_to_f32(bi[idx]) * vsum;
    return f16_bits_to_f32(sc[idx]) * (qv * (1.0f / 7.5f) - vsum);
}

// Activation table for the gate/up MMAs from ntok vectors held in shared fp32
// (token t at vs + t*K). Per 64-group and B set: xtab[(grp*2 + set)*32 +
// lane] = the four B registers {b(even, k 0-15), b(even, k 16-31), b(odd,
// k 0-15), b(odd, k 16-31)} of lane 4g + c, and xg[grp*4 + t] = (2^(E-24)
// (/7.5 for SMOE-Q4), sum of the fixed-point x). The whole table is zeroed
// first: columns of absent tokens stay 0.
template <int FMT>
SMOE_DEVINL void build_xplanes(const float* vs, int ntok, int K, uint4* xtab, float2* xg, int ctid) {
    const int G = K / 64;
    for (int i = ctid; i < G * 64; i += kFusedCThreads) xtab[i] = make_uint4(0u, 0u, 0u, 0u);
    consumer_sync();
    const int warp = ctid >> 5, lane = ctid & 31;
    uint8_t* tb = reinterpret_cast<uint8_t*>(xtab);
    for (int p = warp; p < ntok * G; p += kFusedConsumers) {   // one (token, group) per warp
        const int t = p / G, grp = p - t * G;
        const float* q = vs + size_t(t) * K + grp * 64;
        const float v0 = q[lane], v1 = q[lane + 32];
        float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const int E = m > 0.f ? int((__float_as_uint(m) >> 23) & 0xff) - 127 : 0;
        const int X0 = __float2int_rn(ldexpf(v0, 20 - E)), X1 = __float2int_rn(ldexpf(v1, 20 - E));
        // sum x of the fixed-point values the MMA sees (exact in int), so the
        // bias / offset term cancels against the scale term consistently
        int xs_i = X0 + X1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) xs_i += __shfl_xor_sync(0xffffffffu, xs_i, o);
        if (lane == 0) {
            const float xs = ldexpf(1.0f, E - 24);
            xg[grp * 4 + t] = make_float2(FMT == kFmtAffine ? xs : xs * (1.0f / 7.5f), ldexpf(float(xs_i), E - 20));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = lane + 32 * h;                        // column within the group
            const int X = h ? X1 : X0;
            const int p0 = ((X + 128) & 255) - 128, r = (X - p0) >> 8;
            const int p1 = ((r + 128) & 255) - 128, p2 = (r - p1) >> 8;
            const int odd = j & 1, kk = j >> 1;                 // MMA (even/odd columns), k slot
            const int c = (kk >> 2) & 3, reg = odd * 2 + (kk >> 4), byte = kk & 3;
            uint8_t* e = tb + (size_t(grp) * 64 + (2 * t) * 4 + c) * 16 + reg * 4 + byte;
            e[0] = uint8_t(p0);                                 // set 0, column 2t   (lane 8t + c)
            e[4 * 16] = uint8_t(p1);                            // set 0, column 2t+1 (lane 8t + 4 + c)
            e[32 * 16] = uint8_t(p2);                           // set 1, column 2t
        }
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

SMOE_DEVINL void trace_mark(unsigned long long* tr, int i, bool who = threadIdx.x == 0) {
    if (tr && who) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        if (i < 32) tr[blockIdx.x * 32 + i] = t;
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

SMOE_DEVINL uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
SMOE_DEVINL void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
// Bounded wait on a word another GPU writes (system scope).
SMOE_DEVINL bool spin_sys_until_geq(const uint32_t* p, uint32_t target) {
    for (uint32_t i = 0; i < SMOE_SPIN_LIMIT; ++i) {
        if (ld_acquire_sys(p) >= target) return true;
        if (i > 32) __nanosleep(i > 256 ? 256 : 64);
    }
    return false;
}

// Bounded wait on a word other CTAs of this grid advance with release
// atomics; the acquire load orders the caller's later reads after theirs.
SMOE_DEVINL bool spin_until_geq(const uint32_t* p, uint32_t target) {
    for (uint32_t i = 0; i < SMOE_SPIN_LIMIT; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (v >= target) return true;
        if (i > 32) __nanosleep(64);
    }
    return false;
}

// Geometry of one launch, shared by host (shared-memory sizing) and device.
struct FusedGeom {
    int d, dff, k, ntok, G, Gd;
    TiledGeom tg;
    int stage, nstages;
    int nU, tilesU, outTiles;       // units (slot, 16 hidden rows), units per slot, 16-row output tiles
    int o_xtab, o_xg, o_ysum, o_sbc, o_red, o_hq, o_bar, o_ids, o_w, o_loc, o_ring, total;

    __host__ __device__ void init(int fmt, int d_, int dff_, int k_, int ntok_, int max_smem) {
        d = d_; dff = dff_; k = k_; ntok = ntok_;
        G = d / 64; Gd = dff / 64;
        tg.init(fmt, d, dff);
        stage = int(tg.unit);                  // group scales go straight to o_sbc
        stage = (stage + 127) & ~127;
        tilesU = dff / 16; outTiles = d / 16;
        nU = ntok * k * tilesU;
        int off = 0;
        auto take = [&](int bytes) { int o = off; off += (bytes + 127) & ~127; return o; };
        o_xtab = take(G * 1024);
        o_xg = take(G * 4 * 8);
        const int ys = 4 * ntok * d, ps = 4 * ntok * kRouterMaxE;
        o_ysum = take(ys > ps ? ys : ps);      // also x staging and router softmax scratch
        o_sbc = take(2 * int(tg.dgroup));                // two groups' down scales
        o_red = take(2 * kFusedConsumers * 32 * 4);      // double-buffered partial sums
        o_hq = take(2 * 256);                            // per buffer: h[16], B regs[8], sum
        o_bar = take((2 * 16 + 5) * 8);                 // full[16] empty[16] redF[2] hR[2] routed
        o_ids = take(ntok * k * 4);
        o_w = take(ntok * k * 4);
        o_loc = take(4 * (kFusedMaxTok * kFusedMaxK + 1)); // expert parallel: local slot list + count
        off = (off + 1023) & ~1023;
        o_ring = off;
        nstages = (max_smem - off) / stage;
        // at most 4: the producer copies a group's down scales into the buffer
        // of its parity, which the group two back (4 units earlier) must have
        // finished with - guaranteed when it is at most 4 units ahead
        if (nstages > 4) nstages = 4;
        total = off + nstages * stage;
    }
};

// Expert-parallel exchange (world > 1), one process per GPU. Every rank runs
// the same launch sequence; rank 0 owns x and y. Each rank has a window of
// device memory exported over CUDA IPC; ranks > 0 map rank 0's:
//   flag0  rank 0's x epoch: rank 0 copies x into x0, then releases it;
//   x0     that copy, read by the other ranks with peer loads over NVLink;
//   part0  [world][kFusedMaxTok * d] fp32: rank r's partial output,
//          written by rank r's last CTA with peer stores;
//   done0  ranks whose partial has arrived (system-scope atomics); rank 0's
//          last CTA waits for world - 1, sums, writes y and resets it.
// The epoch of a launch is the rank's count of completed expert-parallel
// launches + 1, kept on the device (so graph replays advance it); every rank
// runs the same launch sequence, so the epochs agree.
// Routing is computed on every rank (same weights, same x, same code: the
// same ids); each rank runs the units of the slots whose expert it holds.
constexpr int kEpMaxWorld = 8;
struct FusedEp {
    int world, rank;
    uint32_t base, nlocal;     // global id of this rank's first expert, experts held
    uint8_t* x0;
    uint32_t* flag0;
    float* part0;
    uint32_t* done0;
    uint32_t part_stride;      // floats per rank in part0
};

struct FusedArgs {
    FfnArgs f;                 // table mode; f.ids/f.wts: routing (written here if rw)
    FusedState* st;
    FusedGeom g;
    const uint16_t* rw;        // optional router phase: W [E x d] bf16 (null: routing given)
    uint32_t E;
    int norm;
    float* logits;             // scratch [ntok x E]
    float* acc;                // scratch [ntok x d] fp32, zero on entry and on exit
    unsigned long long* trace; // optional [grid x 8] phase timestamps (ns), null in production
    FusedEp ep;                // world 0/1: single GPU
};

}  // namespace smoe
