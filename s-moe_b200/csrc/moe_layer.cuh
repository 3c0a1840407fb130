// moe_layer.cuh - the persistent MoE-layer kernel for decode batches of up
// to kLMaxTok tokens (sm_100a), on the tiled expert layout (tiled.cuh).
//
// One launch, one CTA per SM:
//   routing (optional; decode.cpp:280-303): router logit rows spread over
//     the grid, each stored with this launch's tag; every CTA's producer
//     warp then runs the softmax / top-k / renorm of router.cuh on all
//     logits (identical results in every CTA);
//   phase A - gate/up and down (kernels.metal:240-365): the units (slot, 16
//     hidden rows) are split evenly over the CTAs. Per unit the consumer
//     warps run gate/up, the h warp turns the partials into
//     h = silu(Wg.x) * (Wu.x) * w_slot for the unit's 16 rows, and the
//     consumers multiply those 16 h by the unit's 16 columns of W_down (all
//     d_model rows) into the CTA's partial output rows (split-K over d_ff);
//     each CTA stores its partial rows per token, tagged;
//   phase R - combine (decode.cpp:485-499): the row blocks (token, 16 output
//     rows) are split evenly over the CTAs; each sums the partial rows of
//     the CTAs that hold the token's units, in CTA order, as soon as their
//     tags show up, and writes y. Every output row has one owner and a fixed
//     summation order (bitwise reproducible); no grid-wide barrier, no
//     atomics on the data.
// Every byte a CTA needs is streamed by one producer lane with 1-D bulk
// copies (no multicast) into three rings of shared-memory stages: per unit
// its gate/up chunks, its down scales when it starts a new scale group, its
// down columns. Sixteen consumer warps run the dots as integer MMAs on the
// raw codes (arithmetic below).
//
// Gate/up arithmetic: integer tensor-core MMA m16n8k32 (u8 x s8 -> s32).
// A 32-bit word of the fragments holds 8 codes; masking it with 0x0F0F0F0F
// gives the even columns' codes q as u8, with 0xF0F0F0F0 the odd columns'
// 16q - no shifts. The activation of each 64-group becomes fixed point
// X = round(x * 2^(20-E)) (E = exponent of the group's largest |x|, so
// |X| < 2^21) split into signed 8-bit digits X = p0 + 2^8 p1 + 2^16 p2. Two B
// sets carry them: set 0 has (p0, p1) of token t in columns (2t, 2t+1), set
// 1 has p2 in column 2t. Four MMAs per 16 x 64 group give the exact int32
// sums, and per (row, group) sum w.x = scale * sum q x + bias * sum x
// (AFFINE-Q4) or scale * (sum q x / 7.5 - sum x) (SMOE-Q4, the identity of
// kernels.metal:136-143), sum x taken over the same fixed-point values. The
// only roundings are the fixed-point step of x and the fp32 epilogue.
// Down arithmetic: the same fixed-point digits, for h: the h warp
// quantises each unit's 16 h with the exponent of their max|h| into three
// signed byte planes. One MMA m16n8k32 (u8 x s8) covers two 16-row tiles of
// the unit's down columns: k 0-15 multiply the even tile's codes with the
// planes in columns 0-2 of B, k 16-31 the odd tile's with the planes in
// columns 4-6, so all four lanes of a quad hold results; the exact int32
// sums are scaled by 2^(E-20) and the fp32 epilogue applies the down
// matrix's scale (and bias) per row.
//
// Expert parallel (world > 1, one process per GPU, experts [r*E/G,
// (r+1)*E/G) on rank r): every rank routes (the same ids) and runs phase A
// on the units of the slots whose expert it holds and phase R over its own
// CTAs; ranks > 0 store their combined rows into rank 0's window with peer
// stores and count them per row block with system-scope atomics; rank 0's
// owner of that row block waits for the count (bounded), adds the ranks'
// rows in rank order and writes y. x is published by rank 0 (release flag)
// and read by the others with peer loads. No TMA or bulk copy touches peer
// memory.
//
// Every wait is bounded by %globaltimer: LayerArgs.wait_ns from its own
// start, and the whole kernel by 8 x wait_ns. A wait that runs out sets the
// error word and the kernel carries on to its end with whatever shared state
// it has - every index read back from that state is clamped to its valid
// range before it forms an address - so the host sees SMOE_ERR_DEVICE and the
// context stays usable.
#pragma once
#include "ffn_q4.cuh"
#include "router.cuh"
#include "tiled.cuh"

namespace smoe {

constexpr int kLCons = 16;                    // consumer warps
constexpr int kLCThreads = kLCons * 32;
constexpr int kLHWarp = kLCons;               // h warp
constexpr int kLProdWarp = kLCons + 1;        // producer warp (top-k; lane 0 issues the copies)
constexpr int kLThreads = kLCThreads + 64;
constexpr int kLMaxTok = 4;
constexpr int kLMaxK = 16;
constexpr int kLMaxD = 4096;                  // d_model limit (partial rows, accumulators)
constexpr int kLMaxNA = 4;                    // gate/up ring stages (at most)
constexpr int kLMaxND = 3;                    // down-unit ring stages (at most)
constexpr int kLMaxNS = 2;                    // down-scale ring stages (at most)
constexpr int kHRec = 64;                     // one unit's h digit record (shared memory)
constexpr int kEpMaxWorld = 8;
constexpr int kLRedMax = 5;                   // phase R: partial rows per lane (grid <= 160)

struct LayerState {          // device scratch, zero at context creation; the counters zero after every launch
    uint32_t rdone;                 // router logit rows stored (a hint: the logits carry their own tag)
    uint32_t unused;
    uint32_t done;                  // CTAs finished
    uint32_t epoch;                 // expert-parallel launches completed (advanced by the last CTA)
    uint32_t seq;                   // launches completed (advanced by the last CTA): tags this launch's logits
    uint32_t pad[3];
};

// Division by a launch constant d without the integer divide (whose ~100
// cycles of latency sit on the producer's and the phases' critical paths):
// m = ceil(2^32 / d), q = hi32(x * m) = floor(x / d) for x * d < 2^32 (every
// use here: x < 2^22, d < 2^10).
__host__ __device__ inline uint32_t magic_of(uint32_t d) {
    return d <= 1 ? 0u : uint32_t((0x100000000ull + d - 1) / d);
}
SMOE_DEVINL uint32_t divu(uint32_t x, uint32_t d, uint32_t m) { return d <= 1 ? x : __umulhi(x, m); }

SMOE_DEVINL void cons_sync() {
    asm volatile("bar.sync 1, %0;" :: "n"(kLCThreads) : "memory");
}

// Geometry of one launch, shared by host (shared-memory sizing) and device.
struct LayerGeom {
    int d, dff, k, ntok;
    TiledGeom tg;
    int G, tilesU, outTiles, NA, ND, NS;
    int dparts, bpp;           // a down unit streams in dparts parts of bpp 64-row blocks (512 B each)
    uint32_t mg_tilesU, mg_outTiles, mg_G, mg_k;   // division magics (divu below)
    int o_xtab, o_xg, o_red, o_red2, o_hrec, o_bar, o_ids, o_w, o_loc, o_ringA, o_ringD, o_ringS, total;

    __host__ __device__ bool init(int fmt, int d_, int dff_, int k_, int ntok_, int max_smem) {
        d = d_; dff = dff_; k = k_; ntok = ntok_;
        if (!tg.init(fmt, d, dff) || tg.Gc > 32 || ntok < 1 || ntok > kLMaxTok || k < 1 || k > kLMaxK ||
            d > kLMaxD)
            return false;
        G = d / 64; tilesU = dff / 16; outTiles = d / 16;
        dparts = d > 2048 ? 2 : 1;
        bpp = (d / 64 + dparts - 1) / dparts;
        mg_tilesU = magic_of(uint32_t(tilesU));
        mg_outTiles = magic_of(uint32_t(outTiles));
        mg_G = magic_of(uint32_t(G));
        mg_k = magic_of(uint32_t(k));
        int off = 0;
        auto take = [&](int bytes) { int o = off; off += (bytes + 127) & ~127; return o; };
        o_xtab = take(G * 1024);                             // x table
        o_xg = take(G * 4 * 8);
        o_red = take(2 * kLCons * 32 * 4);                   // double-buffered unit partials / router partials
        o_red2 = take(32 * 16 * 4);                          // phase R: [32 CTA lanes][16 rows]
        o_hrec = take(2 * kHRec);                            // double-buffered h digit records
        o_bar = take((2 * kLMaxNA + 2 * kLMaxND + 2 * kLMaxNS + 9) * 8);
        o_ids = take(kLMaxTok * kLMaxK * 4);
        o_w = take(kLMaxTok * kLMaxK * 4);
        o_loc = take(4 * (kLMaxTok * kLMaxK + kLMaxTok + 2));  // local slots, token starts, count
        off = (off + 1023) & ~1023;
        const int fixed = off;
        const int avail = max_smem - fixed;
        const int ca = stageA(), cd = stageD(), cs = stageS();
        // gate/up chunks 3 (else 2) deep, down units 3 (else 2) deep, down
        // scales 2 (else 1: a CTA's units then wait once per new scale group)
        NA = avail >= 3 * ca + 2 * cd + 2 * cs ? 3 : 2;
        ND = avail >= NA * ca + 3 * cd + 2 * cs ? 3 : 2;
        NS = avail >= NA * ca + ND * cd + 2 * cs ? 2 : 1;
        o_ringA = fixed;
        o_ringD = o_ringA + NA * ca;
        o_ringS = o_ringD + ND * cd;
        total = o_ringS + NS * cs;
        return total <= max_smem;
    }
    __host__ __device__ int stageA() const { return int((tg.chunk + 127) & ~127u); }
    __host__ __device__ int stageD() const { return bpp * 512; }
    __host__ __device__ uint32_t dpart_bytes(int p) const {
        const int nb = d / 64 - p * bpp;
        return uint32_t((nb < bpp ? nb : bpp) * 512);
    }
    __host__ __device__ int stageS() const { return int((tg.sgrp + 127) & ~127u); }
};

struct LayerEp {
    int world, rank;
    uint32_t base, nlocal;     // global id of this rank's first expert, experts held
    uint8_t* xw[kEpMaxWorld];  // rank 0: the x area of rank r's window (peer memory), r >= 1
    uint32_t* flagw[kEpMaxWorld];  // rank 0: rank r's x epoch flag (peer memory), r >= 1
    uint32_t* flag;            // ranks > 0: this rank's own x epoch flag (rank 0 advances it)
    unsigned long long* part0; // [world][kLMaxTok * d] tagged rows (epoch << 32 | fp32), in rank 0's window
    uint32_t part_stride;      // entries per rank in part0
};

struct LayerArgs {
    const uint8_t* base;       // tiled experts held here: expert (id - ep.base) at base + i * stride
    uint64_t stride;
    const void* x;             // [ntok x d]
    int x_dtype;
    void* y;                   // [ntok x d] (rank 0)
    int y_dtype;
    const uint32_t* ids_in;    // routing given: [ntok x k] (null when rw)
    const float* wts_in;
    uint32_t* ids_out;         // routing computed: written by CTA 0 (may be null)
    float* wts_out;
    uint32_t n_experts;        // router rows = id bound
    const uint16_t* rw;        // router W [E x d] bf16, null: routing given
    int norm;
    unsigned long long* logits;  // scratch [ntok x E]: (launch tag << 32) | fp32 bits of the logit
    unsigned long long* part;  // scratch partial rows [grid][kLMaxTok][kLMaxD]: (launch tag << 32) | fp32 bits
    LayerState* st;
    uint32_t* err;
    uint64_t wait_ns;          // limit of every wait
    uint32_t mg_grid;          // magic_of(grid size)
    unsigned long long* trace; // optional [grid x 32] phase timestamps (ns)
    LayerGeom g;
    LayerEp ep;
};

// Phase timestamps, in the trace build only (SMOE_TRACE): the code of the
// marks alone adds about 1 us to the kernel (instruction fetch).
SMOE_DEVINL void ltrace(unsigned long long* tr, int i, bool who = threadIdx.x == 0) {
#ifdef SMOE_TRACE
    if (tr && who && i < 32) {
        tr[blockIdx.x * 32 + i] = gtimer();
        tr[(gridDim.x + blockIdx.x) * 32 + i] = clock64();          // same mark in SM cycles
    }
#else
    (void)tr; (void)i; (void)who;
#endif
}

SMOE_DEVINL uint32_t ld_acq_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
SMOE_DEVINL uint32_t ld_acq_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
SMOE_DEVINL void st_rel_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
SMOE_DEVINL void red_rel_gpu(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
// Bounded waits for a counter that other CTAs (gpu scope) or other GPUs
// (sys scope) advance with release operations; false when the deadline passes.
template <bool kSys>
static __device__ __noinline__ bool spin_geq(const uint32_t* p, uint32_t target, const WaitBudget wb) {
    const uint64_t deadline = wb.deadline();
#pragma unroll 1
    for (uint32_t i = 0; i < SMOE_SPIN_LIMIT; ++i) {
        if ((kSys ? ld_acq_sys(p) : ld_acq_gpu(p)) >= target) return true;
        if ((i & 7) == 7 && gtimer() > deadline) return false;
        if (i > 16) __nanosleep(i > 256 ? 256 : 32);
    }
    return false;
}

SMOE_DEVINL void raise_err(uint32_t* err, uint32_t code) { atomicCAS(err, 0u, code); }

SMOE_DEVINL void st_relaxed_gpu_u64(unsigned long long* p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
SMOE_DEVINL uint64_t ld_relaxed_gpu_u64(const unsigned long long* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Expert parallel, phase R: one row block across the ranks, by threads
// 0-15 (row yi, its sum s on this rank). Ranks > 0 store their row into rank
// 0's window tagged with the epoch (one 64-bit peer store: no fence, no
// counter); rank 0 polls its window until every rank's row carries this
// epoch and adds them in rank order. Returns whether this thread writes y.
// Out of line: the single-GPU kernel never runs it.
static __device__ __noinline__ bool ep_combine16(int rank, int world, unsigned long long* part0, uint32_t part_stride,
                                                 uint32_t epoch, float& s, size_t yi, uint32_t* err,
                                                 const WaitBudget wb) {
    if (rank > 0) {
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" :: "l"(part0 + size_t(rank) * part_stride + yi),
                     "l"((uint64_t(epoch) << 32) | __float_as_uint(s)) : "memory");
        return false;
    }
    const uint64_t deadline = wb.deadline();
#pragma unroll 1
    for (int rk = 1; rk < world; ++rk) {
        uint64_t v;
#pragma unroll 1
        for (uint32_t it = 0;; ++it) {
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(part0 + size_t(rk) * part_stride + yi)
                         : "memory");
            if (uint32_t(v >> 32) == epoch) break;
            if ((it & 7) == 7 && gtimer() > deadline) {
                raise_err(err, SMOE_DEVERR_SPIN_TIMEOUT);
                v = 0;
                break;
            }
            if (it >= 8) __nanosleep(64);
        }
        s += __uint_as_float(uint32_t(v));
    }
    return true;
}

// Expert parallel: rank 0 pushes x into another rank's window (peer stores
// by one warp).
static __device__ __noinline__ void ep_push_x(uint8_t* xw, const void* x, uint32_t xbytes, int lane) {
    const uint4* src = static_cast<const uint4*>(x);
    uint4* dst = reinterpret_cast<uint4*>(xw);
#pragma unroll 1
    for (uint32_t i = lane; i < xbytes / 16; i += 32) dst[i] = src[i];
}

// Bounded wait (one warp) for a token's E <= 128 tagged logits of this
// launch: lane l gets logits l + 32j in p[j] (-inf past E). Polls the values
// themselves - the first poll that sees every tag returns them.
static __device__ __noinline__ bool wait_logits(const unsigned long long* lg, int E, uint32_t tag, float (&p)[4],
                                                int lane, const WaitBudget wb) {
    const uint64_t deadline = wb.deadline();
#pragma unroll 1
    for (uint32_t i = 0; i < SMOE_SPIN_LIMIT; ++i) {
        bool ok = true;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = lane + 32 * j;
            p[j] = -INFINITY;
            if (e < E) {
                const uint64_t v = ld_relaxed_gpu_u64(lg + e);
                p[j] = __uint_as_float(uint32_t(v));
                ok = ok && uint32_t(v >> 32) == tag;
            }
        }
        if (__all_sync(0xffffffffu, ok)) return true;
        if ((i & 7) == 7 && gtimer() > deadline) return false;
        if (i > 64) __nanosleep(32);
    }
    return false;
}

// Phase R: one logit row (token t, expert e) by all consumer warps; returns
// this warp's partial sum (reduced across warps by the caller).
SMOE_DEVINL float router_row_part(const LayerArgs& A, const void* xsrc, uint32_t t, uint32_t e, int ctid) {
    const int d = A.g.d;
    float acc = 0.f;
    const uint4* wp = reinterpret_cast<const uint4*>(A.rw + size_t(e) * d);
    #pragma unroll 1
    for (int c = ctid; c < d / 8; c += kLCThreads) {
        const uint4 v = __ldg(wp + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        float xv[8];
        if (A.x_dtype == 0) {
            const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(xsrc) + size_t(t) * d + c * 8);
            const float4 a0 = xp[0], a1 = xp[1];
            xv[0] = a0.x; xv[1] = a0.y; xv[2] = a0.z; xv[3] = a0.w;
            xv[4] = a1.x; xv[5] = a1.y; xv[6] = a1.z; xv[7] = a1.w;
        } else {
            const uint4 b = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(xsrc) + size_t(t) * d + c * 8);
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

// v * 2^e for e in [-200, 200] by two exact power-of-two multiplies (the
// same value ldexpf gives, without its general-case code).
SMOE_DEVINL float pow2i(int e) { return __int_as_float((127 + e) << 23); }   // e in [-126, 127]
SMOE_DEVINL float scale2(float v, int e) {
    const int a = e / 2;
    return (v * pow2i(a)) * pow2i(e - a);
}

// x table of the gate/up MMAs, read straight from global x (ntok x K):
// xtab[(grp*2 + set)*32 + lane] = the four B registers {b(even, k 0-15),
// b(even, k 16-31), b(odd, k 0-15), b(odd, k 16-31)} of lane 4g + c, and
// xg[grp*4 + t] = (2^(E-24) (/7.5 for SMOE-Q4), sum of the fixed-point x).
// Columns of absent tokens stay 0. All consumer threads.
template <int FMT>
SMOE_DEVINL void build_xtab(const void* xsrc, int x_dtype, int ntok, int K, uint4* xtab, float2* xg, int ctid,
                            uint32_t mgG) {
    const int G = K / 64;
    #pragma unroll 1
    for (int i = ctid; i < G * 64; i += kLCThreads) xtab[i] = make_uint4(0u, 0u, 0u, 0u);
    const int warp = ctid >> 5, lane = ctid & 31;
    constexpr int U = 1;
    float v[U][2];
    // first round of loads before the barrier that orders the zeroing
    auto load = [&](int p0) {
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const int p = p0 + q * kLCons;
            v[q][0] = v[q][1] = 0.f;
            if (p < ntok * G) {
                const int t = int(divu(uint32_t(p), uint32_t(G), mgG)), grp = p - t * G;
                const size_t base = size_t(t) * K + grp * 64;
                if (x_dtype == 0) {
                    const float* s = static_cast<const float*>(xsrc) + base;
                    v[q][0] = s[lane];
                    v[q][1] = s[lane + 32];
                } else {
                    const uint16_t* s = static_cast<const uint16_t*>(xsrc) + base;
                    v[q][0] = bf16_bits_to_f32(s[lane]);
                    v[q][1] = bf16_bits_to_f32(s[lane + 32]);
                }
            }
        }
    };
    load(warp);
    cons_sync();
    uint8_t* tb = reinterpret_cast<uint8_t*>(xtab);
    #pragma unroll 1
    for (int p0 = warp; p0 < ntok * G; p0 += U * kLCons) {
        if (p0 != warp) load(p0);
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const int p = p0 + q * kLCons;
            if (p >= ntok * G) break;
            const int t = int(divu(uint32_t(p), uint32_t(G), mgG)), grp = p - t * G;
            const float v0 = v[q][0], v1 = v[q][1];
            float m = fmaxf(fabsf(v0), fabsf(v1));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const int E = m > 0.f ? int((__float_as_uint(m) >> 23) & 0xff) - 127 : 0;
            const int X0 = __float2int_rn(scale2(v0, 20 - E)), X1 = __float2int_rn(scale2(v1, 20 - E));
            int xs_i = X0 + X1;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) xs_i += __shfl_xor_sync(0xffffffffu, xs_i, o);
            if (lane == 0) {
                const float xs = scale2(1.0f, E - 24);
                xg[grp * 4 + t] = make_float2(FMT == kFmtAffine ? xs : xs * (1.0f / 7.5f), scale2(float(xs_i), E - 20));
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = lane + 32 * h;                        // column within the group
                const int X = h ? X1 : X0;
                const int p0d = ((X + 128) & 255) - 128, r = (X - p0d) >> 8;
                const int p1 = ((r + 128) & 255) - 128, p2 = (r - p1) >> 8;
                const int odd = j & 1, kk = j >> 1;                 // MMA (even/odd columns), k slot
                const int c = (kk >> 2) & 3, reg = odd * 2 + (kk >> 4), byte = kk & 3;
                uint8_t* e = tb + (size_t(grp) * 64 + (2 * t) * 4 + c) * 16 + reg * 4 + byte;
                e[0] = uint8_t(p0d);                                // set 0, column 2t   (lane 8t + c)
                e[4 * 16] = uint8_t(p1);                            // set 0, column 2t+1 (lane 8t + 4 + c)
                e[32 * 16] = uint8_t(p2);                           // set 1, column 2t
            }
        }
    }
}

// GW: 64-groups of a gate/up chunk per consumer warp, ceil(Gc / 16);
// DB: 64-row blocks of the output per consumer warp, ceil(d / 1024)
template <int FMT, int GW, int DB>
__global__ void __launch_bounds__(kLThreads, 1) k_moe_layer(LayerArgs A) {
    extern __shared__ __align__(1024) uint8_t sm[];
    const LayerGeom& g = A.g;
    const TiledGeom& tg = g.tg;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool consumer = warp < kLCons;
    uint4* xtab = reinterpret_cast<uint4*>(sm + g.o_xtab);
    float2* xg = reinterpret_cast<float2*>(sm + g.o_xg);
    float* red = reinterpret_cast<float*>(sm + g.o_red);          // [2][16 warps][32]
    float* red2 = reinterpret_cast<float*>(sm + g.o_red2);        // [16 warps][16]
    uint64_t* fullA = reinterpret_cast<uint64_t*>(sm + g.o_bar);
    uint64_t* emptyA = fullA + kLMaxNA;
    uint64_t* fullD = emptyA + kLMaxNA;
    uint64_t* emptyD = fullD + kLMaxND;
    uint64_t* fullS = emptyD + kLMaxND;
    uint64_t* emptyS = fullS + kLMaxNS;
    uint64_t* redF = emptyS + kLMaxNS;                            // [2] unit partials written (16 arrivals)
    uint64_t* redE = redF + 2;                                    // [2] unit partials consumed (1 arrival)
    uint64_t* routed = redE + 2;                                  // s_ids / s_w / s_loc ready (1 arrival)
    uint64_t* hF = routed + 1;                                    // [2] h digit record written (1 arrival)
    uint64_t* hE = hF + 2;                                        // [2] h digit record consumed (16 arrivals)
    uint8_t* hrec = sm + g.o_hrec;                                // [2][kHRec]
    uint32_t* s_ids = reinterpret_cast<uint32_t*>(sm + g.o_ids);
    float* s_w = reinterpret_cast<float*>(sm + g.o_w);
    uint32_t* s_loc = reinterpret_cast<uint32_t*>(sm + g.o_loc);  // local slots in slot order
    uint32_t* s_tok = s_loc + kLMaxTok * kLMaxK;                  // [ntok + 1] first local slot index per token
    uint32_t* s_nloc = s_tok + kLMaxTok + 1;
    uint8_t* ringA = sm + g.o_ringA;
    uint8_t* ringD = sm + g.o_ringD;
    uint8_t* ringS = sm + g.o_ringS;
    const int NA = g.NA, NS = g.NS, k = g.k, d = g.d;
    const uint32_t nslots = uint32_t(g.ntok * k);
    const int cta = blockIdx.x, ncta = gridDim.x;

    ltrace(A.trace, 0);
    // Set-up that reads nothing the previous kernel in the stream writes:
    // with programmatic dependent launch it runs while that kernel drains.
    // Barriers, one per thread of warps 0 and 1.
    if (tid < kLMaxNA) {
        mbar_init(fullA + tid, 1);
        mbar_init(emptyA + tid, kLCons);
    } else if (tid >= 32 && tid < 32 + kLMaxND) {
        mbar_init(fullD + (tid - 32), 1);
        mbar_init(emptyD + (tid - 32), kLCons);
    } else if (tid >= 40 && tid < 40 + kLMaxNS) {
        mbar_init(fullS + (tid - 40), 1);
        mbar_init(emptyS + (tid - 40), kLCons);
    } else if (tid >= 8 && tid < 10) {
        mbar_init(redF + (tid - 8), kLCons);
        mbar_init(redE + (tid - 8), 1);
    } else if (tid >= 12 && tid < 14) {
        mbar_init(hF + (tid - 12), 1);
        mbar_init(hE + (tid - 12), kLCons);
    } else if (tid == 10) {
        mbar_init(routed, 1);
    } else if (tid == 11) {
        // empty routing until it is known (a wait that runs out then finds
        // nothing to do rather than stale shared memory)
        *s_nloc = 0;
#pragma unroll 1
        for (int t = 0; t <= kLMaxTok; ++t) s_tok[t] = 0;
    }
    if (tid < 64) fence_mbar_init();
    const uint64_t t_start = gtimer();      // (the first clock read is slow: taken while the previous kernel drains)
    // the router row this CTA computes first, into L2
    if (A.rw && uint32_t(cta) < A.n_experts * uint32_t(g.ntok) && tid < d / 64)
        asm volatile("prefetch.global.L2 [%0];" :: "l"(A.rw + size_t(uint32_t(cta) % A.n_experts) * d + tid * 64));
    __syncthreads();
    ltrace(A.trace, 31);
    // the next kernel in the stream may start launching its CTAs as this
    // one's exit (its griddepcontrol.wait still waits for all of this grid)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // inputs (x, routing, the launch state) may come from the previous kernel
    asm volatile("griddepcontrol.wait;" ::: "memory");
    ltrace(A.trace, 10);
    // every wait: A.wait_ns from its start, the whole kernel at most 8 x that
    const WaitBudget wb{A.wait_ns, t_start + 8 * A.wait_ns};
    const LayerEp& ep = A.ep;
    const bool epm = ep.world > 1;
    // (read before the barrier below, and so before this CTA's producer
    // counts it done with the launch state: the last CTA to do so advances
    // them)
    const uint32_t epoch = epm ? __ldcg(&A.st->epoch) + 1u : 0u;
    const uint32_t seq = __ldcg(&A.st->seq) + 1u;                 // this launch's tag (never 0 in use)
    ltrace(A.trace, 21);
    // x: the caller's on rank 0; on ranks > 0 the copy rank 0 pushed into this
    // rank's own window (A.x points there), once its flag shows this epoch
    const void* xsrc = A.x;
    if (epm && ep.rank > 0 && tid == 0 && !spin_geq<true>(ep.flag, epoch, wb))
        raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
    __syncthreads();              // (ranks > 0: x is here)
    ltrace(A.trace, 24);
    if (epm && ep.rank == 0 && cta >= ncta - (ep.world - 1) && warp == kLHWarp) {
        // rank r's copy of x is pushed by the h warp of CTA grid - r (idle
        // until the routing is known), then that rank's epoch flag is advanced with
        // a system-scope release (after the warp barrier it orders every
        // lane's stores); the rank reads x and polls the flag locally
        const int r = ncta - cta;
        const uint32_t xbytes = uint32_t(size_t(g.ntok) * d * (A.x_dtype == 0 ? 4 : 2));
#pragma unroll
        for (int q = 1; q < kEpMaxWorld; ++q)
            if (q == r) {
                ep_push_x(ep.xw[q], A.x, xbytes, lane);
                __syncwarp();
                if (lane == 0) st_rel_sys(ep.flagw[q], epoch);
            }
    }
    // routing given: the producer warp's loads of it
    uint32_t pre_id[2] = {0u, 0u};
    float pre_w[2] = {0.f, 0.f};
    if (!A.rw && warp == kLProdWarp) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t i = lane + 32u * q;
            if (i < nslots) {
                pre_id[q] = __ldcg(A.ids_in + i);
                pre_w[q] = __ldcg(A.wts_in + i);
            }
        }
    }

    // The CTA's share of the A units [a0, a1) and the B units [b0, b1), known
    // once the routing (and so the local slot list) is.
    // Everything read back from the routing state is clamped to its valid
    // range before it forms an address: after a wait that ran out, the state
    // may be half written.
    auto nloc = [&]() { return min(*s_nloc, nslots); };
    auto slot_at = [&](uint32_t li) { return min(s_loc[li], nslots - 1u); };
    auto tok_at = [&](int t) { return min(s_tok[t], nloc()); };
    auto a_range = [&](int& a0, int& a1) {
        const int nA = int(nloc()) * g.tilesU;
        a0 = int(divu(uint32_t(cta) * uint32_t(nA), uint32_t(ncta), A.mg_grid));
        a1 = int(divu(uint32_t(cta + 1) * uint32_t(nA), uint32_t(ncta), A.mg_grid));
    };
    // phase R: row blocks (token, 16 output rows) of y
    const int nB = g.ntok * g.outTiles;
    const int b0 = int(divu(uint32_t(cta) * uint32_t(nB), uint32_t(ncta), A.mg_grid)),
              b1 = int(divu(uint32_t(cta + 1) * uint32_t(nB), uint32_t(ncta), A.mg_grid));
    // expert blob of a slot (its id is local: the slot is in s_loc)
    auto expert_of = [&](uint32_t slot) {
        uint32_t e = s_ids[slot] - ep.base;
        if (e >= ep.nlocal) e = 0;
        return A.base + uint64_t(e) * A.stride;
    };
    // local slot list and per-token starts (one warp, after s_ids is final)
    auto finish_routing = [&]() {
        if (!epm) {
            // single GPU: every slot is local unless its id is bad
            bool ok = true;
            #pragma unroll 1
            for (uint32_t sl = lane; sl < nslots; sl += 32) ok = ok && s_ids[sl] < A.n_experts;
            if (__all_sync(0xffffffffu, ok)) {
                #pragma unroll 1
                for (uint32_t sl = lane; sl < nslots; sl += 32) s_loc[sl] = sl;
                if (lane <= g.ntok) s_tok[lane] = uint32_t(lane * k);
                if (lane == 0) *s_nloc = nslots;
                __syncwarp();
                return;
            }
        }
        uint32_t cnt = 0;
        #pragma unroll 1
        for (uint32_t s0 = 0; s0 < nslots; s0 += 32) {
            const uint32_t sl = s0 + lane;
            bool loc = false;
            if (sl < nslots) {
                const uint32_t id = s_ids[sl];
                loc = id < A.n_experts && id - ep.base < ep.nlocal;
            }
            const uint32_t m = __ballot_sync(0xffffffffu, loc);
            if (loc) s_loc[cnt + __popc(m & ((1u << lane) - 1u))] = sl;
            cnt += __popc(m);
        }
        __syncwarp();
        if (lane <= g.ntok) {                      // first local index whose slot belongs to token >= lane
            uint32_t f = 0;
            while (f < cnt && s_loc[f] < uint32_t(lane * k)) ++f;
            s_tok[lane] = f;
        }
        if (lane == 0) *s_nloc = cnt;
        __syncwarp();
    };
    // head start (producer warp, single GPU, all ids valid, s_ids final):
    // every slot is local, so the CTA's A range is known without the routing
    // state - issue its first gate/up chunks before that state is built
    int preA = 0;                              // A items the head start issued
    auto head_start = [&]() {
        if (epm) return;
        bool ok = true;
        #pragma unroll 1
        for (uint32_t sl = lane; sl < nslots; sl += 32) ok = ok && s_ids[sl] < A.n_experts;
        if (__all_sync(0xffffffffu, ok) && lane == 0) {
            const uint32_t nA = nslots * uint32_t(g.tilesU);
            const int a0 = int(divu(uint32_t(cta) * nA, uint32_t(ncta), A.mg_grid));
            const int a1 = int(divu(uint32_t(cta + 1) * nA, uint32_t(ncta), A.mg_grid));
            const int n = min(NA, min(a1 - a0, 2) * int(tg.nchunk));   // units 0 and 1 come first
            int li = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), u = a0 - li * g.tilesU, c = 0;
            #pragma unroll 1
            for (int i = 0; i < n; ++i) {
                mbar_arrive_expect_tx(fullA + i, tg.chunk);
                bulk_g2s(ringA + size_t(i) * g.stageA(), A.base + uint64_t(s_ids[li]) * A.stride + tg.chunk_off(u, c),
                         tg.chunk, fullA + i);
                if (++c == int(tg.nchunk)) {
                    c = 0;
                    if (++u == g.tilesU) { u = 0; ++li; }
                }
            }
            preA = n;
        }
        __syncwarp();
    };
    // producer lane: issue every copy of the CTA, gate/up chunks first
    // Order: the gate/up chunks of units 0 and 1, then per unit n the down
    // scales of n (when n starts a new (slot, scale group)) and its down
    // columns, each after the gate/up chunks of unit n + 1 - the order in
    // which the consumers use them (gate/up of n + 1, then down of n), so
    // every copy lands in the order it is needed. One issue site per ring,
    // no integer division in the loop (each costs ~100 cycles on this lane's
    // critical path): every index advances by counters.
    auto produce = [&]() {
        int a0, a1;
        a_range(a0, a1);
        const int nun = a1 - a0;
        int ali = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), au = a0 - ali * g.tilesU;
        int dli = ali, du = au;
        int iA = 0, stA = 0, rA = 0, stD = 0, rD = 0, stS = 0, rS = 0, sg_li = -1, sg_j = -1;
        ltrace(A.trace, 11, true);
#pragma unroll 1
        for (int s = -1; s < nun; ++s) {
            if (s + 1 < nun) {                          // gate/up chunks of unit s + 1
                const uint8_t* ex = expert_of(slot_at(uint32_t(ali)));
#pragma unroll 1
                for (int c = 0; c < int(tg.nchunk); ++c, ++iA) {
                    if (iA >= preA) {                   // (the head start issued the first preA)
                        if (rA > 0) mbar_wait_e(emptyA + stA, (rA - 1) & 1, wb, A.err);
                        mbar_arrive_expect_tx(fullA + stA, tg.chunk);
                        bulk_g2s(ringA + size_t(stA) * g.stageA(), ex + tg.chunk_off(au, c), tg.chunk, fullA + stA);
                    }
                    if (++stA == NA) { stA = 0; ++rA; }
                }
                if (++au == g.tilesU) { au = 0; ++ali; }
            }
            if (s < 0) continue;
            const uint8_t* ex = expert_of(slot_at(uint32_t(dli)));   // down of unit s
            if (dli != sg_li || (du >> 2) != sg_j) {
                sg_li = dli;
                sg_j = du >> 2;
                if (rS > 0) mbar_wait_e(emptyS + stS, (rS - 1) & 1, wb, A.err);
                mbar_arrive_expect_tx(fullS + stS, tg.sgrp);
                bulk_g2s(ringS + size_t(stS) * g.stageS(), ex + tg.sgrp_off(uint32_t(sg_j)), tg.sgrp, fullS + stS);
                if (++stS == NS) { stS = 0; ++rS; }
            }
#pragma unroll 1
            for (int p = 0; p < g.dparts; ++p) {
                if (rD > 0) mbar_wait_e(emptyD + stD, (rD - 1) & 1, wb, A.err);
                const uint32_t bytes = g.dpart_bytes(p);
                mbar_arrive_expect_tx(fullD + stD, bytes);
                bulk_g2s(ringD + size_t(stD) * g.stageD(), ex + tg.dunit_off(uint32_t(du)) + size_t(p) * g.stageD(), bytes,
                         fullD + stD);
                if (++stD == g.ND) { stD = 0; ++rD; }
            }
            if (++du == g.tilesU) { du = 0; ++dli; }
        }
        ltrace(A.trace, 12, true);
    };

    // ------------------------------------------------------------- routing
    if (A.rw) {
        // logit rows r = cta + i * grid, all consumer warps per row
        const uint32_t rows = A.n_experts * g.ntok;
        #pragma unroll 1
        for (uint32_t r = cta; r < rows; r += ncta) {
            if (consumer) {
                const float v = router_row_part(A, xsrc, r / A.n_experts, r % A.n_experts, tid);
                if (lane == 0) red[warp] = v;
                cons_sync();
                if (tid == 0) {
                    float s = 0.f;
                    for (int w = 0; w < kLCons; ++w) s += red[w];
                    // value and tag in one 64-bit store: a reader that sees
                    // this launch's tag sees the value (no fence)
                    st_relaxed_gpu_u64(A.logits + r, (uint64_t(seq) << 32) | __float_as_uint(s));
                    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" :: "l"(&A.st->rdone) : "memory");
                }
                cons_sync();
            }
        }
        ltrace(A.trace, 1);
        if (warp == kLProdWarp) {
            // the producer warp selects (it then starts the weight stream
            // without a hand-over); one lane waits for the row count (cheap to poll), then the
            // warp reads the tagged logits (and re-reads any that are not
            // this launch's yet: the count is not ordered with the stores)
            if (lane == 0 && !spin_geq<false>(&A.st->rdone, rows, wb)) raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
            __syncwarp();
            ltrace(A.trace, 18, lane == 0);
            #pragma unroll 1
            for (int t = 0; t < g.ntok; ++t) {
                // (the host routes layers of more than 128 experts with k_router)
                float p[4];
                if (!wait_logits(A.logits + size_t(t) * A.n_experts, int(A.n_experts), seq, p, lane, wb))
                    raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
                if (t == 0) ltrace(A.trace, 19, lane == 0);
                warp_topk_regs<4>(p, int(A.n_experts), min(uint32_t(k), A.n_experts), A.norm, s_ids + t * k,
                                  s_w + t * k, lane);
                __syncwarp();
                if (cta == 0 && lane < k) {
                    if (A.ids_out) A.ids_out[t * k + lane] = s_ids[t * k + lane];
                    if (A.wts_out) A.wts_out[t * k + lane] = s_w[t * k + lane];
                }
            }
            __syncwarp();
            ltrace(A.trace, 20, lane == 0);
            head_start();
            finish_routing();
            if (lane == 0) mbar_arrive(routed);
            ltrace(A.trace, 2, lane == 0);
        }
    } else if (warp == kLProdWarp) {
        // routing given (loaded above): into shared memory, then start the
        // weight stream at once
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const uint32_t i = lane + 32u * q;
            if (i < nslots) {
                uint32_t id = pre_id[q];
                if (id >= A.n_experts) {
                    raise_err(A.err, SMOE_DEVERR_BAD_EXPERT);      // skipped: never local
                    id = 0xffffffffu;
                }
                s_ids[i] = id;
                s_w[i] = pre_w[q];
            }
        }
        __syncwarp();
        ltrace(A.trace, 28, lane == 0);
        head_start();
        finish_routing();
        ltrace(A.trace, 29, lane == 0);
        if (lane == 0) mbar_arrive(routed);
        ltrace(A.trace, 2);
    }
    if (warp == kLProdWarp) {       // one call site of the producer loop for both modes
        if (lane == 0) {
            mbar_wait_e(routed, 0, wb, A.err);
            produce();
            // This CTA is done with the launch state (its threads read seq and
            // epoch before the set-up barrier; its row-count wait has passed):
            // the last CTA to get here resets it for the next launch. (No
            // fence: the next launch reads it only after this grid has
            // completed - stream order or griddepcontrol.wait.)
            uint32_t old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&A.st->done) : "memory");
            if (old == uint32_t(ncta) - 1) {
                A.st->done = 0;
                A.st->rdone = 0;
                A.st->seq = seq;
                if (epm) A.st->epoch = epoch;
            }
        }
        __syncwarp();
    }

    if (consumer) {
        // ------------------------------------------------ x table, phase A
        ltrace(A.trace, 30);
        build_xtab<FMT>(xsrc, A.x_dtype, g.ntok, d, xtab, xg, tid, g.mg_G);
        cons_sync();
        ltrace(A.trace, 3);
        mbar_wait_e(routed, 0, wb, A.err);
        int a0, a1;
        a_range(a0, a1);
        const int gr = lane >> 2, cq = lane & 3;
        int iA = 0, stA = 0, rA = 0;
        int ali = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), au = a0 - ali * g.tilesU;
        uint32_t slot = slot_at(uint32_t(ali));
        int tok = int(divu(slot, uint32_t(k), g.mg_k));
        // Down side: unit n - 1 runs after the gate/up of unit n (the h warp
        // turns unit n - 1's partials into its digit record meanwhile). Warp
        // w owns row blocks b = w + 16 i (64 rows each); lanes c = 0 (digit
        // planes 0-1) and c = 1 (plane 2) keep partial sums of rows g, g + 8
        // of each of a block's four tiles, per token, flushed to the CTA's
        // partial rows when the token changes and at the end.
        const int nblk = d >> 6;
        constexpr int DBP = DB == 4 ? 2 : DB;                      // blocks per warp per down part
        float dacc[DB][2][2];
        int dli = ali, du = au, stD = 0, rD = 0, stS = 0, rS = 0, sg_li = -1, sg_j = -1;
#pragma unroll
        for (int i = 0; i < DB; ++i)
#pragma unroll
            for (int pq = 0; pq < 2; ++pq) dacc[i][pq][0] = dacc[i][pq][1] = 0.f;
        auto tok_of = [&](int li) { return int(divu(slot_at(uint32_t(li)), uint32_t(k), g.mg_k)); };
        auto flush = [&](int t) {
            unsigned long long* pr = A.part + (size_t(cta) * kLMaxTok + t) * kLMaxD;
#pragma unroll
            for (int i = 0; i < DB; ++i) {
                const int lb = warp + kLCons * (i % DBP), bk = (i / DBP) * g.bpp + lb;
#pragma unroll
                for (int pq = 0; pq < 2; ++pq)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        // lanes c, c ^ 1: planes 0-1 and plane 2 of tile 2pq + c / 2
                        const float v = dacc[i][pq][h] + __shfl_xor_sync(0xffffffffu, dacc[i][pq][h], 1);
                        if ((cq & 1) == 0 && lb < g.bpp && bk < nblk)
                            st_relaxed_gpu_u64(pr + 64 * bk + 16 * (2 * pq + (cq >> 1)) + gr + 8 * h,
                                               (uint64_t(seq) << 32) | __float_as_uint(v));
                        dacc[i][pq][h] = 0.f;
                    }
            }
        };
        auto down = [&](int n, bool last) {
            if (dli != sg_li || (du >> 2) != sg_j) {             // a new (slot, scale group)
                if (sg_li >= 0) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(emptyS + stS);
                    if (++stS == NS) { stS = 0; ++rS; }
                }
                sg_li = dli;
                sg_j = du >> 2;
                mbar_wait_e(fullS + stS, rS & 1, wb, A.err);
            }
            const int hb = n & 1;
            mbar_wait_e(hF + hb, (n >> 1) & 1, wb, A.err);
            if (last) ltrace(A.trace, 17);
            const uint8_t* rec = hrec + hb * kHRec;
            // One MMA m16n8k32 covers two row tiles: k 0-15 = the even tile's
            // codes x digit planes in columns 0-2, k 16-31 = the odd tile's x the
            // same planes in columns 4-6. Lane c then holds (c even) planes 0-1
            // or (c odd) plane 2 of tile c / 2 of the pair.
            const uint32_t pl = *reinterpret_cast<const uint32_t*>(rec + (gr & 3) * 16 + cq * 4);
            const uint32_t bq[2] = {gr < 3 ? pl : 0u, gr >= 4 && gr < 7 ? pl : 0u};
            const float2 xsv = *reinterpret_cast<const float2*>(rec + 48);
            const float xsl = (cq & 1) ? xsv.x * 65536.0f : xsv.x;
            const float shl = (cq & 1) ? 0.f : xsv.y;              // the sum term once
            const uint8_t* sp = ringS + size_t(stS) * g.stageS();
            constexpr uint32_t lo = 0x0F0F0F0Fu;
#pragma unroll
            for (int i = 0; i < DB; ++i) {
                const int p = i / DBP, lb = warp + kLCons * (i % DBP), bk = p * g.bpp + lb;
                if (i % DBP == 0) {                                   // the part's blocks are in its stage
                    if (i > 0) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(emptyD + stD);
                        if (++stD == g.ND) { stD = 0; ++rD; }
                    }
                    mbar_wait_e(fullD + stD, rD & 1, wb, A.err);
                    if (last && i == 0) ltrace(A.trace, 18);
                }
                const uint8_t* dp = ringD + size_t(stD) * g.stageD();
                if (lb < g.bpp && bk < nblk) {
                    const uint4 wq = *reinterpret_cast<const uint4*>(dp + (lb * 32 + lane) * 16);
#pragma unroll
                    for (int pq = 0; pq < 2; ++pq) {                  // tiles 2pq (low nibbles), 2pq + 1 (high)
                        const uint32_t w0 = pq == 0 ? wq.x : wq.z, w1 = pq == 0 ? wq.y : wq.w;
                        const uint32_t af[4] = {w0 & lo, w1 & lo, (w0 >> 4) & lo, (w1 >> 4) & lo};
                        int dq[4] = {0, 0, 0, 0};
                        mma_u8s8_16832(dq, af, bq);
                        // (for c odd, column 2c + 1 is a zero column: dq[1] = dq[3] = 0)
                        const int r0 = 64 * bk + 16 * (2 * pq + (cq >> 1)) + gr;
                        const float v0 = float(dq[0] + 256 * dq[1]) * xsl, v8 = float(dq[2] + 256 * dq[3]) * xsl;
                        if (FMT == kFmtAffine) {
                            const uint32_t s0 = reinterpret_cast<const uint32_t*>(sp)[r0];
                            const uint32_t s8 = reinterpret_cast<const uint32_t*>(sp)[r0 + 8];
                            dacc[i][pq][0] += fmaf(bf16_bits_to_f32(uint16_t(s0)), v0, bf16_bits_to_f32(uint16_t(s0 >> 16)) * shl);
                            dacc[i][pq][1] += fmaf(bf16_bits_to_f32(uint16_t(s8)), v8, bf16_bits_to_f32(uint16_t(s8 >> 16)) * shl);
                        } else {
                            const uint16_t* sh = reinterpret_cast<const uint16_t*>(sp);
                            dacc[i][pq][0] += f16_bits_to_f32(sh[r0]) * (v0 - shl);
                            dacc[i][pq][1] += f16_bits_to_f32(sh[r0 + 8]) * (v8 - shl);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(hE + hb);
                mbar_arrive(emptyD + stD);
            }
            if (++stD == g.ND) { stD = 0; ++rD; }
            if (++du == g.tilesU) { du = 0; ++dli; }
        };
        #pragma unroll 1
        for (int a = a0; a <= a1; ++a) {
            const int n = a - a0, b = n & 1;
            if (a < a1) {
                float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                #pragma unroll 1
                for (int c = 0; c < int(tg.nchunk); ++c, ++iA) {
                    const int st = stA;
                    mbar_wait_e(fullA + st, rA & 1, wb, A.err);
                    if (++stA == NA) { stA = 0; ++rA; }
                    if (n == 0 && c == 0) ltrace(A.trace, 4);
                    if (iA < 3) ltrace(A.trace, 25 + iA);
                    if (a + 1 == a1 && c + 1 == int(tg.nchunk)) ltrace(A.trace, 14);
                    const uint8_t* sp = ringA + size_t(st) * g.stageA();
                    const uint8_t* sbp = sp + 2 * tg.fragC;          // [gate sb][up sb]
                    uint4 w[GW][2];
    #pragma unroll
                    for (int j = 0; j < GW; ++j) {
                        const int gl = min(warp + j * kLCons, int(tg.Gc) - 1);
    #pragma unroll
                        for (int m = 0; m < 2; ++m)
                            w[j][m] = *reinterpret_cast<const uint4*>(sp + m * tg.fragC + (gl * 32 + lane) * 16);
                    }
    #pragma unroll
                    for (int j = 0; j < GW; ++j) {
                        const int gl = warp + j * kLCons;
                        if (gl < int(tg.Gc)) {
                            const int grp = c * int(tg.Gc) + gl;
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
                                    const uint32_t* sbw = reinterpret_cast<const uint32_t*>(sbp + m * tg.sbC) + gl * 16 + gr;
                                    const uint32_t s0 = sbw[0], s8 = sbw[8];
                                    acc[m][0] += fmaf(bf16_bits_to_f32(uint16_t(s0)), v0 * xv.x,
                                                      bf16_bits_to_f32(uint16_t(s0 >> 16)) * xv.y);
                                    acc[m][1] += fmaf(bf16_bits_to_f32(uint16_t(s8)), v8 * xv.x,
                                                      bf16_bits_to_f32(uint16_t(s8 >> 16)) * xv.y);
                                } else {
                                    const uint16_t* sbh = reinterpret_cast<const uint16_t*>(sbp + m * tg.sbC) + gl * 16 + gr;
                                    acc[m][0] += f16_bits_to_f32(sbh[0]) * fmaf(v0, xv.x, -xv.y);
                                    acc[m][1] += f16_bits_to_f32(sbh[8]) * fmaf(v8, xv.x, -xv.y);
                                }
                            }
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(emptyA + st);          // chunk fully consumed
                }
                // the unit's warp partials -> buffer b (free once the h warp read use n-2)
                if (n >= 2) mbar_wait_e(redE + b, ((n >> 1) - 1) & 1, wb, A.err);
                float* rb = red + (b * kLCons + warp) * 32;
                if (cq == tok) {
                    rb[gr] = acc[0][0];
                    rb[gr + 8] = acc[0][1];
                    rb[16 + gr] = acc[1][0];
                    rb[16 + gr + 8] = acc[1][1];
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(redF + b);
                if (++au == g.tilesU) {
                    au = 0;
                    slot = slot_at(uint32_t(++ali));
                    tok = int(divu(slot, uint32_t(k), g.mg_k));
                }
            }
            if (a == a1) ltrace(A.trace, 20);
            if (n > 0) {
                const int t = tok_of(dli);
                down(n - 1, a == a1);                              // (advances dli, du)
                if (a == a1 || tok_of(dli) != t) flush(t);        // the token's last unit here
            }
            if (a == a1) ltrace(A.trace, 19);
            if (n == 1) ltrace(A.trace, 13);
        }
        ltrace(A.trace, 5);

        ltrace(A.trace, 16);

        // ------------------------------------------------ phase R
        // Row block (token t, rows 16o..16o+15): the sum of the partial rows
        // of the CTAs whose unit ranges hold t's units, in CTA order - thread
        // (j, r) adds CTAs c_lo + j, + 32, ... of row r, then one thread per
        // row adds the 32 in j order (fixed order: bitwise repeatable). The
        // partial rows carry this launch's tag: no grid-wide barrier, each
        // thread polls its own values until every tag is there.
        if (b0 < b1) {
            const int r = tid & 15, j = tid >> 4;
            const uint32_t nA = nloc() * uint32_t(g.tilesU);
            int t = int(divu(uint32_t(b0), uint32_t(g.outTiles), g.mg_outTiles)), o = b0 - t * g.outTiles - 1;
            #pragma unroll 1
            for (int bu = b0; bu < b1; ++bu) {
                if (++o == g.outTiles) { o = 0; ++t; }
                const uint32_t ulo = tok_at(t) * uint32_t(g.tilesU), uhi = tok_at(t + 1) * uint32_t(g.tilesU);
                // CTA c holds units [c nA / grid, (c+1) nA / grid): unit u is in
                // CTA ((u + 1) grid - 1) / nA
                int c_lo = 0, c_hi = -1;
                if (uhi > ulo) {
                    c_lo = int(((ulo + 1) * uint32_t(ncta) - 1) / nA);
                    c_hi = min(int((uhi * uint32_t(ncta) - 1) / nA), ncta - 1);
                }
                float pv[kLRedMax];
                uint32_t need = 0;                                 // bit m: value m still to arrive
                const unsigned long long* col = A.part + size_t(t) * kLMaxD + o * 16 + r;
#pragma unroll
                for (int m = 0; m < kLRedMax; ++m) {
                    const int c = c_lo + j + 32 * m;
                    pv[m] = 0.f;
                    if (c <= c_hi && divu(uint32_t(c + 1) * nA, uint32_t(ncta), A.mg_grid) >
                                         divu(uint32_t(c) * nA, uint32_t(ncta), A.mg_grid))
                        need |= 1u << m;
                }
                const uint64_t deadline = wb.deadline();
                #pragma unroll 1
                for (uint32_t it = 0; need; ++it) {
                    uint64_t v[kLRedMax];
#pragma unroll
                    for (int m = 0; m < kLRedMax; ++m)
                        if (need & (1u << m)) v[m] = ld_relaxed_gpu_u64(col + size_t(c_lo + j + 32 * m) * kLMaxTok * kLMaxD);
#pragma unroll
                    for (int m = 0; m < kLRedMax; ++m)
                        if ((need & (1u << m)) && uint32_t(v[m] >> 32) == seq) {
                            pv[m] = __uint_as_float(uint32_t(v[m]));
                            need &= ~(1u << m);
                        }
                    if (need && (it & 3) == 3 && gtimer() > deadline) {
                        raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
                        break;
                    }
                    if (need && it >= 8) __nanosleep(32);
                }
                if (bu == b0) ltrace(A.trace, 6);
                float s = 0.f;
#pragma unroll
                for (int m = 0; m < kLRedMax; ++m) s += pv[m];
                red2[j * 16 + r] = s;
                cons_sync();
                if (bu == b0) ltrace(A.trace, 15);
                if (tid < 16) {                                   // warp 0, lanes 0-15: row 16o + tid
                    s = 0.f;
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) s += red2[jj * 16 + tid];
                    const size_t yi = size_t(t) * d + o * 16 + tid;
                    const bool write = !epm || ep_combine16(ep.rank, ep.world, ep.part0, ep.part_stride, epoch, s,
                                                            yi, A.err, wb);
                    if (bu == b0) ltrace(A.trace, 22);
                    if (write) {
                        if (A.y_dtype == 0) static_cast<float*>(A.y)[yi] = s;
                        else static_cast<__nv_bfloat16*>(A.y)[yi] = __float2bfloat16_rn(s);
                    }
                }
                cons_sync();
            }
            ltrace(A.trace, 7);
        }
    } else if (warp == kLHWarp) {
        // ------------------------------------------------ h warp
        // per unit: h = silu(gate) * up * w_slot (kernels.metal:61-63) of its
        // 16 rows, then the unit's digit record for the down MMAs: E = the
        // exponent of max|h|, X = round(h 2^(20-E)) = p0 + 2^8 p1 + 2^16 p2
        // (signed bytes) at 0 / 16 / 32, and at 48 the fp32 pair (2^(E-20)
        // (/7.5 for SMOE-Q4), sum X 2^(E-20))
        mbar_wait_e(routed, 0, wb, A.err);
        int a0, a1;
        a_range(a0, a1);
        int hli = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), hu = a0 - hli * g.tilesU;
        #pragma unroll 1
        for (int a = a0; a < a1; ++a, ++hu) {
            if (hu == g.tilesU) { hu = 0; ++hli; }
            const int n = a - a0, b = n & 1;
            const uint32_t slot = slot_at(uint32_t(hli));
            mbar_wait_e(redF + b, (n >> 1) & 1, wb, A.err);
            const float* rb = red + b * kLCons * 32;
            float v = 0.f;                                        // lane = (matrix, row)
#pragma unroll
            for (int w = 0; w < kLCons; ++w) v += rb[w * 32 + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(redE + b);
            const float up = __shfl_down_sync(0xffffffffu, v, 16);
            const float hv = lane < 16 ? v * (1.0f / (1.0f + expf(-v))) * up * s_w[slot] : 0.f;
            float m = fabsf(hv);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            const int E = max(int((__float_as_uint(m) >> 23) & 0xff) - 127, -100);
            const float f = pow2i(20 - E);
            const int X = __float2int_rn(hv * f);
            int sx = X;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
            if (n >= 2) mbar_wait_e(hE + b, ((n >> 1) - 1) & 1, wb, A.err);
            uint8_t* rec = hrec + b * kHRec;
            if (lane < 16) {
                const int d0 = ((X + 128) & 255) - 128, rr = (X - d0) >> 8;
                const int d1 = ((rr + 128) & 255) - 128, d2 = (rr - d1) >> 8;
                rec[lane] = uint8_t(d0);
                rec[16 + lane] = uint8_t(d1);
                rec[32 + lane] = uint8_t(d2);
            }
            if (lane == 0) {
                const float xs = pow2i(E - 20);
                *reinterpret_cast<float2*>(rec + 48) =
                    make_float2(FMT == kFmtAffine ? xs : xs * (1.0f / 7.5f), float(sx) * xs);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(hF + b);
        }
        ltrace(A.trace, 8, lane == 0);
    }

    ltrace(A.trace, 9);
}

}  // namespace smoe
