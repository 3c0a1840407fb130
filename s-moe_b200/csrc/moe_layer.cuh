// moe_layer.cuh - the persistent MoE-layer kernel for decode batches of up
// to kLMaxTok tokens (sm_100a), on the tiled expert layout (tiled.cuh).
//
// One launch, one CTA per SM:
//   routing (optional; decode.cpp:280-303): router logit rows spread over
//     the grid; every CTA then runs the softmax / top-k / renorm of
//     router.cuh on all logits (identical results in every CTA);
//   phase A - gate/up (kernels.metal:240-337): the A units (slot, 16 hidden
//     rows) are split evenly over the CTAs; each yields
//     h = silu(Wg.x) * (Wu.x) * w_slot for its 16 rows, stored as fp32 to a
//     global scratch record (64 B);
//   one grid-wide arrive/wait (every CTA is resident: one CTA per SM);
//   phase B - down + combine (kernels.metal:340-365, decode.cpp:485-499):
//     the B units (token, 16 output rows) are split evenly over the CTAs;
//     each computes its 16 rows of y = sum_slots W_down . h over all of the
//     token's slots and writes them - every output row has exactly one
//     owner, so there are no atomics and the sums are in a fixed order
//     (bitwise reproducible).
// Every byte a CTA needs is streamed by one producer lane with 1-D bulk
// copies (no multicast) into two rings of shared-memory stages - gate/up
// chunks first, then the down tiles - so the down weights are already on
// chip when the grid-wide wait ends. Sixteen consumer warps run the gate/up
// dots as integer MMAs on the raw codes (arithmetic below) and the down
// tiles as bf16 MMAs; warp 16 turns each unit's 16 warp partials into h.
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
// Down arithmetic: the same fixed-point digits, for h: the h warp stores
// each 16-row unit's h as fp32; when phase B loads a token's h, each 64-group
// (four units) is quantised with the exponent of its max|h| into three
// unsigned byte planes (offset 2^21). The down product runs as integer MMAs
// m16n8k16 (u8 x u8), one per unit with the planes in columns 0-2 of B and
// ones in column 3 (to take the offset back out), the four units of a group
// chained into one exact int32 accumulator (odd units' codes shifted down to
// q); per group the sums are scaled by 2^(E-20) and the fp32 epilogue applies
// the down matrix's scale (and bias).
//
// Expert parallel (world > 1, one process per GPU, experts [r*E/G,
// (r+1)*E/G) on rank r): every rank routes (the same ids), runs the A units
// of the slots whose expert it holds, and the B units of every token over its
// local slots; ranks > 0 store their partial rows into rank 0's window with
// peer stores and count them per B unit with system-scope atomics; rank 0's
// owner of that B unit waits for the count (bounded), adds the partials in
// rank order and writes y. x is published by rank 0 (release flag) and read
// by the others with peer loads. No TMA or bulk copy touches peer memory.
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
constexpr int kLMaxNA = 4;                    // gate/up ring stages (at most)
constexpr int kLMaxNB = 16;                   // down ring stages (at most)
constexpr int kHRec = 64;                      // one unit's h: 16 fp32
constexpr int kHGrp = 4 * kHRec;               // one 64-group's digit record in shared memory
constexpr int kEpMaxWorld = 8;

struct LayerState {          // device scratch, zero at context creation; the counters zero after every launch
    uint32_t rdone;                 // router logit rows stored (a hint: the logits carry their own tag)
    uint32_t arrive;                // CTAs past phase A
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
    int G, tilesU, outTiles, NA, NB;
    uint32_t mg_tilesU, mg_outTiles, mg_Gd, mg_G, mg_k;   // division magics (divu below)
    int o_xtab, o_xg, o_red, o_red2, o_bar, o_ids, o_w, o_loc, o_ringA, o_ringB, total;

    __host__ __device__ bool init(int fmt, int d_, int dff_, int k_, int ntok_, int max_smem) {
        d = d_; dff = dff_; k = k_; ntok = ntok_;
        if (!tg.init(fmt, d, dff) || tg.Gc > 32 || ntok < 1 || ntok > kLMaxTok || k < 1 || k > kLMaxK) return false;
        G = d / 64; tilesU = dff / 16; outTiles = d / 16;
        mg_tilesU = magic_of(uint32_t(tilesU));
        mg_outTiles = magic_of(uint32_t(outTiles));
        mg_Gd = magic_of(tg.Gd);
        mg_G = magic_of(uint32_t(G));
        mg_k = magic_of(uint32_t(k));
        int off = 0;
        auto take = [&](int bytes) { int o = off; off += (bytes + 127) & ~127; return o; };
        const int xt = G * 1024, hr = k * tilesU * kHRec;    // x table, then (phase B) one token's h records
        o_xtab = take(xt > hr ? xt : hr);
        o_xg = take(G * 4 * 8);
        const int rs = 2 * kLCons * 32 * 4, ps = 4 * kLMaxTok * kRouterMaxE;
        o_red = take(rs);                                    // double-buffered unit partials / router partials
        o_red2 = take(kLCons * 16 * 4);
        o_bar = take((2 * kLMaxNA + 2 * kLMaxNB + 5) * 8);
        o_ids = take(kLMaxTok * kLMaxK * 4);
        o_w = take(kLMaxTok * kLMaxK * 4);
        o_loc = take(4 * (kLMaxTok * kLMaxK + kLMaxTok + 2));  // local slots, token starts, count
        (void)ps;
        off = (off + 1023) & ~1023;
        const int fixed = off;
        const int avail = max_smem - fixed;
        const int ca = int((tg.chunk + 127) & ~127u), cb = int((tg.btile + 127) & ~127u);
        NA = 3;
        if (avail < 3 * ca + 2 * cb) NA = 2;
        if (NA > kLMaxNA) NA = kLMaxNA;
        NB = (avail - NA * ca) / cb;
        if (NB > kLMaxNB) NB = kLMaxNB;
        if (NB < 2) return false;
        o_ringA = fixed;
        o_ringB = fixed + NA * ca;
        total = o_ringB + NB * cb;
        return total <= max_smem;
    }
    __host__ __device__ int stageA() const { return int((tg.chunk + 127) & ~127u); }
    __host__ __device__ int stageB() const { return int((tg.btile + 127) & ~127u); }
};

struct LayerEp {
    int world, rank;
    uint32_t base, nlocal;     // global id of this rank's first expert, experts held
    uint8_t* x0;               // rank 0's copy of x (peer memory on ranks > 0)
    uint32_t* flag0;           // rank 0's x epoch
    float* part0;              // [world][kLMaxTok * d] partial rows, in rank 0's window
    uint32_t* cnt0;            // [kLMaxTok * d/16] partial B units arrived, in rank 0's window
    uint32_t part_stride;      // floats per rank in part0
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
    uint8_t* hbuf;             // scratch h, fp32 [ntok*k][d_ff/16][16]
    LayerState* st;
    uint32_t* err;
    uint64_t wait_ns;          // limit of every wait
    uint32_t mg_grid;          // magic_of(grid size)
    unsigned long long* trace; // optional [grid x 32] phase timestamps (ns)
    LayerGeom g;
    LayerEp ep;
};

SMOE_DEVINL void ltrace(unsigned long long* tr, int i, bool who = threadIdx.x == 0) {
    if (tr && who && i < 32) {
        tr[blockIdx.x * 32 + i] = gtimer();
        tr[(gridDim.x + blockIdx.x) * 32 + i] = clock64();          // same mark in SM cycles
    }
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

// Digit record of one (slot, 64-group) of h for the down MMAs, built by a
// half-warp (j = 0..15 its thread, v = h rows 4(j&3)..+3 of unit j>>2): one
// exponent E for the group's 64 values, X = round(h * 2^(20-E)) (|X| <= 2^21)
// offset to Xu = X + 2^21 in [0, 2^22] and split into three unsigned byte
// planes. Plane p holds at p*64 + c*16 + u*4 + b the digit of unit u, row
// 4c + b (lane 4g + c's B register of unit u = one 32-bit word, its four
// units one 16-byte load); at 192 the fp32 pair (2^(E-20) (/7.5 for
// SMOE-Q4), sum of the fixed-point h). The offset comes back out through a
// column of ones in the MMA (sum q * X = sum q * Xu - 2^21 sum q). Every
// lane of the warp calls it; `valid` is the same for the 16 threads of a group.
template <int FMT>
SMOE_DEVINL void h_digits(float4 v, uint8_t* rec, int j, bool valid) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // below 2^-100 every X rounds to 0 anyway; the clamp keeps 2^(20-E) a normal float
    const int E = max(int((__float_as_uint(m) >> 23) & 0xff) - 127, -100);
    const float f = pow2i(20 - E);
    const int X[4] = {__float2int_rn(v.x * f), __float2int_rn(v.y * f), __float2int_rn(v.z * f),
                      __float2int_rn(v.w * f)};
    int sx = X[0] + X[1] + X[2] + X[3];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, o);
    const uint32_t u0 = uint32_t(X[0] + (1 << 21)), u1 = uint32_t(X[1] + (1 << 21)),
                   u2 = uint32_t(X[2] + (1 << 21)), u3 = uint32_t(X[3] + (1 << 21));
    if (valid) {
        uint32_t* w = reinterpret_cast<uint32_t*>(rec + (j & 3) * 16 + (j >> 2) * 4);
#pragma unroll
        for (int p = 0; p < 3; ++p)                      // byte p of each value: plane p
            w[16 * p] = __byte_perm(__byte_perm(u0, u1, 0x0040u + 0x0011u * p),
                                    __byte_perm(u2, u3, 0x0040u + 0x0011u * p), 0x5410u);
        if (j == 0) {
            const float xs = pow2i(E - 20);
            *reinterpret_cast<float2*>(rec + 192) =
                make_float2(FMT == kFmtAffine ? xs : xs * (1.0f / 7.5f), float(sx) * xs);
        }
    }
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
    for (int i = ctid; i < G * 64; i += kLCThreads) xtab[i] = make_uint4(0u, 0u, 0u, 0u);
    const int warp = ctid >> 5, lane = ctid & 31;
    constexpr int U = 2;
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

// GW: 64-groups of a gate/up chunk per consumer warp, ceil(Gc / 16)
template <int FMT, int GW>
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
    uint64_t* fullB = emptyA + kLMaxNA;
    uint64_t* emptyB = fullB + kLMaxNB;
    uint64_t* redF = emptyB + kLMaxNB;                            // [2] unit partials written (16 arrivals)
    uint64_t* redE = redF + 2;                                    // [2] unit partials consumed (1 arrival)
    uint64_t* routed = redE + 2;                                  // s_ids / s_w / s_loc ready (1 arrival)
    uint32_t* s_ids = reinterpret_cast<uint32_t*>(sm + g.o_ids);
    float* s_w = reinterpret_cast<float*>(sm + g.o_w);
    uint32_t* s_loc = reinterpret_cast<uint32_t*>(sm + g.o_loc);  // local slots in slot order
    uint32_t* s_tok = s_loc + kLMaxTok * kLMaxK;                  // [ntok + 1] first local slot index per token
    uint32_t* s_nloc = s_tok + kLMaxTok + 1;
    uint8_t* ringA = sm + g.o_ringA;
    uint8_t* ringB = sm + g.o_ringB;
    const int NA = g.NA, NB = g.NB, k = g.k, d = g.d;
    const uint32_t nslots = uint32_t(g.ntok * k);
    const int cta = blockIdx.x, ncta = gridDim.x;
    __shared__ uint32_t last_cta;

    ltrace(A.trace, 0);
    // inputs (x, routing) may come from the previous kernel in the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");
    ltrace(A.trace, 10);
    // every wait: A.wait_ns from its start, the whole kernel at most 8 x that
    const WaitBudget wb{A.wait_ns, gtimer() + 8 * A.wait_ns};
    const LayerEp& ep = A.ep;
    const bool epm = ep.world > 1;
    const uint32_t epoch = epm ? A.st->epoch + 1u : 0u;           // written by the previous launch only
    const uint32_t seq = A.st->seq + 1u;                          // this launch's tag (never 0 in use)
    // x: the caller's, or on ranks > 0 rank 0's published copy (peer memory)
    const void* xsrc = A.x;
    if (epm) {
        const size_t xbytes = size_t(g.ntok) * d * (A.x_dtype == 0 ? 4 : 2);
        if (ep.rank == 0 && cta == 0) {
            for (size_t i = tid; i < xbytes / 16; i += blockDim.x)
                reinterpret_cast<uint4*>(ep.x0)[i] = reinterpret_cast<const uint4*>(A.x)[i];
        } else if (ep.rank > 0) {
            if (tid == 0 && !spin_geq<true>(ep.flag0, epoch, wb)) raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
            xsrc = ep.x0;
        }
    }
    // routing given: the producer warp's loads of it are issued before the
    // set-up barrier, so their latency overlaps it
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
    // barrier set-up, one barrier per thread of warp 0 and 1
    if (tid < kLMaxNA) {
        mbar_init(fullA + tid, 1);
        mbar_init(emptyA + tid, kLCons);
    } else if (tid >= 32 && tid < 32 + kLMaxNB) {
        mbar_init(fullB + (tid - 32), 1);
        mbar_init(emptyB + (tid - 32), kLCons);
    } else if (tid >= 8 && tid < 10) {
        mbar_init(redF + (tid - 8), kLCons);
        mbar_init(redE + (tid - 8), 1);
    } else if (tid == 10) {
        mbar_init(routed, 1);
    } else if (tid == 11) {
        // empty routing until it is known (a wait that runs out then finds
        // nothing to do rather than stale shared memory)
        *s_nloc = 0;
        for (int t = 0; t <= kLMaxTok; ++t) s_tok[t] = 0;
    }
    if (tid < 64) fence_mbar_init();
    __syncthreads();              // (ranks > 0: rank 0's x is published; rank 0 CTA 0: x0 is written)
    ltrace(A.trace, 31);
    if (epm && ep.rank == 0 && cta == 0 && tid == 0) {
        __threadfence_system();
        st_rel_sys(ep.flag0, epoch);
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
            for (uint32_t sl = lane; sl < nslots; sl += 32) ok = ok && s_ids[sl] < A.n_experts;
            if (__all_sync(0xffffffffu, ok)) {
                for (uint32_t sl = lane; sl < nslots; sl += 32) s_loc[sl] = sl;
                if (lane <= g.ntok) s_tok[lane] = uint32_t(lane * k);
                if (lane == 0) *s_nloc = nslots;
                __syncwarp();
                return;
            }
        }
        uint32_t cnt = 0;
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
        for (uint32_t sl = lane; sl < nslots; sl += 32) ok = ok && s_ids[sl] < A.n_experts;
        if (__all_sync(0xffffffffu, ok) && lane == 0) {
            const uint32_t nA = nslots * uint32_t(g.tilesU);
            const int a0 = int(divu(uint32_t(cta) * nA, uint32_t(ncta), A.mg_grid));
            const int a1 = int(divu(uint32_t(cta + 1) * nA, uint32_t(ncta), A.mg_grid));
            const int n = min(NA, (a1 - a0) * int(tg.nchunk));
            int li = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), u = a0 - li * g.tilesU, c = 0;
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
    auto produce = [&]() {
        int a0, a1;
        a_range(a0, a1);
        const int nAi = (a1 - a0) * int(tg.nchunk);
        int nBi = 0;
        {
            int t = int(divu(uint32_t(b0), uint32_t(g.outTiles), g.mg_outTiles)), o = b0 - t * g.outTiles;
            for (int b = b0; b < b1; ++b) {
                nBi += max(int(tok_at(t + 1)) - int(tok_at(t)), 0);
                if (++o == g.outTiles) { o = 0; ++t; }
            }
        }
        // One issue site (code size: this runs cold once per launch), and no
        // integer division in the loop (each costs ~100 cycles of latency on
        // this lane's critical path): every index advances by counters.
        // Order: the first NA gate/up chunks, the first NB down parts, then
        // the rest of each as stages free up.
        int iA = 0, iB = 0;
        int ali = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), au = a0 - ali * g.tilesU, ac = 0;          // next A item: (local slot, unit, chunk)
        int stA = 0, rA = 0, stB = 0, rB = 0;
        for (; iA < preA; ++iA) {              // issued already by the head start below
            if (++ac == int(tg.nchunk)) {
                ac = 0;
                if (++au == g.tilesU) { au = 0; ++ali; }
            }
            if (++stA == NA) { stA = 0; ++rA; }
        }
        int bt = int(divu(uint32_t(b0), uint32_t(g.outTiles), g.mg_outTiles)), bo = b0 - bt * g.outTiles, bb = b0;     // next B part: (token, tile), slot jj
        int jj = b0 < b1 ? int(tok_at(bt)) : 0;
        ltrace(A.trace, 11, true);
        const int limA0 = min(NA, nAi), limB0 = min(NB, nBi);
#pragma unroll 1
        for (int step = 0; step < 4; ++step) {
#ifdef SMOE_EXP_BFIRST
            const bool isA = (step & 1) == 1;
#else
            const bool isA = (step & 1) == 0;
#endif
            const int lim = isA ? (step < 2 ? limA0 : nAi) : (step < 2 ? limB0 : nBi);
            if (step == 1) ltrace(A.trace, 17, true);
#pragma unroll 1
            while ((isA ? iA : iB) < lim) {
                const int st = isA ? stA : stB, r = isA ? rA : rB;
                uint64_t* full = (isA ? fullA : fullB) + st;
                if (r > 0 && !mbar_wait_b((isA ? emptyA : emptyB) + st, (r - 1) & 1, wb))
                    raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
                uint64_t off;
                uint32_t slot, bytes;
                uint8_t* dst;
                if (isA) {
                    slot = slot_at(uint32_t(ali));
                    off = tg.chunk_off(au, ac);
                    bytes = tg.chunk;
                    dst = ringA + size_t(st) * g.stageA();
                    if (++ac == int(tg.nchunk)) {
                        ac = 0;
                        if (++au == g.tilesU) { au = 0; ++ali; }
                    }
                    ++iA;
                    if (++stA == NA) { stA = 0; ++rA; }
                } else {
                    while (jj >= int(tok_at(bt + 1)) && bb < b1) {   // next B unit (skip tokens without local slots)
                        ++bb;
                        if (++bo == g.outTiles) { bo = 0; ++bt; }
                        jj = int(tok_at(bt));
                    }
                    if (bb >= b1) break;
                    slot = slot_at(uint32_t(jj));
                    off = tg.btile_off(bo);
                    bytes = tg.btile;
                    dst = ringB + size_t(st) * g.stageB();
                    ++jj;
                    ++iB;
                    if (++stB == NB) { stB = 0; ++rB; }
                }
                mbar_arrive_expect_tx(full, bytes);
                bulk_g2s(dst, expert_of(slot) + off, bytes, full);
            }
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
            if (!mbar_wait_b(routed, 0, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
            produce();
        }
        __syncwarp();
    }

    if (consumer) {
        // ------------------------------------------------ x table, phase A
        ltrace(A.trace, 30);
        build_xtab<FMT>(xsrc, A.x_dtype, g.ntok, d, xtab, xg, tid, g.mg_G);
        cons_sync();
        ltrace(A.trace, 3);
        if (!mbar_wait_b(routed, 0, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
        int a0, a1;
        a_range(a0, a1);
        const int gr = lane >> 2, cq = lane & 3;
        int iA = 0, stA = 0, rA = 0;
        int ali = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), au = a0 - ali * g.tilesU;
        uint32_t slot = slot_at(uint32_t(ali));
        int tok = int(divu(slot, uint32_t(k), g.mg_k));
        #pragma unroll 1
        for (int a = a0; a < a1; ++a) {
            const int n = a - a0, b = n & 1;
            float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
            #pragma unroll 1
            for (int c = 0; c < int(tg.nchunk); ++c, ++iA) {
                const int st = stA;
                if (!mbar_wait_b(fullA + st, rA & 1, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
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
            if (n >= 2 && !mbar_wait_b(redE + b, ((n >> 1) - 1) & 1, wb))
                raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
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
        ltrace(A.trace, 5);

        // ------------------------------------------------ phase B
        if (b0 < b1) {
            // the first wave's down parts stream in during phase A: wait for
            // them before the grid-wide wait, which is the longer one
            int pre_w = 0;
            {
                const int t0 = int(divu(uint32_t(b0), uint32_t(g.outTiles), g.mg_outTiles)), l0 = int(tok_at(t0));
                pre_w = min(NB, max(l0, min(int(tok_at(t0 + 1)), l0 + k)) - l0);
                #pragma unroll 1
                for (int q = 0; q < pre_w; ++q)
                    if (!mbar_wait_b(fullB + q, 0, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
            }
            if (tid == 0 && !spin_geq<false>(&A.st->arrive, uint32_t(ncta), wb))
                raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
            cons_sync();
            ltrace(A.trace, 6);
            uint8_t* hsm = reinterpret_cast<uint8_t*>(xtab);          // the x table is no longer needed
            int cur = -1, stB = 0, rB = 0;
            const uint32_t bones = gr == 3 ? 0x01010101u : 0u;        // B column 3 of the down MMAs
            const int cmul = cq == 0 ? 256 : -32;
            int t = int(divu(uint32_t(b0), uint32_t(g.outTiles), g.mg_outTiles)), o = b0 - t * g.outTiles - 1;
            #pragma unroll 1
            for (int bu = b0; bu < b1; ++bu) {
                if (++o == g.outTiles) { o = 0; ++t; }
                const int ls = int(tok_at(t)), le = max(ls, min(int(tok_at(t + 1)), ls + k));
                if (t != cur) {
                    // this token's h (local slots ls..le) into shared memory as
                    // digit records, one per (slot, 64-group): 16 threads (a
                    // half-warp) per group, 4 values each
                    if (cur >= 0) cons_sync();                        // the previous token's are done with
                    const float4* src = reinterpret_cast<const float4*>(A.hbuf + size_t(ls) * g.tilesU * kHRec);
                    const int n16 = (le - ls) * g.tilesU * (kHRec / 16);   // a multiple of 16
                    constexpr int U = 4;
#pragma unroll 1
                    for (int base = 0; base < n16; base += U * kLCThreads) {
                        float4 v[U];
#pragma unroll
                        for (int q = 0; q < U; ++q) {
                            const int i = base + q * kLCThreads + tid;
                            v[q] = i < n16 ? __ldcg(src + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int q = 0; q < U; ++q) {
                            const int i = base + q * kLCThreads + tid;
                            h_digits<FMT>(v[q], hsm + size_t(i >> 4) * kHGrp, i & 15, i < n16);
                        }
                    }
                    cons_sync();
                    if (cur < 0) ltrace(A.trace, 16);
                    cur = t;
                }
                // The token's parts (local slots) stream through the ring in
                // waves of at most NB: every warp waits for all parts of a
                // wave, takes its share of the wave's (part, 64-group)
                // items, then releases all of the wave's stages. (A warp
                // releases a stage only after that stage's new data arrived,
                // so its arrival always counts toward the right round.)
                float y0 = 0.f, y8 = 0.f;
                #pragma unroll 1
                for (int w0 = ls; w0 < le; w0 += NB) {
                    const int W = min(NB, le - w0);
                    if (pre_w > 0) {
                        pre_w = 0;                    // the first wave: waited for above
                    } else {
                        int sb = stB, rb = rB;
                        #pragma unroll 1
                        for (int q = 0; q < W; ++q) {
                            if (!mbar_wait_b(fullB + sb, rb & 1, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
                            if (++sb == NB) { sb = 0; ++rb; }
                        }
                    }
                    if (w0 == ls && bu == b0) ltrace(A.trace, 13);
                    const bool tr_items = w0 == ls && bu == b0;
                    // this warp's items [i0, i1) of the wave's W x Gd (part, group) items
                    const int nit = W * int(tg.Gd);
                    const int i0 = (warp * nit) >> 4, i1 = ((warp + 1) * nit) >> 4;   // kLCons == 16
                    int iq = int(divu(uint32_t(i0), tg.Gd, g.mg_Gd)), ig = i0 - iq * int(tg.Gd);
                    int sidx = stB + iq;
                    if (sidx >= NB) sidx -= NB;
                    #pragma unroll 2
                    for (int it = i0; it < i1; ++it) {
                        // one (part, 64-group): four int8 MMAs m16n8k16, one per
                        // 16-column unit, B = the unit's digit planes in columns 0-2
                        const uint8_t* sp = ringB + size_t(sidx) * g.stageB();
                        const uint4 wq = *reinterpret_cast<const uint4*>(sp + (ig * 32 + lane) * 16);
                        const uint8_t* rec = hsm + (size_t(w0 + iq - ls) * tg.Gd + ig) * kHGrp;
                        const uint4 bq = gr < 3 ? *reinterpret_cast<const uint4*>(rec + gr * 64 + cq * 16)
                                                : make_uint4(bones, bones, bones, bones);   // column 3: ones
                        const float2 xsv = *reinterpret_cast<const float2*>(rec + 192);
                        // one exponent for the group: the four unit MMAs chain
                        // into one exact int32 accumulator
                        constexpr uint32_t lo = 0x0F0F0F0Fu;
                        int dq[4] = {0, 0, 0, 0};
                        {
                            const uint32_t a0[2] = {wq.x & lo, wq.y & lo};
                            mma_u8u8_16816(dq, a0, bq.x);
                            const uint32_t a1[2] = {(wq.x >> 4) & lo, (wq.y >> 4) & lo};
                            mma_u8u8_16816(dq, a1, bq.y);
                            const uint32_t a2[2] = {wq.z & lo, wq.w & lo};
                            mma_u8u8_16816(dq, a2, bq.z);
                            const uint32_t a3[2] = {(wq.z >> 4) & lo, (wq.w >> 4) & lo};
                            mma_u8u8_16816(dq, a3, bq.w);
                        }
                        // columns 0, 1 (planes p0, p1) are in lane c = 0, column 2 (p2)
                        // in c = 1: each of the two lanes scales its own columns and
                        // keeps its own partial (added together once per B unit)
                        if (cq < 2) {
                            // lane 0: p0 + 256 p1; lane 1: 65536 (p2 - 32 * ones) - exact
                            const float xs = cq == 0 ? xsv.x : xsv.x * 65536.0f;
                            const float s0 = float(dq[0] + cmul * dq[1]) * xs;
                            const float s8 = float(dq[2] + cmul * dq[3]) * xs;
                            const float sh = cq == 0 ? xsv.y : 0.f;          // the sum term once
                            const uint8_t* sbp = sp + tg.bcodes;
                            if (FMT == kFmtAffine) {
                                const uint32_t* sbw = reinterpret_cast<const uint32_t*>(sbp) + ig * 16 + gr;
                                const uint32_t w0s = sbw[0], w8s = sbw[8];
                                y0 += fmaf(bf16_bits_to_f32(uint16_t(w0s)), s0, bf16_bits_to_f32(uint16_t(w0s >> 16)) * sh);
                                y8 += fmaf(bf16_bits_to_f32(uint16_t(w8s)), s8, bf16_bits_to_f32(uint16_t(w8s >> 16)) * sh);
                            } else {
                                const uint16_t* sbh = reinterpret_cast<const uint16_t*>(sbp) + ig * 16 + gr;
                                y0 += f16_bits_to_f32(sbh[0]) * (s0 - sh);
                                y8 += f16_bits_to_f32(sbh[8]) * (s8 - sh);
                            }
                        }
                        if (++ig == int(tg.Gd)) {
                            ig = 0;
                            ++iq;
                            if (++sidx == NB) sidx = 0;
                        }
                    }
                    if (tr_items) ltrace(A.trace, 21, lane == 0 && warp == 0);
                    __syncwarp();
                    if (lane == 0) {
                        int sb = stB;
                        #pragma unroll 1
                        for (int q = 0; q < W; ++q) {
                            mbar_arrive(emptyB + sb);
                            if (++sb == NB) sb = 0;
                        }
                    }
                    stB += W;                                         // W <= NB
                    if (stB >= NB) { stB -= NB; ++rB; }
                }
                y0 += __shfl_down_sync(0xffffffffu, y0, 1);         // + the p2 columns' partial
                y8 += __shfl_down_sync(0xffffffffu, y8, 1);
                if (cq == 0) {
                    red2[warp * 16 + gr] = y0;
                    red2[warp * 16 + gr + 8] = y8;
                }
                cons_sync();
                if (bu == b0) ltrace(A.trace, 15);
                if (tid < 16) {                                   // warp 0, lanes 0-15: row 16o + tid
                    float s = 0.f;
#pragma unroll
                    for (int w = 0; w < kLCons; ++w) s += red2[w * 16 + tid];
                    const size_t yi = size_t(t) * d + o * 16 + tid;
                    bool write = true;
                    if (epm && ep.rank > 0) {
                        __stcg(ep.part0 + size_t(ep.rank) * ep.part_stride + yi, s);
                        __threadfence_system();
                        __syncwarp(0xffffu);
                        if (tid == 0) atomicAdd_system(ep.cnt0 + bu, 1u);
                        write = false;
                    } else if (epm) {
                        if (tid == 0 && !spin_geq<true>(ep.cnt0 + bu, uint32_t(ep.world - 1), wb))
                            raise_err(A.err, SMOE_DEVERR_SPIN_TIMEOUT);
                        __syncwarp(0xffffu);
                        for (int r = 1; r < ep.world; ++r) s += __ldcv(ep.part0 + size_t(r) * ep.part_stride + yi);
                        __syncwarp(0xffffu);
                        if (tid == 0) ep.cnt0[bu] = 0u;           // ready for the next launch
                    }
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
        if (!mbar_wait_b(routed, 0, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
        int a0, a1;
        a_range(a0, a1);
        int hli = int(divu(uint32_t(a0), uint32_t(g.tilesU), g.mg_tilesU)), hu = a0 - hli * g.tilesU;
        #pragma unroll 1
        for (int a = a0; a < a1; ++a, ++hu) {
            if (hu == g.tilesU) { hu = 0; ++hli; }
            const int n = a - a0, b = n & 1;
            const uint32_t li = uint32_t(hli), u = uint32_t(hu);
            const uint32_t slot = slot_at(li);
            if (!mbar_wait_b(redF + b, (n >> 1) & 1, wb)) raise_err(A.err, SMOE_DEVERR_MBAR_TIMEOUT);
            const float* rb = red + b * kLCons * 32;
            float v = 0.f;                                        // lane = (matrix, row)
#pragma unroll
            for (int w = 0; w < kLCons; ++w) v += rb[w * 32 + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(redE + b);
            const float up = __shfl_down_sync(0xffffffffu, v, 16);
            if (lane < 16)                                        // kernels.metal:61-63
                reinterpret_cast<float*>(A.hbuf + (size_t(li) * g.tilesU + u) * kHRec)[lane] =
                    v * (1.0f / (1.0f + expf(-v))) * up * s_w[slot];
        }
        // phase A of this CTA is done: publish for phase B of all CTAs (the
        // warp barrier orders every lane's record stores before lane 0's
        // gpu-scope release)
        __syncwarp();
        if (lane == 0) red_rel_gpu(&A.st->arrive, 1u);
        ltrace(A.trace, 8, lane == 0);
    }

    // the next kernel in the stream may start its launch now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // ------------------------------------------------- last CTA: reset state
    __syncthreads();
    if (tid == 0) {
        uint32_t old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&A.st->done) : "memory");
        last_cta = (old == uint32_t(ncta) - 1) ? 1u : 0u;
        if (last_cta) {
            A.st->arrive = 0;
            A.st->done = 0;
            A.st->rdone = 0;
            A.st->seq = seq;
            if (epm) A.st->epoch = epoch;
        }
        // (no fence: the next launch reads these only after this grid has
        // completed - stream order or griddepcontrol.wait)
    }
    ltrace(A.trace, 9);
}

}  // namespace smoe
