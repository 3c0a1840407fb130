// sampler.cuh - token sampler of sampler.hpp:33-157 on sm_100a.
//
// One thread-block cluster of 8 CTAs x 1024 threads per row; each CTA keeps
// its eighth of the vocabulary in shared memory for all passes, and the
// cluster exchanges partial results through distributed shared memory:
//   1. repetition penalty over the last 256 history ids, each distinct
//      non-exempt id once, in place (sampler.hpp:42-70), written back;
//   2. greedy argmax when T < 1e-4, lowest index on ties (sampler.hpp:73-83);
//   3. max, then e = exp((s - max)/T) for every entry, bit-identical to the
//      reference's glibc expf (expf_ref below), and the reference's
//      sequential fp32 sum of all e reproduced exactly (seqsum.cuh)
//      (sampler.hpp:86-129);
//   4. top-K candidates by e via a 4 x 8-bit radix select (K = max(top_k,1)
//      <= 1024), ties at the threshold taken lowest index first;
//   5. CTA 0 sorts the K candidates (e desc, index asc) and walks the top-p /
//      top-k cutoff and the draw with the reference's float operations
//      (sampler.hpp:132-156).
// Bit-exactness: every e equals the reference's, the sum is its sequential
// fp32 sum, the cutoff and draw are its float operations; ties between equal
// e values are ordered by index here and unspecified in the reference's heap
// + sort.
#pragma once
#include <cooperative_groups.h>
#include "smoe_common.cuh"
#include "seqsum.cuh"

namespace smoe {
namespace cg = cooperative_groups;

struct SamplerRowDev {      // layout of SmoeSamplerRow
    float temperature, top_p;
    uint32_t top_k;
    float rep_penalty, u;
    uint32_t history_len;
};

struct SamplerArgs {
    float* logits;
    uint32_t V;
    const SamplerRowDev* rows;
    const uint32_t* hist;
    uint32_t hstride;
    uint32_t* tokens;
    unsigned long long* trace;   // optional [8 x 8] phase timestamps of row 0 (profiling aid)
};

SMOE_DEVINL void samp_mark(unsigned long long* tr, int i) {
    if (tr && threadIdx.x == 0 && blockIdx.y == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        tr[blockIdx.x * 8 + i] = t;
    }
}

// the same mark from a given thread (the workers' first thread)
SMOE_DEVINL void samp_mark_w(unsigned long long* tr, int i) {
    if (tr && blockIdx.y == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        tr[blockIdx.x * 8 + i] = t;
    }
}

constexpr int kSampCluster = 8;
constexpr int kSampThreads = 1024;
constexpr int kSampCand = 1024;

// e = exp(x) for the sampler exactly as the reference computes it.
// sampler.hpp:116 calls std::exp on a float, i.e. glibc's expf, whose x86-64
// build on CPUs with FMA (every host of a B200) is the table-driven method of
// Szabolcs Nagy (ARM optimized-routines, glibc >= 2.28, e_expf.c): with N = 32,
//   z = x N/ln2 = k + r, |r| <= 1/2 (k by adding and subtracting 1.5*2^52),
//   2^(k/N) = T[k mod N] with k/N added to its exponent field,
//   2^(r/N) ~ 1 + C2 r + C1 r^2 + C0 r^3 (C = the published degree-3 exp2
//   coefficients scaled by 1/N, 1/N^2, 1/N^3),
// all in double with the FMA build's fused multiply-adds, rounded to float
// once. T[i] holds the bits of 2^(i/N) (correctly rounded; computed from the
// definition) minus i << 47. Every step is an IEEE-exact double operation, so
// the result equals the CPU's bit for bit: the restatement in
// oracle/smoe_oracle.c (or_expf_ref) reproduces glibc 2.39's expf on every
// float in [-104, 88] (tests/test_oracle.py), and the GPU sampler tests
// compare with the compiled reference.
__device__ __align__(256) const uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

SMOE_DEVINL float expf_ref(float x) {
    if (x < -0x1.9fe368p6f) return 0.0f;                 // below: the reference underflows to +0
    constexpr double N = 32.0;
    constexpr double C0 = 0x1.c6af84b912394p-5 / N / N / N, C1 = 0x1.ebfce50fac4f3p-3 / N / N,
                     C2 = 0x1.62e42ff0c52d6p-1 / N;
    constexpr double InvLn2N = 0x1.71547652b82fep+0 * N, Shift = 0x1.8p+52;
    const double xd = (double)x;
    const double kd0 = __fma_rn(InvLn2N, xd, Shift);
    const uint64_t ki = (uint64_t)__double_as_longlong(kd0);
    const double kd = __dsub_rn(kd0, Shift);
    const double r = __fma_rn(InvLn2N, xd, -kd);
    const uint64_t t = __ldg(&kExp2Tab[ki & 31u]) + (ki << 47);
    const double sc = __longlong_as_double((long long)t);
    const double zc = __fma_rn(C0, r, C1);
    const double r2 = __dmul_rn(r, r);
    double y = __fma_rn(C2, r, 1.0);
    y = __fma_rn(zc, r2, y);
    y = __dmul_rn(y, sc);
    return __double2float_rn(y);
}

SMOE_DEVINL uint32_t score_key(float s) {
    uint32_t u = __float_as_uint(s);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0u;        // NaN: never a candidate
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
SMOE_DEVINL float key_score(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <typename T, typename Op>
SMOE_DEVINL T block_reduce(T v, T* red, Op op) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    v = red[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) v = op(v, red[i]);
    return v;
}

// exclusive block scan of a u32 (1024 threads)
SMOE_DEVINL uint32_t block_exscan(uint32_t v, uint32_t* red, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    __syncthreads();
    if (lane == 31) red[warp] = inc;
    __syncthreads();
    uint32_t base = 0, tot = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
        if (i < warp) base += red[i];
        tot += red[i];
    }
    *total = tot;
    return base + inc - v;
}

// ---- worker synchronisation while warp 0 of CTA 0 walks the exact sum:
// the other warps of CTA 0 and every warp of the other CTAs ("workers")
// synchronise among themselves only.
// Within a CTA: named barrier 1 over its workers (992 or 1024 threads).
SMOE_DEVINL void worker_bar(int nwork) {
    asm volatile("bar.sync 1, %0;" :: "r"(nwork) : "memory");
}
// Across the cluster: every CTA's worker 0 arrives (release, cluster scope)
// on the same mbarrier of all 8 CTAs, then every worker waits (acquire) for
// its own CTA's barrier to complete the phase (8 arrivals). Two barriers
// used alternately: a CTA can only arrive for sync k + 1 after every CTA
// has arrived for sync k, so an arrival never lands in an older phase. The
// wait is bounded (a %globaltimer deadline); running out lets the kernel
// finish with a wrong token instead of hanging.
struct WorkerClusterSync {
    uint64_t* bars;            // [2] mbarriers in this CTA's shared memory, count kSampCluster
    uint32_t par[2];
    int use;
    SMOE_DEVINL void sync(int wtid, int nwork) {
        asm volatile("fence.acq_rel.cluster;" ::: "memory");
        worker_bar(nwork);                                   // this CTA's workers are done writing
        uint64_t* b = bars + use;
        if (wtid == 0) {
            const uint32_t a = smem_u32(b);
#pragma unroll 1
            for (uint32_t r = 0; r < uint32_t(kSampCluster); ++r)
                asm volatile("{ .reg .b32 ra; mapa.shared::cluster.u32 ra, %0, %1;\n"
                             " mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra]; }"
                             :: "r"(a), "r"(r) : "memory");
        }
        const uint64_t deadline = gtimer() + SMOE_WAIT_NS_DEFAULT;
#pragma unroll 1
        for (uint32_t i = 0;; ++i) {
            uint32_t ok;
            asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
                         " selp.u32 %0, 1, 0, p; }"
                         : "=r"(ok) : "r"(smem_u32(b)), "r"(par[use]) : "memory");
            if (ok || ((i & 15) == 15 && gtimer() > deadline)) break;
        }
        par[use] ^= 1u;
        use ^= 1;
    }
};

// exclusive scan of a u32 over the workers of this CTA (nwork threads, worker
// index wtid); *total = the sum over them
SMOE_DEVINL uint32_t worker_exscan(uint32_t v, uint32_t* red, uint32_t* total, int wtid, int nwork) {
    const int lane = wtid & 31, ww = wtid >> 5, nww = nwork >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    worker_bar(nwork);
    if (lane == 31) red[ww] = inc;
    worker_bar(nwork);
    uint32_t base = 0, tot = 0;
    for (int i = 0; i < nww; ++i) {
        if (i < ww) base += red[i];
        tot += red[i];
    }
    *total = tot;
    return base + inc - v;
}

struct SampPub {            // per-CTA values read by the cluster
    float fval;
    uint32_t uidx;
    double dsum;
    uint32_t n_gt, n_eq;
};

__global__ void __cluster_dims__(kSampCluster, 1, 1) __launch_bounds__(kSampThreads, 1)
k_sample(SamplerArgs a) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    __shared__ uint32_t hist[2][256];
    __shared__ uint32_t tot[256];
    __shared__ unsigned long long cand[kSampCand];
    __shared__ float probs[kSampCand];
    __shared__ float redf[32];
    __shared__ uint32_t redu[32];
    __shared__ SampPub pub;
    __shared__ SeqShared seqsh;
    __shared__ uint32_t sel_prefix, sel_krem;
    __shared__ uint64_t wbars[2];

    cg::cluster_group cl = cg::this_cluster();
    const int rank = (int)cl.block_rank();
    const int tid = threadIdx.x;
    const uint32_t row = blockIdx.y;
    const SamplerRowDev P = a.rows[row];
    const uint32_t V = a.V;
    const uint32_t L = (((V + kSampCluster - 1) / kSampCluster) + 3u) & ~3u;
    const uint32_t lo = min(V, rank * L);
    const uint32_t n = min(V - lo, L);
    float* s = reinterpret_cast<float*>(smem_raw);
    // per-warp radix histograms [32][256] after the slice
    uint32_t (*whist)[256] = reinterpret_cast<uint32_t (*)[256]>(smem_raw + size_t(L) * 4);
    float* lg = a.logits + size_t(row) * V;

    samp_mark(a.trace, 0);
    if (tid == 0) {
        mbar_init(&wbars[0], kSampCluster);
        mbar_init(&wbars[1], kSampCluster);
        fence_mbar_init();             // visible cluster-wide by the first cluster barrier below
    }
    for (uint32_t i = tid; i < n; i += kSampThreads) s[i] = lg[lo + i];
    __syncthreads();
    samp_mark(a.trace, 1);

    // ---- 1. repetition penalty (sampler.hpp:42-70)
    if (P.rep_penalty != 1.0f) {
        const uint32_t hl = P.history_len;
        const uint32_t start = hl > 256u ? hl - 256u : 0u;
        const uint32_t* h = a.hist + size_t(row) * a.hstride;
        const uint32_t i = start + tid;
        if (tid < 256 && i < hl) {
            const uint32_t t = h[i];
            bool skip = (t == 13 || t == 11 || t == 198 || t == 271 || t == 30 || t == 0 ||
                         t == 151643 || t == 151645);
            for (uint32_t j = start; j < i && !skip; ++j)
                if (h[j] == t) skip = true;
            if (!skip && t >= lo && t < lo + n) {
                float v = s[t - lo];
                v = (v <= 0.0f) ? __fmul_rn(v, P.rep_penalty) : __fdiv_rn(v, P.rep_penalty);
                s[t - lo] = v;
                lg[t] = v;
            }
        }
        __syncthreads();
    }

    // ---- 2. greedy (sampler.hpp:73-83)
    if (P.temperature < 1e-4f) {
        float best = -1e38f;
        uint32_t bi = 0xffffffffu;
        for (uint32_t i = tid; i < n; i += kSampThreads)
            if (s[i] > best) { best = s[i]; bi = lo + i; }
        // (value, index): larger value, then smaller index
        const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (lane == 0) { redf[warp] = best; redu[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < 32; ++w)
                if (redf[w] > best || (redf[w] == best && redu[w] < bi)) { best = redf[w]; bi = redu[w]; }
            pub.fval = best;
            pub.uidx = bi;
        }
        cl.sync();
        if (rank == 0 && tid == 0) {
            for (int r = 1; r < kSampCluster; ++r) {
                const SampPub* o = cl.map_shared_rank(&pub, r);
                if (o->fval > best || (o->fval == best && o->uidx < bi)) { best = o->fval; bi = o->uidx; }
            }
            a.tokens[row] = (bi == 0xffffffffu) ? 0u : bi;
        }
        cl.sync();
        return;
    }

    // ---- 3. max and softmax denominator
    float mx = -INFINITY;
    for (uint32_t i = tid; i < n; i += kSampThreads) mx = fmaxf(mx, s[i]);
    mx = block_reduce(mx, redf, [](float x, float y) { return fmaxf(x, y); });
    if (tid == 0) pub.fval = mx;
    cl.sync();
    mx = -INFINITY;
    for (int r = 0; r < kSampCluster; ++r) mx = fmaxf(mx, cl.map_shared_rank(&pub, r)->fval);
    {   // the reference's max starts from scores[0]: a NaN there poisons it
        const float s0 = *cl.map_shared_rank(s, 0);
        if (s0 != s0) mx = s0;
    }
    cl.sync();     // every CTA has read rank 0's s[0] before any e overwrites it
    const float T = P.temperature;
    // e_v = exp((s_v - max) / T) as the reference's expf computes it, in place of s; then the
    // reference's sequential fp32 sum of all e_v, reproduced exactly
    const uint32_t C = (L + kSampThreads - 1) / kSampThreads;
    {
        const uint32_t c0 = min(n, tid * C), cnt = min(n, c0 + C) - c0;
        float v[kSeqMaxC];                       // independent evaluations, unrolled for ILP
#pragma unroll
        for (int q = 0; q < kSeqMaxC; ++q)
            if (q < (int)cnt) v[q] = expf_ref(__fdiv_rn(__fsub_rn(s[c0 + q], mx), T));
#pragma unroll
        for (int q = 0; q < kSeqMaxC; ++q)
            if (q < (int)cnt) s[c0 + q] = v[q];
    }
    __syncthreads();
    samp_mark(a.trace, 2);
    seq_summarise_cluster(cl, s, n, L, V, C, &seqsh, a.trace);

    // From here warp 0 of CTA 0 walks the exact sum (43 us of serial work)
    // while the other warps - the workers - select, collect and sort the
    // top-K candidates; they meet again at the cluster barrier before the
    // draw. The walker reads every CTA's e values and summaries remotely, so
    // every CTA stays resident until that barrier.
    uint32_t K = P.top_k < 1u ? 1u : P.top_k;
    if (K > (uint32_t)kSampCand) K = kSampCand;
    if (K > V) K = V;
    if (rank == 0 && (tid >> 5) == 0) {
        seq_walk(cl, s, L, V, C, &seqsh, a.trace);
    } else {
        const int wtid = rank == 0 ? tid - 32 : tid, nwork = rank == 0 ? kSampThreads - 32 : kSampThreads;
        const int w0 = rank == 0 ? 1 : 0;                 // first worker warp of this CTA
        WorkerClusterSync csync{wbars, {0u, 0u}, 0};
        // ---- 4. radix select of the K-th largest score key
        uint32_t prefix = 0, mask = 0, krem = K;
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            uint32_t* hh = hist[pass & 1];
            uint32_t* wh = whist[tid >> 5];
            for (int b = tid & 31; b < 256; b += 32) wh[b] = 0;
            __syncwarp();
            for (uint32_t i = wtid; i < n; i += nwork) {
                const uint32_t key = score_key(s[i]);
                if ((key & mask) == prefix) atomicAdd(&wh[(key >> shift) & 255u], 1u);
            }
            worker_bar(nwork);
            if (wtid < 256) {
                uint32_t t = 0;
                for (int w = w0; w < kSampThreads / 32; ++w) t += whist[w][wtid];
                hh[wtid] = t;
            }
            csync.sync(wtid, nwork);
            if (wtid < 256) {
                uint32_t t = 0;
                for (int r = 0; r < kSampCluster; ++r) t += cl.map_shared_rank(hh, r)[wtid];
                tot[wtid] = t;
            }
            worker_bar(nwork);
            if (wtid < 32) {
                // the highest bin b >= 1 whose count from bin 255 down reaches krem,
                // else bin 0; cum = count above b. Lane l scans bins 255 - 8l ..
                // 248 - 8l; the lane holding the answer walks its 8 bins.
                const int lane = wtid;
                uint32_t v[8], sl = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    v[q] = tot[255 - 8 * lane - q];
                    sl += v[q];
                }
                uint32_t incl = sl;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                const unsigned m = __ballot_sync(0xffffffffu, incl >= krem);
                const int owner = m ? __ffs(m) - 1 : 31;
                if (lane == owner) {
                    uint32_t cum = incl - sl;
                    int b = 0;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const int bin = 255 - 8 * lane - q;
                        if (bin == 0) break;
                        if (cum + v[q] >= krem) { b = bin; break; }
                        cum += v[q];
                    }
                    sel_krem = krem - cum;
                    sel_prefix = prefix | (uint32_t(b) << shift);
                }
            }
            worker_bar(nwork);
            krem = sel_krem;
            prefix = sel_prefix;
            mask |= 255u << shift;
            // (hist[pass & 1] is next written two passes later, after a
            // cluster barrier that follows every CTA's reads of it)
        }
        const uint32_t thr = prefix;   // key of the K-th largest; krem ties to take
        if (wtid == 0) samp_mark_w(a.trace, 4);

        // ---- collect candidates into CTA 0 (contiguous chunk per worker keeps
        // the tie order = index order)
        const uint32_t chunk = (n + nwork - 1) / nwork;
        const uint32_t b0 = min(n, wtid * chunk), b1 = min(n, b0 + chunk);
        uint32_t ngt = 0, neq = 0;
        for (uint32_t i = b0; i < b1; ++i) {
            const uint32_t key = score_key(s[i]);
            ngt += key > thr;
            neq += key == thr;
        }
        // one scan of both counts, packed (each CTA total < 2^16: its slice
        // holds at most 24,576 entries: vocab <= 8 x 1024 x kSeqMaxC)
        uint32_t cta_both;
        const uint32_t off_both = worker_exscan((ngt << 16) | neq, redu, &cta_both, wtid, nwork);
        const uint32_t off_gt = off_both >> 16, off_eq = off_both & 0xffffu;
        const uint32_t cta_gt = cta_both >> 16, cta_eq = cta_both & 0xffffu;
        if (wtid == 0) { pub.n_gt = cta_gt; pub.n_eq = cta_eq; }
        csync.sync(wtid, nwork);
        uint32_t all_gt = 0, gt_before = 0, eq_before = 0;
        for (int r = 0; r < kSampCluster; ++r) {
            const SampPub* o = cl.map_shared_rank(&pub, r);
            all_gt += o->n_gt;
            if (r < rank) { gt_before += o->n_gt; eq_before += o->n_eq; }
        }
        unsigned long long* cand0 = cl.map_shared_rank(cand, 0);
        {
            uint32_t pg = gt_before + off_gt, pe = eq_before + off_eq;
            for (uint32_t i = b0; i < b1; ++i) {
                const uint32_t key = score_key(s[i]);
                const unsigned long long packed =
                    (static_cast<unsigned long long>(key) << 32) | (~(lo + i) & 0xffffffffu);
                if (key > thr) cand0[pg++] = packed;
                else if (key == thr) {
                    if (pe < krem) cand0[all_gt + pe] = packed;
                    ++pe;
                }
            }
        }
        csync.sync(wtid, nwork);
        if (wtid == 0) samp_mark_w(a.trace, 5);

        // ---- 5. sort (score desc, index asc), CTA 0's workers
        if (rank == 0) {
            uint32_t N2 = 1;
            while (N2 < K) N2 <<= 1;
            for (uint32_t i = K + wtid; i < N2; i += nwork) cand[i] = 0ull;
            worker_bar(nwork);
            for (uint32_t size = 2; size <= N2; size <<= 1) {
                for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                    for (uint32_t i = wtid; i < N2; i += nwork) {
                        const uint32_t j = i ^ stride;
                        if (j > i) {
                            const bool desc = (i & size) == 0;
                            const unsigned long long x = cand[i], y = cand[j];
                            if (desc ? (x < y) : (x > y)) { cand[i] = y; cand[j] = x; }
                        }
                    }
                    worker_bar(nwork);
                }
            }
            if (wtid == 0) samp_mark_w(a.trace, 6);
        }
    }
    cl.sync();                    // the walk is done and the candidates are sorted
    if (rank != 0) return;        // no CTA's shared memory is read remotely any more
    const float inv_sum = __fdiv_rn(1.0f, seqsh.result);
    for (uint32_t i = tid; i < K; i += kSampThreads) {
        const float e = key_score(uint32_t(cand[i] >> 32));    // keys are the e values
        probs[i] = __fmul_rn(e, inv_sum);
    }
    __syncthreads();
    if (tid == 0) {
        float cum = 0.0f;
        uint32_t tl = 0;
        for (uint32_t i = 0; i < K; ++i) {
            cum = __fadd_rn(cum, probs[i]);
            ++tl;
            if (cum >= P.top_p || tl >= P.top_k) break;
        }
        const float rv = __fmul_rn(P.u, cum);
        float run = 0.0f;
        uint32_t tok = ~uint32_t(cand[tl - 1] & 0xffffffffu);
        for (uint32_t i = 0; i < tl; ++i) {
            run = __fadd_rn(run, probs[i]);
            if (rv <= run) { tok = ~uint32_t(cand[i] & 0xffffffffu); break; }
        }
        a.tokens[row] = tok;
    }
    samp_mark(a.trace, 7);
}

inline size_t sampler_smem_bytes(uint32_t V) {
    const uint32_t L = (((V + kSampCluster - 1) / kSampCluster) + 3u) & ~3u;
    return size_t(L) * 4 + size_t(kSampThreads / 32) * 256 * 4;
}

}  // namespace smoe
