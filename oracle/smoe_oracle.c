/*
 * smoe_oracle.c - TEST INFRASTRUCTURE ONLY.
 *
 * Plain-C CPU restatement of the S-MoE decode hot path. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline legs may load it; the
 * product library (libsmoe_cuda.so) never links or calls it.
 *
 * What it restates (file:line in the reference project):
 *   - bf16 -> f32                 common.hpp:237-242
 *   - scalar gate matvec          common.hpp:294-306 (sequential fp32 sum)
 *   - softmax + top-k + renorm    scout/scout.cpp:77-123, decode.cpp:280-303
 *   - SMOE-Q4 dequant             compute/kernels.metal:90-105,
 *                                 scripts/shatter_moe.py:371-387
 *                                 (w = (q - 7.5) / 7.5 * s, s fp16, group 64,
 *                                  two codes per byte, LSB first)
 *   - AFFINE-Q4 (benchmark format) w = scale * q + bias, scale/bias bf16
 *   - gate/up/SiLU/down           compute/kernels.metal:61-63, 240-365
 *   - expert blob layout          scripts/shatter_moe.py:627-674
 *   - weighted combine            decode.cpp:481-509 (axpy in rank order)
 *   - token sampler               sampler.hpp:33-157
 *   - the sampler's expf          glibc e_expf.c (FMA build), called by
 *                                 sampler.hpp:116 through std::exp(float)
 *
 * The sampler restatement is pinned against the reference's own compiled
 * sampler.hpp (oracle/_ref/libsmoe_ref.so) in tests/test_oracle.py; the Q4
 * format is pinned against shatter_moe.py's quantiser via committed golden
 * fixtures (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define FMT_SMOE_Q4   0
#define FMT_AFFINE_Q4 1
#define GROUP 64

/* ---------------------------------------------------------------- numbers */

float or_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t or_f32_to_bf16(float f) {           /* round to nearest even */
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    uint32_t r = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + r) >> 16);
}

float or_f16_to_f32(uint16_t h) {
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t u;
    if (e == 0) {
        if (m == 0) u = s;
        else {                                   /* subnormal */
            float f = ldexpf((float)m, -24);
            memcpy(&u, &f, 4);
            u |= s;
        }
    } else if (e == 31) u = s | 0x7f800000u | (m << 13);
    else u = s | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t or_f32_to_f16(float f) {            /* round to nearest even */
    uint32_t u;
    memcpy(&u, &f, 4);
    uint32_t s = (u >> 16) & 0x8000u;
    int32_t e = (int32_t)((u >> 23) & 0xff) - 127 + 15;
    uint32_t m = u & 0x7fffffu;
    if (((u >> 23) & 0xff) == 0xff) return (uint16_t)(s | 0x7c00u | (m ? 0x200u : 0));
    if (e >= 31) return (uint16_t)(s | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)s;
        m |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t hm = m >> shift, rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1))) hm++;
        return (uint16_t)(s | hm);
    }
    uint32_t hm = m >> 13, rem = m & 0x1fffu;
    uint32_t out = s | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1))) out++;
    return (uint16_t)out;
}

/* --------------------------------------------------- seeded synthetic data
 * Counter-based: element i of stream `stream` under `seed` is a pure
 * function of (seed, stream, i), so any slice can be regenerated anywhere. */

static inline uint64_t mix64(uint64_t z) {     /* splitmix64 finaliser */
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
static inline uint64_t ctr(uint64_t seed, uint64_t stream, uint64_t i) {
    return mix64(mix64(seed * 0x100000001b3ull ^ stream) + i);
}
static inline double u01(uint64_t r) {         /* (0,1), 53 bits */
    return ((double)(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}
static inline double normal_at(uint64_t seed, uint64_t stream, uint64_t i) {
    /* Box-Muller on two counter draws; one normal per index */
    double a = u01(ctr(seed, stream, 2 * i)), b = u01(ctr(seed, stream, 2 * i + 1));
    return sqrt(-2.0 * log(a)) * cos(6.283185307179586 * b);
}

void or_gen_normal_f32(uint64_t seed, uint64_t stream, uint64_t n, float mean, float std, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = (float)(mean + std * normal_at(seed, stream, i));
}
void or_gen_normal_bf16(uint64_t seed, uint64_t stream, uint64_t n, float mean, float std, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = or_f32_to_bf16((float)(mean + std * normal_at(seed, stream, i)));
}
void or_gen_uniform_bf16(uint64_t seed, uint64_t stream, uint64_t n, float lo, float hi, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = or_f32_to_bf16((float)(lo + (hi - lo) * u01(ctr(seed, stream, i))));
}
void or_gen_uniform_f16(uint64_t seed, uint64_t stream, uint64_t n, float lo, float hi, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = or_f32_to_f16((float)(lo + (hi - lo) * u01(ctr(seed, stream, i))));
}
/* uniform bytes: two uniform 4-bit codes per byte */
void or_gen_bytes(uint64_t seed, uint64_t stream, uint64_t n, uint8_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)(n / 8); ++i) {
        uint64_t r = ctr(seed, stream, i);
        memcpy(out + 8 * i, &r, 8);
    }
    for (uint64_t i = n & ~7ull; i < n; ++i) out[i] = (uint8_t)ctr(seed, stream, i);
}
/* uniform integers in [0, m) */
void or_gen_ids(uint64_t seed, uint64_t stream, uint64_t n, uint32_t m, uint32_t* out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = (uint32_t)(u01(ctr(seed, stream, i)) * m);
}

/* ------------------------------------------------------------ blob layout
 * One expert = three matrices gate [dff x d], up [dff x d], down [d x dff];
 * per matrix: nibbles (rows*cols/2 B, row-major, K-contiguous, LSB first),
 * then scales (rows*cols/64 x 2 B), then - AFFINE only - biases (same size).
 * No internal padding (shatter_moe.py:627-674 for the SMOE-Q4 case). */
void or_blob_layout(int fmt, uint32_t d, uint32_t dff, uint64_t off[9], uint64_t* total) {
    uint64_t rows[3] = {dff, dff, d}, cols[3] = {d, d, dff}, cur = 0;
    for (int m = 0; m < 3; ++m) {
        uint64_t nib = rows[m] * cols[m] / 2, sc = rows[m] * cols[m] / GROUP * 2;
        off[3 * m + 0] = cur; cur += nib;
        off[3 * m + 1] = cur; cur += sc;
        off[3 * m + 2] = cur; if (fmt == FMT_AFFINE_Q4) cur += sc;
    }
    *total = cur;
}

/* weight (r, c) of one quantised matrix */
static inline double deq(int fmt, const uint8_t* nib, const uint16_t* sc, const uint16_t* bi,
                         uint32_t cols, uint32_t r, uint32_t c) {
    uint64_t wi = (uint64_t)r * cols + c;
    uint32_t q = (nib[wi >> 1] >> ((wi & 1) * 4)) & 0xf;
    uint64_t g = wi / GROUP;
    if (fmt == FMT_SMOE_Q4) return ((double)q - 7.5) * (1.0 / 7.5) * (double)or_f16_to_f32(sc[g]);
    return (double)or_bf16_to_f32(sc[g]) * (double)q + (double)or_bf16_to_f32(bi[g]);
}

/* Dense dequantised copy (fp32) of one matrix, in the float operations of
 * shatter_moe.py:371-387 ((q - 7.5) / 7.5 * s, all float32). */
void or_dequant(int fmt, const uint8_t* nib, const uint16_t* sc, const uint16_t* bi,
                uint32_t rows, uint32_t cols, float* out) {
    for (uint64_t wi = 0; wi < (uint64_t)rows * cols; ++wi) {
        float q = (float)((nib[wi >> 1] >> ((wi & 1) * 4)) & 0xf);
        uint64_t g = wi / GROUP;
        if (fmt == FMT_SMOE_Q4) out[wi] = ((q - 7.5f) / 7.5f) * or_f16_to_f32(sc[g]);
        else out[wi] = or_bf16_to_f32(sc[g]) * q + or_bf16_to_f32(bi[g]);
    }
}

/* One row . x in fp32, with the per-group epilogue of kernels.metal:140-143,
 * 200 (Sum q.x and Sum x per group, scale applied once per group). */
static float row_dot_f32(int fmt, const uint8_t* nib, const uint16_t* sc, const uint16_t* bi,
                         uint32_t cols, uint32_t r, const float* x) {
    float acc = 0.0f;
    const uint8_t* rp = nib + (uint64_t)r * cols / 2;
    for (uint32_t g0 = 0; g0 < cols; g0 += GROUP) {
        float a = 0.0f, xs = 0.0f;
        for (uint32_t c = g0; c < g0 + GROUP; ++c) {
            uint32_t q = (rp[c >> 1] >> ((c & 1) * 4)) & 0xf;
            a += (float)q * x[c];
            xs += x[c];
        }
        uint64_t g = ((uint64_t)r * cols + g0) / GROUP;
        if (fmt == FMT_SMOE_Q4) acc += or_f16_to_f32(sc[g]) * (a * (1.0f / 7.5f) - xs);
        else acc += or_bf16_to_f32(sc[g]) * a + or_bf16_to_f32(bi[g]) * xs;
    }
    return acc;
}
static double row_dot_f64(int fmt, const uint8_t* nib, const uint16_t* sc, const uint16_t* bi,
                          uint32_t cols, uint32_t r, const double* x) {
    double acc = 0.0;
    for (uint32_t c = 0; c < cols; ++c) acc += deq(fmt, nib, sc, bi, cols, r, c) * x[c];
    return acc;
}

/* kernels.metal:61-63 */
static inline float silu_f(float v) { return v * (1.0f / (1.0f + expf(-v))); }
static inline double silu_d(double v) { return v / (1.0 + exp(-v)); }

/*
 * One expert FFN: y = W_down . (silu(W_gate . x) * (W_up . x)).
 * blob: the expert's bytes in the layout of or_blob_layout.
 * precise != 0: fp64 accumulation everywhere (error analysis).
 * hidden_out (optional, d_ff floats): the SwiGLU hidden vector.
 */
void or_expert_ffn(int fmt, const uint8_t* blob, uint32_t d, uint32_t dff,
                   const float* x, float* y, int precise, float* hidden_out) {
    uint64_t off[9], tot;
    or_blob_layout(fmt, d, dff, off, &tot);
#define NIB(m) (blob + off[3 * (m)])
#define SC(m) ((const uint16_t*)(blob + off[3 * (m) + 1]))
#define BI(m) ((const uint16_t*)(blob + off[3 * (m) + 2]))
    if (precise) {
        double* xd = (double*)malloc(sizeof(double) * (d > dff ? d : dff));
        double* hd = (double*)malloc(sizeof(double) * dff);
        for (uint32_t i = 0; i < d; ++i) xd[i] = x[i];
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < dff; ++r) {
            double g = row_dot_f64(fmt, NIB(0), SC(0), BI(0), d, (uint32_t)r, xd);
            double u = row_dot_f64(fmt, NIB(1), SC(1), BI(1), d, (uint32_t)r, xd);
            hd[r] = silu_d(g) * u;
        }
        if (hidden_out) for (uint32_t r = 0; r < dff; ++r) hidden_out[r] = (float)hd[r];
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < d; ++r) y[r] = (float)row_dot_f64(fmt, NIB(2), SC(2), BI(2), dff, (uint32_t)r, hd);
        free(xd);
        free(hd);
        return;
    }
    float* h = (float*)malloc(sizeof(float) * dff);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < dff; ++r) {
        float g = row_dot_f32(fmt, NIB(0), SC(0), BI(0), d, (uint32_t)r, x);
        float u = row_dot_f32(fmt, NIB(1), SC(1), BI(1), d, (uint32_t)r, x);
        h[r] = silu_f(g) * u;
    }
    if (hidden_out) memcpy(hidden_out, h, sizeof(float) * dff);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < d; ++r) y[r] = row_dot_f32(fmt, NIB(2), SC(2), BI(2), dff, (uint32_t)r, h);
    free(h);
#undef NIB
#undef SC
#undef BI
}

/* --------------------------------------------------------------- router */

/* common.hpp:294-306: sequential fp32 sum of bf16(W[e,j]) * x[j] */
void or_matvec_bf16(float* out, const uint16_t* w, const float* x, uint32_t rows, uint32_t cols) {
    for (uint32_t i = 0; i < rows; ++i) {
        float s = 0.0f;
        const uint16_t* wr = w + (uint64_t)i * cols;
        for (uint32_t j = 0; j < cols; ++j) s += or_bf16_to_f32(wr[j]) * x[j];
        out[i] = s;
    }
}

/* scout.cpp:77-123 with norm=false, then decode.cpp:296-303 renorm */
uint32_t or_topk_renorm(const float* logits, uint32_t n, uint32_t k, int norm,
                        uint32_t* ids, float* w) {
    float* p = (float*)malloc(sizeof(float) * n);
    uint32_t* idx = (uint32_t*)malloc(sizeof(uint32_t) * n);
    uint32_t cnt = k < n ? k : n;
    float mx = logits[0];
    for (uint32_t i = 1; i < n; ++i) if (logits[i] > mx) mx = logits[i];
    float se = 0.0f;
    for (uint32_t i = 0; i < n; ++i) { p[i] = expf(logits[i] - mx); idx[i] = i; se += p[i]; }
    float inv = se > 0.0f ? 1.0f / se : 0.0f;
    for (uint32_t i = 0; i < n; ++i) p[i] *= inv;
    for (uint32_t s = 0; s < cnt; ++s) {
        uint32_t b = s;
        for (uint32_t i = s + 1; i < n; ++i) if (p[i] > p[b]) b = i;
        float tf = p[s]; p[s] = p[b]; p[b] = tf;
        uint32_t ti = idx[s]; idx[s] = idx[b]; idx[b] = ti;
        ids[s] = idx[s];
        w[s] = p[s];
    }
    float ws = 0.0f;
    for (uint32_t s = 0; s < cnt; ++s) ws += w[s];
    float wi = (norm && ws > 0.0f) ? 1.0f / ws : 1.0f;
    for (uint32_t s = 0; s < cnt; ++s) w[s] = w[s] * wi;
    free(p);
    free(idx);
    return cnt;
}

uint32_t or_route(const float* x, const uint16_t* gate_w, uint32_t n_experts, uint32_t d,
                  uint32_t k, int norm, float* logits, uint32_t* ids, float* w) {
    or_matvec_bf16(logits, gate_w, x, n_experts, d);
    return or_topk_renorm(logits, n_experts, k, norm, ids, w);
}

/*
 * Whole MoE layer for one token: route, run the k chosen experts, combine
 * routed[i] += w_e * y_e[i] in rank order (decode.cpp:485-499, axpy_f32).
 * experts: base of the layer arena, expert e at experts + e * blob_stride.
 * ids/wts (optional, k each) receive the routing.
 */
void or_moe_layer(int fmt, const float* x, const uint16_t* gate_w, uint32_t n_experts,
                  uint32_t d, uint32_t dff, uint32_t k, int norm,
                  const uint8_t* experts, uint64_t blob_stride, int precise,
                  float* routed, uint32_t* ids_out, float* w_out) {
    float* logits = (float*)malloc(sizeof(float) * n_experts);
    uint32_t ids[64];
    float w[64];
    uint32_t nk = or_route(x, gate_w, n_experts, d, k, norm, logits, ids, w);
    float* ye = (float*)malloc(sizeof(float) * d);
    for (uint32_t i = 0; i < d; ++i) routed[i] = 0.0f;
    for (uint32_t e = 0; e < nk; ++e) {
        or_expert_ffn(fmt, experts + (uint64_t)ids[e] * blob_stride, d, dff, x, ye, precise, NULL);
        for (uint32_t i = 0; i < d; ++i) routed[i] += w[e] * ye[i];
    }
    if (ids_out) memcpy(ids_out, ids, nk * sizeof(uint32_t));
    if (w_out) memcpy(w_out, w, nk * sizeof(float));
    free(ye);
    free(logits);
}

int or_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* -------------------------------------------------------------- sampler
 * sampler.hpp:33-157. `u` is the value generate_canonical<float,24> would
 * return for the engine's draw; scratch_k the heap size (0 -> max(top_k,1024)
 * as main.cpp:324). Heap + sort restated with the same comparisons; among
 * exactly equal probabilities the order may differ from libstdc++'s sort. */
typedef struct { float p; uint32_t v; } ProbTok;

static void sift_down(ProbTok* h, uint32_t i, uint32_t n) {
    for (;;) {
        uint32_t l = 2 * i + 1;
        if (l >= n) break;
        uint32_t m = (h[l].p < h[i].p) ? l : i;
        uint32_t r = l + 1;
        if (r < n && h[r].p < h[m].p) m = r;
        if (m == i) break;
        ProbTok t = h[i]; h[i] = h[m]; h[m] = t;
        i = m;
    }
}
static int cmp_desc(const void* a, const void* b) {
    const ProbTok* x = (const ProbTok*)a;
    const ProbTok* y = (const ProbTok*)b;
    if (x->p > y->p) return -1;
    if (x->p < y->p) return 1;
    return (x->v < y->v) ? -1 : (x->v > y->v);
}

uint32_t or_sample_token(float* scores, uint32_t V, float T, float top_p, uint32_t top_k,
                         float rep, const uint32_t* hist, uint32_t hist_len, float u,
                         uint32_t scratch_k) {
    if (rep != 1.0f) {
        uint32_t start = hist_len > 256 ? hist_len - 256 : 0;
        for (uint32_t i = start; i < hist_len; ++i) {
            uint32_t t = hist[i];
            if (t == 13 || t == 11 || t == 198 || t == 271 || t == 30 || t == 0 ||
                t == 151643 || t == 151645) continue;
            int seen = 0;
            for (uint32_t j = start; j < i; ++j) if (hist[j] == t) { seen = 1; break; }
            if (seen) continue;
            if (scores[t] <= 0) scores[t] *= rep;
            else scores[t] /= rep;
        }
    }
    if (T < 1e-4f) {
        float best = -1e38f;
        uint32_t bt = 0;
        for (uint32_t v = 0; v < V; ++v) if (scores[v] > best) { best = scores[v]; bt = v; }
        return bt;
    }
    float mx = scores[0];
    for (uint32_t v = 1; v < V; ++v) if (scores[v] > mx) mx = scores[v];
    if (scratch_k == 0) scratch_k = top_k > 1024 ? top_k : 1024;
    uint32_t K = scratch_k < 1 ? 1 : scratch_k;
    if (K > V) K = V;
    ProbTok* h = (ProbTok*)malloc(sizeof(ProbTok) * K);
    float se = 0.0f;
    uint32_t hl = 0;
    for (uint32_t v = 0; v < V; ++v) {
        float e = expf((scores[v] - mx) / T);
        se += e;
        if (hl < K) {
            h[hl].p = e; h[hl].v = v;
            if (++hl == K) for (uint32_t i = K / 2; i-- > 0;) sift_down(h, i, K);
        } else if (e > h[0].p) {
            h[0].p = e; h[0].v = v;
            sift_down(h, 0, K);
        }
    }
    qsort(h, hl, sizeof(ProbTok), cmp_desc);
    float inv = 1.0f / se, cum = 0.0f;
    uint32_t tl = 0;
    for (uint32_t i = 0; i < hl; ++i) {
        h[i].p *= inv;
        cum += h[i].p;
        tl++;
        if (cum >= top_p || tl >= top_k) break;
    }
    float rv = u * cum, run = 0.0f;
    uint32_t out = h[tl - 1].v;
    for (uint32_t i = 0; i < tl; ++i) {
        run += h[i].p;
        if (rv <= run) { out = h[i].v; break; }
    }
    free(h);
    return out;
}

/* libstdc++ generate_canonical<float,24> of one 32-bit mt19937 word:
 * float(word) / 2^32, clamped below 1 (the draw the engine feeds the sampler) */
float or_canonical_from_word(uint32_t w) {
    float r = (float)w / 4294967296.0f;
    if (r >= 1.0f) r = nextafterf(1.0f, 0.0f);
    return r;
}

/* glibc's expf as the reference's sampler.hpp:116 runs it on x86-64 hosts
 * with FMA: the table-driven method of ARM optimized-routines (Szabolcs
 * Nagy; glibc e_expf.c since 2.28). N = 32; z = x*N/ln2 = k + r (k by adding
 * and subtracting 1.5*2^52); 2^(k/N) = T[k mod N] with k/N added to the
 * exponent field; 2^(r/N) ~ 1 + C2 r + C1 r^2 + C0 r^3 with the published
 * exp2 coefficients scaled by 1/N^i; the FMA build fuses the multiply-adds
 * (written out here as fma() - the file is compiled with
 * -ffp-contract=off). T[i] = bits(2^(i/N), correctly rounded) - (i << 47).
 * or_expf_mismatches() compares it with the libm expf of this host over a
 * range of float bit patterns (tests/test_oracle.py: every float in
 * [-104, 88]). The CUDA sampler (expf_ref) performs the same operations. */
static const uint64_t kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

float or_expf_ref(float x) {
    if (x < -0x1.9fe368p6f) return 0.0f;
    if (x > 0x1.62e42ep6f) return INFINITY;
    const double N = 32.0;
    const double C0 = 0x1.c6af84b912394p-5 / N / N / N, C1 = 0x1.ebfce50fac4f3p-3 / N / N,
                 C2 = 0x1.62e42ff0c52d6p-1 / N;
    const double InvLn2N = 0x1.71547652b82fep+0 * N, Shift = 0x1.8p+52;
    const double xd = (double)x;
    const double kd0 = fma(InvLn2N, xd, Shift);
    uint64_t ki;
    memcpy(&ki, &kd0, 8);
    const double kd = kd0 - Shift;
    const double r = fma(InvLn2N, xd, -kd);
    const uint64_t t = kExp2Tab[ki & 31u] + (ki << 47);
    double sc;
    memcpy(&sc, &t, 8);
    const double zc = fma(C0, r, C1);
    const double r2 = r * r;
    double y = fma(C2, r, 1.0);
    y = fma(zc, r2, y);
    y = y * sc;
    return (float)y;
}

void or_expf_batch(const float* x, float* y, long n) {
#pragma omp parallel for schedule(static)
    for (long i = 0; i < n; ++i) y[i] = or_expf_ref(x[i]);
}

/* Float bit patterns lo..hi (inclusive, same sign) on which or_expf_ref and
 * this host's libm expf differ. */
long or_expf_mismatches(uint32_t lo, uint32_t hi) {
    long bad = 0;
#pragma omp parallel for schedule(static) reduction(+ : bad)
    for (long u = (long)lo; u <= (long)hi; ++u) {
        const uint32_t w = (uint32_t)u;
        float x;
        memcpy(&x, &w, 4);
        const float a = or_expf_ref(x), b = expf(x);
        if (memcmp(&a, &b, 4) != 0) ++bad;
    }
    return bad;
}
