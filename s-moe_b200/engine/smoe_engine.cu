// smoe_engine - the decode engine's host loop in C++ over libsmoe_cuda.
//
// The reference engine (main.cpp:401-711, serve.hpp:47-103) prefills a
// prompt layer-major (prefill.cpp), then decodes one token per step
// (decode.cpp) and samples it (sampler.hpp), either once (--tokens-in) or
// per request line on stdin (--serve: "GEN <max_tokens> [t= p= k= r=]
// <csv ids>" / "RESET", answered by the ids then "fin=<stop|length>
// <<DONE>>", or "<<ERR reason>>"). This program does the same with every
// compute step a libsmoe_cuda entry on one CUDA stream: the decode step is
// captured once as a CUDA graph (embedding, L x (input norm, attention
// layer, post norm, MoE layer), final norm, LM head, sampler, position and
// history bookkeeping), the prompt but its last token goes through the
// layer-major prefill entries, and the host only writes each step's uniform
// draw (std::mt19937 + generate_canonical<float,24>, main.cpp:316 and
// sampler.hpp) and reads the sampled id back.
//
// Weights: --weights DIR (raw little-endian tensors, listed in DIR/meta.txt)
// or seeded random ones with the benchmark's distributions (--shape 30b |
// 235b); --vault FILE takes the experts of a .smoe vault (SMOE-Q4) instead.
// The trunk weights of a real model live in the reference's separate scout
// file, which this program does not read (random trunk with --vault).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <random>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

#include "../../include/smoe_cuda.h"

namespace {

#define CUDA_OK(x)                                                                          \
    do {                                                                                    \
        cudaError_t e_ = (x);                                                               \
        if (e_ != cudaSuccess) {                                                            \
            std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            std::exit(2);                                                                   \
        }                                                                                   \
    } while (0)
#define SMOE_OK_(x)                                                                         \
    do {                                                                                    \
        int r_ = (x);                                                                       \
        if (r_ != SMOE_OK) {                                                                \
            std::fprintf(stderr, "libsmoe_cuda error %d (%s) at %s:%d\n", r_, smoe_cuda_last_error(), \
                         __FILE__, __LINE__);                                               \
            std::exit(3);                                                                   \
        }                                                                                   \
    } while (0)

// ---------------------------------------------------------------- random init
__device__ __forceinline__ uint64_t mix64(uint64_t z) {      // splitmix64 finaliser
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ float unif(uint64_t seed, uint64_t i) {           // (0, 1)
    return (float(mix64(seed * 0x9e3779b97f4a7c15ull + i) >> 40) + 0.5f) * (1.0f / 16777216.0f);
}
// kind 0: normal(a, b) as bf16; 1: uniform(a, b) as bf16; 2: uniform(a, b) as fp16; 3: random bytes
__global__ void k_fill(void* out, size_t n, uint64_t seed, int kind, float a, float b) {
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        if (kind == 3) {
            static_cast<uint8_t*>(out)[i] = uint8_t(mix64(seed * 0x9e3779b97f4a7c15ull + i) >> 56);
            continue;
        }
        float v;
        if (kind == 0) {                                     // Box-Muller
            const float u1 = unif(seed, 2 * i), u2 = unif(seed, 2 * i + 1);
            v = a + b * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        } else {
            v = a + (b - a) * unif(seed, i);
        }
        if (kind == 2) {
            __half h = __float2half_rn(v);
            static_cast<uint16_t*>(out)[i] = *reinterpret_cast<uint16_t*>(&h);
        } else {
            __nv_bfloat16 h = __float2bfloat16_rn(v);
            static_cast<uint16_t*>(out)[i] = *reinterpret_cast<uint16_t*>(&h);
        }
    }
}
void fill(void* p, size_t n, uint64_t seed, int kind, float a, float b, cudaStream_t s) {
    k_fill<<<1184, 256, 0, s>>>(p, n, seed, kind, a, b);
    CUDA_OK(cudaGetLastError());
}

// ---------------------------------------------------------------- config
struct Shape {
    uint32_t layers = 48, d = 2048, heads = 32, kv_heads = 4, hd = 128, E = 128, k = 8, dff = 768,
             vocab = 151936, ctx = 4096, fmt = SMOE_FMT_AFFINE_Q4;
    float theta = 1e6f;
    bool norm_topk = true;
    uint32_t q_dim() const { return heads * hd; }
    uint32_t kv_dim() const { return kv_heads * hd; }
};

// vault-layout blob offsets (gate, up, down: nibbles, scales, biases)
uint64_t blob_layout(const Shape& s, uint64_t off[9]) {
    uint64_t cur = 0;
    const uint64_t rc[3][2] = {{s.dff, s.d}, {s.dff, s.d}, {s.d, s.dff}};
    for (int m = 0; m < 3; ++m) {
        const uint64_t nib = rc[m][0] * rc[m][1] / 2, sc = rc[m][0] * rc[m][1] / 64 * 2;
        off[3 * m] = cur;
        cur += nib;
        off[3 * m + 1] = cur;
        cur += sc;
        off[3 * m + 2] = cur;
        if (s.fmt == SMOE_FMT_AFFINE_Q4) cur += sc;
    }
    return cur;
}

struct Args {
    std::string weights, vault, tokens_in, shape = "30b";
    uint32_t layers = 0, max_tokens = 32, top_k = 20, ctx = 4096, seed = 1234;
    float temperature = 0.7f, top_p = 0.8f, rep = 1.1f;
    bool serve = false, raw_ids = true, bench = false;
    uint32_t bench_prompt = 45, bench_gen = 128;
};

std::vector<uint8_t> read_file(const std::string& path) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) {
        std::fprintf(stderr, "cannot open %s\n", path.c_str());
        std::exit(1);
    }
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    std::vector<uint8_t> b(size_t(n > 0 ? n : 0));
    if (n > 0 && std::fread(b.data(), 1, b.size(), f) != b.size()) {
        std::fprintf(stderr, "short read %s\n", path.c_str());
        std::exit(1);
    }
    std::fclose(f);
    return b;
}

// ---------------------------------------------------------------- engine
struct Layer {
    uint16_t *w_q, *w_k, *w_v, *w_o, *router, *in_norm, *post_norm, *q_norm, *k_norm;
    uint8_t* tiled;
    SmoeMoeLayer moe;
    SmoeCudaAttnLayerArgs attn, attn_pf;
};

struct Engine {
    Shape sh;
    SmoeCudaCtx* ctx = nullptr;
    cudaStream_t st = nullptr;
    uint16_t *embed = nullptr, *lm_head = nullptr, *model_norm = nullptr;
    std::vector<Layer> L;
    // decode-step state (device)
    float *hidden, *normed, *attn_o, *ffn_out, *qbuf, *kbuf, *vbuf, *attn_out, *kv, *rope_cos, *rope_sin,
        *inv_freq, *logits;
    uint32_t *token, *pos, *history;
    SmoeSamplerRow* row;
    uint32_t hcap = 8192;
    // prefill chunk state (device)
    static constexpr uint32_t kChunk = 256;
    float *pf_hidden, *pf_normed, *pf_attn_o, *pf_ffn_out, *pf_q, *pf_k, *pf_v, *pf_attn_out, *pf_cos, *pf_sin;
    uint32_t *pf_tokens, *pf_pos;
    // host mirrors
    SmoeSamplerRow* h_row = nullptr;     // pinned
    uint32_t* h_token = nullptr;         // pinned
    cudaGraphExec_t graph = nullptr;
    std::mt19937 rng;

    template <typename T>
    T* dalloc(size_t n) {
        T* p = nullptr;
        CUDA_OK(cudaMalloc(&p, n * sizeof(T)));
        CUDA_OK(cudaMemsetAsync(p, 0, n * sizeof(T), st));
        CUDA_OK(cudaStreamSynchronize(st));          // before any copy on another stream
        return p;
    }

    void init(const Args& a) {
        SmoeCudaInitArgs ia{};
        ia.device = 0;
        ctx = smoe_cuda_init_ex(&ia);
        if (!ctx) {
            std::fprintf(stderr, "smoe_cuda_init_ex: %s\n", smoe_cuda_last_error());
            std::exit(3);
        }
        CUDA_OK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        SMOE_OK_(smoe_cuda_set_stream(ctx, st));
        rng.seed(a.seed);
        if (!a.weights.empty()) load_dir(a);
        else random_model(a);
        alloc_state();
    }

    // DIR/meta.txt: "key value" lines (layers d_model num_heads num_kv_heads
    // head_dim n_experts top_k d_ff vocab rope_theta fmt expert_stride
    // attn_ctx norm_topk); tensors DIR/<name>.bin raw little-endian.
    void load_dir(const Args& a) {
        std::vector<uint8_t> m = read_file(a.weights + "/meta.txt");
        std::string text(m.begin(), m.end());
        uint64_t estride = 0;
        size_t p = 0;
        while (p < text.size()) {
            size_t e = text.find('\n', p);
            if (e == std::string::npos) e = text.size();
            char key[64];
            double v = 0;
            if (std::sscanf(text.substr(p, e - p).c_str(), "%63s %lf", key, &v) == 2) {
                std::string k(key);
                if (k == "layers") sh.layers = uint32_t(v);
                else if (k == "d_model") sh.d = uint32_t(v);
                else if (k == "num_heads") sh.heads = uint32_t(v);
                else if (k == "num_kv_heads") sh.kv_heads = uint32_t(v);
                else if (k == "head_dim") sh.hd = uint32_t(v);
                else if (k == "n_experts") sh.E = uint32_t(v);
                else if (k == "top_k") sh.k = uint32_t(v);
                else if (k == "d_ff") sh.dff = uint32_t(v);
                else if (k == "vocab") sh.vocab = uint32_t(v);
                else if (k == "rope_theta") sh.theta = float(v);
                else if (k == "fmt") sh.fmt = uint32_t(v);
                else if (k == "expert_stride") estride = uint64_t(v);
                else if (k == "attn_ctx") sh.ctx = uint32_t(v);
                else if (k == "norm_topk") sh.norm_topk = v != 0;
            }
            p = e + 1;
        }
        auto up = [&](const std::string& name, size_t n_u16) {
            std::vector<uint8_t> b = read_file(a.weights + "/" + name + ".bin");
            if (b.size() != n_u16 * 2) {
                std::fprintf(stderr, "%s: %zu bytes, expected %zu\n", name.c_str(), b.size(), n_u16 * 2);
                std::exit(1);
            }
            uint16_t* d = dalloc<uint16_t>(n_u16);
            CUDA_OK(cudaMemcpy(d, b.data(), b.size(), cudaMemcpyHostToDevice));
            return d;
        };
        embed = up("embed", size_t(sh.vocab) * sh.d);
        lm_head = up("lm_head", size_t(sh.vocab) * sh.d);
        model_norm = up("model_norm", sh.d);
        uint64_t off[9];
        blob_layout(sh, off);
        L.resize(sh.layers);
        for (uint32_t l = 0; l < sh.layers; ++l) {
            Layer& y = L[l];
            const std::string pre = "layer" + std::to_string(l) + "_";
            y.w_q = up(pre + "w_q", size_t(sh.q_dim()) * sh.d);
            y.w_k = up(pre + "w_k", size_t(sh.kv_dim()) * sh.d);
            y.w_v = up(pre + "w_v", size_t(sh.kv_dim()) * sh.d);
            y.w_o = up(pre + "w_o", size_t(sh.d) * sh.q_dim());
            y.router = up(pre + "router", size_t(sh.E) * sh.d);
            y.in_norm = up(pre + "in_norm", sh.d);
            y.post_norm = up(pre + "post_norm", sh.d);
            y.q_norm = up(pre + "q_norm", sh.hd);
            y.k_norm = up(pre + "k_norm", sh.hd);
            std::vector<uint8_t> eb = read_file(a.weights + "/" + pre + "experts.bin");
            if (eb.size() != size_t(sh.E) * estride) {
                std::fprintf(stderr, "%sexperts: size mismatch\n", pre.c_str());
                std::exit(1);
            }
            uint8_t* arena = dalloc<uint8_t>(eb.size());
            CUDA_OK(cudaMemcpy(arena, eb.data(), eb.size(), cudaMemcpyHostToDevice));
            SmoeMoeLayer v{};
            v.base = arena;
            v.expert_stride = estride;
            std::memcpy(v.off, off, sizeof(off));
            v.n_experts = sh.E; v.d_model = sh.d; v.d_ff = sh.dff; v.fmt = sh.fmt; v.router_w = y.router;
            prepack(y, v, arena);
        }
    }

    void random_model(const Args& a) {
        if (a.shape == "235b") {
            sh.layers = 94; sh.d = 4096; sh.heads = 64; sh.dff = 1536;
        }
        if (a.layers) sh.layers = a.layers;
        sh.ctx = a.ctx;
        uint64_t seed = a.seed;
        auto normal = [&](size_t n, float std) {
            uint16_t* d = dalloc<uint16_t>(n);
            fill(d, n, ++seed, 0, 0.f, std, st);
            return d;
        };
        auto ones = [&](size_t n) {
            uint16_t* d = dalloc<uint16_t>(n);
            fill(d, n, ++seed, 1, 1.f, 1.f, st);
            return d;
        };
        std::vector<uint8_t> vault;
        SmoeVaultInfo vi{};
        if (!a.vault.empty()) {                      // experts (and the arch) from a .smoe vault
            vault = read_file(a.vault);
            SMOE_OK_(smoe_cuda_vault_parse(vault.data(), vault.size(), &vi));
            sh.layers = a.layers ? std::min(a.layers, vi.num_moe_layers) : vi.num_moe_layers;
            sh.d = vi.d_model; sh.E = vi.max_experts_per_layer; sh.dff = vi.gate_rows;
            sh.fmt = SMOE_FMT_SMOE_Q4;
            if (vi.vocab_size) sh.vocab = vi.vocab_size;
            if (vi.has_arch) {
                sh.heads = vi.num_heads; sh.kv_heads = vi.num_kv_heads; sh.hd = vi.head_dim; sh.k = vi.moe_top_k;
                sh.theta = vi.rope_theta; sh.norm_topk = (vi.arch_flags & 1u) != 0;
            }
        }
        embed = normal(size_t(sh.vocab) * sh.d, 0.02f);
        lm_head = normal(size_t(sh.vocab) * sh.d, 0.02f);
        model_norm = ones(sh.d);
        uint64_t off[9];
        const uint64_t blob = blob_layout(sh, off);
        const uint64_t estride = ((vault.empty() ? blob : vi.max_raw_size) + 255) / 256 * 256;
        uint8_t* arena = dalloc<uint8_t>(size_t(sh.E) * estride);     // staging, reused per layer
        L.resize(sh.layers);
        for (uint32_t l = 0; l < sh.layers; ++l) {
            Layer& y = L[l];
            y.w_q = normal(size_t(sh.q_dim()) * sh.d, 0.02f);
            y.w_k = normal(size_t(sh.kv_dim()) * sh.d, 0.02f);
            y.w_v = normal(size_t(sh.kv_dim()) * sh.d, 0.02f);
            y.w_o = normal(size_t(sh.d) * sh.q_dim(), 0.02f);
            y.router = normal(size_t(sh.E) * sh.d, 0.02f);
            y.in_norm = ones(sh.d); y.post_norm = ones(sh.d); y.q_norm = ones(sh.hd); y.k_norm = ones(sh.hd);
            SmoeMoeLayer v{};
            if (!vault.empty()) {
                SMOE_OK_(smoe_cuda_vault_upload_layer(ctx, vault.data(), vault.size(), l, arena, estride, y.router,
                                                      &v));
            } else {
                for (uint32_t e = 0; e < sh.E; ++e) {
                    uint8_t* b = arena + size_t(e) * estride;
                    const uint64_t rc[3] = {uint64_t(sh.dff) * sh.d, uint64_t(sh.dff) * sh.d, uint64_t(sh.d) * sh.dff};
                    for (int m = 0; m < 3; ++m) {
                        fill(b + off[3 * m], rc[m] / 2, ++seed, 3, 0.f, 0.f, st);
                        fill(b + off[3 * m + 1], rc[m] / 64, ++seed, sh.fmt == SMOE_FMT_AFFINE_Q4 ? 1 : 2, 0.001f,
                             0.01f, st);
                        if (sh.fmt == SMOE_FMT_AFFINE_Q4) fill(b + off[3 * m + 2], rc[m] / 64, ++seed, 0, 0.f, 0.01f, st);
                    }
                }
                v.base = arena;
                v.expert_stride = estride;
                std::memcpy(v.off, off, sizeof(off));
                v.n_experts = sh.E; v.d_model = sh.d; v.d_ff = sh.dff; v.fmt = sh.fmt; v.router_w = y.router;
            }
            prepack(y, v, nullptr);
        }
        CUDA_OK(cudaStreamSynchronize(st));
        CUDA_OK(cudaFree(arena));
    }

    // vault layout -> tiled layout (the single-launch layer kernel's); frees `arena` when given
    void prepack(Layer& y, const SmoeMoeLayer& v, uint8_t* arena) {
        const uint64_t tb = smoe_cuda_tiled_expert_bytes(sh.fmt, sh.d, sh.dff);
        if (!tb) {
            std::fprintf(stderr, "shape not supported by the tiled layout\n");
            std::exit(1);
        }
        const uint64_t ts = (tb + 255) / 256 * 256;
        y.tiled = dalloc<uint8_t>(size_t(sh.E) * ts);
        SMOE_OK_(smoe_cuda_prepack_layer(ctx, &v, y.tiled, ts, &y.moe));
        CUDA_OK(cudaStreamSynchronize(st));
        if (arena) CUDA_OK(cudaFree(arena));
    }

    void alloc_state() {
        const uint32_t d = sh.d, q = sh.q_dim(), kv = sh.kv_dim(), half = sh.hd / 2;
        hidden = dalloc<float>(d); normed = dalloc<float>(d); attn_o = dalloc<float>(d); ffn_out = dalloc<float>(d);
        qbuf = dalloc<float>(q); kbuf = dalloc<float>(kv); vbuf = dalloc<float>(kv); attn_out = dalloc<float>(q);
        kv_ = size_t(sh.layers) * 2 * sh.ctx * kv;
        this->kv = dalloc<float>(kv_);
        rope_cos = dalloc<float>(half); rope_sin = dalloc<float>(half);
        logits = dalloc<float>(sh.vocab);
        token = dalloc<uint32_t>(1); pos = dalloc<uint32_t>(1); history = dalloc<uint32_t>(hcap);
        row = dalloc<SmoeSamplerRow>(1);
        std::vector<float> inv(half);                // engine.cpp:351-356
        for (uint32_t i = 0; i < half; ++i)
            inv[i] = float(1.0 / std::pow(double(sh.theta), double(2 * i) / double(sh.hd)));
        inv_freq = dalloc<float>(half);
        CUDA_OK(cudaMemcpy(inv_freq, inv.data(), half * 4, cudaMemcpyHostToDevice));
        const uint32_t C = kChunk;
        pf_hidden = dalloc<float>(size_t(C) * d); pf_normed = dalloc<float>(size_t(C) * d);
        pf_attn_o = dalloc<float>(size_t(C) * d); pf_ffn_out = dalloc<float>(size_t(C) * d);
        pf_q = dalloc<float>(size_t(C) * q); pf_k = dalloc<float>(size_t(C) * kv); pf_v = dalloc<float>(size_t(C) * kv);
        pf_attn_out = dalloc<float>(size_t(C) * q);
        pf_cos = dalloc<float>(size_t(C) * half); pf_sin = dalloc<float>(size_t(C) * half);
        pf_tokens = dalloc<uint32_t>(C); pf_pos = dalloc<uint32_t>(1);
        CUDA_OK(cudaMallocHost(&h_row, sizeof(SmoeSamplerRow)));
        CUDA_OK(cudaMallocHost(&h_token, 4 * kChunk));
        for (uint32_t l = 0; l < sh.layers; ++l) {
            SmoeCudaAttnLayerArgs& t = L[l].attn;
            t = SmoeCudaAttnLayerArgs{};
            t.w_q = L[l].w_q; t.w_k = L[l].w_k; t.w_v = L[l].w_v; t.w_o = L[l].w_o;
            t.q_norm_w = L[l].q_norm; t.k_norm_w = L[l].k_norm;
            t.rope_cos = rope_cos; t.rope_sin = rope_sin; t.normed_in = normed;
            t.qbuf = qbuf; t.kbuf = kbuf; t.vbuf = vbuf;
            t.k_cache = this->kv + size_t(l) * 2 * sh.ctx * kv;
            t.v_cache = t.k_cache + size_t(sh.ctx) * kv;
            t.attn_out = attn_out; t.o_out = attn_o;
            t.d_model = d; t.q_dim = q; t.kv_dim = kv; t.head_dim = sh.hd;
            t.num_heads = sh.heads; t.num_kv_heads = sh.kv_heads; t.slot = 0; t.valid = 1; t.attn_ctx = sh.ctx;
            t.attn_scale = 1.0f / std::sqrt(float(sh.hd));
            SmoeCudaAttnLayerArgs& p = L[l].attn_pf;
            p = t;
            p.rope_cos = pf_cos; p.rope_sin = pf_sin; p.normed_in = pf_normed;
            p.qbuf = pf_q; p.kbuf = pf_k; p.vbuf = pf_v; p.attn_out = pf_attn_out; p.o_out = pf_attn_o;
        }
        CUDA_OK(cudaStreamSynchronize(st));
    }
    size_t kv_ = 0;

    // one token step (decode.cpp:103-231 + MoE, main.cpp:621-641)
    void step() {
        const uint32_t d = sh.d;
        SMOE_OK_(smoe_cuda_embed_bf16(ctx, embed, token, 1, d, hidden));
        SMOE_OK_(smoe_cuda_rope_table(ctx, pos, inv_freq, rope_cos, rope_sin, sh.hd / 2));
        for (uint32_t l = 0; l < sh.layers; ++l) {
            SMOE_OK_(smoe_cuda_rms_norm(ctx, hidden, l ? ffn_out : nullptr, L[l].in_norm, normed, d, 1));
            SMOE_OK_(smoe_cuda_attention_layer_async(ctx, &L[l].attn, pos));
            SMOE_OK_(smoe_cuda_rms_norm(ctx, hidden, attn_o, L[l].post_norm, normed, d, 1));
            SMOE_OK_(smoe_cuda_moe_layer(ctx, &L[l].moe, normed, 0, 1, sh.k, sh.norm_topk, ffn_out, 0, nullptr,
                                         nullptr));
        }
        SMOE_OK_(smoe_cuda_rms_norm(ctx, hidden, ffn_out, model_norm, normed, d, 1));
        SMOE_OK_(smoe_cuda_matvec_bf16(ctx, lm_head, normed, logits, sh.vocab, d));
        SMOE_OK_(smoe_cuda_sample(ctx, logits, sh.vocab, 1, row, history, hcap, token));
        SMOE_OK_(smoe_cuda_decode_advance(ctx, row, history, hcap, token, pos, nullptr, 0));
    }

    void capture() {
        step();                                      // eager once: kernel attributes set outside capture
        CUDA_OK(cudaStreamSynchronize(st));
        cudaGraph_t g;
        CUDA_OK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        step();
        CUDA_OK(cudaStreamEndCapture(st, &g));
        CUDA_OK(cudaGraphInstantiate(&graph, g, 0));
        CUDA_OK(cudaGraphDestroy(g));
    }

    // prefill.cpp:82-465: n tokens at positions base.. through every layer
    void prefill_chunk(const uint32_t* toks, uint32_t n, uint32_t base) {
        std::memcpy(h_token, toks, 4 * n);
        CUDA_OK(cudaMemcpyAsync(pf_tokens, h_token, 4 * n, cudaMemcpyHostToDevice, st));
        CUDA_OK(cudaMemcpyAsync(pf_pos, &base_host(base), 4, cudaMemcpyHostToDevice, st));
        const uint32_t d = sh.d;
        SMOE_OK_(smoe_cuda_embed_bf16(ctx, embed, pf_tokens, n, d, pf_hidden));
        SMOE_OK_(smoe_cuda_rope_tables(ctx, pf_pos, n, inv_freq, pf_cos, pf_sin, sh.hd / 2));
        for (uint32_t l = 0; l < sh.layers; ++l) {
            SMOE_OK_(smoe_cuda_rms_norm(ctx, pf_hidden, l ? pf_ffn_out : nullptr, L[l].in_norm, pf_normed, d, n));
            SMOE_OK_(smoe_cuda_attention_prefill_async(ctx, &L[l].attn_pf, n, pf_pos));
            SMOE_OK_(smoe_cuda_rms_norm(ctx, pf_hidden, pf_attn_o, L[l].post_norm, pf_normed, d, n));
            for (uint32_t i = 0; i < n; i += 4) {    // the layer kernel, 4 tokens per launch
                const uint32_t m = n - i < 4 ? n - i : 4;
                SMOE_OK_(smoe_cuda_moe_layer(ctx, &L[l].moe, pf_normed + size_t(i) * d, 0, m, sh.k, sh.norm_topk,
                                             pf_ffn_out + size_t(i) * d, 0, nullptr, nullptr));
            }
        }
        CUDA_OK(cudaStreamSynchronize(st));          // h_token / base buffers reused next chunk
    }
    uint32_t base_buf = 0;
    uint32_t& base_host(uint32_t b) {
        base_buf = b;
        return base_buf;
    }

    float draw() {                                   // main.cpp:316 + generate_canonical<float,24>
        return smoe_cuda_canonical_from_u32(uint32_t(rng()));
    }

    // Feed tokens [stream positions start .. start + n) and leave the last one
    // in the token slot at position start + n - 1, history = stream[0 .. start + n).
    void feed(const std::vector<uint32_t>& stream, uint32_t start) {
        const uint32_t n = uint32_t(stream.size()) - start;
        for (uint32_t b0 = 0; b0 + 1 < n; b0 += kChunk) {
            const uint32_t m = std::min<uint32_t>(kChunk, n - 1 - b0);
            prefill_chunk(stream.data() + start + b0, m, start + b0);
        }
        const uint32_t last = stream.back(), p = uint32_t(stream.size()) - 1;
        const uint32_t nh = std::min<uint32_t>(uint32_t(stream.size()), hcap);
        CUDA_OK(cudaMemcpy(token, &last, 4, cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(pos, &p, 4, cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(history, stream.data() + stream.size() - nh, 4 * nh, cudaMemcpyHostToDevice));
        h_row->history_len = nh;
    }

    // One request: stream = the whole conversation; KV of positions < lcp is
    // reused (main.cpp:466-500). Emits up to max_tokens ids; returns the
    // stream extended by the generated ids whose KV exists.
    bool generate(std::vector<uint32_t>& stream, uint32_t lcp, uint32_t max_tokens, const SmoeSamplerRow& cfg,
                  std::vector<uint32_t>& out) {
        static const uint32_t kEos[] = {151643u, 151645u};
        if (lcp == 0) CUDA_OK(cudaMemsetAsync(kv, 0, kv_ * 4, st));
        feed(stream, lcp);
        bool eos = false;
        for (uint32_t i = 0; i < max_tokens; ++i) {
            *h_row = SmoeSamplerRow{cfg.temperature, cfg.top_p, cfg.top_k, cfg.rep_penalty, draw(),
                                    h_row->history_len};
            CUDA_OK(cudaMemcpyAsync(row, h_row, sizeof(*h_row), cudaMemcpyHostToDevice, st));
            CUDA_OK(cudaGraphLaunch(graph, st));
            CUDA_OK(cudaMemcpyAsync(h_token, token, 4, cudaMemcpyDeviceToHost, st));
            CUDA_OK(cudaStreamSynchronize(st));
            h_row->history_len = std::min(h_row->history_len + 1, hcap);
            const uint32_t t = h_token[0];
            if (t == kEos[0] || t == kEos[1]) {
                eos = true;
                break;
            }
            out.push_back(t);
            if (i + 1 < max_tokens) stream.push_back(t);   // processed next step: its KV will exist
        }
        SMOE_OK_(smoe_cuda_synchronize(ctx));
        return eos;
    }
};

std::vector<uint32_t> parse_csv(const std::string& s) {
    std::vector<uint32_t> v;
    const char* p = s.c_str();
    while (*p) {
        char* e = nullptr;
        const unsigned long x = std::strtoul(p, &e, 10);
        if (e == p) break;
        v.push_back(uint32_t(x));
        p = e;
        if (*p == ',') ++p;
    }
    return v;
}

// serve.hpp:47-103: "GEN <max_tokens> [t= p= k= r=] <csv>"
bool parse_gen(const std::string& line, uint32_t& max_tokens, SmoeSamplerRow& cfg, std::vector<uint32_t>& toks) {
    size_t p = 4, sp = line.find(' ', p);
    if (sp == std::string::npos) return false;
    max_tokens = uint32_t(std::atoi(line.c_str() + p));
    if (max_tokens == 0 || max_tokens > 8192) return false;
    p = sp + 1;
    while (p < line.size()) {
        size_t fend = line.find(' ', p);
        if (fend == std::string::npos) fend = line.size();
        const size_t eq = line.find('=', p);
        if (eq == std::string::npos || eq >= fend) break;
        const char* val = line.c_str() + eq + 1;
        if (eq == p + 1) {
            switch (line[p]) {
                case 't': cfg.temperature = std::max(0.0f, std::strtof(val, nullptr)); break;
                case 'p': cfg.top_p = std::min(std::max(std::strtof(val, nullptr), 0.01f), 1.0f); break;
                case 'k': cfg.top_k = uint32_t(std::min(std::max(std::strtol(val, nullptr, 10), 1L), 1024L)); break;
                case 'r': {
                    const float r = std::strtof(val, nullptr);
                    if (r > 0.0f) cfg.rep_penalty = r;
                    break;
                }
                default: break;
            }
        }
        p = fend < line.size() ? fend + 1 : fend;
    }
    toks = parse_csv(line.substr(p < line.size() ? p : line.size()));
    return !toks.empty();
}

}  // namespace

int main(int argc, char** argv) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        std::string k = argv[i];
        auto nx = [&]() -> const char* {
            if (i + 1 >= argc) {
                std::fprintf(stderr, "missing value for %s\n", k.c_str());
                std::exit(1);
            }
            return argv[++i];
        };
        if (k == "--weights") a.weights = nx();
        else if (k == "--vault") a.vault = nx();
        else if (k == "--shape") a.shape = nx();
        else if (k == "--layers") a.layers = uint32_t(std::atoi(nx()));
        else if (k == "--ctx") a.ctx = uint32_t(std::atoi(nx()));
        else if (k == "--tokens-in") a.tokens_in = nx();
        else if (k == "--max-tokens") a.max_tokens = uint32_t(std::atoi(nx()));
        else if (k == "--temperature") a.temperature = std::strtof(nx(), nullptr);
        else if (k == "--top-p") a.top_p = std::strtof(nx(), nullptr);
        else if (k == "--top-k") a.top_k = uint32_t(std::atoi(nx()));
        else if (k == "--rep-penalty") a.rep = std::strtof(nx(), nullptr);
        else if (k == "--seed") a.seed = uint32_t(std::atoi(nx()));
        else if (k == "--serve") a.serve = true;
        else if (k == "--bench") a.bench = true;
        else if (k == "--bench-prompt") a.bench_prompt = uint32_t(std::atoi(nx()));
        else if (k == "--bench-gen") a.bench_gen = uint32_t(std::atoi(nx()));
        else {
            std::fprintf(stderr, "unknown option %s\n", k.c_str());
            return 1;
        }
    }
    Engine eng;
    const auto t0 = std::chrono::steady_clock::now();
    eng.init(a);
    eng.capture();
    const double load_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    SmoeSamplerRow cfg{a.temperature, a.top_p, a.top_k, a.rep, 0.5f, 0};
    if (a.bench) {                                   // prompt + generation timing, one JSON line
        std::vector<uint32_t> stream(a.bench_prompt), out;
        std::mt19937 prng(11);
        for (auto& t : stream) t = uint32_t(prng() % eng.sh.vocab);
        eng.generate(stream, 0, 4, cfg, out);        // warm-up
        stream.resize(a.bench_prompt);
        out.clear();
        cudaEvent_t e0, e1, e2;
        CUDA_OK(cudaEventCreate(&e0)); CUDA_OK(cudaEventCreate(&e1)); CUDA_OK(cudaEventCreate(&e2));
        CUDA_OK(cudaEventRecord(e0, eng.st));
        std::vector<uint32_t> first;
        eng.generate(stream, 0, 1, cfg, first);      // prefill + first token
        CUDA_OK(cudaEventRecord(e1, eng.st));
        const auto w0 = std::chrono::steady_clock::now();
        eng.generate(stream, uint32_t(stream.size()) - 1, a.bench_gen, cfg, out);
        const double gen_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - w0).count();
        CUDA_OK(cudaEventSynchronize(e1));
        float ttft_ms = 0;
        CUDA_OK(cudaEventElapsedTime(&ttft_ms, e0, e1));
        std::printf("{\"engine\": \"smoe_engine (C++)\", \"layers\": %u, \"d_model\": %u, \"prompt\": %u, "
                    "\"generated\": %zu, \"ttft_ms\": %.3f, \"tok_per_s\": %.2f, \"load_s\": %.1f}\n",
                    eng.sh.layers, eng.sh.d, a.bench_prompt, out.size(), ttft_ms, double(out.size()) / gen_s,
                    load_s);
        return 0;
    }
    if (!a.serve) {                                  // one-shot (main.cpp --tokens-in)
        std::vector<uint32_t> stream = parse_csv(a.tokens_in), out;
        if (stream.empty()) {
            std::fprintf(stderr, "--tokens-in needs at least one id\n");
            return 1;
        }
        const bool eos = eng.generate(stream, 0, a.max_tokens, cfg, out);
        for (uint32_t t : out) std::printf("%u ", t);
        std::printf("\nfin=%s <<DONE>>\n", eos ? "stop" : "length");
        return 0;
    }
    std::vector<uint32_t> stream;                    // tokens whose KV exists
    char buf[1 << 16];
    std::string line;
    while (std::fgets(buf, sizeof(buf), stdin)) {
        line = buf;
        while (!line.empty() && (line.back() == '\n' || line.back() == '\r')) line.pop_back();
        if (line.empty()) continue;
        if (line == "RESET") {
            stream.clear();
            std::printf("<<DONE>>\n");
            std::fflush(stdout);
            continue;
        }
        uint32_t max_tokens = 0;
        std::vector<uint32_t> full, out;
        if (line.rfind("GEN ", 0) != 0 || !parse_gen(line, max_tokens, cfg, full)) {
            std::printf("<<ERR bad_request>>\n");
            std::fflush(stdout);
            continue;
        }
        if (full.size() > eng.sh.ctx) {
            std::printf("<<ERR ctx_overflow>>\n");
            std::fflush(stdout);
            continue;
        }
        uint32_t lcp = 0;                            // main.cpp:466-480
        while (lcp < stream.size() && lcp < full.size() && stream[lcp] == full[lcp]) ++lcp;
        if (lcp < stream.size()) lcp = 0;
        if (lcp == full.size()) {
            std::printf("<<ERR empty_suffix>>\n");
            std::fflush(stdout);
            continue;
        }
        stream = full;
        const bool eos = eng.generate(stream, lcp, max_tokens, cfg, out);
        for (uint32_t t : out) std::printf("%u ", t);
        std::printf("\nfin=%s <<DONE>>\n", eos ? "stop" : "length");
        std::fflush(stdout);
    }
    return 0;
}
