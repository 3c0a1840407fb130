// smoe_cuda.cu - the C ABI of include/smoe_cuda.h: context, scratch,
// launches and bounded waits. Kernels live in the *.cuh files.
#include <cuda_runtime.h>
#include <cublas_v2.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>

#include "../../include/smoe_cuda.h"
#include "ffn_q4.cuh"
#include "moe_layer.cuh"
#include "router.cuh"
#include "sampler.cuh"
#include "decode.cuh"
#include "ffn_grouped.cuh"

namespace {

thread_local char g_err[512] = "";

void set_err(const char* fmt, const char* a = "", long b = 0) {
    std::snprintf(g_err, sizeof(g_err), fmt, a, b);
}

#define CK(call)                                                                      \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess) {                                                      \
            set_err("CUDA error %s (line %ld)", cudaGetErrorString(e_), (long)__LINE__); \
            return SMOE_ERR_CUDA;                                                     \
        }                                                                             \
    } while (0)

constexpr int kEventRing = 64;
constexpr size_t kBlasWorkspace = size_t(32) << 20;

}  // namespace

struct SmoeCudaCtx {
    int device = 0;
    SmoeCudaInitArgs cfg{};
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    // scratch (device)
    float* hidden = nullptr;        // [max_batch * 16][max_d_ff]
    float* slot_out = nullptr;      // [max(16, 64)][max_d_model]  mirror outputs
    float* in_stage = nullptr;      // [64][max_d_model]           mirror inputs
    float* batch_out = nullptr;     // [64][max_d_model]           token-batch outputs
    float* logits = nullptr;        // [max_batch][max_experts]
    unsigned long long* lpair = nullptr;
    float* attn_part = nullptr;           // decode attention split partials [heads][splits][258]
    uint32_t* attn_cnt = nullptr;         // [heads] splits done (zero between launches)  // layer kernel's tagged logits [kLMaxTok][128] (zero: no tag)
    uint32_t* ids = nullptr;        // [max_batch][16]
    float* wts = nullptr;           // [max_batch][16]
    uint32_t* ticket = nullptr;     // [max_batch]
    uint32_t* err = nullptr;        // device error word
    float* gemv_out = nullptr;      // staging for the mirrored matvec
    float* gemv_in = nullptr;
    // batched trunk GEMMs (cuBLAS bf16, fp32 accumulation)
    cublasHandle_t blas = nullptr;
    void* blas_ws = nullptr;        // cuBLAS workspace (fixed, so graph capture allocates nothing)
    uint16_t* xsplit = nullptr;     // [2][max_batch * max_d_model] bf16 hi / lo planes
    size_t gemv_cap = 0;
    // waits
    cudaEvent_t events[kEventRing] = {};
    uint64_t seq = 0;
    std::atomic<uint64_t> dispatches{0};
    size_t smem_optin = 0;
    int num_sms = 0;
    int gemv_res[2] = {0, 0};        // resident CTAs per SM of k_gemv_set<1>, <2>
    smoe::LayerState* lstate = nullptr;   // layer kernel's grid counters (zero between launches)
    unsigned long long* lpart = nullptr;  // layer kernel's tagged partial rows [num_sms][kLMaxTok][kLMaxD] (zero: no tag)
    uint64_t wait_ns = 0;                 // limit of every device-side wait of the layer kernel
    unsigned long long* trace = nullptr;   // phase timestamps of the layer kernel (profiling aid)
    // expert-grouped batch path: per-expert slot lists, operand tables, per-slot outputs
    uint32_t* g_list = nullptr;      // [max_experts][max_batch * 16]
    uint32_t* g_count = nullptr;     // [max_experts], then the grouped path's lo flag
    uint2* g_xtab = nullptr;         // [max_batch][max_d_model / 16][8]
    float2* g_xgs = nullptr;         // [max_batch][max_d_model / 64]
    uint2* g_htab = nullptr;         // [max_batch * 16][max_d_ff / 16][8]
    float2* g_hgs = nullptr;         // [max_batch * 16][max_d_ff / 64]
    float* g_ys = nullptr;           // [max_batch * 16][max_d_model]
    // expert parallel: this rank's exchange window (IPC-exported) and rank 0's, mapped
    uint8_t* ep_win = nullptr;
    size_t ep_win_bytes = 0;
    uint8_t* ep_peer[smoe::kEpMaxWorld] = {};   // windows of the ranks this one writes to (own: ep_win)
    int ep_world = 0, ep_rank = 0;
};

namespace {

// 0: device (or managed) memory, 1: pinned host memory the GPU can address,
// 2: pageable host memory or unknown.
int mem_kind(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return 2;
    }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) return 0;
    if (at.type == cudaMemoryTypeHost && at.devicePointer == p) return 1;
    return 2;
}

bool is_device_ptr(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

int check_device_err(SmoeCudaCtx* c) {
    uint32_t e = 0;
    CK(cudaMemcpyAsync(&e, c->err, 4, cudaMemcpyDeviceToHost, c->stream));
    CK(cudaStreamSynchronize(c->stream));
    if (e != 0) {
        cudaMemsetAsync(c->err, 0, 4, c->stream);
        set_err("device error flag %s%ld raised by a kernel", "", (long)e);
        return SMOE_ERR_DEVICE;
    }
    return SMOE_OK;
}

int wait_event_bounded(SmoeCudaCtx* c, cudaEvent_t ev) {
    auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaEventQuery(ev);
        if (q == cudaSuccess) return SMOE_OK;
        if (q != cudaErrorNotReady) {
            set_err("CUDA error %s while waiting (%ld)", cudaGetErrorString(q), 0);
            return SMOE_ERR_CUDA;
        }
        auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                      std::chrono::steady_clock::now() - t0).count();
        if (ms > (long)c->cfg.timeout_ms) {
            set_err("wait timed out after %s%ld ms", "", (long)ms);
            return SMOE_ERR_TIMEOUT;
        }
        std::this_thread::yield();
    }
}

template <typename K>
int prep_kernel(SmoeCudaCtx* c, K kern, size_t smem) {
    // (also below 48 KB of dynamic memory: with the kernel's static shared
    // memory the total may still exceed the default limit)
    if (smem > 0) {
        if (smem > c->smem_optin) {
            set_err("kernel needs %s%ld bytes of shared memory", "", (long)smem);
            return SMOE_ERR_ARG;
        }
        // Raise the limit once per (kernel, device, size): later calls, including
        // calls made while a stream is being captured, then issue no attribute call.
        static thread_local struct { const void* f; int dev; size_t smem; } seen[32];
        static thread_local int nseen = 0;
        for (int i = 0; i < nseen; ++i)
            if (seen[i].f == (const void*)kern && seen[i].dev == c->device && seen[i].smem >= smem)
                return SMOE_OK;
        CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (nseen < 32) seen[nseen++] = {(const void*)kern, c->device, smem};
    }
    return SMOE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_ffn_dims(SmoeCudaCtx* c, uint32_t d, uint32_t dff) {
    if (d == 0 || dff == 0 || d % 64 || dff % 64 || d > c->cfg.max_d_model || dff > c->cfg.max_d_ff) {
        set_err("unsupported FFN dims (need multiples of 64 within the context limits) %s%ld", "",
                (long)d);
        return SMOE_ERR_ARG;
    }
    return SMOE_OK;
}

// Launch gate_up then down/combine for a prepared FfnArgs.
// Token batches (> 4 tokens) on the vault layout: the expert-grouped path,
// each expert's weights read once per layer whatever its token count.
// base / e_total: an expert-parallel shard holds experts [base, base + E) of
// e_total (0: the whole layer); its y is the partial sum over its experts.
int launch_grouped(SmoeCudaCtx* c, smoe::FfnArgs& a, int fmt, uint32_t E, uint32_t base = 0, uint32_t e_total = 0) {
    const bool shard = e_total != 0;
    if (!shard) e_total = E;
    const uint32_t nslots = a.ntok * a.k, lcap = c->cfg.max_batch * 16u;
    if (nslots == 0) return SMOE_OK;
    if (nslots > lcap || E > c->cfg.max_experts || !a.ids) {
        set_err("bad grouped FFN arguments %s%ld", "", (long)nslots);
        return SMOE_ERR_ARG;
    }
    const uint32_t d = a.d_model, dff = a.d_ff;
    // gate/up: 32 rows x 2 matrices per CTA; down: 128 rows per CTA
    constexpr int kRbGu = 32, kWnGu = 1;
    if (dff % 256 || d % 128 || dff > 4096) { set_err("grouped FFN needs d_ff % 256 == 0, d_ff <= 4096 and d_model % 128 == 0 %s%ld", "", 0); return SMOE_ERR_ARG; }
    int rc;
    uint32_t* lo_flag = c->g_count + c->cfg.max_experts;
    using namespace smoe;
    smoe::k_group_slots<<<E, 32, 0, c->stream>>>(a.ids, nslots, c->g_list, c->g_count, lcap, lo_flag, c->err,
                                                 base, e_total);
    if ((rc = prep_kernel(c, k_build_tabs<kTabMma>, size_t(d / 4) * 8))) return rc;
    if ((rc = prep_kernel(c, k_build_tabs<kTabTc>, size_t(dff / 4) * 8))) return rc;
    k_build_tabs<kTabMma><<<a.ntok, 256, size_t(d / 4) * 8, c->stream>>>(a.x, a.x_dtype == 1, d, c->g_xtab, c->g_xgs,
                                                                        lo_flag);
    smoe::GroupedArgs g{};
    g.base = a.base;
    g.stride = a.stride;
    for (int i = 0; i < 9; ++i) g.off[i] = a.off[i];
    g.list = c->g_list;
    g.count = c->g_count;
    g.lcap = lcap;
    g.d_model = d;
    g.d_ff = dff;
    g.err = c->err;
    smoe::GroupedArgs g1 = g, g2 = g;
    g1.tab = c->g_xtab; g1.gs = c->g_xgs; g1.tab_div = a.k; g1.out = c->hidden; g1.lo_flag = lo_flag;
    g2.tab = c->g_htab; g2.gs = c->g_hgs; g2.tab_div = 1; g2.out = c->g_ys; g2.lo_flag = nullptr;
    const size_t s1 = grouped_smem_bytes(d, 2, kRbGu, kWnGu), s2 = TcSmem::bytes(dff / 64);
    auto run = [&](auto k1, auto k2) -> int {
        int r;
        if ((r = prep_kernel(c, k1, s1)) || (r = prep_kernel(c, k2, s2))) return r;
        k1<<<dim3(dff / kRbGu, E), 256, s1, c->stream>>>(g1);
        k_build_tabs<kTabTc><<<nslots, 256, size_t(dff / 4) * 8, c->stream>>>(c->hidden, 0, dff, c->g_htab, c->g_hgs,
                                                                              nullptr);
        k2<<<dim3(d / 128, E), 256, s2, c->stream>>>(g2);
        return SMOE_OK;
    };
    // the 30B shape (d_model 2048) runs the gate/up kernel with compile-time K
    const bool k30b = d == 2048;
    if (fmt == SMOE_FMT_AFFINE_Q4)
        rc = k30b ? run(k_ffn_grouped<kFmtAffine, 2, kRbGu, kWnGu, 2048>, k_ffn_down_tc<kFmtAffine>)
                  : run(k_ffn_grouped<kFmtAffine, 2, kRbGu, kWnGu, 0>, k_ffn_down_tc<kFmtAffine>);
    else
        rc = k30b ? run(k_ffn_grouped<kFmtSmoe, 2, kRbGu, kWnGu, 2048>, k_ffn_down_tc<kFmtSmoe>)
                  : run(k_ffn_grouped<kFmtSmoe, 2, kRbGu, kWnGu, 0>, k_ffn_down_tc<kFmtSmoe>);
    if (rc) return rc;
    smoe::k_combine_slots<<<dim3((d + 255) / 256, a.ntok), 256, 0, c->stream>>>(c->g_ys, a.wts, a.k, d, a.y,
                                                                               a.y_dtype, shard ? a.ids : nullptr,
                                                                               base, E);
    CK(cudaGetLastError());
    c->dispatches += 6;
    return SMOE_OK;
}

int launch_ffn(SmoeCudaCtx* c, smoe::FfnArgs& a, int fmt) {
    const uint32_t nslots = a.ntok * a.k;
    if (nslots == 0) return SMOE_OK;
    if (nslots > c->cfg.max_batch * 16u) {
        set_err("too many (token, expert) slots %s%ld", "", (long)nslots);
        return SMOE_ERR_ARG;
    }
    a.hidden = c->hidden;
    a.err = c->err;
    const size_t s1 = smoe::gate_up_smem_bytes(a.d_model), s2 = smoe::down_smem_bytes(a.d_ff);
    int rc;
    dim3 g1(a.d_ff / 16, nslots), g2(a.d_model / 16, a.ntok);
    if (fmt == SMOE_FMT_AFFINE_Q4) {
        if ((rc = prep_kernel(c, smoe::k_gate_up<smoe::kFmtAffine>, s1))) return rc;
        if ((rc = prep_kernel(c, smoe::k_down_combine<smoe::kFmtAffine>, s2))) return rc;
        smoe::k_gate_up<smoe::kFmtAffine><<<g1, 256, s1, c->stream>>>(a);
        smoe::k_down_combine<smoe::kFmtAffine><<<g2, 256, s2, c->stream>>>(a);
    } else {
        if ((rc = prep_kernel(c, smoe::k_gate_up<smoe::kFmtSmoe>, s1))) return rc;
        if ((rc = prep_kernel(c, smoe::k_down_combine<smoe::kFmtSmoe>, s2))) return rc;
        smoe::k_gate_up<smoe::kFmtSmoe><<<g1, 256, s1, c->stream>>>(a);
        smoe::k_down_combine<smoe::kFmtSmoe><<<g2, 256, s2, c->stream>>>(a);
    }
    CK(cudaGetLastError());
    c->dispatches += 2;
    return SMOE_OK;
}

// The persistent MoE-layer kernel (moe_layer.cuh): one CTA per SM, all
// resident at once (one CTA fills an SM's shared memory; the grid is the SM
// count), so its grid-wide wait is safe; every wait is bounded anyway.
// Returns SMOE_ERR_UNSUPPORTED when the shape does not fit, so the caller can
// use another path.
struct LayerCall {
    const SmoeMoeLayer* L;       // tiled layer (the experts held here)
    uint32_t n_experts;          // router rows / id bound
    uint32_t expert_base;        // id of the first expert held here
    const void* x; int x_dtype;
    void* y; int y_dtype;
    const uint32_t* ids_in; const float* wts_in;
    uint32_t* ids_out; float* wts_out;
    const uint16_t* rw; int norm;
    uint32_t k, batch;
    const smoe::LayerEp* ep;
};

}  // namespace
namespace smoe {
// One small copy of the caller's x from pinned host memory into device
// scratch, one 16-byte piece per thread. Launched as a programmatic
// dependent: the read over the host link is issued before waiting for the
// previous kernel (which may still read the scratch), and the layer kernel
// that follows may start its set-up at once.
__global__ void k_stage_in(const uint4* __restrict__ src, uint4* __restrict__ dst, uint32_t n16) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (i < n16) v = src[i];
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (i < n16) dst[i] = v;
}
}  // namespace smoe
namespace {

int launch_layer(SmoeCudaCtx* c, const LayerCall& q) {
    const int fmt = int(q.L->fmt & ~uint32_t(SMOE_LAYOUT_TILED));
    if (q.batch > (uint32_t)smoe::kLMaxTok || q.k > (uint32_t)smoe::kLMaxK || q.L->d_ff > c->cfg.max_d_ff ||
        c->num_sms > 32 * smoe::kLRedMax ||
        (q.rw && (q.n_experts > 128u || q.L->d_model % 8)))
        return SMOE_ERR_UNSUPPORTED;
    if (!aligned16(q.x) || (q.y && !aligned16(q.y))) {            // whole-vector loads
        set_err("layer kernel needs 16-byte aligned x and y %s%ld", "", 0);
        return SMOE_ERR_ARG;
    }
    smoe::LayerArgs A{};
    if (!A.g.init(fmt, (int)q.L->d_model, (int)q.L->d_ff, (int)q.k, (int)q.batch, (int)c->smem_optin - 1024))
        return SMOE_ERR_UNSUPPORTED;
    // x and y may be pinned host buffers (as the reference's engine passes
    // them): x is then staged into device scratch by one small copy kernel,
    // and the layer kernel stores y's rows straight into the host buffer -
    // no memcpy in between (a memcpy per call costs several microseconds).
    const void* xin = q.x;
    const int xk = mem_kind(q.x), yk = q.y ? mem_kind(q.y) : 0;
    if (xk == 2 || yk == 2) {
        set_err("layer x / y must be device memory or pinned host memory %s%ld", "", 0);
        return SMOE_ERR_ARG;
    }
    if (xk == 1) {
        const uint32_t n16 = uint32_t(size_t(q.batch) * q.L->d_model * (q.x_dtype == 0 ? 4 : 2) / 16);
        cudaLaunchConfig_t sc{};
        cudaLaunchAttribute sa[1];
        sa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        sa[0].val.programmaticStreamSerializationAllowed = 1;
        sc.gridDim = dim3((n16 + 255) / 256);               // n16 <= 4 x 4096 x 4 / 16: at most 16 CTAs
        sc.blockDim = dim3(256);
        sc.stream = c->stream;
        sc.attrs = sa;
        sc.numAttrs = 1;
        const uint4* xs = static_cast<const uint4*>(q.x);
        uint4* xd = reinterpret_cast<uint4*>(c->in_stage);
        CK(cudaLaunchKernelEx(&sc, smoe::k_stage_in, xs, xd, n16));
        c->dispatches += 1;
        xin = c->in_stage;
    }
    A.base = q.L->base;
    A.stride = q.L->expert_stride;
    A.x = xin; A.x_dtype = q.x_dtype;
    A.y = q.y; A.y_dtype = q.y_dtype;
    A.ids_in = q.ids_in; A.wts_in = q.wts_in;
    A.ids_out = q.ids_out; A.wts_out = q.wts_out;
    A.n_experts = q.n_experts;
    A.rw = q.rw;
    A.norm = q.norm;
    A.logits = c->lpair;
    A.part = c->lpart;
    A.st = c->lstate;
    A.err = c->err;
    A.wait_ns = c->wait_ns;
    A.mg_grid = smoe::magic_of(uint32_t(c->num_sms));
    A.trace = c->trace;
    if (q.ep) {
        A.ep = *q.ep;
    } else {
        A.ep.world = 1;
        A.ep.base = 0;
        A.ep.nlocal = q.n_experts;
    }
    const size_t smem = (size_t)A.g.total;
    const int gw = (int(A.g.tg.Gc) + smoe::kLCons - 1) / smoe::kLCons;   // 1 or 2 (Gc <= 32)
    const int dbi = A.g.d <= 1024 ? 0 : A.g.d <= 2048 ? 1 : 2;           // 64-row blocks per warp: 1, 2, 4
    using smoe::k_moe_layer;
    using smoe::kFmtAffine;
    using smoe::kFmtSmoe;
#define SMOE_LAYER_K(F, G) {(void*)k_moe_layer<F, G, 1>, (void*)k_moe_layer<F, G, 2>, (void*)k_moe_layer<F, G, 4>}
    static void* const kerns[2][2][3] = {{SMOE_LAYER_K(kFmtSmoe, 1), SMOE_LAYER_K(kFmtSmoe, 2)},
                                         {SMOE_LAYER_K(kFmtAffine, 1), SMOE_LAYER_K(kFmtAffine, 2)}};
#undef SMOE_LAYER_K
    void* kern = kerns[fmt == SMOE_FMT_AFFINE_Q4 ? 1 : 0][gw - 1][dbi];
    int rc = prep_kernel(c, kern, smem);
    if (rc) return rc;
    cudaLaunchConfig_t lc{};
    lc.blockDim = dim3(smoe::kLThreads);
    lc.dynamicSmemBytes = smem;
    lc.stream = c->stream;
    lc.gridDim = dim3(c->num_sms);
    // programmatic dependent launch: the kernel's set-up overlaps the
    // previous kernel's tail; it waits for it in griddepcontrol.wait
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    void* args[] = {&A};
    CK(cudaLaunchKernelExC(&lc, kern, args));
    c->dispatches += 1;
    return SMOE_OK;
}

void* record_handle(SmoeCudaCtx* c) {
    const uint64_t s = ++c->seq;
    if (cudaEventRecord(c->events[s % kEventRing], c->stream) != cudaSuccess) {
        set_err("cudaEventRecord failed %s%ld", "", 0);
        return nullptr;
    }
    return reinterpret_cast<void*>(static_cast<uintptr_t>(s));
}

int wait_handle(SmoeCudaCtx* c, void* h) {
    const uint64_t s = reinterpret_cast<uintptr_t>(h);
    if (s == 0 || s > c->seq || c->seq - s >= (uint64_t)kEventRing) {
        set_err("stale or invalid wait handle %s%ld", "", (long)s);
        return SMOE_ERR_ARG;
    }
    return wait_event_bounded(c, c->events[s % kEventRing]);
}

// Copy an activation the caller passed (host or device) into device memory.
const float* stage_input(SmoeCudaCtx* c, const float* in, size_t n) {
    if (is_device_ptr(in)) return in;
    if (cudaMemcpyAsync(c->in_stage, in, n * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return nullptr;
    return c->in_stage;
}

}  // namespace

extern "C" {

const char* smoe_cuda_last_error(void) { return g_err; }

float smoe_cuda_canonical_from_u32(uint32_t w) {
    float r = (float)w / 4294967296.0f;
    if (r >= 1.0f) r = std::nextafter(1.0f, 0.0f);
    return r;
}

SmoeCudaCtx* smoe_cuda_init_ex(const SmoeCudaInitArgs* args) {
    SmoeCudaInitArgs a = args ? *args : SmoeCudaInitArgs{};
    if (!args) cudaGetDevice(&a.device);
    if (!a.max_d_model) a.max_d_model = 8192;
    if (!a.max_d_ff) a.max_d_ff = 4096;
    if (!a.max_experts) a.max_experts = 512;
    if (!a.max_batch) a.max_batch = 256;
    if (!a.max_vocab) a.max_vocab = 262144;
    if (!a.timeout_ms) a.timeout_ms = 10000;
    if (!a.device_wait_us) a.device_wait_us = 1000000;
    if (a.max_experts > (uint32_t)smoe::kRouterMaxE) {
        set_err("max_experts above %s%ld", "", (long)smoe::kRouterMaxE);
        return nullptr;
    }
    auto* c = new (std::nothrow) SmoeCudaCtx();
    if (!c) return nullptr;
    c->device = a.device;
    c->cfg = a;
    c->wait_ns = uint64_t(a.device_wait_us) * 1000u;
    auto fail = [&](cudaError_t e) {
        set_err("init failed: %s (%ld)", cudaGetErrorString(e), 0);
        smoe_cuda_destroy(c);
        return (SmoeCudaCtx*)nullptr;
    };
    cudaError_t e;
    if ((e = cudaSetDevice(a.device)) != cudaSuccess) return fail(e);
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, a.device);
    c->smem_optin = (size_t)optin;
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, a.device);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c->gemv_res[0], smoe::k_gemv_set<1>, smoe::kGemvThreads, 0);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&c->gemv_res[1], smoe::k_gemv_set<2>, smoe::kGemvThreads, 0);
    if (c->gemv_res[0] < 1) c->gemv_res[0] = 1;
    if (c->gemv_res[1] < 1) c->gemv_res[1] = 1;
    if ((e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking)) != cudaSuccess) return fail(e);
    c->stream = c->own_stream;
    const size_t slots = size_t(a.max_batch) * 16;
    if ((e = cudaMalloc(&c->hidden, slots * a.max_d_ff * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->slot_out, size_t(SMOE_MAX_FFN_BATCH) * a.max_d_model * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->batch_out, size_t(SMOE_MAX_FFN_BATCH) * a.max_d_model * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->in_stage, size_t(SMOE_MAX_FFN_BATCH) * a.max_d_model * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->logits, size_t(a.max_batch) * a.max_experts * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->lpair, size_t(smoe::kLMaxTok) * 128 * 8)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->attn_part, size_t(smoe::kAttnMaxHeads) * smoe::kAttnSplits * 258 * 4)) != cudaSuccess)
        return fail(e);
    if ((e = cudaMalloc(&c->attn_cnt, size_t(smoe::kAttnMaxHeads) * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->ids, size_t(a.max_batch) * 16 * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->wts, size_t(a.max_batch) * 16 * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->ticket, size_t(a.max_batch) * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->err, 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->lstate, sizeof(smoe::LayerState))) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->lpart, size_t(c->num_sms) * smoe::kLMaxTok * smoe::kLMaxD * 8)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_list, size_t(a.max_experts) * slots * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_count, size_t(a.max_experts + 1) * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_xtab, size_t(a.max_batch) * a.max_d_model * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_xgs, size_t(a.max_batch) * (a.max_d_model / 64) * 8)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_htab, slots * a.max_d_ff * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_hgs, slots * (a.max_d_ff / 64) * 8)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->g_ys, slots * a.max_d_model * 4)) != cudaSuccess) return fail(e);
    cudaMemsetAsync(c->lstate, 0, sizeof(smoe::LayerState), c->stream);
    cudaMemsetAsync(c->lpair, 0, size_t(smoe::kLMaxTok) * 128 * 8, c->stream);
    cudaMemsetAsync(c->attn_cnt, 0, size_t(smoe::kAttnMaxHeads) * 4, c->stream);
    cudaMemsetAsync(c->lpart, 0, size_t(c->num_sms) * smoe::kLMaxTok * smoe::kLMaxD * 8, c->stream);
    c->gemv_cap = a.max_vocab > a.max_d_model ? a.max_vocab : a.max_d_model;
    if ((e = cudaMalloc(&c->gemv_out, c->gemv_cap * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->gemv_in, size_t(a.max_d_model) * 4)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->blas_ws, kBlasWorkspace)) != cudaSuccess) return fail(e);
    if ((e = cudaMalloc(&c->xsplit, size_t(2) * a.max_batch * a.max_d_model * 2)) != cudaSuccess) return fail(e);
    if (cublasCreate(&c->blas) != CUBLAS_STATUS_SUCCESS ||
        cublasSetWorkspace(c->blas, c->blas_ws, kBlasWorkspace) != CUBLAS_STATUS_SUCCESS) {
        set_err("init failed: cuBLAS handle %s%ld", "", 0);
        smoe_cuda_destroy(c);
        return nullptr;
    }
    cudaMemsetAsync(c->ticket, 0, size_t(a.max_batch) * 4, c->stream);
    cudaMemsetAsync(c->hidden, 0, slots * a.max_d_ff * 4, c->stream);
    cudaMemsetAsync(c->err, 0, 4, c->stream);
    for (auto& ev : c->events)
        if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess) return fail(e);
    if ((e = cudaStreamSynchronize(c->stream)) != cudaSuccess) return fail(e);
    return c;
}

SmoeCudaCtx* smoe_cuda_init(size_t slot_bytes) {
    (void)slot_bytes;
    SmoeCudaInitArgs a{};
    cudaGetDevice(&a.device);
    return smoe_cuda_init_ex(&a);
}

void smoe_cuda_destroy(SmoeCudaCtx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->own_stream) cudaStreamSynchronize(c->own_stream);
    if (c->blas) cublasDestroy(c->blas);
    for (int r = 0; r < smoe::kEpMaxWorld; ++r)
        if (c->ep_peer[r] && c->ep_peer[r] != c->ep_win) cudaIpcCloseMemHandle(c->ep_peer[r]);
    if (c->ep_win) cudaFree(c->ep_win);
    for (auto& ev : c->events)
        if (ev) cudaEventDestroy(ev);
    void* bufs[] = {c->g_list, c->g_count, c->g_xtab, c->g_xgs, c->g_htab, c->g_hgs, c->g_ys, c->lstate, c->lpair, c->lpart, c->attn_part, c->attn_cnt, c->hidden, c->slot_out, c->in_stage, c->batch_out, c->logits, c->ids,
                    c->wts, c->ticket, c->err, c->gemv_out, c->gemv_in, c->blas_ws, c->xsplit};
    for (void* b : bufs)
        if (b) cudaFree(b);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

int smoe_cuda_set_stream(SmoeCudaCtx* c, void* s) {
    if (!c) return SMOE_ERR_ARG;
    c->stream = s ? static_cast<cudaStream_t>(s) : c->own_stream;
    return SMOE_OK;
}

void* smoe_cuda_get_stream(SmoeCudaCtx* c) { return c ? c->stream : nullptr; }

int smoe_cuda_synchronize(SmoeCudaCtx* c) {
    if (!c) return SMOE_ERR_ARG;
    cudaEvent_t ev = c->events[(c->seq + 1) % kEventRing];
    ++c->seq;
    CK(cudaEventRecord(ev, c->stream));
    int rc = wait_event_bounded(c, ev);
    if (rc) return rc;
    return check_device_err(c);
}

uint64_t smoe_cuda_kernel_dispatches(const SmoeCudaCtx* c) { return c ? c->dispatches.load() : 0; }

}  // extern "C"

namespace smoe {
__global__ void k_expf_ref(const float* x, float* y, uint32_t n) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = expf_ref(x[i]);
}
}  // namespace smoe

extern "C" {

// Test aid, not part of the public header: the sampler's e = expf(x)
// (expf_ref of sampler.cuh) over n device floats, on `stream`.
int smoe_cuda_debug_expf(const float* x, float* y, uint32_t n, void* stream) {
    if (!x || !y) return SMOE_ERR_ARG;
    const uint32_t blocks = n / 256 + 1 < 148u * 16u ? n / 256 + 1 : 148u * 16u;
    smoe::k_expf_ref<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
    return cudaGetLastError() == cudaSuccess ? SMOE_OK : SMOE_ERR_CUDA;
}

// Profiling aid, not part of the public header: record per-CTA phase
// timestamps of the fused layer kernel into `buf` ([num_SMs x 8] u64, device;
// NULL turns it off).
int smoe_cuda_debug_trace(SmoeCudaCtx* c, void* buf) {
    if (!c) return SMOE_ERR_ARG;
    c->trace = static_cast<unsigned long long*>(buf);
    return SMOE_OK;
}

void smoe_cuda_register_buffer(SmoeCudaCtx* c, const void* p, size_t n) {
    if (!c || !p || !n || is_device_ptr(p)) return;
    if (cudaHostRegister(const_cast<void*>(p), n, cudaHostRegisterDefault) != cudaSuccess)
        cudaGetLastError();   // already registered or not registrable: copies still work
}

}  // extern "C"

// ------------------------------------------------------ mirrored entries
namespace {

// Pointer-mode FfnArgs for SMOE-Q4 expert column j.
bool set_ptr_expert(smoe::FfnArgs& a, int j, const uint8_t* pg, const uint16_t* sg,
                    const uint8_t* pu, const uint16_t* su, const uint8_t* pd, const uint16_t* sd) {
    const void* ps[6] = {pg, sg, pu, su, pd, sd};
    for (const void* p : ps)
        if (!p || !aligned16(p)) return false;
    a.p_nib[j][0] = pg; a.p_sc[j][0] = sg; a.p_bi[j][0] = sg;
    a.p_nib[j][1] = pu; a.p_sc[j][1] = su; a.p_bi[j][1] = su;
    a.p_nib[j][2] = pd; a.p_sc[j][2] = sd; a.p_bi[j][2] = sd;
    return true;
}

int mirror_check(SmoeCudaCtx* c, uint32_t gate_rows, uint32_t gate_cols, uint32_t down_rows,
                 uint32_t down_cols, uint32_t group_size, uint32_t bits) {
    if (!c) { set_err("null context %s%ld", "", 0); return SMOE_ERR_ARG; }
    if (bits != 4 || group_size != 64) {
        set_err("only SMOE-Q4 with group 64 is implemented (bits %s%ld)", "", (long)bits);
        return SMOE_ERR_UNSUPPORTED;
    }
    if (down_rows != gate_cols || down_cols != gate_rows) {
        set_err("inconsistent FFN dims %s%ld", "", (long)down_rows);
        return SMOE_ERR_ARG;
    }
    return check_ffn_dims(c, gate_cols, gate_rows);
}

}  // namespace

extern "C" {

void* smoe_cuda_fused_ffn(SmoeCudaCtx* c, const uint8_t* pg, const uint16_t* sg,
                          const uint8_t* pu, const uint16_t* su, const uint8_t* pd,
                          const uint16_t* sd, const float* input_vec, float* hidden_vec,
                          float* output_vec, uint32_t gate_rows, uint32_t gate_cols,
                          uint32_t down_rows, uint32_t down_cols, uint32_t group_size,
                          uint32_t bits, uint32_t expert_index) {
    (void)hidden_vec;
    (void)output_vec;   // fetched by smoe_cuda_wait, as the reference does
    SmoeExpertBlob b{pg, sg, pu, su, pd, sd, expert_index};
    return smoe_cuda_fused_ffn_group(c, &b, 1, input_vec, gate_rows, gate_cols, down_rows,
                                     down_cols, group_size, bits);
}

void* smoe_cuda_fused_ffn_group(SmoeCudaCtx* c, const SmoeExpertBlob* ex, uint32_t n,
                                const float* input_vec, uint32_t gate_rows, uint32_t gate_cols,
                                uint32_t down_rows, uint32_t down_cols, uint32_t group_size,
                                uint32_t bits) {
    if (mirror_check(c, gate_rows, gate_cols, down_rows, down_cols, group_size, bits)) return nullptr;
    if (!ex || n == 0 || n > SMOE_MAX_ACTIVE) {
        set_err("bad expert group size %s%ld", "", (long)n);
        return nullptr;
    }
    smoe::FfnArgs a{};
    // slots are laid out by column; the per-slot output goes to slot_out[slot]
    // so the caller's `slot` numbering is honoured by a final scatter.
    uint32_t maxslot = 0;
    for (uint32_t j = 0; j < n; ++j) {
        if (!set_ptr_expert(a, j, ex[j].packed_gate, ex[j].scales_gate, ex[j].packed_up,
                            ex[j].scales_up, ex[j].packed_down, ex[j].scales_down)) {
            set_err("null or unaligned expert pointer (expert %s%ld)", "", (long)j);
            return nullptr;
        }
        if (ex[j].slot >= SMOE_MAX_FFN_BATCH - SMOE_MAX_ACTIVE) {
            set_err("slot out of range %s%ld", "", (long)ex[j].slot);
            return nullptr;
        }
        if (ex[j].slot > maxslot) maxslot = ex[j].slot;
    }
    const float* x = stage_input(c, input_vec, gate_cols);
    if (!x) { set_err("input copy failed %s%ld", "", 0); return nullptr; }
    a.x = x;
    a.x_dtype = SMOE_DTYPE_F32;
    a.per_slot = 1;
    a.d_model = gate_cols;
    a.d_ff = gate_rows;
    a.k = n;
    a.ntok = 1;
    // kernel writes column j to slot_out + (64 - 16 + j) rows region, then we
    // move each to the caller's slot (device-to-device, tiny).
    float* tmp = c->slot_out + size_t(SMOE_MAX_FFN_BATCH - SMOE_MAX_ACTIVE) * c->cfg.max_d_model;
    a.y = tmp;
    // per-slot output rows are d_model apart
    if (launch_ffn(c, a, SMOE_FMT_SMOE_Q4)) return nullptr;
    for (uint32_t j = 0; j < n; ++j) {
        if (cudaMemcpyAsync(c->slot_out + size_t(ex[j].slot) * c->cfg.max_d_model,
                            tmp + size_t(j) * gate_cols, size_t(gate_cols) * 4,
                            cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess) {
            set_err("slot scatter failed %s%ld", "", 0);
            return nullptr;
        }
    }
    return record_handle(c);
}

void smoe_cuda_wait(SmoeCudaCtx* c, void* h, float* out, uint32_t slot, uint32_t cols) {
    if (!c || !out || slot >= SMOE_MAX_FFN_BATCH - SMOE_MAX_ACTIVE || cols > c->cfg.max_d_model) {
        set_err("bad wait arguments %s%ld", "", (long)slot);
        return;
    }
    if (wait_handle(c, h)) return;
    if (cudaMemcpy(out, c->slot_out + size_t(slot) * c->cfg.max_d_model, size_t(cols) * 4,
                   cudaMemcpyDefault) != cudaSuccess)
        set_err("output copy failed %s%ld", "", 0);
}

void* smoe_cuda_fused_ffn_batch(SmoeCudaCtx* c, const uint8_t* pg, const uint16_t* sg,
                                const uint8_t* pu, const uint16_t* su, const uint8_t* pd,
                                const uint16_t* sd, const float* input_mat, uint32_t batch,
                                uint32_t gate_rows, uint32_t gate_cols, uint32_t down_rows,
                                uint32_t down_cols, uint32_t group_size, uint32_t bits) {
    if (mirror_check(c, gate_rows, gate_cols, down_rows, down_cols, group_size, bits)) return nullptr;
    if (batch == 0 || batch > SMOE_MAX_FFN_BATCH || gate_cols > SMOE_MAX_FFN_BATCH_DIM ||
        gate_rows > SMOE_MAX_FFN_BATCH_DIM) {
        set_err("batch/dims exceed the staging limits %s%ld", "", (long)batch);
        return nullptr;
    }
    smoe::FfnArgs a{};
    if (!set_ptr_expert(a, 0, pg, sg, pu, su, pd, sd)) {
        set_err("null or unaligned expert pointer %s%ld", "", 0);
        return nullptr;
    }
    const float* x = stage_input(c, input_mat, size_t(batch) * gate_cols);
    if (!x) { set_err("input copy failed %s%ld", "", 0); return nullptr; }
    a.x = x;
    a.x_dtype = SMOE_DTYPE_F32;
    a.per_slot = 1;
    a.d_model = gate_cols;
    a.d_ff = gate_rows;
    a.k = 1;
    a.ntok = batch;
    a.y = c->batch_out;           // [batch x d_model], contiguous
    if (launch_ffn(c, a, SMOE_FMT_SMOE_Q4)) return nullptr;
    return record_handle(c);
}

void smoe_cuda_wait_ffn_batch(SmoeCudaCtx* c, void* h, float* out, uint32_t batch, uint32_t cols) {
    if (!c || !out || batch > SMOE_MAX_FFN_BATCH || cols > c->cfg.max_d_model) {
        set_err("bad wait arguments %s%ld", "", (long)batch);
        return;
    }
    if (wait_handle(c, h)) return;
    if (cudaMemcpy(out, c->batch_out, size_t(batch) * cols * 4, cudaMemcpyDefault) != cudaSuccess)
        set_err("output copy failed %s%ld", "", 0);
}

}  // extern "C"

namespace {
// One bf16 GEMV of the mirrored entries, asynchronous: host or device input
// and output (host ones are staged through the context's buffers, in stream
// order, so consecutive calls may reuse them).
int matvec_one(SmoeCudaCtx* c, const uint16_t* w, const float* in, float* out, uint32_t rows, uint32_t cols) {
    if (!c || !w || !in || !out || cols == 0 || cols % 8 || cols > c->cfg.max_d_model || !aligned16(w)) {
        set_err("bad matvec arguments %s%ld", "", (long)cols);
        return SMOE_ERR_ARG;
    }
    const bool out_dev = is_device_ptr(out);
    if (!out_dev && rows > c->gemv_cap) {
        set_err("matvec rows exceed staging %s%ld", "", (long)rows);
        return SMOE_ERR_ARG;
    }
    const float* x = in;
    if (!is_device_ptr(in)) {
        CK(cudaMemcpyAsync(c->gemv_in, in, size_t(cols) * 4, cudaMemcpyHostToDevice, c->stream));
        x = c->gemv_in;
    }
    float* y = out_dev ? out : c->gemv_out;
    const uint32_t blocks = (rows + 7) / 8 < 148u * 8u ? (rows + 7) / 8 : 148u * 8u;
    const size_t smem = size_t(cols) * 4;
    int rc = prep_kernel(c, smoe::k_gemv_bf16, smem);
    if (rc) return rc;
    smoe::k_gemv_bf16<<<blocks, 256, smem, c->stream>>>(w, x, y, rows, cols);
    CK(cudaGetLastError());
    c->dispatches += 1;
    if (!out_dev) CK(cudaMemcpyAsync(out, y, size_t(rows) * 4, cudaMemcpyDeviceToHost, c->stream));
    return SMOE_OK;
}
}  // namespace

extern "C" {

void smoe_cuda_scout_matvec_bf16(SmoeCudaCtx* c, const uint16_t* w, const float* in, float* out,
                                 uint32_t rows, uint32_t cols) {
    if (matvec_one(c, w, in, out, rows, cols) == SMOE_OK)
        smoe_cuda_synchronize(c);   // synchronous, as metal_bridge.h:157
}

// metal_bridge.h:199-206: dispatch i may read what an earlier one wrote; the
// context's single stream orders them.
void smoe_cuda_scout_matvec_batch_bf16(SmoeCudaCtx* c, const uint16_t** weights, const float** inputs,
                                       float** outputs, const uint32_t* rows, const uint32_t* cols,
                                       uint32_t count) {
    if (!c || (count && (!weights || !inputs || !outputs || !rows || !cols))) {
        set_err("bad matvec batch arguments %s%ld", "", (long)count);
        return;
    }
    for (uint32_t i = 0; i < count; ++i)
        if (matvec_one(c, weights[i], inputs[i], outputs[i], rows[i], cols[i]) != SMOE_OK) return;
    smoe_cuda_synchronize(c);
}

// metal_bridge.h:212-219: the caller guarantees distinct outputs that no
// dispatch reads, so no ordering between them is needed; on one stream they
// run back to back (each kernel fills the GPU on its own at these sizes).
void smoe_cuda_scout_matvec_group_bf16(SmoeCudaCtx* c, const uint16_t** weights, const float** inputs,
                                       float** outputs, const uint32_t* rows, const uint32_t* cols,
                                       uint32_t count) {
    smoe_cuda_scout_matvec_batch_bf16(c, weights, inputs, outputs, rows, cols, count);
}

// ------------------------------------------------------- native entries
int smoe_cuda_router_topk(SmoeCudaCtx* c, const uint16_t* w, const void* x, int x_dtype,
                          uint32_t E, uint32_t d, uint32_t batch, uint32_t k, int norm,
                          uint32_t* ids, float* wts, float* logits) {
    if (!c || !w || !x || !ids || !wts) { set_err("null argument %s%ld", "", 0); return SMOE_ERR_ARG; }
    if (E == 0 || E > c->cfg.max_experts || d % 8 || d > c->cfg.max_d_model || k == 0 ||
        k > SMOE_MAX_ACTIVE || k > E || batch == 0 || batch > c->cfg.max_batch ||
        (x_dtype != 0 && x_dtype != 1) || !aligned16(w)) {
        set_err("bad router arguments %s%ld", "", (long)E);
        return SMOE_ERR_ARG;
    }
    smoe::RouterArgs a{w, x, x_dtype, E, d, k, norm, logits ? logits : c->logits, ids, wts,
                       c->ticket, c->err};
    const size_t smem = size_t(d) * 4;
    if (batch >= 16) {                     // one CTA per token (x staged once per token)
        int rc = prep_kernel(c, smoe::k_router_tok, smem);
        if (rc) return rc;
        smoe::k_router_tok<<<batch, 512, smem, c->stream>>>(a);
    } else {                               // rows spread over CTAs (latency at small batch)
        int rc = prep_kernel(c, smoe::k_router, smem);
        if (rc) return rc;
        dim3 g((E + smoe::kRouterRowsPerCta - 1) / smoe::kRouterRowsPerCta, batch);
        smoe::k_router<<<g, 256, smem, c->stream>>>(a);
    }
    CK(cudaGetLastError());
    c->dispatches += 1;
    return SMOE_OK;
}

static int layer_args(SmoeCudaCtx* c, const SmoeMoeLayer* L, smoe::FfnArgs& a) {
    const uint32_t fmt = L ? (L->fmt & ~uint32_t(SMOE_LAYOUT_TILED)) : 99u;
    if (!L || !L->base || (fmt != SMOE_FMT_SMOE_Q4 && fmt != SMOE_FMT_AFFINE_Q4) ||
        L->expert_stride % 16 || !aligned16(L->base)) {
        set_err("bad layer descriptor %s%ld", "", 0);
        return SMOE_ERR_ARG;
    }
    for (int i = 0; i < 9; ++i)
        if (L->off[i] % 16) { set_err("unaligned blob offset %s%ld", "", (long)i); return SMOE_ERR_ARG; }
    int rc = check_ffn_dims(c, L->d_model, L->d_ff);
    if (rc) return rc;
    a.base = L->base;
    a.stride = L->expert_stride;
    for (int i = 0; i < 9; ++i) a.off[i] = L->off[i];
    a.d_model = L->d_model;
    a.d_ff = L->d_ff;
    return SMOE_OK;
}

int smoe_cuda_moe_ffn(SmoeCudaCtx* c, const SmoeMoeLayer* L, const void* x, int x_dtype,
                      const uint32_t* ids, const float* wts, uint32_t k, uint32_t batch,
                      void* y, int y_dtype) {
    if (!c || !x || !ids || !wts || !y) { set_err("null argument %s%ld", "", 0); return SMOE_ERR_ARG; }
    smoe::FfnArgs a{};
    int rc = layer_args(c, L, a);
    if (rc) return rc;
    if (k == 0 || k > SMOE_MAX_ACTIVE || batch == 0 || batch > c->cfg.max_batch ||
        (x_dtype != 0 && x_dtype != 1) || (y_dtype != 0 && y_dtype != 1)) {
        set_err("bad moe_ffn arguments %s%ld", "", (long)k);
        return SMOE_ERR_ARG;
    }
    a.ids = ids;
    a.wts = wts;
    a.x = x;
    a.x_dtype = x_dtype;
    a.y = y;
    a.y_dtype = y_dtype;
    a.per_slot = 0;
    a.k = k;
    a.ntok = batch;
    a.n_experts = L->n_experts;
    const int fmt = int(L->fmt & ~uint32_t(SMOE_LAYOUT_TILED));
    if (L->fmt & SMOE_LAYOUT_TILED) {
        LayerCall q{};
        q.L = L; q.n_experts = L->n_experts;
        q.x = x; q.x_dtype = x_dtype; q.y = y; q.y_dtype = y_dtype;
        q.ids_in = ids; q.wts_in = wts; q.k = k; q.batch = batch;
        rc = launch_layer(c, q);
        if (rc == SMOE_ERR_UNSUPPORTED)
            set_err("tiled layout needs batch <= 4 and a shape whose tiles fit shared memory %s%ld", "", (long)batch);
        return rc;
    }
    // token batches: expert-grouped path (shapes whose tiles it covers)
    if (batch > uint32_t(smoe::kLMaxTok) && L->d_model % 128 == 0 && L->d_ff % 256 == 0 && L->d_ff <= 4096)
        return launch_grouped(c, a, fmt, L->n_experts);
    return launch_ffn(c, a, fmt);
}

int smoe_cuda_moe_layer_shard(SmoeCudaCtx* c, const SmoeMoeLayer* shard, uint32_t n_experts_total,
                              uint32_t expert_base, const void* x, int x_dtype, uint32_t batch, uint32_t k,
                              int norm, float* y_partial, uint32_t* ids_out, float* w_out) {
    if (!c || !shard || !x || !y_partial) { set_err("null argument %s%ld", "", 0); return SMOE_ERR_ARG; }
    smoe::FfnArgs a{};
    int rc = layer_args(c, shard, a);
    if (rc) return rc;
    if ((shard->fmt & SMOE_LAYOUT_TILED) || !shard->router_w || shard->n_experts == 0 ||
        expert_base + shard->n_experts > n_experts_total || k == 0 || k > SMOE_MAX_ACTIVE || batch == 0 ||
        batch > c->cfg.max_batch || (x_dtype != 0 && x_dtype != 1) || shard->d_model % 128 ||
        shard->d_ff % 256 || shard->d_ff > 4096) {
        set_err("bad layer shard (vault layout, d_model %% 128, d_ff %% 256, experts within the layer) %s%ld", "",
                (long)expert_base);
        return SMOE_ERR_ARG;
    }
    uint32_t* ids = ids_out ? ids_out : c->ids;
    float* wts = w_out ? w_out : c->wts;
    // every rank routes over the whole router (identical ids on every rank)
    if ((rc = smoe_cuda_router_topk(c, shard->router_w, x, x_dtype, n_experts_total, shard->d_model, batch, k, norm,
                                    ids, wts, nullptr)))
        return rc;
    a.ids = ids;
    a.wts = wts;
    a.x = x;
    a.x_dtype = x_dtype;
    a.y = y_partial;
    a.y_dtype = 0;
    a.per_slot = 0;
    a.k = k;
    a.ntok = batch;
    a.n_experts = n_experts_total;
    return launch_grouped(c, a, int(shard->fmt), shard->n_experts, expert_base, n_experts_total);
}

int smoe_cuda_moe_layer(SmoeCudaCtx* c, const SmoeMoeLayer* L, const void* x, int x_dtype,
                        uint32_t batch, uint32_t k, int norm, void* y, int y_dtype,
                        uint32_t* ids_out, float* w_out) {
    if (!c || !L) { set_err("null argument %s%ld", "", 0); return SMOE_ERR_ARG; }
    uint32_t* ids = ids_out ? ids_out : c->ids;
    float* wts = w_out ? w_out : c->wts;
    // the layer kernel routes in-kernel up to 128 experts (larger routers:
    // k_router first, then the layer kernel with the routing given)
    if ((L->fmt & SMOE_LAYOUT_TILED) && L->router_w && x && y &&
        aligned16(L->router_w) && L->n_experts >= k && k > 0 && k <= SMOE_MAX_ACTIVE &&
        L->n_experts <= 128u && L->n_experts <= c->cfg.max_experts && (x_dtype == 0 || x_dtype == 1) &&
        (y_dtype == 0 || y_dtype == 1)) {
        smoe::FfnArgs a{};
        int rc = layer_args(c, L, a);
        if (rc) return rc;
        LayerCall q{};
        q.L = L; q.n_experts = L->n_experts;
        q.x = x; q.x_dtype = x_dtype; q.y = y; q.y_dtype = y_dtype;
        q.ids_out = ids; q.wts_out = wts;
        q.rw = L->router_w; q.norm = norm; q.k = k; q.batch = batch;
        rc = launch_layer(c, q);
        if (rc == SMOE_ERR_UNSUPPORTED)
            set_err("tiled layout needs batch <= 4 and a shape whose tiles fit shared memory %s%ld", "", (long)batch);
        return rc;
    }
    int rc = smoe_cuda_router_topk(c, L->router_w, x, x_dtype, L->n_experts, L->d_model, batch,
                                   k, norm, ids, wts, nullptr);
    if (rc) return rc;
    return smoe_cuda_moe_ffn(c, L, x, x_dtype, ids, wts, k, batch, y, y_dtype);
}

// ------------------------------------------------------- dense trunk (decode)
namespace {
// Launch a trunk kernel with programmatic stream serialization: it may start
// while its predecessor drains, and waits for it in pdl_wait().
extern "C++" template <typename... KArgs, typename... Args>
int pdl_launch_smem(SmoeCudaCtx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
    cudaLaunchConfig_t lc{};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = c->stream;
    lc.attrs = at;
    lc.numAttrs = 1;
    c->dispatches += 1;
    return cudaLaunchKernelEx(&lc, kern, KArgs(args)...) == cudaSuccess ? SMOE_OK : SMOE_ERR_CUDA;
}

extern "C++" template <typename... KArgs, typename... Args>
int pdl_launch(SmoeCudaCtx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, Args... args) {
    cudaLaunchConfig_t lc{};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = 0;
    lc.stream = c->stream;
    lc.attrs = at;
    lc.numAttrs = 1;
    c->dispatches += 1;
    return cudaLaunchKernelEx(&lc, kern, KArgs(args)...) == cudaSuccess ? SMOE_OK : SMOE_ERR_CUDA;
}

int gemv_set(SmoeCudaCtx* c, const smoe::GemvSet& g) {
    uint32_t total = 0;
    for (uint32_t m = 0; m < g.nmat; ++m) {
        if (!g.w[m] || !g.y[m] || !aligned16(g.w[m])) { set_err("bad matvec operand %s%ld", "", (long)m); return SMOE_ERR_ARG; }
        total += g.rows[m];
    }
    if (!g.x || g.cols == 0 || g.cols % 8 || g.cols > 16384) { set_err("bad matvec cols %s%ld", "", (long)g.cols); return SMOE_ERR_ARG; }
    if (!aligned16(g.x)) { set_err("matvec input must be 16-byte aligned %s%ld", "", 0); return SMOE_ERR_ARG; }
    // One warp per row while every row's warp fits in one wave of resident
    // CTAs (all weight loads in flight at once); two rows per warp beyond
    // that, and grid-stride only past two rows per resident warp. (A second
    // partial wave costs a whole DRAM round trip: 5120 x 2048 rows at one per
    // warp took 8.6 us against 5.2 us for 4096.)
    const uint32_t warps = smoe::kGemvThreads / 32;
    const uint32_t cap1 = uint32_t(c->num_sms) * uint32_t(c->gemv_res[0]);
    const uint32_t cap2 = uint32_t(c->num_sms) * uint32_t(c->gemv_res[1]);
    const bool pair = total > cap1 * warps;
    const uint32_t units = pair ? (total + 1) / 2 : total;
    const uint32_t want = (units + warps - 1) / warps, cap = pair ? cap2 : cap1;
    auto kern = pair ? smoe::k_gemv_set<2> : (g.cols > 2048 ? smoe::k_gemv_set<1, 16> : smoe::k_gemv_set<1>);
    return pdl_launch(c, kern, dim3(want < cap ? want : cap), dim3(smoe::kGemvThreads), g, total);
}
}  // namespace

int smoe_cuda_matvec_bf16(SmoeCudaCtx* c, const uint16_t* w, const float* x, float* y, uint32_t rows,
                          uint32_t cols) {
    if (!c) { set_err("null context %s%ld", "", 0); return SMOE_ERR_ARG; }
    smoe::GemvSet g{};
    g.w[0] = w;
    g.y[0] = y;
    g.rows[0] = rows;
    g.nmat = 1;
    g.cols = cols;
    g.x = x;
    return gemv_set(c, g);
}

int smoe_cuda_rms_norm(SmoeCudaCtx* c, float* hidden, const float* delta, const uint16_t* w, float* normed,
                       uint32_t n, uint32_t rows) {
    if (!c || !hidden || !w || !normed || n == 0 || rows == 0) { set_err("bad rms_norm arguments %s%ld", "", (long)n); return SMOE_ERR_ARG; }
    return pdl_launch(c, smoe::k_add_rms_norm, dim3(rows), dim3(1024), hidden, delta, w, normed, n);
}

int smoe_cuda_embed_bf16(SmoeCudaCtx* c, const uint16_t* table, const uint32_t* tokens, uint32_t n_tokens,
                         uint32_t d_model, float* out) {
    if (!c || !table || !tokens || !out || n_tokens == 0 || d_model == 0) { set_err("bad embed arguments %s%ld", "", 0); return SMOE_ERR_ARG; }
    return pdl_launch(c, smoe::k_embed, dim3((d_model + 255) / 256, n_tokens), dim3(256), table, tokens, d_model,
                      out);
}

int smoe_cuda_rope_table(SmoeCudaCtx* c, const uint32_t* pos, const float* inv_freq, float* cos_out,
                         float* sin_out, uint32_t half) {
    if (!c || !pos || !inv_freq || !cos_out || !sin_out || half == 0) { set_err("bad rope arguments %s%ld", "", 0); return SMOE_ERR_ARG; }
    return pdl_launch(c, smoe::k_rope_table, dim3((half + 127) / 128), dim3(128), pos, inv_freq, cos_out, sin_out,
                      half);
}

int smoe_cuda_decode_advance(SmoeCudaCtx* c, SmoeSamplerRow* row, uint32_t* history, uint32_t hcap,
                             const uint32_t* token, uint32_t* pos, const float* u_seq, uint32_t u_len) {
    if (!c || !row || !token || !pos || (hcap && !history)) { set_err("bad decode_advance arguments %s%ld", "", 0); return SMOE_ERR_ARG; }
    static_assert(sizeof(SmoeSamplerRow) == sizeof(smoe::SamplerRowDevMut), "row layout");
    return pdl_launch(c, smoe::k_decode_advance, dim3(1), dim3(32),
                      reinterpret_cast<smoe::SamplerRowDevMut*>(row), history, hcap, token, pos, u_seq, u_len);
}

int smoe_cuda_attention_layer_async(SmoeCudaCtx* c, const SmoeCudaAttnLayerArgs* a, const uint32_t* pos) {
    if (!c || !a || !a->w_q || !a->w_k || !a->w_v || !a->w_o || !a->rope_cos || !a->rope_sin ||
        !a->normed_in || !a->qbuf || !a->kbuf || !a->vbuf || !a->k_cache || !a->v_cache || !a->attn_out ||
        !a->o_out || a->head_dim == 0 || a->head_dim > 256 || a->head_dim % 32 || a->num_kv_heads == 0 ||
        a->num_heads % a->num_kv_heads || a->q_dim != a->num_heads * a->head_dim ||
        a->kv_dim != a->num_kv_heads * a->head_dim || a->attn_ctx == 0 || a->attn_ctx > smoe::kAttnMaxCtx ||
        a->num_heads > (uint32_t)smoe::kAttnMaxHeads ||
        (!pos && (a->valid == 0 || a->valid > a->attn_ctx || a->slot >= a->attn_ctx))) {
        set_err("bad attention-layer arguments %s%ld", "", 0);
        return SMOE_ERR_ARG;
    }
    // 1. Q, K, V projections of the normed input (one launch)
    smoe::GemvSet g{};
    g.w[0] = a->w_q; g.y[0] = a->qbuf; g.rows[0] = a->q_dim;
    g.w[1] = a->w_k; g.y[1] = a->kbuf; g.rows[1] = a->kv_dim;
    g.w[2] = a->w_v; g.y[2] = a->vbuf; g.rows[2] = a->kv_dim;
    g.nmat = 3;
    g.cols = a->d_model;
    g.x = a->normed_in;
    int rc = gemv_set(c, g);
    if (rc) return rc;
    // 2. per-head QK norm + RoPE, ring append; 3. attention
    smoe::AttnArgs t{};
    t.q = a->qbuf; t.k = a->kbuf; t.v = a->vbuf;
    t.q_norm_w = a->q_norm_w; t.k_norm_w = a->k_norm_w;
    t.rope_cos = a->rope_cos; t.rope_sin = a->rope_sin;
    t.qbuf = a->qbuf; t.kbuf = a->kbuf; t.vbuf = a->vbuf;
    t.k_cache = a->k_cache; t.v_cache = a->v_cache;
    t.attn_out = a->attn_out;
    t.q_dim = a->q_dim; t.kv_dim = a->kv_dim; t.head_dim = a->head_dim;
    t.num_heads = a->num_heads; t.num_kv_heads = a->num_kv_heads;
    t.slot = a->slot; t.valid = a->valid; t.attn_ctx = a->attn_ctx;
    t.pos = pos;
    t.scale = a->attn_scale;
    t.part = c->attn_part;
    t.cnt = c->attn_cnt;
    // positions split over up to kAttnSplits CTAs per head (>= 32 positions of the ring each)
    const uint32_t splits = std::min<uint32_t>(smoe::kAttnSplits, (a->attn_ctx + 31) / 32);
    rc = pdl_launch(c, smoe::k_attn_decode, dim3(a->num_heads, splits), dim3(smoe::kAttnThreads), t);
    if (rc) return rc;
    // 4. O projection
    smoe::GemvSet o{};
    o.w[0] = a->w_o; o.y[0] = a->o_out; o.rows[0] = a->d_model;
    o.nmat = 1;
    o.cols = a->q_dim;
    o.x = a->attn_out;
    return gemv_set(c, o);
}

namespace {
// X [batch x cols] fp32 -> the two bf16 planes in c->xsplit
int split_planes(SmoeCudaCtx* c, const float* x, size_t n) {
    const size_t blocks = (n + 1023) / 1024;
    return pdl_launch(c, smoe::k_split_bf16, dim3(unsigned(blocks < 1184 ? blocks : 1184)), dim3(1024), x,
                      c->xsplit, n);
}

// Y = W X over the planes already in c->xsplit (n = batch * cols).
// cuBLAS is column-major: row-major W [rows x cols] is A = W^T (cols x rows,
// ld cols), X [batch x cols] is B = X^T (cols x batch, ld cols) and Y [batch
// x rows] is C = Y^T (rows x batch, ld rows); C = A^T B, hi plane then lo
// plane accumulated.
int gemm_planes(SmoeCudaCtx* c, const uint16_t* w, float* y, uint32_t rows, uint32_t cols, uint32_t batch) {
    if (!w || !y || rows == 0 || !aligned16(w)) {
        set_err("bad batched matvec operand %s%ld", "", (long)rows);
        return SMOE_ERR_ARG;
    }
    if (cublasSetStream(c->blas, c->stream) != CUBLAS_STATUS_SUCCESS) {
        set_err("cuBLAS stream %s%ld", "", 0);
        return SMOE_ERR_CUDA;
    }
    const size_t n = size_t(batch) * cols;
    const float one = 1.0f, zero = 0.0f;
    for (int plane = 0; plane < 2; ++plane) {
        const cublasStatus_t st = cublasGemmEx(
            c->blas, CUBLAS_OP_T, CUBLAS_OP_N, int(rows), int(batch), int(cols), &one, w, CUDA_R_16BF, int(cols),
            c->xsplit + plane * n, CUDA_R_16BF, int(cols), plane ? &one : &zero, y, CUDA_R_32F, int(rows),
            CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        if (st != CUBLAS_STATUS_SUCCESS) {
            set_err("cuBLAS GEMM failed %s(status %ld)", "", (long)st);
            return SMOE_ERR_CUDA;
        }
        c->dispatches += 1;
    }
    return SMOE_OK;
}

bool gemm_shape_ok(const SmoeCudaCtx* c, const float* x, uint32_t cols, uint32_t batch) {
    return x && cols && cols % 8 == 0 && batch && batch <= c->cfg.max_batch && cols <= c->cfg.max_d_model;
}
}  // namespace

namespace {
// positions per score block of the GQA attention kernel (shared memory
// [G][blk] floats): the whole ring up to 1024 positions
uint32_t gqa_block(uint32_t attn_ctx) { return attn_ctx < 1024u ? attn_ctx : 1024u; }
size_t gqa_smem_bytes(uint32_t G, uint32_t hd, uint32_t blk) {
    return (size_t(G + 2) * hd + size_t(G) * blk + size_t(smoe::kAttnThreads / 32) * G * hd) * 4;
}
}  // namespace

int smoe_cuda_gemm_bf16(SmoeCudaCtx* c, const uint16_t* w, const float* x, float* y, uint32_t rows,
                        uint32_t cols, uint32_t batch) {
    if (!c) { set_err("null context %s%ld", "", 0); return SMOE_ERR_ARG; }
    if (batch == 1) return smoe_cuda_matvec_bf16(c, w, x, y, rows, cols);
    if (!w || !y || rows == 0 || !aligned16(w) || !gemm_shape_ok(c, x, cols, batch)) {
        set_err("bad batched matvec arguments %s%ld", "", (long)batch);
        return SMOE_ERR_ARG;
    }
    int rc = split_planes(c, x, size_t(batch) * cols);
    if (rc) return rc;
    return gemm_planes(c, w, y, rows, cols, batch);
}

int smoe_cuda_attention_batch_async(SmoeCudaCtx* c, const SmoeCudaAttnLayerArgs* a, uint32_t batch,
                                    uint64_t kv_seq_stride, const uint32_t* pos) {
    if (!c || !a || !pos || batch == 0 || batch > 65535 || !a->w_q || !a->w_k || !a->w_v || !a->w_o ||
        !a->rope_cos || !a->rope_sin || !a->normed_in || !a->qbuf || !a->kbuf || !a->vbuf || !a->k_cache ||
        !a->v_cache || !a->attn_out || !a->o_out || a->head_dim == 0 || a->head_dim > 256 || a->head_dim % 32 ||
        a->num_kv_heads == 0 || a->num_heads % a->num_kv_heads || a->q_dim != a->num_heads * a->head_dim ||
        a->kv_dim != a->num_kv_heads * a->head_dim || a->attn_ctx == 0 || a->attn_ctx > smoe::kAttnMaxCtx ||
        a->num_heads > (uint32_t)smoe::kAttnMaxHeads ||
        (batch > 1 && kv_seq_stride < uint64_t(a->attn_ctx) * a->kv_dim)) {
        set_err("bad batched attention arguments %s%ld", "", (long)batch);
        return SMOE_ERR_ARG;
    }
    int rc;
    if (batch == 1) {
        if ((rc = smoe_cuda_matvec_bf16(c, a->w_q, a->normed_in, a->qbuf, a->q_dim, a->d_model))) return rc;
        if ((rc = smoe_cuda_matvec_bf16(c, a->w_k, a->normed_in, a->kbuf, a->kv_dim, a->d_model))) return rc;
        if ((rc = smoe_cuda_matvec_bf16(c, a->w_v, a->normed_in, a->vbuf, a->kv_dim, a->d_model))) return rc;
    } else {                             // the normed rows split into planes once for Q, K and V
        if (!gemm_shape_ok(c, a->normed_in, a->d_model, batch) || !gemm_shape_ok(c, a->attn_out, a->q_dim, batch)) {
            set_err("batched attention: batch or width above the context's limits %s%ld", "", (long)batch);
            return SMOE_ERR_ARG;
        }
        if ((rc = split_planes(c, a->normed_in, size_t(batch) * a->d_model))) return rc;
        if ((rc = gemm_planes(c, a->w_q, a->qbuf, a->q_dim, a->d_model, batch))) return rc;
        if ((rc = gemm_planes(c, a->w_k, a->kbuf, a->kv_dim, a->d_model, batch))) return rc;
        if ((rc = gemm_planes(c, a->w_v, a->vbuf, a->kv_dim, a->d_model, batch))) return rc;
    }
    smoe::AttnArgs t{};
    t.q = a->qbuf; t.k = a->kbuf; t.v = a->vbuf;
    t.q_norm_w = a->q_norm_w; t.k_norm_w = a->k_norm_w;
    t.rope_cos = a->rope_cos; t.rope_sin = a->rope_sin;
    t.qbuf = a->qbuf; t.kbuf = a->kbuf; t.vbuf = a->vbuf;
    t.k_cache = a->k_cache; t.v_cache = a->v_cache;
    t.attn_out = a->attn_out;
    t.q_dim = a->q_dim; t.kv_dim = a->kv_dim; t.head_dim = a->head_dim;
    t.num_heads = a->num_heads; t.num_kv_heads = a->num_kv_heads;
    t.attn_ctx = a->attn_ctx;
    t.pos = pos;
    t.scale = a->attn_scale;
    t.part = c->attn_part;
    t.cnt = c->attn_cnt;
    t.kv_seq_stride = size_t(kv_seq_stride);
    // batch x heads CTAs cover the GPU: one split per head (no partials).
    // Head groups whose ring is shared by several query heads take the
    // GQA kernel (each ring read once per group) when its tiles fit.
    const uint32_t G = a->num_heads / a->num_kv_heads;
    const uint32_t blk = gqa_block(a->attn_ctx);
    const size_t gqa_smem = gqa_smem_bytes(G, a->head_dim, blk);
    t.blk = blk;
    if (batch > 1 && a->head_dim == 128 && (size_t(G) * blk) % 4 == 0 &&   // float4 partials aligned
        G <= uint32_t(smoe::kAttnGqaMaxG) && gqa_smem <= c->smem_optin && aligned16(a->k_cache) &&
        aligned16(a->v_cache) && aligned16(a->qbuf) && aligned16(a->attn_out) && kv_seq_stride % 4 == 0) {
        auto kern = G <= 8 ? smoe::k_attn_batch_gqa<8> : smoe::k_attn_batch_gqa<16>;
        if ((rc = prep_kernel(c, kern, gqa_smem))) return rc;
        rc = pdl_launch_smem(c, kern, dim3(a->num_kv_heads, batch), dim3(smoe::kAttnThreads), gqa_smem, t);
    } else {
        const uint32_t splits = batch > 1 ? 1u : std::min<uint32_t>(smoe::kAttnSplits, (a->attn_ctx + 31) / 32);
        rc = pdl_launch(c, smoe::k_attn_decode, dim3(a->num_heads, splits, batch), dim3(smoe::kAttnThreads), t);
    }
    if (rc) return rc;
    return smoe_cuda_gemm_bf16(c, a->w_o, a->attn_out, a->o_out, a->d_model, a->q_dim, batch);
}

int smoe_cuda_rope_tables(SmoeCudaCtx* c, const uint32_t* pos, uint32_t n, const float* inv_freq, float* cos_out,
                          float* sin_out, uint32_t half) {
    if (!c || !pos || !inv_freq || !cos_out || !sin_out || half == 0 || n == 0 || n > 65535) {
        set_err("bad rope table arguments %s%ld", "", (long)n);
        return SMOE_ERR_ARG;
    }
    return pdl_launch(c, smoe::k_rope_tables, dim3((half + 127) / 128, n), dim3(128), pos, inv_freq, cos_out,
                      sin_out, half);
}

int smoe_cuda_attention_prefill_async(SmoeCudaCtx* c, const SmoeCudaAttnLayerArgs* a, uint32_t n_tokens,
                                      const uint32_t* pos) {
    const uint32_t G = a && a->num_kv_heads ? a->num_heads / a->num_kv_heads : 0;
    const uint32_t blk = a ? gqa_block(a->attn_ctx) : 0;
    const size_t smem = a ? gqa_smem_bytes(G, a->head_dim, blk) : 0;
    if (!c || !a || !pos || n_tokens == 0 || !a->w_q || !a->w_k || !a->w_v || !a->w_o || !a->rope_cos ||
        !a->rope_sin || !a->normed_in || !a->qbuf || !a->kbuf || !a->vbuf || !a->k_cache || !a->v_cache ||
        !a->attn_out || !a->o_out || a->num_kv_heads == 0 || a->num_heads % a->num_kv_heads ||
        a->q_dim != a->num_heads * a->head_dim || a->kv_dim != a->num_kv_heads * a->head_dim ||
        a->attn_ctx == 0 || a->attn_ctx > smoe::kAttnMaxCtx || n_tokens > a->attn_ctx) {
        set_err("bad prefill attention arguments %s%ld", "", (long)n_tokens);
        return SMOE_ERR_ARG;
    }
    if (a->head_dim != 128 || G > uint32_t(smoe::kAttnGqaMaxG) || (size_t(G) * blk) % 4 ||
        smem > c->smem_optin || !aligned16(a->k_cache) || !aligned16(a->v_cache) || !aligned16(a->qbuf) ||
        !aligned16(a->attn_out)) {
        set_err("prefill attention needs head_dim 128, <= 16 query heads per KV head and aligned rings %s%ld", "",
                (long)a->head_dim);
        return SMOE_ERR_UNSUPPORTED;
    }
    int rc;
    if (n_tokens == 1) {
        if ((rc = smoe_cuda_matvec_bf16(c, a->w_q, a->normed_in, a->qbuf, a->q_dim, a->d_model))) return rc;
        if ((rc = smoe_cuda_matvec_bf16(c, a->w_k, a->normed_in, a->kbuf, a->kv_dim, a->d_model))) return rc;
        if ((rc = smoe_cuda_matvec_bf16(c, a->w_v, a->normed_in, a->vbuf, a->kv_dim, a->d_model))) return rc;
    } else {
        if (!gemm_shape_ok(c, a->normed_in, a->d_model, n_tokens) || !gemm_shape_ok(c, a->attn_out, a->q_dim, n_tokens)) {
            set_err("prefill chunk or width above the context's limits %s%ld", "", (long)n_tokens);
            return SMOE_ERR_ARG;
        }
        if ((rc = split_planes(c, a->normed_in, size_t(n_tokens) * a->d_model))) return rc;
        if ((rc = gemm_planes(c, a->w_q, a->qbuf, a->q_dim, a->d_model, n_tokens))) return rc;
        if ((rc = gemm_planes(c, a->w_k, a->kbuf, a->kv_dim, a->d_model, n_tokens))) return rc;
        if ((rc = gemm_planes(c, a->w_v, a->vbuf, a->kv_dim, a->d_model, n_tokens))) return rc;
    }
    rc = pdl_launch(c, smoe::k_prefill_kv, dim3(a->num_kv_heads, n_tokens), dim3(32), (const float*)a->kbuf,
                    (const float*)a->vbuf, a->k_norm_w, a->rope_cos, a->rope_sin, a->k_cache, a->v_cache, a->kv_dim,
                    a->head_dim, a->attn_ctx, pos);
    if (rc) return rc;
    smoe::AttnArgs t{};
    t.q = a->qbuf; t.k = a->kbuf; t.v = a->vbuf;
    t.q_norm_w = a->q_norm_w; t.k_norm_w = a->k_norm_w;
    t.rope_cos = a->rope_cos; t.rope_sin = a->rope_sin;
    t.qbuf = a->qbuf; t.kbuf = a->kbuf; t.vbuf = a->vbuf;
    t.k_cache = a->k_cache; t.v_cache = a->v_cache;
    t.attn_out = a->attn_out;
    t.q_dim = a->q_dim; t.kv_dim = a->kv_dim; t.head_dim = a->head_dim;
    t.num_heads = a->num_heads; t.num_kv_heads = a->num_kv_heads;
    t.attn_ctx = a->attn_ctx;
    t.pos = pos;
    t.scale = a->attn_scale;
    t.kv_seq_stride = 0;                 // one sequence: every token's window is in the same ring
    t.prefill = 1;
    t.blk = blk;
    auto kern = G <= 8 ? smoe::k_attn_batch_gqa<8> : smoe::k_attn_batch_gqa<16>;
    if ((rc = prep_kernel(c, kern, smem))) return rc;
    rc = pdl_launch_smem(c, kern, dim3(a->num_kv_heads, n_tokens), dim3(smoe::kAttnThreads), smem, t);
    if (rc) return rc;
    return smoe_cuda_gemm_bf16(c, a->w_o, a->attn_out, a->o_out, a->d_model, a->q_dim, n_tokens);
}

int smoe_cuda_decode_advance_batch(SmoeCudaCtx* c, SmoeSamplerRow* rows, uint32_t* history, uint32_t hcap,
                                   const uint32_t* tokens, uint32_t batch, uint32_t* pos, const float* u_seq,
                                   uint32_t u_len) {
    if (!c || !rows || !tokens || !pos || (hcap && !history) || batch == 0 || batch > 1024) {
        set_err("bad decode_advance_batch arguments %s%ld", "", (long)batch);
        return SMOE_ERR_ARG;
    }
    return pdl_launch(c, smoe::k_decode_advance_batch, dim3(1), dim3((batch + 31) / 32 * 32),
                      reinterpret_cast<smoe::SamplerRowDevMut*>(rows), history, hcap, tokens, batch, pos, u_seq,
                      u_len);
}

int smoe_cuda_attention_layer(SmoeCudaCtx* c, const SmoeCudaAttnLayerArgs* a) {
    int rc = smoe_cuda_attention_layer_async(c, a, nullptr);
    if (rc) return rc;
    return smoe_cuda_synchronize(c);      // o_out valid on return, as metal_bridge.h:163-169
}

// ----------------------------------------------------------- expert parallel
namespace {
// Exchange window of a rank (rank 0's is the one used): x epoch flag, x copy,
// [kEpMaxWorld][kLMaxTok * max_d_model] partial rows, [kLMaxTok *
// max_d_model/16] partial-unit counts.
constexpr size_t kEpFlagOff = 0, kEpXOff = 256;
size_t ep_x_bytes(const SmoeCudaCtx* c) { return size_t(smoe::kLMaxTok) * c->cfg.max_d_model * 4; }
size_t ep_part_stride(const SmoeCudaCtx* c) { return size_t(smoe::kLMaxTok) * c->cfg.max_d_model; }
size_t ep_part_off(const SmoeCudaCtx* c) { return kEpXOff + ep_x_bytes(c); }
size_t ep_win_size(const SmoeCudaCtx* c) {
    return ep_part_off(c) + size_t(smoe::kEpMaxWorld) * ep_part_stride(c) * 8;   // tagged rows, 8 B each
}
}  // namespace

int smoe_cuda_ep_export(SmoeCudaCtx* c, SmoeEpHandle* out) {
    if (!c || !out) { set_err("null argument %s%ld", "", 0); return SMOE_ERR_ARG; }
    if (!c->ep_win) {
        c->ep_win_bytes = ep_win_size(c);
        CK(cudaMalloc(&c->ep_win, c->ep_win_bytes));
        CK(cudaMemset(c->ep_win, 0, c->ep_win_bytes));
    }
    cudaIpcMemHandle_t h;
    static_assert(sizeof(h) <= sizeof(out->bytes), "IPC handle size");
    CK(cudaIpcGetMemHandle(&h, c->ep_win));
    memset(out->bytes, 0, sizeof(out->bytes));
    memcpy(out->bytes, &h, sizeof(h));
    return SMOE_OK;
}

int smoe_cuda_ep_attach(SmoeCudaCtx* c, int rank, int world, const SmoeEpHandle* handles) {
    if (!c || !handles || world < 1 || world > smoe::kEpMaxWorld || rank < 0 || rank >= world || !c->ep_win) {
        set_err("bad expert-parallel attach (rank %s%ld)", "", (long)rank);
        return SMOE_ERR_ARG;
    }
    for (int r = 0; r < smoe::kEpMaxWorld; ++r) {
        if (c->ep_peer[r] && c->ep_peer[r] != c->ep_win) cudaIpcCloseMemHandle(c->ep_peer[r]);
        c->ep_peer[r] = nullptr;
    }
    cudaIpcMemHandle_t mine;
    CK(cudaIpcGetMemHandle(&mine, c->ep_win));
    // rank 0 writes x into every rank's window; the others write their rows
    // into rank 0's
    for (int r = 0; r < world; ++r) {
        if (r != 0 && rank != 0) continue;
        if (r == rank || memcmp(&mine, handles[r].bytes, sizeof(mine)) == 0) {
            c->ep_peer[r] = c->ep_win;    // this rank, or a window this process owns
        } else {
            cudaIpcMemHandle_t h;
            memcpy(&h, handles[r].bytes, sizeof(h));
            void* p = nullptr;
            CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
            c->ep_peer[r] = static_cast<uint8_t*>(p);
        }
    }
    c->ep_rank = rank;
    c->ep_world = world;
    // a fresh exchange: window and this rank's epoch count start at 0 (every
    // rank attaches before any rank launches an expert-parallel layer)
    CK(cudaMemsetAsync(c->ep_win, 0, c->ep_win_bytes, c->stream));
    CK(cudaMemsetAsync(&c->lstate->epoch, 0, sizeof(uint32_t), c->stream));
    CK(cudaStreamSynchronize(c->stream));
    return SMOE_OK;
}

int smoe_cuda_moe_layer_ep(SmoeCudaCtx* c, const SmoeMoeLayer* shard, uint32_t n_experts_total,
                           uint32_t expert_base, const void* x, int x_dtype, uint32_t batch, uint32_t k,
                           int norm, void* y, int y_dtype, uint32_t* ids_out, float* w_out) {
    if (!c || !shard || !c->ep_peer[0]) { set_err("expert parallel not attached %s%ld", "", 0); return SMOE_ERR_ARG; }
    const bool r0 = c->ep_rank == 0;
    if (!(shard->fmt & SMOE_LAYOUT_TILED) || !shard->router_w || !aligned16(shard->router_w) ||
        n_experts_total < k || k == 0 || k > SMOE_MAX_ACTIVE || n_experts_total > c->cfg.max_experts ||
        expert_base + shard->n_experts > n_experts_total || (x_dtype != 0 && x_dtype != 1) ||
        (y_dtype != 0 && y_dtype != 1) || batch == 0 || (r0 && (!x || !y))) {
        set_err("bad expert-parallel layer arguments %s%ld", "", (long)k);
        return SMOE_ERR_ARG;
    }
    smoe::FfnArgs a{};
    int rc = layer_args(c, shard, a);
    if (rc) return rc;
    smoe::LayerEp ep{};
    ep.world = c->ep_world;
    ep.rank = c->ep_rank;
    ep.base = expert_base;
    ep.nlocal = shard->n_experts;
    for (int r = 1; r < c->ep_world; ++r)
        if (r0) {
            ep.xw[r] = c->ep_peer[r] + kEpXOff;
            ep.flagw[r] = reinterpret_cast<uint32_t*>(c->ep_peer[r] + kEpFlagOff);
        }
    ep.flag = reinterpret_cast<uint32_t*>(c->ep_win + kEpFlagOff);
    ep.part0 = reinterpret_cast<unsigned long long*>(c->ep_peer[0] + ep_part_off(c));
    ep.part_stride = uint32_t(ep_part_stride(c));
    LayerCall q{};
    q.L = shard;
    q.n_experts = n_experts_total;
    q.expert_base = expert_base;
    q.x = r0 ? x : c->ep_win + kEpXOff;              // ranks > 0 read the copy rank 0 pushed here
    q.x_dtype = x_dtype;
    q.y = r0 ? y : nullptr;                          // (only rank 0 writes y)
    q.y_dtype = y_dtype;
    q.ids_out = ids_out;
    q.wts_out = w_out;
    q.rw = shard->router_w;
    q.norm = norm;
    q.k = k;
    q.batch = batch;
    q.ep = &ep;
    if (c->ep_world == 1) {                          // a world of one: plain single-GPU layer
        ep.world = 1;
    }
    rc = launch_layer(c, q);
    if (rc == SMOE_ERR_UNSUPPORTED)
        set_err("tiled layout needs batch <= 4 and a shape whose tiles fit shared memory %s%ld", "", (long)batch);
    return rc;
}

int smoe_cuda_sample(SmoeCudaCtx* c, float* logits, uint32_t vocab, uint32_t batch,
                     const SmoeSamplerRow* rows, const uint32_t* history, uint32_t hstride,
                     uint32_t* tokens) {
    if (!c || !logits || !rows || !tokens || vocab == 0 || vocab > c->cfg.max_vocab ||
        vocab > uint32_t(smoe::kSampCluster) * smoe::kSampThreads * smoe::kSeqMaxC || batch == 0 ||
        batch > 65535u || (hstride && !history)) {
        set_err("bad sampler arguments %s%ld", "", (long)vocab);
        return SMOE_ERR_ARG;
    }
    static_assert(sizeof(SmoeSamplerRow) == sizeof(smoe::SamplerRowDev), "row layout");
    smoe::SamplerArgs a{logits, vocab, reinterpret_cast<const smoe::SamplerRowDev*>(rows),
                        history, hstride, tokens, c->trace};
    const size_t smem = smoe::sampler_smem_bytes(vocab);
    int rc = prep_kernel(c, smoe::k_sample, smem);
    if (rc) return rc;
    dim3 g(smoe::kSampCluster, batch);
    smoe::k_sample<<<g, smoe::kSampThreads, smem, c->stream>>>(a);
    CK(cudaGetLastError());
    c->dispatches += 1;
    return SMOE_OK;
}

}  // extern "C"

extern "C" {

uint64_t smoe_cuda_tiled_expert_bytes(uint32_t fmt, uint32_t d, uint32_t dff) {
    fmt &= ~uint32_t(SMOE_LAYOUT_TILED);
    if ((fmt != SMOE_FMT_SMOE_Q4 && fmt != SMOE_FMT_AFFINE_Q4) || !d || !dff || d % 64 || dff % 64) return 0;
    smoe::TiledGeom t;
    if (!t.init((int)fmt, d, dff)) return 0;
    return t.expert;
}

int smoe_cuda_prepack_layer(SmoeCudaCtx* c, const SmoeMoeLayer* src, void* dst, uint64_t dst_stride,
                            SmoeMoeLayer* out) {
    if (!c || !src || !dst || !out) { set_err("null argument %s%ld", "", 0); return SMOE_ERR_ARG; }
    if (src->fmt & SMOE_LAYOUT_TILED) { set_err("layer is already tiled %s%ld", "", 0); return SMOE_ERR_ARG; }
    smoe::FfnArgs a{};
    int rc = layer_args(c, src, a);
    if (rc) return rc;
    const uint64_t need = smoe_cuda_tiled_expert_bytes(src->fmt, src->d_model, src->d_ff);
    if (dst_stride < need || dst_stride % 256 || !aligned16(dst)) {
        set_err("dst_stride below the tiled expert size or not a multiple of 256 (%s%ld)", "", (long)need);
        return SMOE_ERR_ARG;
    }
    smoe::PrepackArgs p{};
    p.src = src->base;
    p.src_stride = src->expert_stride;
    for (int i = 0; i < 9; ++i) p.off[i] = src->off[i];
    p.dst = static_cast<uint8_t*>(dst);
    p.dst_stride = dst_stride;
    p.fmt = (int)src->fmt;
    if (!p.tg.init((int)src->fmt, src->d_model, src->d_ff)) { set_err("shape has no tiled layout %s%ld", "", 0); return SMOE_ERR_ARG; }
    dim3 grid(2 * (src->d_ff / 16) + src->d_ff / 64, src->n_experts);
    smoe::k_prepack<<<grid, 256, 0, c->stream>>>(p);
    CK(cudaGetLastError());
    c->dispatches += 1;
    *out = *src;
    out->base = static_cast<const uint8_t*>(dst);
    out->expert_stride = dst_stride;
    for (int i = 0; i < 9; ++i) out->off[i] = 0;
    out->fmt = src->fmt | SMOE_LAYOUT_TILED;
    return SMOE_OK;
}

}  // extern "C"
