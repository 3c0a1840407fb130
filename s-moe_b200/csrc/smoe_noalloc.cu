// smoe_noalloc.cu - the expert-FFN entry point that allocates nothing.
//
// smoe_cuda_moe_ffn needs a context, and creating a context allocates device
// scratch with cudaMalloc. Some hosts cannot do that: an engine whose device
// memory is handed out by its own arena or pool (all of HBM reserved up
// front), code running inside a framework callback where allocation is
// forbidden, or a process that must not add allocations after start-up.
// smoe_cuda_moe_ffn_noalloc serves them: the only memory it needs besides
// the caller's inputs and outputs - the SwiGLU hidden vectors between the
// gate/up and the down kernels, and a device error word - lives in the
// file-scope array below, which every GPU that loads this library holds
// until the process exits.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <thread>

#include "../../include/smoe_cuda.h"
#include "ffn_q4.cuh"

namespace {

// Hidden vectors for up to kNoAllocHiddenFloats (slot, row) values, i.e.
// batch * k * d_ff <= 65536 (256 KiB), plus the error word at the end.
constexpr size_t kNoAllocHiddenFloats = 65536;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocHiddenFloats + 64];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};   // device address of the array, per device

thread_local char g_na_err[256] = "";

int fail(int code, const char* msg, long v) {
    std::snprintf(g_na_err, sizeof(g_na_err), "moe_ffn_noalloc: %s (%ld)", msg, v);
    return code;
}

// Once per device, with that device current: the array's name is only a
// host-side stand-in, so ask the runtime for its real device address.
int scratch_for_current_device(float** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return fail(SMOE_ERR_CUDA, "no current device", dev);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return fail(SMOE_ERR_CUDA, cudaGetErrorString(e), dev);
        g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_scratch_ptr[dev];
    return SMOE_OK;
}

template <typename K>
int smem_limit(K kern, size_t smem) {
    if (smem <= 48 * 1024) return SMOE_OK;
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (smem > (size_t)optin) return fail(SMOE_ERR_ARG, "shape needs more shared memory than the GPU has", (long)smem);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(SMOE_ERR_CUDA, "cudaFuncSetAttribute failed", (long)smem);
    return SMOE_OK;
}

}  // namespace

extern "C" {

const char* smoe_cuda_noalloc_last_error(void) { return g_na_err; }

int smoe_cuda_moe_ffn_noalloc(const SmoeMoeLayer* L, const void* x, int x_dtype,
                              const uint32_t* ids, const float* weights, uint32_t k,
                              uint32_t batch, void* y, int y_dtype, void* stream) {
    if (!L || !L->base || !x || !ids || !weights || !y)
        return fail(SMOE_ERR_ARG, "null argument", 0);
    if (L->fmt & SMOE_LAYOUT_TILED)
        return fail(SMOE_ERR_ARG, "the tiled layout is not supported here; pass the vault layout", (long)L->fmt);
    if (L->fmt != SMOE_FMT_SMOE_Q4 && L->fmt != SMOE_FMT_AFFINE_Q4)
        return fail(SMOE_ERR_ARG, "unknown weight format", (long)L->fmt);
    if (L->d_model == 0 || L->d_ff == 0 || L->d_model % 64 || L->d_ff % 64)
        return fail(SMOE_ERR_ARG, "d_model and d_ff must be multiples of 64", (long)L->d_model);
    if (k == 0 || k > SMOE_MAX_ACTIVE || batch == 0 || (x_dtype != 0 && x_dtype != 1) ||
        (y_dtype != 0 && y_dtype != 1))
        return fail(SMOE_ERR_ARG, "bad k, batch or dtype", (long)k);
    if ((reinterpret_cast<uintptr_t>(L->base) | L->expert_stride) & 15u)
        return fail(SMOE_ERR_ARG, "expert arena not 16-byte aligned", 0);
    for (int i = 0; i < 9; ++i)
        if (L->off[i] % 16) return fail(SMOE_ERR_ARG, "unaligned blob offset", i);
    const size_t need = size_t(batch) * k * L->d_ff;
    if (need > kNoAllocHiddenFloats)
        return fail(SMOE_ERR_ARG, "batch * k * d_ff exceeds the fixed scratch of 65536 floats",
                    (long)need);
    float* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;

    smoe::FfnArgs a{};
    a.base = L->base;
    a.stride = L->expert_stride;
    for (int i = 0; i < 9; ++i) a.off[i] = L->off[i];
    a.ids = ids;
    a.wts = weights;
    a.x = x;
    a.x_dtype = x_dtype;
    a.hidden = scratch;                                           // fully written before read
    a.err = reinterpret_cast<uint32_t*>(scratch + kNoAllocHiddenFloats);
    a.y = y;
    a.y_dtype = y_dtype;
    a.per_slot = 0;
    a.d_model = L->d_model;
    a.d_ff = L->d_ff;
    a.k = k;
    a.ntok = batch;
    a.n_experts = L->n_experts;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(a.err, 0, sizeof(uint32_t), s) != cudaSuccess)   // the one word that must start at 0
        return fail(SMOE_ERR_CUDA, "clearing the error word failed", 0);
    const size_t s1 = smoe::gate_up_smem_bytes(L->d_model), s2 = smoe::down_smem_bytes(L->d_ff);
    dim3 g1(L->d_ff / 16, batch * k), g2(L->d_model / 16, batch);
    if (L->fmt == SMOE_FMT_AFFINE_Q4) {
        if ((rc = smem_limit(smoe::k_gate_up<smoe::kFmtAffine>, s1))) return rc;
        if ((rc = smem_limit(smoe::k_down_combine<smoe::kFmtAffine>, s2))) return rc;
        smoe::k_gate_up<smoe::kFmtAffine><<<g1, 256, s1, s>>>(a);
        smoe::k_down_combine<smoe::kFmtAffine><<<g2, 256, s2, s>>>(a);
    } else {
        if ((rc = smem_limit(smoe::k_gate_up<smoe::kFmtSmoe>, s1))) return rc;
        if ((rc = smem_limit(smoe::k_down_combine<smoe::kFmtSmoe>, s2))) return rc;
        smoe::k_gate_up<smoe::kFmtSmoe><<<g1, 256, s1, s>>>(a);
        smoe::k_down_combine<smoe::kFmtSmoe><<<g2, 256, s2, s>>>(a);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(SMOE_ERR_CUDA, cudaGetErrorString(e), 0);
    return SMOE_OK;
}

// The device error word of the calls above (bounded waits that ran out, an
// expert id past the layer): wait (bounded, polling) until `stream` is idle,
// read the word, clear it. Allocates nothing either.
int smoe_cuda_noalloc_check(void* stream, uint32_t timeout_ms) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(s);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return fail(SMOE_ERR_CUDA, cudaGetErrorString(q), 0);
        const long ms = (long)std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (ms > (long)timeout_ms) return fail(SMOE_ERR_TIMEOUT, "stream still busy after (ms)", ms);
        std::this_thread::yield();
    }
    uint32_t word = 0;          // the stream is idle: the copy returns at once
    cudaError_t e = cudaMemcpyFromSymbolAsync(&word, g_noalloc_scratch, sizeof(word),
                                              kNoAllocHiddenFloats * sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(SMOE_ERR_CUDA, cudaGetErrorString(e), 0);
    if (word != 0) {
        e = cudaMemsetAsync(scratch + kNoAllocHiddenFloats, 0, sizeof(uint32_t), s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail(SMOE_ERR_CUDA, cudaGetErrorString(e), 0);
        return fail(SMOE_ERR_DEVICE, "a kernel raised device error code", (long)word);
    }
    return SMOE_OK;
}

}  // extern "C"
