/*
 * smoe_cuda_compat.h - name shim for the reference engine.
 *
 * Lets src/decode.cpp, src/prefill.cpp and src/main.cpp of the reference
 * compile unchanged against libsmoe_cuda: make their
 * #include "compute/metal_bridge.h" resolve to a one-line file that includes
 * this header (tests/test_compat_compile.py checks exactly that). Every
 * smoe_metal_X of metal_bridge.h (:47-224) is an inline forwarder to the
 * smoe_cuda_X of smoe_cuda.h with the same arguments and the reference's
 * return type. Weight pointers handed to the FFN entries must be device
 * pointers into the resident expert arena.
 */
#pragma once
#include "smoe_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The reference forward-declares `struct SmoeMetalCtx;` on its own
 * (scout.hpp:27, engine.hpp), so it stays a distinct incomplete type here; a
 * SmoeMetalCtx* is a SmoeCudaCtx*. */
struct SmoeMetalCtx;
typedef struct SmoeMetalCtx SmoeMetalCtx;
#define SMOE_CUDA_CTX(c) ((SmoeCudaCtx*)(c))

/* metal_bridge.h:171-194: same fields, same order. */
typedef SmoeCudaAttnLayerArgs SmoeAttnLayerArgs;

static inline SmoeMetalCtx* smoe_metal_init(size_t slot_bytes) {
    return (SmoeMetalCtx*)smoe_cuda_init(slot_bytes);
}
static inline void smoe_metal_destroy(SmoeMetalCtx* ctx) { smoe_cuda_destroy(SMOE_CUDA_CTX(ctx)); }

static inline void* smoe_metal_fused_ffn(SmoeMetalCtx* ctx, const uint8_t* packed_gate,
                                         const uint16_t* scales_gate, const uint8_t* packed_up,
                                         const uint16_t* scales_up, const uint8_t* packed_down,
                                         const uint16_t* scales_down, const float* input_vec,
                                         float* hidden_vec, float* output_vec, uint32_t gate_rows,
                                         uint32_t gate_cols, uint32_t down_rows, uint32_t down_cols,
                                         uint32_t group_size, uint32_t bits, uint32_t expert_index) {
    return smoe_cuda_fused_ffn(SMOE_CUDA_CTX(ctx), packed_gate, scales_gate, packed_up, scales_up,
                               packed_down, scales_down, input_vec, hidden_vec, output_vec, gate_rows,
                               gate_cols, down_rows, down_cols, group_size, bits, expert_index);
}

static inline void smoe_metal_wait(SmoeMetalCtx* ctx, void* handle, float* output_vec,
                                   uint32_t expert_index, uint32_t cols) {
    smoe_cuda_wait(SMOE_CUDA_CTX(ctx), handle, output_vec, expert_index, cols);
}

static inline void* smoe_metal_fused_ffn_group(SmoeMetalCtx* ctx, const SmoeExpertBlob* experts,
                                               uint32_t n_experts, const float* input_vec,
                                               uint32_t gate_rows, uint32_t gate_cols,
                                               uint32_t down_rows, uint32_t down_cols,
                                               uint32_t group_size, uint32_t bits) {
    return smoe_cuda_fused_ffn_group(SMOE_CUDA_CTX(ctx), experts, n_experts, input_vec, gate_rows,
                                     gate_cols, down_rows, down_cols, group_size, bits);
}

static inline void* smoe_metal_fused_ffn_batch(SmoeMetalCtx* ctx, const uint8_t* packed_gate,
                                               const uint16_t* scales_gate, const uint8_t* packed_up,
                                               const uint16_t* scales_up, const uint8_t* packed_down,
                                               const uint16_t* scales_down, const float* input_mat,
                                               uint32_t batch, uint32_t gate_rows, uint32_t gate_cols,
                                               uint32_t down_rows, uint32_t down_cols,
                                               uint32_t group_size, uint32_t bits) {
    return smoe_cuda_fused_ffn_batch(SMOE_CUDA_CTX(ctx), packed_gate, scales_gate, packed_up, scales_up,
                                     packed_down, scales_down, input_mat, batch, gate_rows, gate_cols,
                                     down_rows, down_cols, group_size, bits);
}

static inline void smoe_metal_wait_ffn_batch(SmoeMetalCtx* ctx, void* handle, float* out_mat,
                                             uint32_t batch, uint32_t cols) {
    smoe_cuda_wait_ffn_batch(SMOE_CUDA_CTX(ctx), handle, out_mat, batch, cols);
}

static inline void smoe_metal_scout_matvec_bf16(SmoeMetalCtx* ctx, const uint16_t* weight,
                                                const float* input_vec, float* output_vec,
                                                uint32_t rows, uint32_t cols) {
    smoe_cuda_scout_matvec_bf16(SMOE_CUDA_CTX(ctx), weight, input_vec, output_vec, rows, cols);
}

/* metal_bridge.h:196 returns void and reports failures on stderr; the status
 * of smoe_cuda_attention_layer is kept in smoe_cuda_last_error(). */
static inline void smoe_metal_attention_layer(SmoeMetalCtx* ctx, const SmoeAttnLayerArgs* args) {
    (void)smoe_cuda_attention_layer(SMOE_CUDA_CTX(ctx), args);
}

static inline void smoe_metal_scout_matvec_batch_bf16(SmoeMetalCtx* ctx, const uint16_t** weights,
                                                      const float** inputs, float** outputs,
                                                      const uint32_t* rows, const uint32_t* cols,
                                                      uint32_t count) {
    smoe_cuda_scout_matvec_batch_bf16(SMOE_CUDA_CTX(ctx), weights, inputs, outputs, rows, cols, count);
}

static inline void smoe_metal_scout_matvec_group_bf16(SmoeMetalCtx* ctx, const uint16_t** weights,
                                                      const float** inputs, float** outputs,
                                                      const uint32_t* rows, const uint32_t* cols,
                                                      uint32_t count) {
    smoe_cuda_scout_matvec_group_bf16(SMOE_CUDA_CTX(ctx), weights, inputs, outputs, rows, cols, count);
}

static inline void smoe_metal_register_buffer(SmoeMetalCtx* ctx, const void* ptr, size_t size_in_bytes) {
    smoe_cuda_register_buffer(SMOE_CUDA_CTX(ctx), ptr, size_in_bytes);
}

static inline uint64_t smoe_metal_kernel_dispatches(const SmoeMetalCtx* ctx) {
    return smoe_cuda_kernel_dispatches((const SmoeCudaCtx*)ctx);
}

#ifdef __cplusplus
}  /* extern "C" */
#endif
