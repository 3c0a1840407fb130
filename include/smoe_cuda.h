/*
 * smoe_cuda.h - C ABI of the B200 (sm_100a) decode hot path of S-MoE.
 *
 * Drop-in for the reference's compute interface src/compute/metal_bridge.h:
 * every smoe_metal_X there has a smoe_cuda_X here with the same argument
 * meaning (see smoe_cuda_compat.h for the name shim), plus native entries for
 * the router (decode.cpp:280-303 -> scout.cpp:77-123, host code in the
 * reference), the whole MoE layer and the token sampler (sampler.hpp:33-157,
 * host code in the reference).
 *
 * Conventions
 *   - Pure C, <stdint.h>/<stddef.h>/<stdbool.h> only; no CUDA types.
 *   - Weight pointers are DEVICE pointers into a resident expert arena (the
 *     reference passes unified-memory host pointers).
 *   - Activation pointers of the mirrored entries may be host or device
 *     memory (detected per call); the native entries take device pointers
 *     and run asynchronously on the context's stream.
 *   - int-returning entries give an SMOE_* status; pointer-returning mirrored
 *     entries keep the reference's NULL-on-failure contract. The message of
 *     the last failure is in smoe_cuda_last_error().
 *   - One context per (thread, device). No allocation after init: all
 *     scratch is sized by SmoeCudaInitArgs.
 *   - Every host wait is bounded by timeout_ms and returns SMOE_ERR_TIMEOUT.
 */
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

/* ---------------------------------------------------------------- status */
#define SMOE_OK               0
#define SMOE_ERR_ARG          1   /* bad argument / unsupported shape        */
#define SMOE_ERR_CUDA         2   /* CUDA runtime error                      */
#define SMOE_ERR_TIMEOUT      3   /* bounded host or device wait ran out     */
#define SMOE_ERR_NCCL         4
#define SMOE_ERR_DEVICE       5   /* a kernel raised its error flag          */
#define SMOE_ERR_UNSUPPORTED  6

/* ----------------------------------------------------------- formats */
/* SMOE-Q4 (vault format, shatter_moe.py:331-387): w = (q - 7.5)/7.5 * s,
 * fp16 s per group of 64, no bias. AFFINE-Q4: w = scale*q + bias, bf16 scale
 * and bf16 bias per group of 64. Both: 2 codes per byte, LSB first,
 * row-major, K (input dim) contiguous. */
#define SMOE_FMT_SMOE_Q4   0
#define SMOE_FMT_AFFINE_Q4 1

#define SMOE_DTYPE_F32  0
#define SMOE_DTYPE_BF16 1

#define SMOE_MAX_ACTIVE        16     /* scout.hpp:32 MAX_ACTIVE            */
#define SMOE_MAX_FFN_BATCH     64     /* metal_bridge.h:134                 */
#define SMOE_MAX_FFN_BATCH_DIM 16384  /* metal_bridge.h:135                 */
#define SMOE_MAX_TOP_K_SAMPLE  1024   /* main.cpp:323 TOP_K_PROTOCOL_CAP    */

typedef struct SmoeCudaCtx SmoeCudaCtx;

/* ------------------------------------------------------------ lifecycle */
typedef struct {
    int      device;        /* CUDA ordinal                                 */
    uint32_t max_d_model;   /* 0 -> 8192                                    */
    uint32_t max_d_ff;      /* 0 -> 4096                                    */
    uint32_t max_experts;   /* router width, 0 -> 512                       */
    uint32_t max_batch;     /* tokens per call, 0 -> 256                    */
    uint32_t max_vocab;     /* sampler rows, 0 -> 262144                    */
    uint32_t timeout_ms;    /* host waits, 0 -> 10000                       */
    uint32_t device_wait_us;/* limit of every wait inside the MoE-layer
                               kernel (other CTAs, other GPUs, bulk copies),
                               0 -> 1000000; a wait that runs out raises
                               SMOE_ERR_DEVICE at the next synchronize     */
} SmoeCudaInitArgs;

/* Mirror of smoe_metal_init (metal_bridge.h:47): defaults, current device.
 * slot_bytes is accepted for signature compatibility. NULL on failure. */
SmoeCudaCtx* smoe_cuda_init(size_t slot_bytes);
SmoeCudaCtx* smoe_cuda_init_ex(const SmoeCudaInitArgs* args);
/* metal_bridge.h:50. NULL-safe. */
void smoe_cuda_destroy(SmoeCudaCtx* ctx);
/* Message of the last failure on this thread ("" if none). */
const char* smoe_cuda_last_error(void);
/* Run subsequent work on an external cudaStream_t (NULL -> own stream). */
int smoe_cuda_set_stream(SmoeCudaCtx* ctx, void* cuda_stream);
void* smoe_cuda_get_stream(SmoeCudaCtx* ctx);
/* Bounded wait for all work on the context's stream; also reports a device
 * error flag raised by any kernel since the previous call. */
int smoe_cuda_synchronize(SmoeCudaCtx* ctx);

/* ------------------------------------------------ mirrored FFN entries */
/* metal_bridge.h:74-90. One expert, returns a wait handle (NULL on error).
 * hidden_vec is accepted for compatibility; the context owns its scratch. */
void* smoe_cuda_fused_ffn(SmoeCudaCtx* ctx,
                          const uint8_t* packed_gate, const uint16_t* scales_gate,
                          const uint8_t* packed_up, const uint16_t* scales_up,
                          const uint8_t* packed_down, const uint16_t* scales_down,
                          const float* input_vec, float* hidden_vec, float* output_vec,
                          uint32_t gate_rows, uint32_t gate_cols,
                          uint32_t down_rows, uint32_t down_cols,
                          uint32_t group_size, uint32_t bits, uint32_t expert_index);

/* metal_bridge.h:92. Waits for `handle` then copies slot `expert_index`'s
 * output (cols floats) into output_vec (host or device). */
void smoe_cuda_wait(SmoeCudaCtx* ctx, void* handle, float* output_vec,
                    uint32_t expert_index, uint32_t cols);

/* metal_bridge.h:106-114 */
typedef struct {
    const uint8_t*  packed_gate;
    const uint16_t* scales_gate;
    const uint8_t*  packed_up;
    const uint16_t* scales_up;
    const uint8_t*  packed_down;
    const uint16_t* scales_down;
    uint32_t        slot;
} SmoeExpertBlob;

/* metal_bridge.h:116-125. n_experts <= SMOE_MAX_ACTIVE same-shape SMOE-Q4
 * experts on one input vector; fetch each with smoe_cuda_wait(slot). */
void* smoe_cuda_fused_ffn_group(SmoeCudaCtx* ctx, const SmoeExpertBlob* experts,
                                uint32_t n_experts, const float* input_vec,
                                uint32_t gate_rows, uint32_t gate_cols,
                                uint32_t down_rows, uint32_t down_cols,
                                uint32_t group_size, uint32_t bits);

/* metal_bridge.h:137-151. One expert over `batch` <= SMOE_MAX_FFN_BATCH rows
 * of input_mat [batch x gate_cols]; NULL when batch/dims exceed the limits. */
void* smoe_cuda_fused_ffn_batch(SmoeCudaCtx* ctx,
                                const uint8_t* packed_gate, const uint16_t* scales_gate,
                                const uint8_t* packed_up, const uint16_t* scales_up,
                                const uint8_t* packed_down, const uint16_t* scales_down,
                                const float* input_mat, uint32_t batch,
                                uint32_t gate_rows, uint32_t gate_cols,
                                uint32_t down_rows, uint32_t down_cols,
                                uint32_t group_size, uint32_t bits);

/* metal_bridge.h:153-154: out_mat [batch x cols] (host or device). */
void smoe_cuda_wait_ffn_batch(SmoeCudaCtx* ctx, void* handle, float* out_mat,
                              uint32_t batch, uint32_t cols);

/* metal_bridge.h:157-162: bf16 W [rows x cols] . fp32 x, synchronous. */
void smoe_cuda_scout_matvec_bf16(SmoeCudaCtx* ctx, const uint16_t* weight,
                                 const float* input_vec, float* output_vec,
                                 uint32_t rows, uint32_t cols);

/* metal_bridge.h:199-206: `count` GEMVs outputs[i] = weights[i] . inputs[i]
 * (rows[i] x cols[i] bf16, fp32 vectors, host or device), in order - a
 * dispatch may read an earlier one's output. Synchronous. */
void smoe_cuda_scout_matvec_batch_bf16(SmoeCudaCtx* ctx, const uint16_t** weights,
                                       const float** inputs, float** outputs,
                                       const uint32_t* rows, const uint32_t* cols, uint32_t count);

/* metal_bridge.h:212-219: the same for dispatches with distinct outputs that
 * no dispatch reads (no ordering needed between them). Synchronous. */
void smoe_cuda_scout_matvec_group_bf16(SmoeCudaCtx* ctx, const uint16_t** weights,
                                       const float** inputs, float** outputs,
                                       const uint32_t* rows, const uint32_t* cols, uint32_t count);

/* metal_bridge.h:221. Pins a host buffer (cudaHostRegister); device
 * pointers are accepted and ignored. */
void smoe_cuda_register_buffer(SmoeCudaCtx* ctx, const void* ptr, size_t size_in_bytes);

/* metal_bridge.h:224. Number of kernels this context has launched. */
uint64_t smoe_cuda_kernel_dispatches(const SmoeCudaCtx* ctx);

/* ------------------------------------------------------ native entries */
/* A layer's resident experts: expert e's blob at base + e * expert_stride,
 * matrix m (0 gate [d_ff x d_model], 1 up, 2 down [d_model x d_ff]) with its
 * nibbles / scales / biases at offsets off[3m+0..2] inside the blob
 * (biases ignored for SMOE-Q4). All offsets and the stride 16-byte aligned. */
typedef struct {
    const uint8_t*  base;
    uint64_t        expert_stride;
    uint64_t        off[9];
    uint32_t        n_experts;
    uint32_t        d_model;
    uint32_t        d_ff;
    uint32_t        fmt;          /* SMOE_FMT_*                              */
    const uint16_t* router_w;     /* bf16 [n_experts x d_model]              */
} SmoeMoeLayer;

/* Tiled device layout of a layer's experts, made once at load time by
 * smoe_cuda_prepack_layer (no counterpart in the reference, whose experts
 * stay in the vault layout). Set as a flag in SmoeMoeLayer.fmt: the fused
 * single-launch MoE path needs it; the vault layout is served by the
 * two-kernel path. Per expert: d_ff/16 gate+up tiles then d_model/16 down
 * tiles, each tile one contiguous block (nibbles in MMA-fragment order,
 * then transposed scales, then biases). Same byte count as the vault layout. */
#define SMOE_LAYOUT_TILED 0x100

/* Bytes of one expert in the tiled layout (0 for unsupported shapes). */
uint64_t smoe_cuda_tiled_expert_bytes(uint32_t fmt, uint32_t d_model, uint32_t d_ff);

/* Re-lay out every expert of `src` (vault layout, device) into `dst`
 * (device, n_experts * dst_stride bytes, dst_stride >= the tiled size and a
 * multiple of 256) and describe the result in *out (base dst, fmt |
 * SMOE_LAYOUT_TILED, router_w copied). Asynchronous on the context stream. */
int smoe_cuda_prepack_layer(SmoeCudaCtx* ctx, const SmoeMoeLayer* src, void* dst,
                            uint64_t dst_stride, SmoeMoeLayer* out);

/* ---- .smoe vault (common.hpp:52-183, written by shatter_moe.py): the
 * reader of main.cpp:96-198 and a device uploader. The vault is passed as
 * host bytes (e.g. the caller's mmap); nothing here needs a GPU except the
 * upload. */
typedef struct {
    uint32_t version, num_moe_layers, max_experts_per_layer, total_experts;
    uint32_t group_size, bits, d_model, vocab_size, ffn_dim;
    uint64_t table_offset, data_offset;
    /* v2 arch block (has_arch 0 for a v1 vault) */
    uint32_t has_arch, arch_flags, num_heads, num_kv_heads, head_dim, moe_top_k;
    uint32_t moe_ffn_dim, dense_ffn_dim, shared_expert_ffn_dim, num_hidden_layers;
    float    rope_theta, rms_norm_eps;
    char     model_type[24];
    /* expert layout from the first expert's descriptors (main.cpp:170-198) */
    uint32_t gate_rows, gate_cols, up_rows, up_cols, down_rows, down_cols;
    uint64_t gate_packed_offset, gate_scales_offset, up_packed_offset, up_scales_offset;
    uint64_t down_packed_offset, down_scales_offset;
    uint64_t max_raw_size;        /* largest expert blob, unpadded bytes */
} SmoeVaultInfo;

/* Header, arch block, tensor descriptors and table bounds (main.cpp:96-198:
 * magic, version 1..2, a v2 vault's arch block valid, SiLU, top_k <= 16,
 * head_dim <= 256, heads divisible). SMOE_OK or SMOE_ERR_ARG /
 * SMOE_ERR_UNSUPPORTED with smoe_cuda_vault_last_error(). Host only. */
int smoe_cuda_vault_parse(const void* vault, uint64_t size, SmoeVaultInfo* out);
/* Byte offset and unpadded size of (layer, expert)'s blob. Host only. */
int smoe_cuda_vault_expert(const void* vault, uint64_t size, uint32_t layer, uint32_t expert,
                           uint64_t* offset, uint64_t* raw_size);
/* Copy every expert blob of `layer` into the device arena dst (expert e at
 * dst + e * dst_stride; dst_stride >= max_raw_size, 16-byte multiple), one
 * cudaMemcpyAsync per expert on the context stream, and describe the result
 * in *out (SMOE-Q4 vault layout, router_w stored as given). 4-bit group-64
 * vaults only (a 2-bit vault: SMOE_ERR_UNSUPPORTED). The vault bytes must
 * stay valid until the stream has run the copies. */
int smoe_cuda_vault_upload_layer(SmoeCudaCtx* ctx, const void* vault, uint64_t size, uint32_t layer,
                                 void* dst, uint64_t dst_stride, const uint16_t* router_w,
                                 SmoeMoeLayer* out);
const char* smoe_cuda_vault_last_error(void);

/* Expert parallel for token batches (BASELINE config 3 at batch 32: the
 * 235B layer's experts sharded over the GPUs, combined with NCCL). Every
 * rank passes the same x and routes it over the whole router
 * (shard->router_w: [n_experts_total x d_model]); shard holds experts
 * [expert_base, expert_base + shard->n_experts) in the vault layout; the
 * expert-grouped FFN runs only this rank's slots and y_partial [batch x
 * d_model] fp32 receives their weighted sum in rank order (zero rows where
 * no local expert was chosen). The layer output is the sum of the ranks'
 * partials (an NCCL reduce or all-reduce of y_partial by the caller; sum
 * order across ranks differs from the one-GPU rank order, ~1e-7
 * relative). ids_out / w_out (optional, device): the routing. */
int smoe_cuda_moe_layer_shard(SmoeCudaCtx* ctx, const SmoeMoeLayer* shard, uint32_t n_experts_total,
                              uint32_t expert_base, const void* x, int x_dtype, uint32_t batch,
                              uint32_t k, int norm, float* y_partial, uint32_t* ids_out,
                              float* w_out);

/* Router of decode.cpp:280-303 for `batch` tokens: logits = W . x (bf16 W,
 * fp32 accumulate), softmax over n_experts, top-k by probability (lowest
 * index wins ties), renormalised over the k when norm_topk. Outputs (device):
 * ids [batch x k] u32 in rank order, weights [batch x k] f32, logits
 * [batch x n_experts] (optional, may be NULL). x: [batch x d_model]. */
int smoe_cuda_router_topk(SmoeCudaCtx* ctx, const uint16_t* router_w, const void* x,
                          int x_dtype, uint32_t n_experts, uint32_t d_model,
                          uint32_t batch, uint32_t k, int norm_topk,
                          uint32_t* ids, float* weights, float* logits);

/* Expert FFN + weighted combine for `batch` tokens whose routing is already
 * on the device (ids/weights [batch x k]): y[t] = sum_j w[t,j] * FFN_{ids[t,j]}(x[t])
 * accumulated in rank order j = 0..k-1 (decode.cpp:485-499).
 * y: [batch x d_model] in y_dtype. */
int smoe_cuda_moe_ffn(SmoeCudaCtx* ctx, const SmoeMoeLayer* layer, const void* x,
                      int x_dtype, const uint32_t* ids, const float* weights,
                      uint32_t k, uint32_t batch, void* y, int y_dtype);

/* Router + expert FFN + combine, all on the device. ids_out / w_out
 * (optional, device, [batch x k]) receive the routing. On the tiled layout
 * (and for smoe_cuda_moe_ffn on it) x and y may also be pinned host memory
 * (cudaHostAlloc / cudaHostRegister): x is staged by a small copy kernel and
 * y's rows are stored straight into the host buffer, with no memcpy call;
 * pageable host memory is rejected with SMOE_ERR_ARG. */
int smoe_cuda_moe_layer(SmoeCudaCtx* ctx, const SmoeMoeLayer* layer, const void* x,
                        int x_dtype, uint32_t batch, uint32_t k, int norm_topk,
                        void* y, int y_dtype, uint32_t* ids_out, float* w_out);

/* ---- Expert parallel over the GPUs of one node (one process per GPU).
 * Replaces the per-GPU partial-sum combine that the reference leaves to
 * NCCL (the 235B EP layout: experts [r*E/G, (r+1)*E/G) on rank r, x and y on
 * rank 0). No counterpart in metal_bridge.h, which is single-GPU.
 *
 * Set-up, once per context: every rank calls smoe_cuda_ep_export, the host
 * gathers the handles in rank order by any means (e.g. an all-gather of
 * the 64-byte blobs), and every rank calls smoe_cuda_ep_attach with all of
 * them. The exchange then runs inside the layer kernel over NVLink: rank 0
 * pushes x into every rank's window (peer stores, then a release flag),
 * every rank routes (identical ids), runs the experts it holds and stores
 * its fp32 output rows, tagged with the call's epoch, into rank 0's window;
 * rank 0 adds the ranks' rows in rank order.
 * All ranks must make the same sequence of smoe_cuda_moe_layer_ep calls.
 * Waits on other GPUs are bounded (a rank that never arrives raises
 * SMOE_ERR_DEVICE at the next synchronize instead of hanging). */
typedef struct SmoeEpHandle {
    uint8_t bytes[64];
} SmoeEpHandle;

int smoe_cuda_ep_export(SmoeCudaCtx* ctx, SmoeEpHandle* out);
int smoe_cuda_ep_attach(SmoeCudaCtx* ctx, int rank, int world, const SmoeEpHandle* handles);

/* One MoE layer, expert parallel. shard: this rank's experts
 * [expert_base, expert_base + shard->n_experts) in the tiled layout, with
 * the full router (n_experts_total rows) in shard->router_w. x, y: device
 * buffers on rank 0 (ignored, may be NULL, on other ranks); ids_out / w_out
 * (optional) receive the routing on every rank. */
int smoe_cuda_moe_layer_ep(SmoeCudaCtx* ctx, const SmoeMoeLayer* shard, uint32_t n_experts_total,
                           uint32_t expert_base, const void* x, int x_dtype, uint32_t batch,
                           uint32_t k, int norm_topk, void* y, int y_dtype, uint32_t* ids_out,
                           float* w_out);

/* No counterpart in the reference. For callers that cannot call cudaMalloc -
 * engines whose device memory is all reserved by their own pool, code run
 * inside callbacks where allocation is forbidden - this is smoe_cuda_moe_ffn
 * (same arguments and results, device pointers, asynchronous on `stream`, a
 * cudaStream_t or NULL) without a context: it allocates nothing. Its only
 * scratch is one fixed array compiled into the library, which every GPU that
 * loads the library holds until the process exits. Limits: batch * k * d_ff
 * <= 65536 (256 KiB of hidden vectors); larger calls return SMOE_ERR_ARG.
 * Vault layout only (layers with SMOE_LAYOUT_TILED set return SMOE_ERR_ARG).
 * The first call on each device looks up the array's device address, so make
 * that call before any stream capture. All calls share the array: calls that
 * overlap on the GPU (different streams, or different host threads) race.
 * The message of a failure is in smoe_cuda_noalloc_last_error(). */
int smoe_cuda_moe_ffn_noalloc(const SmoeMoeLayer* layer, const void* x, int x_dtype,
                              const uint32_t* ids, const float* weights, uint32_t k,
                              uint32_t batch, void* y, int y_dtype, void* stream);
const char* smoe_cuda_noalloc_last_error(void);
/* Companion status call of smoe_cuda_moe_ffn_noalloc, allocating nothing
 * either: waits (bounded by timeout_ms, polling) until `stream` is idle, then
 * reads and clears the library's device error word. SMOE_ERR_DEVICE when a
 * call since the previous check raised it (an expert id >= layer->n_experts,
 * whose slot then used expert 0's weights, or a bounded device wait that ran
 * out), SMOE_ERR_TIMEOUT when the stream stayed busy. */
int smoe_cuda_noalloc_check(void* stream, uint32_t timeout_ms);

/* ------------------------------------------------------------- sampler */
/* One row of sampler state (sampler.hpp:11-17 SamplerConfig + the draw). */
typedef struct {
    float    temperature;   /* < 1e-4 -> greedy                             */
    float    top_p;
    uint32_t top_k;         /* 0..SMOE_MAX_TOP_K_SAMPLE                     */
    float    rep_penalty;   /* 1.0 -> none                                  */
    float    u;             /* generate_canonical<float,24> draw in [0,1)   */
    uint32_t history_len;   /* entries of this row's history                */
} SmoeSamplerRow;

/* sampler.hpp:33-157 for `batch` rows. logits: device [batch x vocab] fp32,
 * mutated in place by the repetition penalty exactly as the reference does.
 * rows: device [batch]. history: device [batch x history_stride] u32.
 * tokens: device [batch] u32. */
int smoe_cuda_sample(SmoeCudaCtx* ctx, float* logits, uint32_t vocab, uint32_t batch,
                     const SmoeSamplerRow* rows, const uint32_t* history,
                     uint32_t history_stride, uint32_t* tokens);

/* Host helper: the float libstdc++'s generate_canonical<float,24> makes of
 * one 32-bit std::mt19937 word (what sample_token consumes per call). */
float smoe_cuda_canonical_from_u32(uint32_t word);

/* ---- Dense trunk of a decode step around the MoE layer. All pointers are
 * device pointers; calls are asynchronous on the context stream unless
 * stated (so a whole decode step can be captured in one CUDA graph).
 * Not bit-exact with the reference's CPU loops (tree reductions, CUDA
 * exp/cos/sin), like the reference's own Metal attention. */

/* Mirror of SmoeAttnLayerArgs (metal_bridge.h:171-194), same fields. */
typedef struct SmoeCudaAttnLayerArgs {
    const uint16_t* w_q;        /* [q_dim x d_model] bf16 */
    const uint16_t* w_k;        /* [kv_dim x d_model] bf16 */
    const uint16_t* w_v;        /* [kv_dim x d_model] bf16 */
    const uint16_t* w_o;        /* [d_model x q_dim] bf16 */
    const uint16_t* q_norm_w;   /* [head_dim] bf16, NULL: no QK norm */
    const uint16_t* k_norm_w;
    const float*    rope_cos;   /* [head_dim/2] for this token's position */
    const float*    rope_sin;
    const float*    normed_in;  /* [d_model] post input-norm hidden */
    float*          qbuf;       /* [q_dim] scratch (normed + roped Q on exit) */
    float*          kbuf;       /* [kv_dim] */
    float*          vbuf;       /* [kv_dim] */
    float*          k_cache;    /* layer base of the KV ring [attn_ctx x kv_dim] */
    float*          v_cache;
    float*          attn_out;   /* [q_dim] scratch */
    float*          o_out;      /* [d_model] result */
    uint32_t d_model, q_dim, kv_dim, head_dim, num_heads, num_kv_heads;
    uint32_t slot;              /* ring write slot (ctx_pos % attn_ctx) */
    uint32_t valid;             /* attended positions incl. current */
    uint32_t attn_ctx;          /* ring capacity (<= 8192) */
    float    attn_scale;        /* 1/sqrt(head_dim) */
} SmoeCudaAttnLayerArgs;

/* smoe_metal_attention_layer (metal_bridge.h:196): QKV -> per-head QK
 * RMSNorm -> RoPE -> ring append -> GQA attention -> O. Synchronous. */
int smoe_cuda_attention_layer(SmoeCudaCtx* ctx, const SmoeCudaAttnLayerArgs* args);
/* The same, asynchronous. pos (device, optional): the token's position;
 * when given it overrides slot/valid (slot = pos % attn_ctx, valid =
 * min(pos + 1, attn_ctx)) so graph replays follow the position. */
int smoe_cuda_attention_layer_async(SmoeCudaCtx* ctx, const SmoeCudaAttnLayerArgs* args,
                                    const uint32_t* pos);

/* y[r] = sum_j W[r, j] x[j] (matvec_bf16, common.hpp:293-306), device
 * pointers, asynchronous; cols % 8 == 0, cols <= 16384. */
int smoe_cuda_matvec_bf16(SmoeCudaCtx* ctx, const uint16_t* w, const float* x, float* y,
                          uint32_t rows, uint32_t cols);
/* For each of `rows` rows: hidden += delta (delta may be NULL), then
 * normed = rms_norm_bf16(hidden, w) (common.hpp:245-256, eps 1e-6). */
int smoe_cuda_rms_norm(SmoeCudaCtx* ctx, float* hidden, const float* delta, const uint16_t* w,
                       float* normed, uint32_t n, uint32_t rows);
/* out[t] = bf16 embedding row tokens[t] as fp32 (decode.cpp:103-107). */
int smoe_cuda_embed_bf16(SmoeCudaCtx* ctx, const uint16_t* table, const uint32_t* tokens,
                         uint32_t n_tokens, uint32_t d_model, float* out);
/* cos/sin of float(*pos) * inv_freq[i], i < half (decode.cpp:113-118). */
int smoe_cuda_rope_table(SmoeCudaCtx* ctx, const uint32_t* pos, const float* inv_freq,
                         float* cos_out, float* sin_out, uint32_t half);
/* End of a decode step on the device: append *token to the row's history
 * (history_len < hcap), ++*pos, and row->u = u_seq[*pos % u_len] when
 * u_seq is given. */
int smoe_cuda_decode_advance(SmoeCudaCtx* ctx, SmoeSamplerRow* row, uint32_t* history,
                             uint32_t hcap, const uint32_t* token, uint32_t* pos,
                             const float* u_seq, uint32_t u_len);

/* ---- Batched decode: `batch` sequences at one shared position, each with
 * its own KV ring (256 sequences; the reference decodes
 * one sequence at a time and batches tokens only per expert in prefill,
 * prefill.cpp:321-417, kernels.metal:662-769). */

/* Y[b][r] = sum_j W[r, j] X[b][j] for b < batch: matvec_bf16
 * (common.hpp:293-306) over a batch of fp32 rows. batch == 1 is
 * smoe_cuda_matvec_bf16. Larger batches run on the tensor cores (cuBLAS bf16
 * GEMM, fp32 accumulation) over X split into two bf16 planes (hi = bf16(x),
 * lo = bf16(x - hi)), which keeps the activations to ~2^-17 relative.
 * batch <= max_batch, cols <= max_d_model, cols % 8 == 0. Asynchronous. */
int smoe_cuda_gemm_bf16(SmoeCudaCtx* ctx, const uint16_t* w, const float* x, float* y,
                        uint32_t rows, uint32_t cols, uint32_t batch);

/* The attention layer (decode.cpp:150-231) for `batch` sequences at the
 * device position *pos: normed_in [batch x d_model], qbuf/attn_out [batch x
 * q_dim], kbuf/vbuf [batch x kv_dim], o_out [batch x d_model]; sequence b's
 * rings at k_cache / v_cache + b * kv_seq_stride floats. slot/valid are
 * ignored (pos decides them). Asynchronous. */
int smoe_cuda_attention_batch_async(SmoeCudaCtx* ctx, const SmoeCudaAttnLayerArgs* args,
                                    uint32_t batch, uint64_t kv_seq_stride, const uint32_t* pos);

/* ---- Layer-major prefill (prefill.cpp:82-465): the prompt's tokens, all
 * but the last, go through each layer together, in chunks; the last prompt
 * token then takes the normal decode step, which samples. */

/* RoPE tables of n consecutive positions *pos + t (decode.cpp:113-118 per
 * token): cos_out / sin_out [n x half]. */
int smoe_cuda_rope_tables(SmoeCudaCtx* ctx, const uint32_t* pos, uint32_t n, const float* inv_freq,
                          float* cos_out, float* sin_out, uint32_t half);

/* The attention layer for a chunk of n_tokens of ONE sequence at positions
 * *pos .. *pos + n_tokens - 1 (prefill.cpp:131-268): Q/K/V of all tokens,
 * QK RMSNorm + RoPE at each token's position (rope_cos / rope_sin: [n_tokens
 * x head_dim/2], smoe_cuda_rope_tables), every token's K/V appended to the
 * ring, then causal attention (token t attends to the newest min(*pos + t +
 * 1, attn_ctx) positions), O projection. Buffers as the batched entry
 * ([n_tokens x width]); one ring (k_cache / v_cache). n_tokens <= max_batch
 * and <= attn_ctx; head_dim 128 (else SMOE_ERR_UNSUPPORTED). As in the
 * reference, a chunk that wraps the ring overwrites positions its earlier
 * tokens would still see. slot/valid ignored. Asynchronous. */
int smoe_cuda_attention_prefill_async(SmoeCudaCtx* ctx, const SmoeCudaAttnLayerArgs* args,
                                      uint32_t n_tokens, const uint32_t* pos);

/* End of a batched decode step: tokens[b] joins rows[b]'s history (history
 * [batch x hcap]), ++*pos, and rows[b].u = u_seq[(*pos * batch + b) % u_len]
 * when u_seq is given. batch <= 1024. */
int smoe_cuda_decode_advance_batch(SmoeCudaCtx* ctx, SmoeSamplerRow* rows, uint32_t* history,
                                   uint32_t hcap, const uint32_t* tokens, uint32_t batch,
                                   uint32_t* pos, const float* u_seq, uint32_t u_len);

#ifdef __cplusplus
}  /* extern "C" */
#endif
