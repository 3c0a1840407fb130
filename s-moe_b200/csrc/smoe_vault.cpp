// smoe_vault.cpp - .smoe vault reader and device uploader.
//
// The vault format is the reference's (common.hpp:52-183, written by
// scripts/shatter_moe.py:627-674 and :1044-1099): a 64-byte header at offset
// 0, `total_experts` 48-byte expert entries at table_offset, then 3 44-byte
// tensor descriptors per expert (gate, up, down), the 128-byte arch block at
// reserved_ext (v2), and page-aligned expert blobs from data_offset, each
// [gate nibbles][gate fp16 scales][up ...][down ...]. The checks follow the
// engine's reader (main.cpp:96-198). The engine mmaps the vault and hands
// blob pointers to the compute layer; here a layer's blobs are copied once
// into a device arena (one cudaMemcpyAsync per expert), after which the
// layer is an ordinary SmoeMoeLayer (SMOE-Q4, vault layout) that
// smoe_cuda_prepack_layer can re-lay out for the single-launch layer kernel.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

#include "../../include/smoe_cuda.h"

namespace {

#pragma pack(push, 1)
struct VaultHeader {                 // common.hpp:57-72
    uint8_t magic[8];
    uint32_t version, num_moe_layers, max_experts_per_layer, total_experts;
    uint64_t table_offset, data_offset;
    uint32_t group_size, bits, d_model, vocab_size, ffn_dim, reserved_ext;
};
struct VaultArch {                   // common.hpp:96-113
    uint8_t magic[4];
    uint32_t block_version, block_size, flags;
    float rope_theta;
    uint32_t num_heads, num_kv_heads, head_dim, moe_top_k, moe_ffn_dim, dense_ffn_dim, shared_expert_ffn_dim,
        activation, num_hidden_layers;
    float rms_norm_eps;
    char model_type[24];
    uint8_t reserved[44];
};
struct VaultEntry {                  // common.hpp:143-152
    uint32_t layer_id, expert_id;
    uint64_t byte_offset, raw_size, padded_size;
    uint32_t group_size;
    uint64_t num_groups;
    uint8_t reserved[4];
};
struct VaultDesc {                   // common.hpp:166-176
    uint8_t tensor_type, ndim, reserved_0[2];
    uint32_t rows, cols;
    uint64_t packed_offset, packed_size, scales_offset, scales_size;
};
#pragma pack(pop)
static_assert(sizeof(VaultHeader) == 64 && sizeof(VaultArch) == 128 && sizeof(VaultEntry) == 48 &&
                  sizeof(VaultDesc) == 44, "vault record sizes");

constexpr uint8_t kMagic[8] = {'S', 'M', 'O', 'E', 0xDE, 0xEA, 0x00, 0x01};   // common.hpp:44-47
constexpr uint8_t kArchMagic[4] = {'S', 'A', 'R', 'C'};

thread_local char g_verr[256] = "";

int fail(int code, const char* msg, unsigned long long v = 0) {
    std::snprintf(g_verr, sizeof(g_verr), "%s (%llu)", msg, v);
    return code;
}

bool in_file(uint64_t off, uint64_t len, uint64_t size) { return off <= size && len <= size - off; }

// Header, arch block and the table bounds; entries and descriptors are read
// in place (the vault is byte-packed, so through memcpy).
int parse(const uint8_t* v, uint64_t size, SmoeVaultInfo* out) {
    if (!v || !out) return fail(SMOE_ERR_ARG, "null argument");
    std::memset(out, 0, sizeof(*out));
    VaultHeader h;
    if (size < sizeof(h)) return fail(SMOE_ERR_ARG, "vault too small", size);
    std::memcpy(&h, v, sizeof(h));
    if (std::memcmp(h.magic, kMagic, 8) != 0) return fail(SMOE_ERR_ARG, "bad magic: not a .smoe vault");
    if (h.version < 1 || h.version > 2) return fail(SMOE_ERR_ARG, "unsupported vault version", h.version);
    const uint64_t tbytes = uint64_t(h.total_experts) * sizeof(VaultEntry);
    const uint64_t dbytes = uint64_t(h.total_experts) * 3 * sizeof(VaultDesc);
    if (h.total_experts == 0 || !in_file(h.table_offset, tbytes + dbytes, size))
        return fail(SMOE_ERR_ARG, "expert table outside the vault", h.table_offset);
    out->version = h.version;
    out->num_moe_layers = h.num_moe_layers;
    out->max_experts_per_layer = h.max_experts_per_layer;
    out->total_experts = h.total_experts;
    out->table_offset = h.table_offset;
    out->data_offset = h.data_offset;
    out->group_size = h.group_size;
    out->bits = h.bits;
    out->d_model = h.d_model;
    out->vocab_size = h.vocab_size;
    out->ffn_dim = h.ffn_dim;
    if (h.version >= 2) {            // main.cpp:124-158: a v2 vault needs a valid arch block
        VaultArch a;
        if (h.reserved_ext == 0 || uint64_t(h.reserved_ext) + sizeof(a) > h.data_offset ||
            !in_file(h.reserved_ext, sizeof(a), size))
            return fail(SMOE_ERR_ARG, "v2 vault has no valid arch-block offset", h.reserved_ext);
        std::memcpy(&a, v + h.reserved_ext, sizeof(a));
        if (std::memcmp(a.magic, kArchMagic, 4) != 0 || a.block_size != sizeof(VaultArch) || a.block_version != 1)
            return fail(SMOE_ERR_ARG, "corrupt arch block", h.reserved_ext);
        if (a.activation != 0) return fail(SMOE_ERR_UNSUPPORTED, "activation is not SiLU", a.activation);
        if (a.moe_top_k == 0 || a.moe_top_k > SMOE_MAX_ACTIVE || a.head_dim == 0 || a.head_dim > 256 ||
            a.num_heads == 0 || a.num_kv_heads == 0 || a.num_heads % a.num_kv_heads != 0)
            return fail(SMOE_ERR_ARG, "arch block values out of engine limits", a.moe_top_k);
        out->has_arch = 1;
        out->arch_flags = a.flags;
        out->rope_theta = a.rope_theta;
        out->num_heads = a.num_heads;
        out->num_kv_heads = a.num_kv_heads;
        out->head_dim = a.head_dim;
        out->moe_top_k = a.moe_top_k;
        out->moe_ffn_dim = a.moe_ffn_dim;
        out->dense_ffn_dim = a.dense_ffn_dim;
        out->shared_expert_ffn_dim = a.shared_expert_ffn_dim;
        out->num_hidden_layers = a.num_hidden_layers;
        out->rms_norm_eps = a.rms_norm_eps;
        std::memcpy(out->model_type, a.model_type, sizeof(out->model_type));
        out->model_type[sizeof(out->model_type) - 1] = 0;
    }
    // main.cpp:170-198: the first expert's descriptors give every expert's layout
    VaultDesc d[3];
    std::memcpy(d, v + h.table_offset + tbytes, sizeof(d));
    for (int m = 0; m < 3; ++m)
        if (d[m].tensor_type != m || d[m].rows == 0 || d[m].cols == 0)
            return fail(SMOE_ERR_ARG, "bad tensor descriptor", m);
    out->gate_rows = d[0].rows; out->gate_cols = d[0].cols;
    out->up_rows = d[1].rows; out->up_cols = d[1].cols;
    out->down_rows = d[2].rows; out->down_cols = d[2].cols;
    out->gate_packed_offset = d[0].packed_offset; out->gate_scales_offset = d[0].scales_offset;
    out->up_packed_offset = d[1].packed_offset; out->up_scales_offset = d[1].scales_offset;
    out->down_packed_offset = d[2].packed_offset; out->down_scales_offset = d[2].scales_offset;
    uint64_t maxraw = 0;
    for (uint32_t i = 0; i < h.total_experts; ++i) {
        VaultEntry e;
        std::memcpy(&e, v + h.table_offset + uint64_t(i) * sizeof(e), sizeof(e));
        if (!in_file(e.byte_offset, e.raw_size, size)) return fail(SMOE_ERR_ARG, "expert blob outside the vault", i);
        if (e.layer_id >= h.num_moe_layers || e.expert_id >= h.max_experts_per_layer)
            return fail(SMOE_ERR_ARG, "expert entry out of range", i);
        if (e.raw_size > maxraw) maxraw = e.raw_size;
    }
    out->max_raw_size = maxraw;
    return SMOE_OK;
}

}  // namespace

extern "C" {

const char* smoe_cuda_vault_last_error(void) { return g_verr; }

int smoe_cuda_vault_parse(const void* vault, uint64_t size, SmoeVaultInfo* out) {
    return parse(static_cast<const uint8_t*>(vault), size, out);
}

int smoe_cuda_vault_expert(const void* vault, uint64_t size, uint32_t layer, uint32_t expert, uint64_t* offset,
                           uint64_t* raw_size) {
    SmoeVaultInfo info;
    int rc = parse(static_cast<const uint8_t*>(vault), size, &info);
    if (rc) return rc;
    const uint8_t* v = static_cast<const uint8_t*>(vault);
    for (uint32_t i = 0; i < info.total_experts; ++i) {
        VaultEntry e;
        std::memcpy(&e, v + info.table_offset + uint64_t(i) * sizeof(e), sizeof(e));
        if (e.layer_id == layer && e.expert_id == expert) {
            if (offset) *offset = e.byte_offset;
            if (raw_size) *raw_size = e.raw_size;
            return SMOE_OK;
        }
    }
    return fail(SMOE_ERR_ARG, "no such expert in the vault", (unsigned long long)layer * 65536ull + expert);
}

int smoe_cuda_vault_upload_layer(SmoeCudaCtx* ctx, const void* vault, uint64_t size, uint32_t layer, void* dst,
                                 uint64_t dst_stride, const uint16_t* router_w, SmoeMoeLayer* out) {
    if (!ctx || !dst || !out) return fail(SMOE_ERR_ARG, "null argument");
    SmoeVaultInfo info;
    int rc = parse(static_cast<const uint8_t*>(vault), size, &info);
    if (rc) return rc;
    if (layer >= info.num_moe_layers) return fail(SMOE_ERR_ARG, "layer beyond the vault", layer);
    if (info.bits != 4 || info.group_size != 64)
        return fail(SMOE_ERR_UNSUPPORTED, "only 4-bit group-64 (SMOE-Q4) vaults are uploaded; bits", info.bits);
    const uint32_t dff = info.gate_rows, d = info.gate_cols;
    if (info.up_rows != dff || info.up_cols != d || info.down_rows != d || info.down_cols != dff || d % 64 ||
        dff % 64)
        return fail(SMOE_ERR_ARG, "inconsistent expert shapes", d);
    const uint64_t offs[6] = {info.gate_packed_offset, info.gate_scales_offset, info.up_packed_offset,
                              info.up_scales_offset, info.down_packed_offset, info.down_scales_offset};
    for (uint64_t o : offs)
        if (o % 16) return fail(SMOE_ERR_UNSUPPORTED, "tensor offsets inside the blob must be 16-byte aligned", o);
    if (dst_stride < info.max_raw_size || dst_stride % 16 || (reinterpret_cast<uintptr_t>(dst) & 15u))
        return fail(SMOE_ERR_ARG, "destination stride below the largest blob or unaligned", dst_stride);
    cudaStream_t s = static_cast<cudaStream_t>(smoe_cuda_get_stream(ctx));
    const uint8_t* v = static_cast<const uint8_t*>(vault);
    uint32_t seen = 0;
    for (uint32_t i = 0; i < info.total_experts; ++i) {
        VaultEntry e;
        std::memcpy(&e, v + info.table_offset + uint64_t(i) * sizeof(e), sizeof(e));
        if (e.layer_id != layer) continue;
        cudaError_t ce = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + uint64_t(e.expert_id) * dst_stride,
                                         v + e.byte_offset, e.raw_size, cudaMemcpyHostToDevice, s);
        if (ce != cudaSuccess) return fail(SMOE_ERR_CUDA, cudaGetErrorString(ce), i);
        ++seen;
    }
    if (seen != info.max_experts_per_layer)
        return fail(SMOE_ERR_ARG, "layer is missing experts in the vault; found", seen);
    std::memset(out, 0, sizeof(*out));
    out->base = static_cast<const uint8_t*>(dst);
    out->expert_stride = dst_stride;
    for (int m = 0; m < 3; ++m) {
        out->off[3 * m] = offs[2 * m];
        out->off[3 * m + 1] = offs[2 * m + 1];
        out->off[3 * m + 2] = 0;
    }
    out->n_experts = info.max_experts_per_layer;
    out->d_model = d;
    out->d_ff = dff;
    out->fmt = SMOE_FMT_SMOE_Q4;
    out->router_w = router_w;
    return SMOE_OK;
}

}  // extern "C"
