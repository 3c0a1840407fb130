"""Python host binding of the C ABI in include/smoe_cuda.h (ctypes).

Mirrors the reference's compute interface (src/compute/metal_bridge.h) name
for name with the ``smoe_cuda_`` prefix, plus the native router / MoE-layer /
sampler entries. Device buffers are passed as integer addresses or as
objects with ``data_ptr()`` (torch tensors). There is no CPU fallback: if
libsmoe_cuda.so is missing or no GPU is present, calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SMOE_CUDA_LIB") or os.path.join(HERE, "libsmoe_cuda.so")   # override: another build of the library

SMOE_OK = 0
SMOE_ERR_ARG, SMOE_ERR_CUDA, SMOE_ERR_TIMEOUT, SMOE_ERR_DEVICE = 1, 2, 3, 5
STATUS = {0: "OK", 1: "ERR_ARG", 2: "ERR_CUDA", 3: "ERR_TIMEOUT", 4: "ERR_NCCL",
          5: "ERR_DEVICE", 6: "ERR_UNSUPPORTED"}
FMT_SMOE_Q4 = 0
FMT_AFFINE_Q4 = 1
LAYOUT_TILED = 0x100
DTYPE_F32 = 0
DTYPE_BF16 = 1
MAX_ACTIVE = 16
MAX_FFN_BATCH = 64

# Every symbol include/smoe_cuda.h declares (checked by the CPU tests).
EXPORTS = [
    "smoe_cuda_init", "smoe_cuda_init_ex", "smoe_cuda_destroy", "smoe_cuda_last_error",
    "smoe_cuda_set_stream", "smoe_cuda_get_stream", "smoe_cuda_synchronize",
    "smoe_cuda_fused_ffn", "smoe_cuda_wait", "smoe_cuda_fused_ffn_group",
    "smoe_cuda_fused_ffn_batch", "smoe_cuda_wait_ffn_batch", "smoe_cuda_scout_matvec_bf16",
    "smoe_cuda_register_buffer", "smoe_cuda_kernel_dispatches", "smoe_cuda_router_topk",
    "smoe_cuda_moe_ffn", "smoe_cuda_moe_layer", "smoe_cuda_sample",
    "smoe_cuda_canonical_from_u32", "smoe_cuda_moe_ffn_noalloc", "smoe_cuda_noalloc_last_error",
    "smoe_cuda_noalloc_check", "smoe_cuda_scout_matvec_batch_bf16", "smoe_cuda_scout_matvec_group_bf16",
    "smoe_cuda_tiled_expert_bytes", "smoe_cuda_prepack_layer",
    "smoe_cuda_ep_export", "smoe_cuda_ep_attach", "smoe_cuda_moe_layer_ep",
    "smoe_cuda_attention_layer", "smoe_cuda_attention_layer_async", "smoe_cuda_matvec_bf16",
    "smoe_cuda_rms_norm", "smoe_cuda_embed_bf16", "smoe_cuda_rope_table", "smoe_cuda_decode_advance",
    "smoe_cuda_gemm_bf16", "smoe_cuda_attention_batch_async", "smoe_cuda_decode_advance_batch",
    "smoe_cuda_rope_tables", "smoe_cuda_attention_prefill_async",
    "smoe_cuda_vault_parse", "smoe_cuda_vault_expert", "smoe_cuda_vault_upload_layer", "smoe_cuda_vault_last_error",
    "smoe_cuda_moe_layer_shard",
]


class VaultInfo(C.Structure):
    """SmoeVaultInfo (a parsed .smoe vault header, arch block and layout)."""
    _fields_ = [(n, C.c_uint32) for n in ("version", "num_moe_layers", "max_experts_per_layer", "total_experts",
                                          "group_size", "bits", "d_model", "vocab_size", "ffn_dim")] + \
              [("table_offset", C.c_uint64), ("data_offset", C.c_uint64)] + \
              [(n, C.c_uint32) for n in ("has_arch", "arch_flags", "num_heads", "num_kv_heads", "head_dim",
                                          "moe_top_k", "moe_ffn_dim", "dense_ffn_dim", "shared_expert_ffn_dim",
                                          "num_hidden_layers")] + \
              [("rope_theta", C.c_float), ("rms_norm_eps", C.c_float), ("model_type", C.c_char * 24)] + \
              [(n, C.c_uint32) for n in ("gate_rows", "gate_cols", "up_rows", "up_cols", "down_rows", "down_cols")] + \
              [(n, C.c_uint64) for n in ("gate_packed_offset", "gate_scales_offset", "up_packed_offset",
                                          "up_scales_offset", "down_packed_offset", "down_scales_offset",
                                          "max_raw_size")]


class AttnLayerArgs(C.Structure):
    """SmoeCudaAttnLayerArgs (device pointers)."""
    _fields_ = [(n, C.c_void_p) for n in ("w_q", "w_k", "w_v", "w_o", "q_norm_w", "k_norm_w", "rope_cos",
                                          "rope_sin", "normed_in", "qbuf", "kbuf", "vbuf", "k_cache",
                                          "v_cache", "attn_out", "o_out")] + \
              [(n, C.c_uint32) for n in ("d_model", "q_dim", "kv_dim", "head_dim", "num_heads",
                                         "num_kv_heads", "slot", "valid", "attn_ctx")] + \
              [("attn_scale", C.c_float)]


class EpHandle(C.Structure):
    _fields_ = [("bytes", C.c_uint8 * 64)]


def ep_partition(n_experts: int, world: int, rank: int):
    """Experts held by `rank`: [base, base + count) of an even split (the
    235B layout: 128 experts over 8 GPUs -> 16 each)."""
    if world < 1 or not 0 <= rank < world or n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    return rank * per, per


class SmoeCudaError(RuntimeError):
    pass


def ep_exchange_handles(mine: bytes, world: int, group=None, timeout_s: float = 60.0):
    """All-gather every rank's 64-byte exchange-window handle in rank order
    (what ep_attach expects) over a torch.distributed group (gloo is enough).
    A rank that never joins makes the others raise SmoeCudaError after
    timeout_s instead of waiting forever."""
    import datetime
    import torch
    import torch.distributed as dist
    if len(mine) != 64:
        raise ValueError("an exchange handle is 64 bytes")
    if world == 1:
        return [mine]
    t = torch.frombuffer(bytearray(mine), dtype=torch.uint8)
    out = [torch.empty(64, dtype=torch.uint8) for _ in range(world)]
    try:
        work = dist.all_gather(out, t, group=group, async_op=True)
        if not work.wait(timeout=datetime.timedelta(seconds=timeout_s)):
            raise SmoeCudaError("expert-parallel handle exchange timed out")
    except RuntimeError as e:             # gloo reports the missing peer as an error
        raise SmoeCudaError(f"expert-parallel handle exchange failed: {e}") from e
    return [bytes(o.numpy().tobytes()) for o in out]


class InitArgs(C.Structure):
    _fields_ = [("device", C.c_int), ("max_d_model", C.c_uint32), ("max_d_ff", C.c_uint32),
                ("max_experts", C.c_uint32), ("max_batch", C.c_uint32),
                ("max_vocab", C.c_uint32), ("timeout_ms", C.c_uint32),
                ("device_wait_us", C.c_uint32)]


class ExpertBlob(C.Structure):
    _fields_ = [("packed_gate", C.c_void_p), ("scales_gate", C.c_void_p),
                ("packed_up", C.c_void_p), ("scales_up", C.c_void_p),
                ("packed_down", C.c_void_p), ("scales_down", C.c_void_p),
                ("slot", C.c_uint32)]


class MoeLayer(C.Structure):
    _fields_ = [("base", C.c_void_p), ("expert_stride", C.c_uint64), ("off", C.c_uint64 * 9),
                ("n_experts", C.c_uint32), ("d_model", C.c_uint32), ("d_ff", C.c_uint32),
                ("fmt", C.c_uint32), ("router_w", C.c_void_p)]


class SamplerRow(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_p", C.c_float), ("top_k", C.c_uint32),
                ("rep_penalty", C.c_float), ("u", C.c_float), ("history_len", C.c_uint32)]


_lib = None


def lib():
    """Load libsmoe_cuda.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SmoeCudaError(f"{LIB_PATH} not built (python s-moe_b200/build.py)")
        L = C.CDLL(LIB_PATH)
        vp, u32, u64, i32, f32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int, C.c_float
        L.smoe_cuda_init.argtypes = [C.c_size_t]
        L.smoe_cuda_init.restype = vp
        L.smoe_cuda_init_ex.argtypes = [C.POINTER(InitArgs)]
        L.smoe_cuda_init_ex.restype = vp
        L.smoe_cuda_destroy.argtypes = [vp]
        L.smoe_cuda_last_error.restype = C.c_char_p
        L.smoe_cuda_set_stream.argtypes = [vp, vp]
        L.smoe_cuda_get_stream.argtypes = [vp]
        L.smoe_cuda_get_stream.restype = vp
        L.smoe_cuda_synchronize.argtypes = [vp]
        L.smoe_cuda_fused_ffn.argtypes = [vp] * 10 + [u32] * 7
        L.smoe_cuda_fused_ffn.restype = vp
        L.smoe_cuda_wait.argtypes = [vp, vp, vp, u32, u32]
        L.smoe_cuda_fused_ffn_group.argtypes = [vp, C.POINTER(ExpertBlob), u32, vp] + [u32] * 6
        L.smoe_cuda_fused_ffn_group.restype = vp
        L.smoe_cuda_fused_ffn_batch.argtypes = [vp] * 8 + [u32] * 7
        L.smoe_cuda_fused_ffn_batch.restype = vp
        L.smoe_cuda_wait_ffn_batch.argtypes = [vp, vp, vp, u32, u32]
        L.smoe_cuda_scout_matvec_bf16.argtypes = [vp, vp, vp, vp, u32, u32]
        L.smoe_cuda_scout_matvec_batch_bf16.argtypes = [vp, vp, vp, vp, vp, vp, u32]
        L.smoe_cuda_scout_matvec_group_bf16.argtypes = [vp, vp, vp, vp, vp, vp, u32]
        L.smoe_cuda_register_buffer.argtypes = [vp, vp, C.c_size_t]
        L.smoe_cuda_kernel_dispatches.argtypes = [vp]
        L.smoe_cuda_kernel_dispatches.restype = u64
        L.smoe_cuda_router_topk.argtypes = [vp, vp, vp, i32, u32, u32, u32, u32, i32, vp, vp, vp]
        L.smoe_cuda_moe_ffn.argtypes = [vp, C.POINTER(MoeLayer), vp, i32, vp, vp, u32, u32, vp, i32]
        L.smoe_cuda_moe_layer.argtypes = [vp, C.POINTER(MoeLayer), vp, i32, u32, u32, i32, vp,
                                          i32, vp, vp]
        L.smoe_cuda_sample.argtypes = [vp, vp, u32, u32, vp, vp, u32, vp]
        L.smoe_cuda_ep_export.argtypes = [vp, C.POINTER(EpHandle)]
        L.smoe_cuda_attention_layer.argtypes = [vp, C.POINTER(AttnLayerArgs)]
        L.smoe_cuda_attention_layer_async.argtypes = [vp, C.POINTER(AttnLayerArgs), vp]
        L.smoe_cuda_matvec_bf16.argtypes = [vp, vp, vp, vp, u32, u32]
        L.smoe_cuda_rms_norm.argtypes = [vp, vp, vp, vp, vp, u32, u32]
        L.smoe_cuda_embed_bf16.argtypes = [vp, vp, vp, u32, u32, vp]
        L.smoe_cuda_rope_table.argtypes = [vp, vp, vp, vp, vp, u32]
        L.smoe_cuda_decode_advance.argtypes = [vp, vp, vp, u32, vp, vp, vp, u32]
        L.smoe_cuda_gemm_bf16.argtypes = [vp, vp, vp, vp, u32, u32, u32]
        L.smoe_cuda_attention_batch_async.argtypes = [vp, C.POINTER(AttnLayerArgs), u32, u64, vp]
        L.smoe_cuda_decode_advance_batch.argtypes = [vp, vp, vp, u32, vp, u32, vp, vp, u32]
        L.smoe_cuda_rope_tables.argtypes = [vp, vp, u32, vp, vp, vp, u32]
        L.smoe_cuda_vault_parse.argtypes = [vp, u64, C.POINTER(VaultInfo)]
        L.smoe_cuda_vault_expert.argtypes = [vp, u64, u32, u32, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
        L.smoe_cuda_vault_upload_layer.argtypes = [vp, vp, u64, u32, vp, u64, vp, C.POINTER(MoeLayer)]
        L.smoe_cuda_vault_last_error.restype = C.c_char_p
        L.smoe_cuda_attention_prefill_async.argtypes = [vp, C.POINTER(AttnLayerArgs), u32, vp]
        L.smoe_cuda_ep_attach.argtypes = [vp, i32, i32, C.POINTER(EpHandle)]
        L.smoe_cuda_moe_layer_ep.argtypes = [vp, C.POINTER(MoeLayer), u32, u32, vp, i32, u32, u32, i32,
                                             vp, i32, vp, vp]
        L.smoe_cuda_moe_layer_shard.argtypes = [vp, C.POINTER(MoeLayer), u32, u32, vp, i32, u32, u32, i32, vp,
                                                vp, vp]
        L.smoe_cuda_moe_ffn_noalloc.argtypes = [C.POINTER(MoeLayer), vp, i32, vp, vp, u32, u32, vp,
                                                i32, vp]
        L.smoe_cuda_noalloc_last_error.restype = C.c_char_p
        L.smoe_cuda_noalloc_check.argtypes = [vp, u32]
        L.smoe_cuda_tiled_expert_bytes.argtypes = [u32, u32, u32]
        L.smoe_cuda_tiled_expert_bytes.restype = u64
        L.smoe_cuda_prepack_layer.argtypes = [vp, C.POINTER(MoeLayer), vp, u64, C.POINTER(MoeLayer)]
        L.smoe_cuda_debug_expf.argtypes = [vp, vp, u32, vp]
        L.smoe_cuda_canonical_from_u32.argtypes = [u32]
        L.smoe_cuda_canonical_from_u32.restype = f32
        _lib = L
    return _lib


def ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):          # numpy (host memory)
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)}")


def last_error() -> str:
    return lib().smoe_cuda_last_error().decode()


def check(rc: int, what: str = "") -> None:
    if rc != SMOE_OK:
        raise SmoeCudaError(f"{what}: {STATUS.get(rc, rc)}: {last_error()}")


def canonical_from_u32(word: int) -> float:
    return float(lib().smoe_cuda_canonical_from_u32(word))


class Context:
    """One smoe_cuda context (scratch, stream, event ring) on one device."""

    def __init__(self, device: int = 0, max_d_model=0, max_d_ff=0, max_experts=0,
                 max_batch=0, max_vocab=0, timeout_ms=0, device_wait_us=0):
        a = InitArgs(device, max_d_model, max_d_ff, max_experts, max_batch, max_vocab, timeout_ms,
                     device_wait_us)
        self.L = lib()
        self.h = self.L.smoe_cuda_init_ex(C.byref(a))
        if not self.h:
            raise SmoeCudaError(f"smoe_cuda_init_ex failed: {last_error()}")

    def close(self):
        if self.h:
            self.L.smoe_cuda_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -------------------------------------------------------------- plumbing
    def set_stream(self, stream_handle: int | None):
        check(self.L.smoe_cuda_set_stream(self.h, stream_handle), "set_stream")

    def synchronize(self):
        check(self.L.smoe_cuda_synchronize(self.h), "synchronize")

    def dispatches(self) -> int:
        return int(self.L.smoe_cuda_kernel_dispatches(self.h))

    # ------------------------------------------------------------ mirrored
    def fused_ffn_group(self, blobs, input_vec, gate_rows, gate_cols, group_size=64, bits=4):
        arr = (ExpertBlob * len(blobs))(*blobs)
        h = self.L.smoe_cuda_fused_ffn_group(self.h, arr, len(blobs), ptr(input_vec), gate_rows,
                                             gate_cols, gate_cols, gate_rows, group_size, bits)
        if not h:
            raise SmoeCudaError(f"fused_ffn_group: {last_error()}")
        return h

    def fused_ffn(self, pg, sg, pu, su, pd, sd, input_vec, gate_rows, gate_cols, expert_index,
                  group_size=64, bits=4):
        h = self.L.smoe_cuda_fused_ffn(self.h, ptr(pg), ptr(sg), ptr(pu), ptr(su), ptr(pd), ptr(sd),
                                       ptr(input_vec), None, None, gate_rows, gate_cols, gate_cols,
                                       gate_rows, group_size, bits, expert_index)
        if not h:
            raise SmoeCudaError(f"fused_ffn: {last_error()}")
        return h

    def wait(self, handle, output_vec, slot, cols):
        self.L.smoe_cuda_wait(self.h, handle, ptr(output_vec), slot, cols)

    def fused_ffn_batch(self, pg, sg, pu, su, pd, sd, input_mat, batch, gate_rows, gate_cols,
                        group_size=64, bits=4):
        h = self.L.smoe_cuda_fused_ffn_batch(self.h, ptr(pg), ptr(sg), ptr(pu), ptr(su), ptr(pd),
                                             ptr(sd), ptr(input_mat), batch, gate_rows, gate_cols,
                                             gate_cols, gate_rows, group_size, bits)
        if not h:
            raise SmoeCudaError(f"fused_ffn_batch: {last_error()}")
        return h

    def wait_ffn_batch(self, handle, out_mat, batch, cols):
        self.L.smoe_cuda_wait_ffn_batch(self.h, handle, ptr(out_mat), batch, cols)

    def scout_matvec_bf16(self, weight, input_vec, output_vec, rows, cols):
        self.L.smoe_cuda_scout_matvec_bf16(self.h, ptr(weight), ptr(input_vec), ptr(output_vec),
                                           rows, cols)

    # -------------------------------------------------------------- native
    def router_topk(self, router_w, x, x_dtype, n_experts, d_model, batch, k, norm, ids, weights,
                    logits=None):
        check(self.L.smoe_cuda_router_topk(self.h, ptr(router_w), ptr(x), x_dtype, n_experts,
                                           d_model, batch, k, int(norm), ptr(ids), ptr(weights),
                                           ptr(logits)), "router_topk")

    def moe_ffn(self, layer: MoeLayer, x, x_dtype, ids, weights, k, batch, y, y_dtype):
        check(self.L.smoe_cuda_moe_ffn(self.h, C.byref(layer), ptr(x), x_dtype, ptr(ids),
                                       ptr(weights), k, batch, ptr(y), y_dtype), "moe_ffn")

    def moe_layer(self, layer: MoeLayer, x, x_dtype, batch, k, norm, y, y_dtype, ids=None,
                  weights=None):
        check(self.L.smoe_cuda_moe_layer(self.h, C.byref(layer), ptr(x), x_dtype, batch, k,
                                         int(norm), ptr(y), y_dtype, ptr(ids), ptr(weights)),
              "moe_layer")

    # ---- expert parallel (one process per GPU)
    def ep_export(self) -> bytes:
        h = EpHandle()
        check(self.L.smoe_cuda_ep_export(self.h, C.byref(h)), "ep_export")
        return bytes(h.bytes)

    def ep_attach(self, rank: int, world: int, handles):
        arr = (EpHandle * world)()
        for r, b in enumerate(handles):
            C.memmove(arr[r].bytes, bytes(b), 64)
        check(self.L.smoe_cuda_ep_attach(self.h, rank, world, arr), "ep_attach")

    def moe_layer_shard(self, shard: MoeLayer, n_experts_total, expert_base, x, x_dtype, batch, k, norm, y_partial,
                        ids=None, w=None):
        check(self.L.smoe_cuda_moe_layer_shard(self.h, C.byref(shard), n_experts_total, expert_base, ptr(x), x_dtype,
                                               batch, k, int(norm), ptr(y_partial), ptr(ids), ptr(w)),
              "moe_layer_shard")

    def moe_layer_ep(self, shard: MoeLayer, n_experts_total, expert_base, x, x_dtype, batch, k, norm,
                     y, y_dtype, ids=None, weights=None):
        check(self.L.smoe_cuda_moe_layer_ep(self.h, C.byref(shard), n_experts_total, expert_base,
                                            ptr(x), x_dtype, batch, k, int(norm), ptr(y), y_dtype,
                                            ptr(ids), ptr(weights)), "moe_layer_ep")

    def prepack_layer(self, layer: MoeLayer, dst, dst_stride: int) -> MoeLayer:
        """Tiled copy of a vault-layout layer (dst: device buffer of
        n_experts * dst_stride bytes, kept alive by the caller)."""
        out = MoeLayer()
        check(self.L.smoe_cuda_prepack_layer(self.h, C.byref(layer), ptr(dst), dst_stride,
                                             C.byref(out)), "prepack_layer")
        return out

    # ---- dense trunk
    def attention_layer(self, args: AttnLayerArgs, pos=None, sync=False):
        if sync:
            check(self.L.smoe_cuda_attention_layer(self.h, C.byref(args)), "attention_layer")
        else:
            check(self.L.smoe_cuda_attention_layer_async(self.h, C.byref(args), ptr(pos)), "attention_layer")

    def matvec_bf16(self, w, x, y, rows, cols):
        check(self.L.smoe_cuda_matvec_bf16(self.h, ptr(w), ptr(x), ptr(y), rows, cols), "matvec_bf16")

    def rms_norm(self, hidden, delta, w, normed, n, rows=1):
        check(self.L.smoe_cuda_rms_norm(self.h, ptr(hidden), ptr(delta), ptr(w), ptr(normed), n, rows), "rms_norm")

    def embed_bf16(self, table, tokens, n_tokens, d_model, out):
        check(self.L.smoe_cuda_embed_bf16(self.h, ptr(table), ptr(tokens), n_tokens, d_model, ptr(out)),
              "embed_bf16")

    def rope_table(self, pos, inv_freq, cos_out, sin_out, half):
        check(self.L.smoe_cuda_rope_table(self.h, ptr(pos), ptr(inv_freq), ptr(cos_out), ptr(sin_out), half),
              "rope_table")

    def decode_advance(self, row, history, hcap, token, pos, u_seq=None, u_len=0):
        check(self.L.smoe_cuda_decode_advance(self.h, ptr(row), ptr(history), hcap, ptr(token), ptr(pos),
                                              ptr(u_seq), u_len), "decode_advance")

    # ---- batched decode (sequences at one shared position)
    def gemm_bf16(self, w, x, y, rows, cols, batch):
        check(self.L.smoe_cuda_gemm_bf16(self.h, ptr(w), ptr(x), ptr(y), rows, cols, batch), "gemm_bf16")

    def attention_batch(self, args: AttnLayerArgs, batch, kv_seq_stride, pos):
        check(self.L.smoe_cuda_attention_batch_async(self.h, C.byref(args), batch, kv_seq_stride, ptr(pos)),
              "attention_batch")

    def vault_upload_layer(self, vault, layer, dst, dst_stride, router_w) -> MoeLayer:
        """Copy a vault layer's expert blobs into the device arena dst."""
        p, n = _vault_bytes(vault)
        out = MoeLayer()
        rc = self.L.smoe_cuda_vault_upload_layer(self.h, p, n, layer, ptr(dst), dst_stride, ptr(router_w),
                                                 C.byref(out))
        if rc:
            raise SmoeCudaError(f"vault_upload_layer: {STATUS.get(rc, rc)}: " + self.L.smoe_cuda_vault_last_error().decode())
        return out

    def rope_tables(self, pos, n, inv_freq, cos_out, sin_out, half):
        check(self.L.smoe_cuda_rope_tables(self.h, ptr(pos), n, ptr(inv_freq), ptr(cos_out), ptr(sin_out), half),
              "rope_tables")

    def attention_prefill(self, args: AttnLayerArgs, n_tokens, pos):
        check(self.L.smoe_cuda_attention_prefill_async(self.h, C.byref(args), n_tokens, ptr(pos)),
              "attention_prefill")

    def decode_advance_batch(self, rows, history, hcap, tokens, batch, pos, u_seq=None, u_len=0):
        check(self.L.smoe_cuda_decode_advance_batch(self.h, ptr(rows), ptr(history), hcap, ptr(tokens), batch,
                                                    ptr(pos), ptr(u_seq), u_len), "decode_advance_batch")

    def sample(self, logits, vocab, batch, rows, history, history_stride, tokens):
        check(self.L.smoe_cuda_sample(self.h, ptr(logits), vocab, batch, ptr(rows), ptr(history),
                                      history_stride, ptr(tokens)), "sample")


def _vault_bytes(vault):
    """(pointer, size) of a vault held in host memory (numpy uint8 array or bytes)."""
    import numpy as np
    a = np.frombuffer(vault, np.uint8) if isinstance(vault, (bytes, bytearray, memoryview)) else vault
    return a.ctypes.data, a.nbytes


def vault_parse(vault) -> VaultInfo:
    """Parse a .smoe vault (host bytes); raises SmoeCudaError with the reader's message."""
    p, n = _vault_bytes(vault)
    info = VaultInfo()
    rc = lib().smoe_cuda_vault_parse(p, n, C.byref(info))
    if rc:
        raise SmoeCudaError(f"vault_parse: {STATUS.get(rc, rc)}: " + lib().smoe_cuda_vault_last_error().decode())
    return info


def vault_expert(vault, layer: int, expert: int):
    """(byte offset, unpadded size) of one expert blob."""
    p, n = _vault_bytes(vault)
    off, raw = C.c_uint64(), C.c_uint64()
    rc = lib().smoe_cuda_vault_expert(p, n, layer, expert, C.byref(off), C.byref(raw))
    if rc:
        raise SmoeCudaError(f"vault_expert: {STATUS.get(rc, rc)}: " + lib().smoe_cuda_vault_last_error().decode())
    return off.value, raw.value


def make_layer(base, stride, off, n_experts, d_model, d_ff, fmt, router_w) -> MoeLayer:
    L = MoeLayer()
    L.base = ptr(base)
    L.expert_stride = stride
    for i in range(9):
        L.off[i] = off[i]
    L.n_experts = n_experts
    L.d_model = d_model
    L.d_ff = d_ff
    L.fmt = fmt
    L.router_w = ptr(router_w)
    return L


def blob_layout(fmt: int, d_model: int, d_ff: int):
    """Byte offsets of the 9 tensors of one vault expert blob - per matrix
    (gate [d_ff x d_model], up, down [d_model x d_ff]) nibbles, scales (one
    16-bit value per 64 weights), biases (AFFINE-Q4 only) - and the blob's
    byte count without padding (shatter_moe.py:627-674)."""
    off, cur = [], 0
    for rows, cols in ((d_ff, d_model), (d_ff, d_model), (d_model, d_ff)):
        nib, sc = rows * cols // 2, rows * cols // 64 * 2
        off.append(cur)
        cur += nib
        off.append(cur)
        cur += sc
        off.append(cur)
        if fmt == FMT_AFFINE_Q4:
            cur += sc
    return off, cur


def expert_bytes(fmt: int, d_model: int, d_ff: int) -> int:
    """Bytes one expert's FFN reads (the vault blob without padding)."""
    return blob_layout(fmt, d_model, d_ff)[1]


def tiled_stride(fmt: int, d_model: int, d_ff: int) -> int:
    """Per-expert stride (bytes, 256-aligned) of the tiled layout."""
    b = int(lib().smoe_cuda_tiled_expert_bytes(fmt, d_model, d_ff))
    if b == 0:
        raise SmoeCudaError("unsupported shape for the tiled layout")
    return (b + 255) // 256 * 256
