"""CPU oracle loader - TEST INFRASTRUCTURE ONLY.

ctypes bindings for
  * ``liboracle.so``        - the plain-C restatement of the decode hot path
                              (``smoe_oracle.c``; every function cites the
                              reference file:line it restates), and
  * ``_ref/libsmoe_ref.so`` - the reference project's own CPU code
                              (``sampler.hpp``, ``scout/scout.cpp::top_k``,
                              ``common.hpp::matvec_bf16``) compiled unmodified
                              by ``ref_shim.cpp``.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs import this module. The product path (``libsmoe_cuda.so``) never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libsmoe_ref.so")

FMT_SMOE_Q4 = 0
FMT_AFFINE_Q4 = 1
GROUP = 64

_P = np.ctypeslib.ndpointer
_f32 = _P(np.float32, flags="C_CONTIGUOUS")
_u32 = _P(np.uint32, flags="C_CONTIGUOUS")
_u16 = _P(np.uint16, flags="C_CONTIGUOUS")
_u8 = _P(np.uint8, flags="C_CONTIGUOUS")
_u64 = _P(np.uint64, flags="C_CONTIGUOUS")

_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        L = C.CDLL(LIB_PATH)
        u64, u32, f32, i32 = C.c_uint64, C.c_uint32, C.c_float, C.c_int
        L.or_gen_normal_f32.argtypes = [u64, u64, u64, f32, f32, _f32]
        L.or_gen_normal_bf16.argtypes = [u64, u64, u64, f32, f32, _u16]
        L.or_gen_uniform_bf16.argtypes = [u64, u64, u64, f32, f32, _u16]
        L.or_gen_uniform_f16.argtypes = [u64, u64, u64, f32, f32, _u16]
        L.or_gen_bytes.argtypes = [u64, u64, u64, _u8]
        L.or_gen_ids.argtypes = [u64, u64, u64, u32, _u32]
        L.or_blob_layout.argtypes = [i32, u32, u32, _u64, C.POINTER(u64)]
        L.or_expert_ffn.argtypes = [i32, _u8, u32, u32, _f32, _f32, i32, C.c_void_p]
        L.or_dequant.argtypes = [i32, C.c_void_p, C.c_void_p, C.c_void_p, u32, u32, _f32]
        L.or_matvec_bf16.argtypes = [_f32, _u16, _f32, u32, u32]
        L.or_topk_renorm.argtypes = [_f32, u32, u32, i32, _u32, _f32]
        L.or_topk_renorm.restype = u32
        L.or_route.argtypes = [_f32, _u16, u32, u32, u32, i32, _f32, _u32, _f32]
        L.or_route.restype = u32
        L.or_moe_layer.argtypes = [i32, _f32, _u16, u32, u32, u32, u32, i32, C.c_void_p,
                                   u64, i32, _f32, C.c_void_p, C.c_void_p]
        L.or_sample_token.argtypes = [_f32, u32, f32, f32, u32, f32, _u32, u32, f32, u32]
        L.or_sample_token.restype = u32
        L.or_canonical_from_word.argtypes = [u32]
        L.or_canonical_from_word.restype = f32
        L.or_set_threads.argtypes = [i32]
        L.or_set_threads.restype = i32
        L.or_f32_to_bf16.argtypes = [f32]
        L.or_f32_to_bf16.restype = C.c_uint16
        L.or_expf_ref.argtypes = [f32]
        L.or_expf_ref.restype = f32
        L.or_expf_batch.argtypes = [_f32, _f32, C.c_long]
        L.or_expf_mismatches.argtypes = [u32, u32]
        L.or_expf_mismatches.restype = C.c_long
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref():
    """The reference's own compiled CPU code (None if it was not built)."""
    global _ref
    if _ref is None:
        if not ref_available():
            return None
        R = C.CDLL(REF_PATH)
        u32, f32, i32 = C.c_uint32, C.c_float, C.c_int
        R.ref_mt_next_after_inject.argtypes = [u32]
        R.ref_mt_next_after_inject.restype = u32
        R.ref_canonical_from_word.argtypes = [u32]
        R.ref_canonical_from_word.restype = f32
        R.ref_mt19937_words.argtypes = [u32, u32, _u32]
        R.ref_sample_token.argtypes = [_f32, u32, f32, f32, u32, f32, _u32, u32, u32, u32]
        R.ref_sample_token.restype = u32
        R.ref_top_k.argtypes = [_f32, u32, u32, _u32, _f32, i32]
        R.ref_top_k.restype = u32
        R.ref_matvec_bf16.argtypes = [_f32, _u16, _f32, u32, u32]
        R.ref_rms_norm_bf16.argtypes = [_f32, _u16, u32]
        R.ref_route.argtypes = [_f32, _u16, u32, u32, u32, i32, _f32, _u32, _f32]
        R.ref_route.restype = u32
        _ref = R
    return _ref


# ------------------------------------------------------------------ data
def normal_f32(seed, stream, n, mean=0.0, std=1.0):
    out = np.empty(n, np.float32)
    lib().or_gen_normal_f32(seed, stream, n, mean, std, out)
    return out


def normal_bf16(seed, stream, n, mean=0.0, std=1.0):
    out = np.empty(n, np.uint16)
    lib().or_gen_normal_bf16(seed, stream, n, mean, std, out)
    return out


def uniform_bf16(seed, stream, n, lo, hi):
    out = np.empty(n, np.uint16)
    lib().or_gen_uniform_bf16(seed, stream, n, lo, hi, out)
    return out


def uniform_f16(seed, stream, n, lo, hi):
    out = np.empty(n, np.uint16)
    lib().or_gen_uniform_f16(seed, stream, n, lo, hi, out)
    return out


def random_bytes(seed, stream, n):
    out = np.empty(n, np.uint8)
    lib().or_gen_bytes(seed, stream, n, out)
    return out


def random_ids(seed, stream, n, m):
    out = np.empty(n, np.uint32)
    lib().or_gen_ids(seed, stream, n, m, out)
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even, same as the C oracle."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = 0x7FFF + ((u >> 16) & 1)
    out = ((u + r) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return out


def blob_layout(fmt, d, dff):
    off = np.zeros(9, np.uint64)
    tot = C.c_uint64()
    lib().or_blob_layout(fmt, d, dff, off, C.byref(tot))
    return [int(o) for o in off], int(tot.value)


def make_experts(fmt, n_experts, d, dff, seed, blob_align=256, first=0):
    """Layer arena of n_experts blobs with the benchmark's distributions.

    Nibbles uniform in [0, 15]; AFFINE: scale bf16 ~ U(0.001, 0.01), bias bf16
    ~ N(0, 0.01^2); SMOE: fp16 scale ~ U(0.001, 0.01). Expert e has its own
    generator streams, so experts [first, first + n_experts) of a layer are
    the same whichever range is made. Returns (arena uint8 [n_experts,
    stride], stride, offsets)."""
    off, tot = blob_layout(fmt, d, dff)
    stride = (tot + blob_align - 1) // blob_align * blob_align
    arena = np.zeros((n_experts, stride), np.uint8)
    for i in range(n_experts):
        e = first + i
        b = arena[i]
        for m in range(3):
            rows, cols = (dff, d) if m < 2 else (d, dff)
            nb = rows * cols // 2
            ng = rows * cols // GROUP
            st = 1000 + 16 * e + 4 * m
            b[off[3 * m]:off[3 * m] + nb] = random_bytes(seed, st, nb)
            if fmt == FMT_AFFINE_Q4:
                b[off[3 * m + 1]:off[3 * m + 1] + 2 * ng] = uniform_bf16(seed, st + 1, ng, 0.001, 0.01).view(np.uint8)
                b[off[3 * m + 2]:off[3 * m + 2] + 2 * ng] = normal_bf16(seed, st + 2, ng, 0.0, 0.01).view(np.uint8)
            else:
                b[off[3 * m + 1]:off[3 * m + 1] + 2 * ng] = uniform_f16(seed, st + 1, ng, 0.001, 0.01).view(np.uint8)
    return arena, stride, off


# -------------------------------------------------------------- compute
def expert_ffn(fmt, blob: np.ndarray, d, dff, x: np.ndarray, precise=True):
    y = np.empty(d, np.float32)
    lib().or_expert_ffn(fmt, np.ascontiguousarray(blob), d, dff,
                        np.ascontiguousarray(x, np.float32), y, int(precise), None)
    return y


def dequant(fmt, blob: np.ndarray, d, dff, m):
    """Dense fp32 copy of matrix m (0 gate, 1 up, 2 down) of one expert blob."""
    off, _ = blob_layout(fmt, d, dff)
    rows, cols = (dff, d) if m < 2 else (d, dff)
    out = np.empty(rows * cols, np.float32)
    base = blob.ctypes.data
    lib().or_dequant(fmt, base + off[3 * m], base + off[3 * m + 1], base + off[3 * m + 2],
                     rows, cols, out)
    return out.reshape(rows, cols)


def route(x, gate_w_bf16, n_experts, d, k, norm=True):
    logits = np.empty(n_experts, np.float32)
    ids = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    n = lib().or_route(np.ascontiguousarray(x, np.float32), gate_w_bf16, n_experts, d, k,
                       int(norm), logits, ids, w)
    return ids[:n], w[:n], logits


def moe_layer(fmt, x, gate_w_bf16, arena, stride, n_experts, d, dff, k, norm=True,
              precise=True):
    out = np.empty(d, np.float32)
    ids = np.zeros(k, np.uint32)
    w = np.zeros(k, np.float32)
    lib().or_moe_layer(fmt, np.ascontiguousarray(x, np.float32), gate_w_bf16, n_experts, d,
                       dff, k, int(norm), arena.ctypes.data, stride, int(precise), out,
                       ids.ctypes.data, w.ctypes.data)
    return out, ids, w


def sample_token(scores, temperature, top_p, top_k, rep, history, u, scratch_k=0):
    """Restated sampler; mutates `scores` (float32) in place like the reference."""
    h = np.ascontiguousarray(history, np.uint32)
    return int(lib().or_sample_token(scores, scores.size, temperature, top_p, top_k, rep,
                                     h, h.size, u, scratch_k))


def ref_sample_token(scores, temperature, top_p, top_k, rep, history, word, scratch_k=0):
    """The reference's sample_token, fed the 32-bit draw `word`."""
    h = np.ascontiguousarray(history, np.uint32)
    return int(ref().ref_sample_token(scores, scores.size, temperature, top_p, top_k, rep,
                                      h, h.size, word, scratch_k))


def canonical_from_word(word: int) -> float:
    return float(lib().or_canonical_from_word(word))


def set_threads(n: int) -> int:
    return int(lib().or_set_threads(n))


def expf_ref(x: np.ndarray) -> np.ndarray:
    """The reference sampler's expf (glibc's FMA build), restated."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().or_expf_batch(x, y, x.size)
    return y


def expf_mismatches(lo_bits: int, hi_bits: int) -> int:
    """Float bit patterns in [lo_bits, hi_bits] where the restated expf and
    this host's libm expf differ."""
    return int(lib().or_expf_mismatches(lo_bits, hi_bits))
