"""CPU: the .smoe vault reader of the library (smoe_cuda_vault_parse /
_expert) on a vault written by the reference's own writer pieces and
accepted by its validate_vault (tests/golden/make_golden.py), and the
reader's rejections (main.cpp:96-198: magic, version, arch block,
activation, table bounds). Also: the blobs the reader locates hold the
reference quantiser's format, checked by the oracle's FFN over the
reference's own dequantisation (shatter_moe.py:371-387 restated)."""
import os
import struct

import numpy as np
import pytest

import oracle as O
import smoe_cuda as S

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = np.load(os.path.join(HERE, "golden", "vault.npz"))


def vault():
    return FIX["vault"].copy()


def test_parse_fields():
    v = vault()
    info = S.vault_parse(v)
    L, E, d, dff = (int(FIX[k]) for k in ("layers", "experts", "d_model", "d_ff"))
    assert (info.version, info.num_moe_layers, info.max_experts_per_layer, info.total_experts) == (2, L, E, L * E)
    assert (info.group_size, info.bits, info.d_model, info.ffn_dim) == (64, 4, d, dff)
    assert info.data_offset == int(FIX["data_offset"]) and info.table_offset == 64
    assert info.has_arch == 1 and info.model_type == b"qwen3_moe"
    assert (info.num_heads, info.num_kv_heads, info.head_dim, info.moe_top_k, info.moe_ffn_dim) == (4, 2, 32, 2, dff)
    assert info.arch_flags == 0b011 and info.rope_theta == 1e6 and abs(info.rms_norm_eps - 1e-6) < 1e-12
    desc = FIX["desc"]
    assert (info.gate_rows, info.gate_cols, info.up_rows, info.up_cols, info.down_rows, info.down_cols) == (
        desc[0, 0], desc[0, 1], desc[1, 0], desc[1, 1], desc[2, 0], desc[2, 1])
    assert (info.gate_packed_offset, info.gate_scales_offset, info.up_packed_offset, info.up_scales_offset,
            info.down_packed_offset, info.down_scales_offset) == tuple(int(x) for x in desc[:, 2:].reshape(-1))
    for l, e, off, raw in FIX["entries"]:
        assert S.vault_expert(v, int(l), int(e)) == (int(off), int(raw))
    assert info.max_raw_size == int(FIX["entries"][:, 3].max())
    with pytest.raises(S.SmoeCudaError):
        S.vault_expert(v, 0, E)


def _corrupt(edit):
    v = bytearray(vault().tobytes())
    edit(v)
    return np.frombuffer(bytes(v), np.uint8)


@pytest.mark.parametrize("name,edit", [
    ("magic", lambda v: v.__setitem__(slice(0, 4), b"XMOE")),
    ("version", lambda v: v.__setitem__(slice(8, 12), struct.pack("<I", 3))),
    ("no arch offset", lambda v: v.__setitem__(slice(60, 64), struct.pack("<I", 0))),
    ("arch magic", lambda v: v.__setitem__(slice(int(FIX["arch_offset"]), int(FIX["arch_offset"]) + 4), b"XARC")),
    ("activation", lambda v: v.__setitem__(slice(int(FIX["arch_offset"]) + 48, int(FIX["arch_offset"]) + 52),
                                          struct.pack("<I", 1))),
    ("top_k", lambda v: v.__setitem__(slice(int(FIX["arch_offset"]) + 32, int(FIX["arch_offset"]) + 36),
                                     struct.pack("<I", 17))),
    ("blob past end", lambda v: v.__setitem__(slice(64 + 8, 64 + 16), struct.pack("<Q", len(v)))),
    ("expert id", lambda v: v.__setitem__(slice(64 + 4, 64 + 8), struct.pack("<I", 99))),
])
def test_parse_rejects(name, edit):
    with pytest.raises(S.SmoeCudaError):
        S.vault_parse(_corrupt(edit))


def test_parse_rejects_truncated():
    with pytest.raises(S.SmoeCudaError):
        S.vault_parse(vault()[:100])


def test_blobs_are_reference_q4():
    """The blob at the located offset is the reference's SMOE-Q4 expert:
    the oracle FFN over it equals an fp64 FFN over the reference
    dequantisation formula (q - 7.5) / 7.5 * fp16 scale per 64 weights."""
    v = vault()
    info = S.vault_parse(v)
    d, dff = int(FIX["d_model"]), int(FIX["d_ff"])
    off, raw = S.vault_expert(v, 1, 2)
    blob = v[off:off + raw]

    def dense(po, so, rows, cols):
        nib = blob[po:po + rows * cols // 2]
        q = np.empty(rows * cols, np.float64)
        q[0::2], q[1::2] = nib & 15, nib >> 4
        sc = blob[so:so + rows * cols // 64 * 2].view(np.float16).astype(np.float64)
        return ((q - 7.5) / 7.5 * np.repeat(sc, 64)).reshape(rows, cols)
    g = dense(info.gate_packed_offset, info.gate_scales_offset, dff, d)
    u = dense(info.up_packed_offset, info.up_scales_offset, dff, d)
    dn = dense(info.down_packed_offset, info.down_scales_offset, d, dff)
    x = np.random.default_rng(4).standard_normal(d).astype(np.float32)
    gx, ux = g @ x, u @ x
    ref = dn @ (gx / (1 + np.exp(-gx)) * ux)
    got = O.expert_ffn(O.FMT_SMOE_Q4, blob, d, dff, x)
    assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-5
