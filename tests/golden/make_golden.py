"""Generate the committed golden fixtures (run in the build container only).

Sources of truth, all from the reference project itself:
  * Q4 format: ``scripts/shatter_moe.py`` ``build_expert_blob`` /
    ``quantize_smoeq4`` / ``dequantize_smoeq4`` (imported from the reference
    tree) quantise seeded float weights; the dense dequantised matrices and an
    fp64 SwiGLU FFN over them are stored as the expected outputs.
  * Sampler / router: the reference's ``sampler.hpp`` and ``scout.cpp::top_k``
    compiled unmodified into ``oracle/_ref/libsmoe_ref.so``.

Usage:  python tests/golden/make_golden.py <reference-root>
Writes: tests/golden/q4_expert.npz, vault.npz, sampler.npz, router.npz
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402


def q4_fixture(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    import shatter_moe as S  # reference quantiser = format definition

    d, dff = 256, 128
    rng = np.random.default_rng(1234)
    tensors = {
        "gate": rng.normal(0, 0.02, (dff, d)).astype(np.float32),
        "up": rng.normal(0, 0.02, (dff, d)).astype(np.float32),
        "down": rng.normal(0, 0.02, (d, dff)).astype(np.float32),
    }
    blob, descs = S.build_expert_blob(tensors, 64, bits=4)
    blob = np.frombuffer(blob, np.uint8).copy()
    dense = []
    for td in descs:
        packed = blob[td.packed_offset:td.packed_offset + td.packed_size]
        scales = blob[td.scales_offset:td.scales_offset + td.scales_size].view(np.float16)
        w = S.dequantize_smoeq4(packed, scales, td.rows * td.cols, 64)
        dense.append(w.reshape(td.rows, td.cols).astype(np.float64))
    xs = rng.normal(0, 1, (4, d)).astype(np.float32)
    ys = []
    for x in xs:
        g = dense[0] @ x.astype(np.float64)
        u = dense[1] @ x.astype(np.float64)
        h = g / (1.0 + np.exp(-g)) * u
        ys.append(dense[2] @ h)
    offs = np.array([[td.packed_offset, td.packed_size, td.scales_offset, td.scales_size]
                     for td in descs], np.int64)
    np.savez_compressed(os.path.join(HERE, "q4_expert.npz"), blob=blob, offsets=offs,
                        d=d, dff=dff, x=xs, y=np.array(ys), gate=dense[0].astype(np.float32),
                        up=dense[1].astype(np.float32), down=dense[2].astype(np.float32))


def vault_fixture(ref_root: str):
    """A two-layer, four-expert SMOE-Q4 vault (d_model 128, expert d_ff 64)
    written with the reference writer's own pieces: ``build_expert_blob``
    (quantise + blob layout), ``HEADER_FMT`` / ``EXPERT_ENTRY_FMT`` /
    ``TENSOR_DESC_FMT`` records, ``build_arch_block``, the layout rules of its
    ``main`` (table after the header, descriptors after the table, arch block
    64-byte aligned after them, blobs from the next page, each padded to a
    page), then accepted by the reference's ``validate_vault``. Stored with
    the expected header / arch values and every blob's offset and size."""
    sys.path.insert(0, os.path.join(ref_root, "scripts"))
    import tempfile
    import shatter_moe as S

    L, E, d, dff = 2, 4, 128, 64
    rng = np.random.default_rng(77)
    blobs, metas = [], []
    for l in range(L):
        for e in range(E):
            t = {"gate": rng.normal(0, 0.05, (dff, d)).astype(np.float32),
                 "up": rng.normal(0, 0.05, (dff, d)).astype(np.float32),
                 "down": rng.normal(0, 0.05, (d, dff)).astype(np.float32)}
            blob, descs = S.build_expert_blob(t, 64, bits=4)
            blobs.append(blob)
            metas.append((l, e, descs))
    n = len(blobs)
    meta_bytes = S.HEADER_FMT.size + n * S.EXPERT_ENTRY_FMT.size + n * 3 * S.TENSOR_DESC_FMT.size
    arch_offset = S._align_up(meta_bytes, 64)
    data_offset = S._align_up(arch_offset + S.ARCH_FMT.size, S.PAGE_SIZE)
    arch = {"norm_topk_prob": True, "has_qk_norm": True, "has_dense_layer_0": False, "rope_theta": 1e6,
            "num_heads": 4, "num_kv_heads": 2, "head_dim": 32, "moe_top_k": 2, "moe_ffn_dim": dff,
            "dense_ffn_dim": 0, "shared_expert_ffn_dim": 0, "activation": 0, "num_hidden_layers": L,
            "rms_norm_eps": 1e-6, "model_type": "qwen3_moe"}
    body, entries, cur = [], [], data_offset
    for blob in blobs:
        padded = S._align_up(len(blob), S.PAGE_SIZE)
        entries.append((cur, len(blob), padded))
        body.append(blob + b"\x00" * (padded - len(blob)))
        cur += padded
    head = bytearray(S.HEADER_FMT.pack(S.SMOE_MAGIC, S.SMOE_VERSION, L, E, n, S.HEADER_FMT.size, data_offset, 64,
                                       4, d, 512, dff, arch_offset))
    for (l, e, descs), (off, raw, pad) in zip(metas, entries):
        groups = sum(td.num_groups for td in descs)
        head += S.EXPERT_ENTRY_FMT.pack(l, e, off, raw, pad, 64, groups)
    for (_, _, descs) in metas:
        for td in descs:
            head += S.TENSOR_DESC_FMT.pack(td.tensor_type, 2, td.rows, td.cols, td.packed_offset, td.packed_size,
                                           td.scales_offset, td.scales_size)
    head += b"\x00" * (arch_offset - len(head))
    head += S.build_arch_block(arch)
    head += b"\x00" * (data_offset - len(head))
    vault = bytes(head) + b"".join(body)
    with tempfile.TemporaryDirectory() as tmp:          # the reference's own reader accepts it
        path = os.path.join(tmp, "fixture.smoe")
        with open(path, "wb") as f:
            f.write(vault)
        S.validate_vault(S.Path(path))
    d0 = metas[0][2]
    np.savez_compressed(os.path.join(HERE, "vault.npz"), vault=np.frombuffer(vault, np.uint8),
                        layers=L, experts=E, d_model=d, d_ff=dff, data_offset=data_offset, arch_offset=arch_offset,
                        entries=np.array([(l, e, off, raw) for (l, e, _), (off, raw, _) in zip(metas, entries)],
                                         np.int64),
                        desc=np.array([[td.rows, td.cols, td.packed_offset, td.scales_offset] for td in d0],
                                      np.int64))


def sampler_fixture():
    V = 151936
    cases = []
    # (seed, T, top_p, top_k, rep, hist_len): config-0 case plus edge cases
    plan = [(s, 0.7, 0.8, 20, 1.1, 64) for s in range(24)]
    plan += [(100, 0.0, 0.9, 50, 1.1, 64),     # greedy
             (101, 1e-5, 0.9, 50, 1.0, 0),     # greedy, no penalty, empty history
             (102, 1.0, 1.0, 1024, 1.1, 300),  # max top_k, history over the 256 window
             (103, 0.6, 0.95, 40, 1.1, 128),
             (104, 1.0, 0.01, 40, 1.3, 128),   # top_p floor
             (105, 0.7, 0.8, 1, 1.1, 64),      # top_k 1
             (106, 0.7, 0.8, 0, 1.1, 64)]      # top_k 0 (reference keeps one)
    logits, hists, words, params, toks, hlens = [], [], [], [], [], []
    for (s, T, p, k, r, hl) in plan:
        sc = O.normal_f32(s, 1, V, 0.0, 2.0)
        h = np.zeros(300, np.uint32)
        hh = O.random_ids(s, 2, hl, V)
        if s == 102:
            hh[:8] = [13, 11, 198, 271, 30, 0, 151643, 151645]   # exempt ids
            hh[10:20] = hh[20:30]                                 # repeats
        h[:hl] = hh
        w = int(O.random_ids(s, 3, 1, 1 << 24)[0]) << 8
        tok = O.ref_sample_token(sc.copy(), T, p, k, r, hh, w)
        logits.append(sc)
        hists.append(h)
        hlens.append(hl)
        words.append(w)
        params.append((T, p, float(k), r))
        toks.append(tok)
    # logits are regenerated from their seed by the oracle's counter RNG; a
    # checksum of each array pins the generator.
    sums = np.array([np.float64(l.astype(np.float64).sum()) for l in logits])
    seeds = np.array([c[0] for c in plan], np.uint64)
    np.savez_compressed(os.path.join(HERE, "sampler.npz"), seed=seeds, logit_sum=sums,
                        hist=np.array(hists), hist_len=np.array(hlens, np.uint32),
                        word=np.array(words, np.uint32), params=np.array(params, np.float32),
                        token=np.array(toks, np.uint32))


def router_fixture():
    R = O.ref()
    d, E, k = 2048, 128, 8
    xs, ws, ids_all, wts_all, lgs = [], [], [], [], []
    for s in range(8):
        x = O.bf16_to_f32(O.normal_bf16(s, 5, d))
        W = O.normal_bf16(s, 6, E * d, 0.0, 0.02)
        lg = np.empty(E, np.float32)
        ids = np.zeros(k, np.uint32)
        wt = np.zeros(k, np.float32)
        R.ref_route(x, W, E, d, k, 1, lg, ids, wt)
        xs.append(x)
        ws.append(W)
        ids_all.append(ids)
        wts_all.append(wt)
        lgs.append(lg)
    wsum = np.array([O.bf16_to_f32(W).astype(np.float64).sum() for W in ws])
    np.savez_compressed(os.path.join(HERE, "router.npz"), seed=np.arange(8, dtype=np.uint64),
                        x=np.array(xs), w_sum=wsum,
                        ids=np.array(ids_all), weights=np.array(wts_all), logits=np.array(lgs))


if __name__ == "__main__":
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("SMOE_REFERENCE_ROOT", "")
    assert ref_root and os.path.isdir(ref_root), "pass the reference project root"
    assert O.ref_available(), "build oracle/_ref first (make -C oracle REF_SRC=...)"
    q4_fixture(ref_root)
    vault_fixture(ref_root)
    sampler_fixture()
    router_fixture()
    print("golden fixtures written to", HERE)
