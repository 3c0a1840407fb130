"""GPU: the C++ engine binary (s-moe_b200/smoe_engine, linked against
libsmoe_cuda) against the Python decode driver on the same weights: the
engine reads a weights directory this test writes (a small Qwen3-MoE-shaped
model, the decode tests' shape), runs the layer-major prefill and greedy
decode (--tokens-in, temperature 0), and must emit the same ids as the
Python driver's prefill + step graph (same kernels in the same order, so
the same logits); the --serve line protocol (GEN with overrides, RESET,
errors) answers as the reference's serve mode (serve.hpp, main.cpp:401-711).
The Python driver is itself checked against the CPU restatement
(test_gpu_decode.py)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from decode_ref import make_weights

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENGINE = os.path.join(ROOT, "s-moe_b200", "smoe_engine")


def small_shape():
    from decode import Shape
    return Shape(layers=2, n_experts=16, top_k=4, vocab=512, attn_ctx=64)


def write_weights(d, sh, W):
    import smoe_cuda as S
    os.makedirs(d, exist_ok=True)
    stride = W["experts"][0][1]
    with open(os.path.join(d, "meta.txt"), "w") as f:
        for k, v in (("layers", sh.layers), ("d_model", sh.d_model), ("num_heads", sh.num_heads),
                     ("num_kv_heads", sh.num_kv_heads), ("head_dim", sh.head_dim), ("n_experts", sh.n_experts),
                     ("top_k", sh.top_k), ("d_ff", sh.d_ff), ("vocab", sh.vocab), ("rope_theta", sh.rope_theta),
                     ("fmt", sh.fmt), ("expert_stride", stride), ("attn_ctx", sh.attn_ctx),
                     ("norm_topk", int(sh.norm_topk))):
            f.write(f"{k} {v}\n")
    for name in ("embed", "lm_head", "model_norm"):
        np.ascontiguousarray(W[name], np.uint16).tofile(os.path.join(d, name + ".bin"))
    for l in range(sh.layers):
        for name in ("w_q", "w_k", "w_v", "w_o", "router", "in_norm", "post_norm", "q_norm", "k_norm"):
            np.ascontiguousarray(W[name][l], np.uint16).tofile(os.path.join(d, f"layer{l}_{name}.bin"))
        arena, st, off = W["experts"][l]
        assert st == stride and list(off) == list(S.blob_layout(sh.fmt, sh.d_model, sh.d_ff)[0])
        np.ascontiguousarray(arena).tofile(os.path.join(d, f"layer{l}_experts.bin"))


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    import build
    build.build_engine()
    sh = small_shape()
    W = make_weights(sh, 33)
    d = str(tmp_path_factory.mktemp("engine_weights"))
    write_weights(d, sh, W)
    return d, sh, W


def test_engine_greedy_matches_python_driver(ctx, model_dir):
    from decode import Decoder, Model
    d, sh, W = model_dir
    prompt = [7, 300, 41, 41, 509, 2, 120, 88, 250, 13]
    n_gen = 12
    r = subprocess.run([ENGINE, "--weights", d, "--tokens-in", ",".join(map(str, prompt)), "--max-tokens",
                        str(n_gen), "--temperature", "0", "--top-k", "1", "--rep-penalty", "1"],
                       capture_output=True, text=True, timeout=180)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    assert lines[-1] == "fin=length <<DONE>>"
    got = [int(t) for t in lines[0].split()]
    model = Model(ctx, sh, weights=W)
    dec = Decoder(model, temperature=0.0, top_p=1.0, top_k=1, rep_penalty=1.0)
    try:
        dec.capture(torch.cuda.Stream())
        want, _, _ = dec.run_prefill(prompt, n_gen)
    finally:                                  # the session context goes back to the tests' stream
        torch.cuda.synchronize()
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    assert got == want


def test_engine_serve_protocol(model_dir):
    d, sh, _ = model_dir
    reqs = ["GEN 5 t=0 k=1 r=1 3,4,5,6", "GEN 4 3,4,5,6,9", "NONSENSE", "GEN 0 1,2", "RESET",
            "GEN 5 t=0 k=1 r=1 3,4,5,6"]
    r = subprocess.run([ENGINE, "--weights", d, "--serve"], input="\n".join(reqs) + "\n", capture_output=True,
                       text=True, timeout=180)
    assert r.returncode == 0, r.stderr[-2000:]
    out = r.stdout.strip().splitlines()
    # replies: ids + fin line per GEN; errors; RESET -> <<DONE>>
    fin = [i for i, s in enumerate(out) if s.startswith("fin=")]
    assert len(fin) == 3
    assert out.count("<<ERR bad_request>>") == 2 and "<<DONE>>" in out
    first = [int(t) for t in out[fin[0] - 1].split()]
    last = [int(t) for t in out[fin[2] - 1].split()]
    assert len(first) == 5 and first == last          # after RESET the same greedy request repeats
    second = [int(t) for t in out[fin[1] - 1].split()]
    assert len(second) == 4
