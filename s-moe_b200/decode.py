"""Batch-1 decode of a Qwen3-MoE-shaped model through libsmoe_cuda.

Host-side restatement of the reference's token step (decode.cpp:103-231 and
the MoE block that follows it, main.cpp:621-641 for the final norm, LM head
and sampler) over the C ABI: every operation is a kernel of the library,
and one whole step - embedding, L x (input norm, attention layer, post norm,
fused MoE layer), final norm, LM head, sampler, bookkeeping - is captured
once as a CUDA graph. The token, its position, the sampler row (history
length, uniform draw) and the history live on the device, so a replay needs
no host work; prompt tokens are written into the token slot before their
step. (During the prompt the sampled token is discarded but still appended
to the device history, which the repetition penalty reads.)

BatchDecoder steps `batch` sequences at one shared position (BASELINE
config 4: 256 sequences of the 30B shape; config 3 at batch 32): each has its
own KV ring, sampler row and history; the trunk matmuls run as batched GEMMs
and the MoE layer takes all the batch's tokens at once (the expert-grouped
path, vault layout).

    python s-moe_b200/decode.py --layers 48 --gen 256                 # 30B-shaped decode, batch 1
    python s-moe_b200/decode.py --batch 256 --gen 128 --ctx 256       # config 4: 256 sequences
    python s-moe_b200/decode.py --shape 235b --gen 128                # config 3, batch 1, one GPU
    python s-moe_b200/decode.py --shape 235b --batch 32 --gen 128 --ctx 256
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time
from dataclasses import dataclass

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import smoe_cuda as S  # noqa: E402


@dataclass
class Shape:
    layers: int = 48
    d_model: int = 2048
    num_heads: int = 32
    num_kv_heads: int = 4
    head_dim: int = 128
    n_experts: int = 128
    top_k: int = 8
    d_ff: int = 768
    vocab: int = 151_936
    rope_theta: float = 1_000_000.0
    norm_topk: bool = True
    attn_ctx: int = 4096
    fmt: int = S.FMT_AFFINE_Q4

    @classmethod
    def qwen3_235b(cls, **kw):
        """Qwen3-235B-A22B shape."""
        base = dict(layers=94, d_model=4096, num_heads=64, num_kv_heads=4, head_dim=128, n_experts=128,
                    top_k=8, d_ff=1536)
        base.update(kw)
        return cls(**base)

    @property
    def q_dim(self):
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self):
        return self.num_kv_heads * self.head_dim


def rope_inv_freq(shape: Shape) -> np.ndarray:
    """engine.cpp:351-356: 1 / theta^(2d / head_dim), in fp32."""
    half = shape.head_dim // 2
    return np.array([1.0 / math.pow(shape.rope_theta, float(2 * d) / float(shape.head_dim))
                     for d in range(half)], np.float32)


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).contiguous()


class Model:
    """Device-resident weights. `weights` (numpy, for tests): dict with
    embed [V*d] u16, lm_head [V*d] u16, model_norm [d] u16, and per layer
    lists in_norm, post_norm [d] u16, q_norm, k_norm [hd] u16, w_q, w_k, w_v,
    w_o u16, router [E*d] u16, experts (arena [E, stride] u8, stride, off)
    in the vault layout. Without `weights`, random weights with the
    benchmark's distributions are generated on the device (seeded)."""

    def __init__(self, ctx: "S.Context", shape: Shape, weights=None, seed: int = 7, layout: str = "tiled"):
        self.ctx, self.shape = ctx, shape
        sh = shape
        dev = "cuda"
        g = torch.Generator(device=dev)
        g.manual_seed(seed)

        def from_np(a):
            return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)

        def randn_bf16(n, std):
            return _bf16(torch.randn(n, generator=g, device=dev) * std).view(torch.int16)

        def ones_bf16(n):
            return _bf16(torch.ones(n, device=dev)).view(torch.int16)

        W = weights
        self.embed = from_np(W["embed"]) if W else randn_bf16(sh.vocab * sh.d_model, 0.02)
        self.lm_head = from_np(W["lm_head"]) if W else randn_bf16(sh.vocab * sh.d_model, 0.02)
        self.model_norm = from_np(W["model_norm"]) if W else ones_bf16(sh.d_model)
        self.layers = []
        tstride = S.tiled_stride(sh.fmt, sh.d_model, sh.d_ff)
        for l in range(sh.layers):
            L = {}
            for name, n in (("w_q", sh.q_dim * sh.d_model), ("w_k", sh.kv_dim * sh.d_model),
                            ("w_v", sh.kv_dim * sh.d_model), ("w_o", sh.d_model * sh.q_dim),
                            ("router", sh.n_experts * sh.d_model)):
                L[name] = from_np(W[name][l]) if W else randn_bf16(n, 0.02)
            for name, n in (("in_norm", sh.d_model), ("post_norm", sh.d_model), ("q_norm", sh.head_dim),
                            ("k_norm", sh.head_dim)):
                L[name] = from_np(W[name][l]) if W else ones_bf16(n)
            if W:
                arena, stride, off = W["experts"][l]
                varena = torch.from_numpy(np.ascontiguousarray(arena)).to(dev)
            else:
                varena, stride, off = self._random_experts(g)
            vault = S.make_layer(varena, stride, off, sh.n_experts, sh.d_model, sh.d_ff, sh.fmt, L["router"])
            if layout in ("vault", "both"):  # batched decode / prefill: the expert-grouped path reads it
                L["vault"], L["vault_buf"] = vault, varena
            if layout == "vault":
                self.layers.append(L)
                continue
            tb = torch.empty(sh.n_experts * tstride, dtype=torch.uint8, device=dev)
            # the arena was written on torch's stream, the prepack runs on the
            # context's: finish the former first, the latter before the arena
            # goes back to torch's allocator
            torch.cuda.synchronize()
            L["tiled"] = ctx.prepack_layer(vault, tb, tstride)
            ctx.synchronize()
            L["tiled_buf"] = tb
            del varena, vault
            self.layers.append(L)
        self.layout = layout
        torch.cuda.synchronize()

    def _random_experts(self, g):
        """Vault-layout arena on the device: codes U{0..15}, AFFINE scale
        bf16 ~ U(0.001, 0.01), bias bf16 ~ N(0, 0.01^2), group 64."""
        sh = self.shape
        off, total = S.blob_layout(sh.fmt, sh.d_model, sh.d_ff)
        stride = (total + 255) // 256 * 256
        arena = torch.zeros(sh.n_experts, stride, dtype=torch.uint8, device="cuda")
        for m in range(3):
            rows, cols = (sh.d_ff, sh.d_model) if m < 2 else (sh.d_model, sh.d_ff)
            nb, ng = rows * cols // 2, rows * cols // 64
            arena[:, off[3 * m]:off[3 * m] + nb] = torch.randint(0, 256, (sh.n_experts, nb), generator=g,
                                                                   device="cuda", dtype=torch.int32).to(torch.uint8)
            sc = _bf16(torch.rand(sh.n_experts, ng, generator=g, device="cuda") * 0.009 + 0.001)
            arena[:, off[3 * m + 1]:off[3 * m + 1] + 2 * ng] = sc.view(torch.uint8).view(sh.n_experts, 2 * ng)
            if sh.fmt == S.FMT_AFFINE_Q4:
                bi = _bf16(torch.randn(sh.n_experts, ng, generator=g, device="cuda") * 0.01)
                arena[:, off[3 * m + 2]:off[3 * m + 2] + 2 * ng] = bi.view(torch.uint8).view(sh.n_experts, 2 * ng)
        return arena, stride, off


class Decoder:
    """One sequence, batch 1. Step graph: see the module docstring."""

    def __init__(self, model: Model, temperature=0.7, top_p=0.8, top_k=20, rep_penalty=1.1,
                 uniforms: np.ndarray | None = None, hcap: int = 8192):
        self.m, self.ctx = model, model.ctx
        sh = model.shape
        f32 = dict(dtype=torch.float32, device="cuda")
        self.hidden = torch.zeros(sh.d_model, **f32)
        self.normed = torch.zeros(sh.d_model, **f32)
        self.attn_o = torch.zeros(sh.d_model, **f32)
        self.ffn_out = torch.zeros(sh.d_model, **f32)
        self.qbuf = torch.zeros(sh.q_dim, **f32)
        self.kbuf = torch.zeros(sh.kv_dim, **f32)
        self.vbuf = torch.zeros(sh.kv_dim, **f32)
        self.attn_out = torch.zeros(sh.q_dim, **f32)
        self.kv = torch.zeros(sh.layers, 2, sh.attn_ctx, sh.kv_dim, **f32)
        self.rope_cos = torch.zeros(sh.head_dim // 2, **f32)
        self.rope_sin = torch.zeros(sh.head_dim // 2, **f32)
        self.inv_freq = torch.from_numpy(rope_inv_freq(sh)).cuda()
        self.logits = torch.zeros(sh.vocab, **f32)
        self.token = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.hcap = hcap
        self.history = torch.zeros(hcap, dtype=torch.int32, device="cuda")
        row = np.zeros(6, np.float32)
        row[0:2] = (temperature, top_p)
        row.view(np.uint32)[2] = top_k
        row[3:5] = (rep_penalty, 0.5)
        row.view(np.uint32)[5] = 0
        self.row = torch.from_numpy(row.view(np.int32)).cuda()
        self.u_seq = torch.from_numpy((uniforms if uniforms is not None else np.full(1, 0.5)).astype(np.float32)).cuda()
        torch.cuda.synchronize()
        self.args = []
        for l, L in enumerate(model.layers):
            a = S.AttnLayerArgs()
            for name in ("w_q", "w_k", "w_v", "w_o"):
                setattr(a, name, L[name].data_ptr())
            a.q_norm_w, a.k_norm_w = L["q_norm"].data_ptr(), L["k_norm"].data_ptr()
            a.rope_cos, a.rope_sin = self.rope_cos.data_ptr(), self.rope_sin.data_ptr()
            a.normed_in = self.normed.data_ptr()
            a.qbuf, a.kbuf, a.vbuf = self.qbuf.data_ptr(), self.kbuf.data_ptr(), self.vbuf.data_ptr()
            a.k_cache, a.v_cache = self.kv[l, 0].data_ptr(), self.kv[l, 1].data_ptr()
            a.attn_out, a.o_out = self.attn_out.data_ptr(), self.attn_o.data_ptr()
            a.d_model, a.q_dim, a.kv_dim = sh.d_model, sh.q_dim, sh.kv_dim
            a.head_dim, a.num_heads, a.num_kv_heads = sh.head_dim, sh.num_heads, sh.num_kv_heads
            a.slot, a.valid, a.attn_ctx = 0, 1, sh.attn_ctx
            a.attn_scale = 1.0 / math.sqrt(sh.head_dim)
            self.args.append(a)
        self.graph = None

    def _step(self):
        """One token step, all on the context stream (decode.cpp:103-231 +
        MoE block, main.cpp:621-641)."""
        c, sh = self.ctx, self.m.shape
        c.embed_bf16(self.m.embed, self.token, 1, sh.d_model, self.hidden)
        c.rope_table(self.pos, self.inv_freq, self.rope_cos, self.rope_sin, sh.head_dim // 2)
        for l, L in enumerate(self.m.layers):
            c.rms_norm(self.hidden, self.ffn_out if l > 0 else None, L["in_norm"], self.normed, sh.d_model)
            c.attention_layer(self.args[l], pos=self.pos)
            c.rms_norm(self.hidden, self.attn_o, L["post_norm"], self.normed, sh.d_model)
            c.moe_layer(L["tiled"], self.normed, S.DTYPE_F32, 1, sh.top_k, sh.norm_topk, self.ffn_out, S.DTYPE_F32)
        c.rms_norm(self.hidden, self.ffn_out, self.m.model_norm, self.normed, sh.d_model)
        c.matvec_bf16(self.m.lm_head, self.normed, self.logits, sh.vocab, sh.d_model)
        c.sample(self.logits, sh.vocab, 1, self.row, self.history, self.hcap, self.token)
        c.decode_advance(self.row, self.history, self.hcap, self.token, self.pos, self.u_seq, self.u_seq.numel())

    # ---- layer-major prefill (prefill.cpp:82-465, main.cpp:532-560)
    def prefill_setup(self, max_chunk: int = 256):
        """Buffers for prompt chunks of up to max_chunk tokens."""
        sh = self.m.shape
        C = max_chunk
        f32 = dict(dtype=torch.float32, device="cuda")
        self.pf_chunk = C
        self.pf_hidden = torch.zeros(C, sh.d_model, **f32)
        self.pf_normed = torch.zeros(C, sh.d_model, **f32)
        self.pf_attn_o = torch.zeros(C, sh.d_model, **f32)
        self.pf_ffn_out = torch.zeros(C, sh.d_model, **f32)
        self.pf_q = torch.zeros(C, sh.q_dim, **f32)
        self.pf_k = torch.zeros(C, sh.kv_dim, **f32)
        self.pf_v = torch.zeros(C, sh.kv_dim, **f32)
        self.pf_attn_out = torch.zeros(C, sh.q_dim, **f32)
        self.pf_cos = torch.zeros(C, sh.head_dim // 2, **f32)
        self.pf_sin = torch.zeros(C, sh.head_dim // 2, **f32)
        self.pf_tokens = torch.zeros(C, dtype=torch.int32, device="cuda")
        self.pf_pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.pf_args = []
        for l, a0 in enumerate(self.args):
            a = S.AttnLayerArgs.from_buffer_copy(a0)
            a.rope_cos, a.rope_sin = self.pf_cos.data_ptr(), self.pf_sin.data_ptr()
            a.normed_in = self.pf_normed.data_ptr()
            a.qbuf, a.kbuf, a.vbuf = self.pf_q.data_ptr(), self.pf_k.data_ptr(), self.pf_v.data_ptr()
            a.attn_out, a.o_out = self.pf_attn_out.data_ptr(), self.pf_attn_o.data_ptr()
            self.pf_args.append(a)

    def _prefill_chunk(self, n: int):
        """Tokens pf_tokens[:n] at positions pf_pos.. through every layer
        (their KV into the rings); the chunk's hidden states are not needed
        afterwards (the last prompt token takes the normal step)."""
        c, sh = self.ctx, self.m.shape
        c.embed_bf16(self.m.embed, self.pf_tokens, n, sh.d_model, self.pf_hidden)
        c.rope_tables(self.pf_pos, n, self.inv_freq, self.pf_cos, self.pf_sin, sh.head_dim // 2)
        for l, L in enumerate(self.m.layers):
            c.rms_norm(self.pf_hidden, self.pf_ffn_out if l > 0 else None, L["in_norm"], self.pf_normed, sh.d_model,
                       rows=n)
            c.attention_prefill(self.pf_args[l], n, self.pf_pos)
            c.rms_norm(self.pf_hidden, self.pf_attn_o, L["post_norm"], self.pf_normed, sh.d_model, rows=n)
            if "vault" in L and n > 4:       # expert-grouped path over the chunk's tokens
                c.moe_layer(L["vault"], self.pf_normed, S.DTYPE_F32, n, sh.top_k, sh.norm_topk, self.pf_ffn_out,
                            S.DTYPE_F32)
            else:                            # the layer kernel, 4 tokens per launch
                for i in range(0, n, 4):
                    m = min(4, n - i)
                    c.moe_layer(L["tiled"], self.pf_normed[i:i + m], S.DTYPE_F32, m, sh.top_k, sh.norm_topk,
                                self.pf_ffn_out[i:i + m], S.DTYPE_F32)

    def prefill(self, toks: torch.Tensor) -> None:
        """All prompt tokens (device int32 [P]) but the last, layer-major in
        chunks, then the device state for the last prompt token's step:
        token, position P - 1, history = the prompt (the sampler's stream),
        and that step's uniform. Device work only (capturable), on the
        current stream."""
        if not hasattr(self, "pf_chunk"):
            self.prefill_setup()
        P = toks.numel()
        for b0 in range(0, P - 1, self.pf_chunk):
            n = min(self.pf_chunk, P - 1 - b0)
            self.pf_tokens[:n].copy_(toks[b0:b0 + n])
            self.pf_pos.fill_(b0)
            self._prefill_chunk(n)
        self.token.copy_(toks[P - 1:P])
        self.pos.fill_(P - 1)
        n_hist = min(P, self.hcap)
        self.history[:n_hist].copy_(toks[P - n_hist:])
        self.row[5:6].fill_(n_hist)
        self.row[4:5].copy_(self.u_seq[(P - 1) % self.u_seq.numel():(P - 1) % self.u_seq.numel() + 1].view(torch.int32))

    def run_prefill(self, prompt: list[int], n_gen: int):
        """Layer-major prefill of the prompt (one CUDA graph for its chunks),
        then n_gen step-graph replays (the first processes the last prompt
        token and samples the first generated one). Returns (generated ids,
        seconds to the first generated token, seconds for all n_gen)."""
        assert self.graph is not None
        self.reset()
        if not hasattr(self, "pf_chunk"):
            self.prefill_setup()
        new = torch.tensor([int(t) for t in prompt], dtype=torch.int32, device="cuda")
        if getattr(self, "pf_graph_len", None) == len(prompt):
            self.pf_prompt.copy_(new)                # the captured graph reads this buffer
        else:
            self.pf_prompt = new
        torch.cuda.synchronize()
        with torch.cuda.stream(self.stream):
            if getattr(self, "pf_graph_len", None) != len(prompt):
                self.prefill(self.pf_prompt)         # eager once (kernel attributes), then capture
                torch.cuda.synchronize()
                self.reset()
                self.pf_graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.pf_graph, stream=self.stream):
                    self.prefill(self.pf_prompt)
                self.pf_graph_len = len(prompt)
                torch.cuda.synchronize()
                self.reset()
            toks = torch.zeros(n_gen, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            ev[0].record(self.stream)
            self.pf_graph.replay()
            self.graph.replay()
            toks[0:1].copy_(self.token)
            ev[1].record(self.stream)
            for i in range(1, n_gen):
                self.graph.replay()
                toks[i:i + 1].copy_(self.token)
            ev[2].record(self.stream)
            torch.cuda.synchronize()
        return toks.cpu().numpy().tolist(), ev[0].elapsed_time(ev[1]) / 1e3, ev[0].elapsed_time(ev[2]) / 1e3

    def capture(self, stream: torch.cuda.Stream):
        self.stream = stream
        self.ctx.set_stream(stream.cuda_stream)
        with torch.cuda.stream(stream):
            self._step()                  # eager once: kernel attributes set before capture
        torch.cuda.synchronize()
        self.reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self._step()
        torch.cuda.synchronize()

    def reset(self):
        torch.cuda.synchronize()
        self.kv.zero_()
        self.pos.zero_()
        self.history.zero_()
        self.row[5] = 0
        torch.cuda.synchronize()

    def run(self, prompt: list[int], n_gen: int):
        """Prompt tokens then n_gen sampled tokens (graph replays); returns
        (generated ids, seconds spent generating, device time)."""
        assert self.graph is not None
        with torch.cuda.stream(self.stream):
            for tok in prompt:
                self.token.fill_(int(tok))
                self.graph.replay()
            toks = torch.zeros(n_gen, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            for i in range(n_gen):
                self.graph.replay()
                toks[i:i + 1].copy_(self.token)
            e1.record(self.stream)
            torch.cuda.synchronize()
        return toks.cpu().numpy().tolist(), e0.elapsed_time(e1) / 1e3


class BatchDecoder:
    """`batch` sequences decoded together at one shared position. Per
    sequence: its own KV ring (attn_ctx positions), sampler row
    (temperature, top_p, top_k, rep_penalty, u, history_len) and history.
    Step graph: embed B tokens, L x (B-row input norm, batched attention
    layer, B-row post norm, MoE layer over the B tokens), final norm, LM head
    as a batched GEMM, B-row sampler, batched bookkeeping. The model must be
    built with layout="vault"."""

    def __init__(self, model: Model, batch: int, rows: np.ndarray | None = None,
                 uniforms: np.ndarray | None = None, hcap: int = 512):
        self.m, self.ctx, self.B = model, model.ctx, batch
        sh = model.shape
        B = batch
        f32 = dict(dtype=torch.float32, device="cuda")
        self.hidden = torch.zeros(B, sh.d_model, **f32)
        self.normed = torch.zeros(B, sh.d_model, **f32)
        self.attn_o = torch.zeros(B, sh.d_model, **f32)
        self.ffn_out = torch.zeros(B, sh.d_model, **f32)
        self.qbuf = torch.zeros(B, sh.q_dim, **f32)
        self.kbuf = torch.zeros(B, sh.kv_dim, **f32)
        self.vbuf = torch.zeros(B, sh.kv_dim, **f32)
        self.attn_out = torch.zeros(B, sh.q_dim, **f32)
        self.kv = torch.zeros(sh.layers, 2, B, sh.attn_ctx, sh.kv_dim, **f32)
        self.rope_cos = torch.zeros(sh.head_dim // 2, **f32)
        self.rope_sin = torch.zeros(sh.head_dim // 2, **f32)
        self.inv_freq = torch.from_numpy(rope_inv_freq(sh)).cuda()
        self.logits = torch.zeros(B, sh.vocab, **f32)
        self.tokens = torch.zeros(B, dtype=torch.int32, device="cuda")
        self.pos = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.hcap = hcap
        self.history = torch.zeros(B, hcap, dtype=torch.int32, device="cuda")
        if rows is None:
            rows = batch_rows(B)
        self.rows0 = np.ascontiguousarray(rows, np.float32).copy()
        self.rows = torch.from_numpy(self.rows0.view(np.int32)).cuda()
        self.u_seq = torch.from_numpy((uniforms if uniforms is not None else np.full(1, 0.5)).astype(np.float32)).cuda()
        torch.cuda.synchronize()
        self.args = []
        for l, L in enumerate(model.layers):
            a = S.AttnLayerArgs()
            for name in ("w_q", "w_k", "w_v", "w_o"):
                setattr(a, name, L[name].data_ptr())
            a.q_norm_w, a.k_norm_w = L["q_norm"].data_ptr(), L["k_norm"].data_ptr()
            a.rope_cos, a.rope_sin = self.rope_cos.data_ptr(), self.rope_sin.data_ptr()
            a.normed_in = self.normed.data_ptr()
            a.qbuf, a.kbuf, a.vbuf = self.qbuf.data_ptr(), self.kbuf.data_ptr(), self.vbuf.data_ptr()
            a.k_cache, a.v_cache = self.kv[l, 0].data_ptr(), self.kv[l, 1].data_ptr()
            a.attn_out, a.o_out = self.attn_out.data_ptr(), self.attn_o.data_ptr()
            a.d_model, a.q_dim, a.kv_dim = sh.d_model, sh.q_dim, sh.kv_dim
            a.head_dim, a.num_heads, a.num_kv_heads = sh.head_dim, sh.num_heads, sh.num_kv_heads
            a.slot, a.valid, a.attn_ctx = 0, 1, sh.attn_ctx
            a.attn_scale = 1.0 / math.sqrt(sh.head_dim)
            self.args.append(a)
        self.kv_seq_stride = sh.attn_ctx * sh.kv_dim
        self.graph = None

    def _step(self):
        c, sh, B = self.ctx, self.m.shape, self.B
        c.embed_bf16(self.m.embed, self.tokens, B, sh.d_model, self.hidden)
        c.rope_table(self.pos, self.inv_freq, self.rope_cos, self.rope_sin, sh.head_dim // 2)
        for l, L in enumerate(self.m.layers):
            c.rms_norm(self.hidden, self.ffn_out if l > 0 else None, L["in_norm"], self.normed, sh.d_model, rows=B)
            c.attention_batch(self.args[l], B, self.kv_seq_stride, self.pos)
            c.rms_norm(self.hidden, self.attn_o, L["post_norm"], self.normed, sh.d_model, rows=B)
            c.moe_layer(L["vault"], self.normed, S.DTYPE_F32, B, sh.top_k, sh.norm_topk, self.ffn_out, S.DTYPE_F32)
        c.rms_norm(self.hidden, self.ffn_out, self.m.model_norm, self.normed, sh.d_model, rows=B)
        c.gemm_bf16(self.m.lm_head, self.normed, self.logits, sh.vocab, sh.d_model, B)
        c.sample(self.logits, sh.vocab, B, self.rows, self.history, self.hcap, self.tokens)
        c.decode_advance_batch(self.rows, self.history, self.hcap, self.tokens, B, self.pos, self.u_seq,
                               self.u_seq.numel())

    def capture(self, stream: torch.cuda.Stream):
        self.stream = stream
        self.ctx.set_stream(stream.cuda_stream)
        with torch.cuda.stream(stream):
            self._step()
        torch.cuda.synchronize()
        self.reset()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=stream):
            self._step()
        torch.cuda.synchronize()

    def reset(self):
        torch.cuda.synchronize()
        self.kv.zero_()
        self.pos.zero_()
        self.history.zero_()
        self.rows.copy_(torch.from_numpy(self.rows0.view(np.int32)))
        torch.cuda.synchronize()

    def run(self, prompts: np.ndarray, n_gen: int):
        """prompts [B, P] token ids (one prompt per sequence, fed in step), then
        n_gen sampled steps; returns (generated ids [n_gen, B], seconds)."""
        assert self.graph is not None
        pr = torch.from_numpy(np.ascontiguousarray(prompts.T, np.int32)).cuda()
        with torch.cuda.stream(self.stream):
            for p in range(pr.shape[0]):
                self.tokens.copy_(pr[p])
                self.graph.replay()
            toks = torch.zeros(n_gen, self.B, dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            for i in range(n_gen):
                self.graph.replay()
                toks[i].copy_(self.tokens)
            e1.record(self.stream)
            torch.cuda.synchronize()
        return toks.cpu().numpy(), e0.elapsed_time(e1) / 1e3


def batch_rows(B: int, seed: int = 5) -> np.ndarray:
    """BASELINE config 4 sampler rows: temperature in {0.6, 0.7, 1.0}, top-k
    in {20, 40}, top-p in {0.8, 0.95}, repetition penalty 1.1, a seeded
    uniform each; history starts empty. [B, 6] float32 (top_k and
    history_len as uint32 bits)."""
    rng = np.random.default_rng(seed)
    rows = np.zeros((B, 6), np.float32)
    rows[:, 0] = np.array([0.6, 0.7, 1.0], np.float32)[np.arange(B) % 3]
    rows[:, 1] = np.array([0.8, 0.95], np.float32)[np.arange(B) % 2]
    rows.view(np.uint32)[:, 2] = np.array([20, 40])[(np.arange(B) // 2) % 2]
    rows[:, 3] = 1.1
    rows[:, 4] = (rng.integers(0, 1 << 24, B) / (1 << 24)).astype(np.float32)
    rows.view(np.uint32)[:, 5] = 0
    return rows


def per_token_bytes(sh: Shape) -> int:
    """Weights one batch-1 token reads: top-k experts, attention, router, LM head."""
    attn = (2 * sh.q_dim + 2 * sh.kv_dim) * sh.d_model * 2
    return (sh.layers * (sh.top_k * S.expert_bytes(sh.fmt, sh.d_model, sh.d_ff) + attn
                         + sh.n_experts * sh.d_model * 2) + sh.vocab * sh.d_model * 2)


def profile_steps(dec, n: int = 1) -> None:
    """n step-graph replays between cudaProfilerStart / Stop, for
    `ncu --profile-from-start off` (the graph's kernels one by one)."""
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    with torch.cuda.stream(dec.stream):
        for _ in range(n):
            dec.graph.replay()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def run_batched(ctx, sh: Shape, batch: int, prompt: int, gen: int, seed: int = 11, profile: bool = False) -> dict:
    t0 = time.time()
    model = Model(ctx, sh, layout="vault")
    t_load = time.time() - t0
    rng = np.random.default_rng(seed)
    dec = BatchDecoder(model, batch, uniforms=rng.integers(0, 1 << 24, 1 << 16).astype(np.float64) / (1 << 24),
                       hcap=max(512, prompt + gen + 16))
    dec.capture(torch.cuda.Stream())
    prompts = rng.integers(0, sh.vocab, (batch, prompt))
    dec.run(prompts, 4)                                  # warm-up
    dec.reset()
    toks, t = dec.run(prompts, gen)
    ctx.synchronize()
    if profile:
        profile_steps(dec)
    out = {"batch": batch, "tok_per_s": round(batch * gen / t, 1), "ms_per_step": round(1e3 * t / gen, 3),
           "load_s": round(t_load, 1), "first_tokens_seq0": toks[:8, 0].tolist()}
    del dec, model
    torch.cuda.empty_cache()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", choices=["30b", "235b"], default="30b")
    ap.add_argument("--layers", type=int, default=0, help="0: the shape's own layer count")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=4096, help="KV ring positions per sequence")
    ap.add_argument("--prompt", type=int, default=45)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--profile", action="store_true",
                    help="after the timed run, one more step between cudaProfilerStart/Stop (ncu "
                         "--profile-from-start off)")
    args = ap.parse_args()
    sh = Shape.qwen3_235b() if args.shape == "235b" else Shape()
    if args.layers:
        sh.layers = args.layers
    sh.attn_ctx = args.ctx
    name = "Qwen3-235B-A22B" if args.shape == "235b" else "Qwen3-30B-A3B"
    ctx = S.Context(0)
    if args.batch > 1:
        out = run_batched(ctx, sh, args.batch, args.prompt, args.gen, profile=args.profile)
        out["workload"] = (f"{name}-shaped decode, {sh.layers} layers, batch {args.batch}, prompt {args.prompt}, "
                           f"{args.gen} generated per sequence (random weights)")
        print(json.dumps(out))
        ctx.close()
        return
    t0 = time.time()
    model = Model(ctx, sh)
    t_load = time.time() - t0
    rng = np.random.default_rng(11)
    dec = Decoder(model, uniforms=rng.integers(0, 1 << 24, 4096).astype(np.float64) / (1 << 24))
    dec.capture(torch.cuda.Stream())
    prompt = rng.integers(0, sh.vocab, args.prompt).tolist()
    dec.run(prompt, 8)                                   # warm-up
    dec.reset()
    toks, t = dec.run(prompt, args.gen)
    ctx.synchronize()
    if args.profile:
        profile_steps(dec)
    ptb = per_token_bytes(sh)
    print(json.dumps({"workload": f"{name}-shaped decode, {sh.layers} layers, batch 1, prompt "
                                  f"{args.prompt}, {args.gen} generated (random weights)",
                      "tok_per_s": round(args.gen / t, 2), "ms_per_token": round(1e3 * t / args.gen, 4),
                      "load_s": round(t_load, 1), "weights_gb_per_token": round(ptb / 1e9, 3),
                      "achieved_gbs": round(ptb * args.gen / t / 1e9, 1),
                      "first_tokens": toks[:8]}))
    ctx.close()


if __name__ == "__main__":
    main()
