"""GPU: a layer uploaded from a .smoe vault (smoe_cuda_vault_upload_layer;
the vault written by the reference's writer pieces, tests/golden/vault.npz)
runs the MoE layer like any resident layer: router + experts + combine
against the oracle over the same blobs, on the vault layout and after
prepacking to the tiled layout. Tolerance as the other FFN tests (1e-4 of
max|ref|)."""
import os

import numpy as np
import pytest
import torch

import oracle as O
import smoe_cuda as S
from gpu_util import dev, rel_err

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
FIX = np.load(os.path.join(HERE, "golden", "vault.npz"))


@pytest.mark.parametrize("layer", [0, 1])
def test_vault_layer_upload_and_run(ctx, layer):
    v = FIX["vault"].copy()
    info = S.vault_parse(v)
    E, d, dff, k = info.max_experts_per_layer, info.d_model, info.ffn_dim, info.moe_top_k
    stride = (info.max_raw_size + 255) // 256 * 256
    arena = torch.zeros(E * stride, dtype=torch.uint8, device="cuda")
    router = O.normal_bf16(30 + layer, 6, E * d, 0.0, 0.5)
    drouter = dev(router)
    torch.cuda.synchronize()
    L = ctx.vault_upload_layer(v, layer, arena, stride, drouter)
    ctx.synchronize()
    # the same blobs, host side, for the oracle
    host = np.zeros((E, stride), np.uint8)
    for e in range(E):
        off, raw = S.vault_expert(v, layer, e)
        host[e, :raw] = v[off:off + raw]
    assert np.array_equal(arena.cpu().numpy().reshape(E, stride), host)
    B = 3
    X = O.normal_bf16(40 + layer, 5, B * d)
    layers = [("vault", L, None)]
    tst = S.tiled_stride(S.FMT_SMOE_Q4, d, dff)
    if tst:
        tb = torch.empty(E * tst, dtype=torch.uint8, device="cuda")
        layers.append(("tiled", ctx.prepack_layer(L, tb, tst), tb))
        ctx.synchronize()
    for name, desc, _ in layers:
        y = torch.zeros(B, d, dtype=torch.float32, device="cuda")
        ids = torch.zeros(B, k, dtype=torch.int32, device="cuda")
        w = torch.zeros(B, k, dtype=torch.float32, device="cuda")
        ctx.moe_layer(desc, dev(X), S.DTYPE_BF16, B, k, True, y, S.DTYPE_F32, ids, w)
        ctx.synchronize()
        got, gid = y.cpu().numpy(), ids.cpu().numpy().view(np.uint32)
        for t in range(B):
            x = O.bf16_to_f32(X[t * d:(t + 1) * d])
            ref, rids, _ = O.moe_layer(O.FMT_SMOE_Q4, x, router, host, stride, E, d, dff, k)
            assert (gid[t] == rids).all(), name
            assert rel_err(got[t], ref) < 1e-4, name


def test_vault_upload_rejects_small_stride(ctx):
    v = FIX["vault"].copy()
    info = S.vault_parse(v)
    arena = torch.zeros(info.max_experts_per_layer * 4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(S.SmoeCudaError):
        ctx.vault_upload_layer(v, 0, arena, 4096, None)
