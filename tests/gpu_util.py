"""Helpers for the GPU parity tests: device copies of oracle data."""
import numpy as np
import torch

import oracle as O
import smoe_cuda as S


_SIGNED = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32,
           np.dtype(np.uint64): np.int64}


def dev(a: np.ndarray) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if a.dtype in _SIGNED:
        a = a.view(_SIGNED[a.dtype])
    return torch.from_numpy(a).cuda()


def rel_err(got, ref) -> float:
    """max_i |got_i - ref_i| / max_j |ref_j| (the FFN tolerance metric)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bf16_dev_to_f32(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16).astype(np.uint32).__lshift__(16).view(np.float32)


class Layer:
    """A synthetic MoE layer resident on the device (config-1 distributions)."""

    def __init__(self, fmt, n_experts, d, dff, seed, router=True):
        self.fmt, self.E, self.d, self.dff = fmt, n_experts, d, dff
        self.arena, self.stride, self.off = O.make_experts(fmt, n_experts, d, dff, seed)
        self.router_w = O.normal_bf16(seed, 6, n_experts * d, 0.0, 0.02)
        self.d_arena = dev(self.arena)
        self.d_router = dev(self.router_w)
        self.desc = S.make_layer(self.d_arena, self.stride, self.off, n_experts, d, dff, fmt,
                                 self.d_router)


def tiled(ctx, layer: "Layer"):
    """Prepack a Layer into the tiled device layout; returns (desc, buffer)."""
    stride = S.tiled_stride(layer.fmt, layer.d, layer.dff)
    buf = torch.empty(layer.E * stride, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()          # the arena was copied on torch's stream
    desc = ctx.prepack_layer(layer.desc, buf, stride)
    ctx.synchronize()
    return desc, buf
