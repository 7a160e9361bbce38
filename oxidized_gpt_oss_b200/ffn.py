"""SwiGLU — mirror of src/ffn.rs of the reference.

The reference's ``swiglu(gate, up)`` (src/ffn.rs:5-13) is the plain
``silu(g) * u``. gpt-oss experts use the clamped form, which is what this
library computes (and fuses into the mlp1 epilogue of the MoE kernels):
``g <- min(g, limit); u <- clamp(u, -limit, limit); g * sigmoid(alpha g) * (u + 1)``.
"""
from __future__ import annotations

import torch

from . import abi
from .mxfp4 import context

ALPHA = 1.702
LIMIT = 7.0


def swiglu(gate: torch.Tensor, up: torch.Tensor, alpha: float = ALPHA, limit: float = LIMIT, *,
           ctx: abi.Context | None = None) -> torch.Tensor:
    if gate.shape != up.shape:
        raise ValueError(f"gate and up shapes differ: {tuple(gate.shape)} vs {tuple(up.shape)}")
    if gate.dtype != torch.float32 or up.dtype != torch.float32 or not (gate.is_cuda and up.is_cuda):
        raise ValueError("gate and up must be float32 CUDA tensors")
    g = gate.contiguous()
    u = up.contiguous()
    out = torch.empty_like(g)
    c = context(ctx)
    abi.check(c.lib.oxg_swiglu(c.handle, g.data_ptr(), u.data_ptr(), g.numel(), float(alpha), float(limit),
                               out.data_ptr()), c.handle)
    return out
