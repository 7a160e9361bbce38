"""MoE layer — mirror of src/moe.rs of the reference.

``MoELayer.forward(hidden)`` replaces ``MoELayer::forward(&self, hidden_states,
compute) -> Result<MetalBuffer>`` (src/moe.rs:16-100): router, top-k +
softmax, permutation, expert MLPs with the clamped SwiGLU fused in, and the
weighted combine, all in liboxg_b200.so. The layer's packed MXFP4 weights are
uploaded once (``oxg_moe_upload``) and stay resident in HBM.

Differences from the reference's buffers, by design: activations in are bf16
(the reference keeps every buffer as f16, src/utils.rs:9-32) and outputs are
f32 (the reference rounds them to f16).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import abi
from .mxfp4 import context

_WEIGHT_KEYS = ("router_w", "router_b", "w1_blocks", "w1_scales", "b1", "w2_blocks", "w2_scales", "b2")


def _ptr(a):
    if a is None:
        return None
    if isinstance(a, torch.Tensor):
        return a.data_ptr()
    return a.ctypes.data


class MoELayer:
    """One uploaded MoE block.

    ``weights`` holds the arrays named in ``_WEIGHT_KEYS`` (numpy or torch,
    host or CUDA) plus ``hidden``, ``intermediate``, ``n_experts``, ``top_k``,
    ``alpha`` and ``limit`` (see ``synth.moe_layer``).
    """

    _next_layer = 0

    def __init__(self, weights: dict, *, ctx: abi.Context | None = None, layer: int | None = None,
                 experts: tuple[int, int] | None = None):
        """experts: (begin, count) to keep only that range of experts resident
        (expert parallelism: ``dispatch`` / ``experts`` / ``combine``)."""
        self.ctx = context(ctx)
        if layer is None:
            layer = MoELayer._next_layer
            MoELayer._next_layer += 1
        self.layer = layer
        self.hidden = int(weights["hidden"])
        self.intermediate = int(weights["intermediate"])
        self.n_experts = int(weights["n_experts"])
        self.top_k = int(weights["top_k"])
        self.expert_begin, self.expert_count = experts if experts is not None else (0, self.n_experts)
        dims = abi.MoeDims(self.hidden, self.intermediate, self.n_experts, self.top_k,
                           float(weights["alpha"]), float(weights["limit"]))
        keep = {}
        for k in _WEIGHT_KEYS:
            v = weights.get(k)
            if isinstance(v, np.ndarray):
                v = np.ascontiguousarray(v)
            elif isinstance(v, torch.Tensor):
                v = v.contiguous()
            keep[k] = v
        w = abi.MoeWeights(*[_ptr(keep[k]) for k in _WEIGHT_KEYS])
        if experts is None:
            abi.check(self.ctx.lib.oxg_moe_upload(self.ctx.handle, self.layer, ctypes.byref(dims), ctypes.byref(w)),
                      self.ctx.handle)
        else:
            abi.check(self.ctx.lib.oxg_moe_upload_shard(self.ctx.handle, self.layer, ctypes.byref(dims),
                                                        ctypes.byref(w), int(experts[0]), int(experts[1])),
                      self.ctx.handle)

    def reserve(self, n_tokens: int) -> None:
        abi.check(self.ctx.lib.oxg_moe_reserve(self.ctx.handle, self.layer, int(n_tokens)), self.ctx.handle)

    def forward(self, hidden: torch.Tensor, *, mode: int = abi.OXG_MODE_AUTO,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """hidden: [T, H] bf16 CUDA tensor -> [T, H] f32 CUDA tensor."""
        if hidden.dim() != 2 or hidden.shape[1] != self.hidden:
            raise ValueError(f"hidden must be [T, {self.hidden}], got {tuple(hidden.shape)}")
        if hidden.dtype not in (torch.bfloat16, torch.int16) or not hidden.is_cuda:
            raise ValueError("hidden must be a bf16 CUDA tensor")
        x = hidden.contiguous()
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.float32, device=x.device)
        c = context(self.ctx)
        abi.check(c.lib.oxg_moe_forward(c.handle, self.layer, x.data_ptr(), T, out.data_ptr(), mode,
                                        abi.OXG_PRECISION_PARITY), c.handle)
        return out

    __call__ = forward

    def forward_host(self, x_host: np.ndarray | torch.Tensor, y_host=None, *, mode: int = abi.OXG_MODE_AUTO):
        """Host buffers in and out (pinned for full speed); waits for the result."""
        T = x_host.shape[0]
        if y_host is None:
            y_host = torch.empty((T, self.hidden), dtype=torch.float32, pin_memory=True)
        c = context(self.ctx)
        abi.check(c.lib.oxg_moe_forward_host(c.handle, self.layer, _ptr(x_host), T, _ptr(y_host), mode,
                                             abi.OXG_PRECISION_PARITY), c.handle)
        return y_host

    def route(self, hidden: torch.Tensor):
        """Routing tap: (idx [T, k] int32, weights [T, k] f32, logits [T, E] f32)."""
        x = hidden.contiguous()
        T = x.shape[0]
        idx = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        logits = torch.empty((T, self.n_experts), dtype=torch.float32, device=x.device)
        c = context(self.ctx)
        abi.check(c.lib.oxg_moe_route(c.handle, self.layer, x.data_ptr(), T, idx.data_ptr(), w.data_ptr(),
                                      logits.data_ptr()), c.handle)
        return idx, w, logits

    def last_counts(self) -> np.ndarray:
        counts = np.zeros(self.n_experts, dtype=np.int32)
        abi.check(self.ctx.lib.oxg_moe_last_counts(self.ctx.handle, counts.ctypes.data, self.n_experts),
                  self.ctx.handle)
        return counts

    # ---- expert parallelism (see include/oxg_b200.h) --------------------------
    def dispatch(self, hidden: torch.Tensor):
        """Routes ``hidden`` [T, H] and lays its T*k slot rows out expert-major:
        (rows [T*k, H] f16, row_scale [T*k] f32, counts [E] int32),
        all on the device."""
        x = hidden.contiguous()
        T = x.shape[0]
        S = T * self.top_k
        rows = torch.empty((S, self.hidden), dtype=torch.float16, device=x.device)
        scale = torch.empty((S,), dtype=torch.float32, device=x.device)
        counts = torch.empty((self.n_experts,), dtype=torch.int32, device=x.device)
        c = context(self.ctx)
        abi.check(c.lib.oxg_moe_dispatch(c.handle, self.layer, x.data_ptr(), T, rows.data_ptr(),
                                         scale.data_ptr(), counts.data_ptr()), c.handle)
        return rows, scale, counts

    def experts(self, rows: torch.Tensor, row_scale: torch.Tensor, seg_counts) -> torch.Tensor:
        """Resident experts over received rows; seg_counts [n_src, expert_count]
        (host) rows per (source, resident expert) in row order. -> [R, H] f32."""
        seg = np.ascontiguousarray(np.asarray(seg_counts, dtype=np.int32).reshape(-1, self.expert_count))
        R = int(seg.sum())
        if R != rows.shape[0]:
            raise ValueError(f"seg_counts sum to {R} rows, rows has {rows.shape[0]}")
        y = torch.empty((R, self.hidden), dtype=torch.float32, device=rows.device)
        c = context(self.ctx)
        abi.check(c.lib.oxg_moe_experts(c.handle, self.layer, rows.data_ptr() if R else None,
                                        row_scale.data_ptr() if R else None, seg.shape[0], seg.ctypes.data,
                                        y.data_ptr() if R else None), c.handle)
        return y

    def combine(self, y_rows: torch.Tensor, n_tokens: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Weighted top-k combine of the rows returned in dispatch order -> [T, H] f32."""
        if out is None:
            out = torch.empty((n_tokens, self.hidden), dtype=torch.float32, device=y_rows.device)
        c = context(self.ctx)
        abi.check(c.lib.oxg_moe_combine(c.handle, self.layer, y_rows.data_ptr(), int(n_tokens), out.data_ptr()),
                  c.handle)
        return out

    def release(self) -> None:
        abi.check(self.ctx.lib.oxg_moe_release(self.ctx.handle, self.layer), self.ctx.handle)
