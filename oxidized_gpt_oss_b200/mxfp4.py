"""MXFP4 dequantisation — mirror of src/mxfp4.rs of the reference.

``dequantize_mxfp4(blocks, scales, rows, cols)`` keeps the reference's
signature and meaning (src/mxfp4.rs:15): ``blocks`` are packed E2M1 codes
(low nibble = even element), ``scales`` one per 32-element block, the result
``rows * cols`` bf16 bit patterns. Inputs are CUDA tensors; the work runs in
liboxg_b200.so on torch's current stream. Shape violations raise
``ValueError`` with the reference's assert text where the reference panics.
"""
from __future__ import annotations

import torch

from . import abi

_default_ctx = None


def context(ctx: abi.Context | None = None) -> abi.Context:
    """The given context, or a per-process default one on the current device,
    bound to torch's current stream."""
    global _default_ctx
    if ctx is None:
        if _default_ctx is None:
            _default_ctx = abi.Context(torch.cuda.current_device())
        ctx = _default_ctx
    ctx.set_stream(torch.cuda.current_stream())
    return ctx


def dequantize_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, rows: int, cols: int, *,
                     ctx: abi.Context | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """blocks: uint8 CUDA tensor; scales: int16/uint16 (bf16 bits) or uint8 (E8M0).

    Returns an int16 tensor of rows*cols bf16 bit patterns."""
    if not (blocks.is_cuda and scales.is_cuda):
        raise ValueError("blocks and scales must be CUDA tensors")
    blocks = blocks.contiguous()
    scales = scales.contiguous()
    if scales.dtype == torch.uint8:
        fmt = abi.OXG_SCALE_E8M0
    elif scales.dtype in (torch.int16, torch.uint16, torch.bfloat16):
        fmt = abi.OXG_SCALE_BF16
    else:
        raise ValueError(f"unsupported scale dtype {scales.dtype}")
    c = context(ctx)
    if out is None:
        out = torch.empty(max(rows * cols, 0), dtype=torch.int16, device=blocks.device)
    st = c.lib.oxg_dequant_mxfp4(c.handle, blocks.data_ptr(), blocks.numel(), scales.data_ptr(),
                                 scales.numel(), fmt, rows, cols, out.data_ptr())
    if st == abi.OXG_ERR_SHAPE:
        raise ValueError(c.lib.oxg_last_error(c.handle).decode())
    abi.check(st, c.handle)
    return out
