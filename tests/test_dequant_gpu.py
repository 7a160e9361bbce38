"""MXFP4 -> bf16 dequantisation on the GPU through the C ABI: bit-exact against
the reference's known-answer tests (committed fixtures) and the oracle."""
import json
import os

import numpy as np
import pytest

from oracle import oracle
from oxidized_gpt_oss_b200 import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _dq(blocks_np, scales_np, rows, cols, **kw):
    import torch
    from oxidized_gpt_oss_b200.mxfp4 import dequantize_mxfp4
    b = torch.from_numpy(np.ascontiguousarray(blocks_np)).cuda()
    s = torch.from_numpy(np.ascontiguousarray(scales_np).view(np.int16) if scales_np.dtype == np.uint16
                         else np.ascontiguousarray(scales_np)).cuda()
    out = dequantize_mxfp4(b, s, rows, cols, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)


def test_kat_4x64_bit_exact(cuda_ctx):
    kat = json.load(open(os.path.join(GOLDEN, "mxfp4_kat_4x64.json")))
    out = _dq(np.array(kat["blocks"], np.uint8), np.array(kat["scales_bf16"], np.uint16), kat["rows"], kat["cols"])
    assert out.tolist() == kat["expected_bf16"]


def test_integration_sanity_2x32(cuda_ctx):
    g = json.load(open(os.path.join(GOLDEN, "mxfp4_sanity_2x32.json")))
    out = _dq(np.array(g["blocks"], np.uint8), np.array(g["scales_bf16"], np.uint16), g["rows"], g["cols"])
    assert out.tolist() == g["expected_bf16"]
    v = synth.bf16_bits_to_f32(out)
    assert abs(v.mean()) < 1.0 and v.std() > 0.0


def test_every_code_times_every_e8m0_scale(cuda_ctx):
    # 256 scales x all 256 byte values: covers 0 -> 0.0, 255 -> inf, subnormal
    # products and -0.0, each compared bit for bit with the oracle.
    scales = np.arange(256, dtype=np.uint8)
    rows, cols = 256, 512
    blocks = np.tile(np.arange(256, dtype=np.uint8), rows)
    sc = np.repeat(scales, cols // 32)
    out = _dq(blocks, sc, rows, cols)
    ref = oracle.dequantize_mxfp4_e8m0(blocks, sc, rows, cols)
    assert np.array_equal(out, ref)


def test_bf16_scales_with_rounding_and_nan(cuda_ctx):
    rng = np.random.default_rng(1)
    rows, cols = 64, 256
    blocks = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    sc = synth.f32_to_bf16_bits(rng.standard_normal(rows * cols // 32).astype(np.float32) * 3)
    sc[:4] = [0x7FC0, 0x7F80, 0xFF80, 0x0001]  # NaN, +inf, -inf, subnormal
    out = _dq(blocks, sc, rows, cols)
    ref = oracle.dequantize_mxfp4(blocks, sc, rows, cols)
    assert np.array_equal(out, ref)


def test_unaligned_pointers_take_the_byte_path(cuda_ctx):
    import torch
    from oxidized_gpt_oss_b200.mxfp4 import dequantize_mxfp4
    rng = np.random.default_rng(2)
    rows, cols = 33, 96
    blocks = rng.integers(0, 256, rows * cols // 2 + 1, dtype=np.uint8)
    sc = rng.integers(100, 140, rows * cols // 32, dtype=np.uint8)
    b = torch.from_numpy(blocks).cuda()[1:]
    out = torch.empty(rows * cols + 1, dtype=torch.int16, device="cuda")
    dequantize_mxfp4(b, torch.from_numpy(sc).cuda(), rows, cols, out=out[1:])
    torch.cuda.synchronize()
    got = out[1:].cpu().numpy().view(np.uint16)
    assert np.array_equal(got, oracle.dequantize_mxfp4_e8m0(blocks[1:], sc, rows, cols))


@pytest.mark.parametrize("rows,cols,nb,ns,msg", [
    (2, 48, 48, 2, "cols must be divisible by 32, got 48"),
    (2, 64, 63, 4, "blocks length mismatch: expected 64, got 63"),
    (2, 64, 64, 3, "scales length mismatch: expected 4, got 3"),
])
def test_shape_errors_mirror_reference(cuda_ctx, rows, cols, nb, ns, msg):
    import torch
    from oxidized_gpt_oss_b200.mxfp4 import dequantize_mxfp4
    with pytest.raises(ValueError, match=msg):
        dequantize_mxfp4(torch.zeros(nb, dtype=torch.uint8, device="cuda"),
                         torch.zeros(ns, dtype=torch.int16, device="cuda"), rows, cols)


def test_empty_tensor(cuda_ctx):
    out = _dq(np.zeros(0, np.uint8), np.zeros(0, np.uint8), 0, 64)
    assert out.size == 0


def test_full_layer_bit_exact():
    """The standalone dequant workload at full size: 32 x 5760 x 2880 plus
    32 x 2880 x 2880 elements, E8M0 scales in [110, 135], bit-exact."""
    import torch
    from oxidized_gpt_oss_b200.mxfp4 import dequantize_mxfp4
    (w1, s1, r1, c1), (w2, s2, r2, c2) = synth.dequant_tensors(seed=0)
    for blocks, scales, rows, cols in ((w1, s1, r1, c1), (w2, s2, r2, c2)):
        out = dequantize_mxfp4(torch.from_numpy(blocks).cuda(), torch.from_numpy(scales).cuda(), rows, cols)
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        ref = oracle.dequantize_mxfp4_e8m0(blocks, scales, rows, cols)
        assert np.array_equal(got, ref)
        del out, got, ref
