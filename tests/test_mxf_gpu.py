"""Block-scaled tensor-core expert path (OXG_MODE_MXF4) against the oracle.

The E2M1 weights and their E8M0 scales go straight into
tcgen05.mma.kind::mxf8f6f4; x enters as two E4M3 terms per element and the
SwiGLU output as four (one UE8M0 exponent per 32-element block). Same bar as
every MoE parity test: max |err| <= 2e-2 and sum|err| / sum|ref| <= 1e-3
against the fp64-accumulating oracle, plus agreement with the in-register-
dequant decode path (OXG_MODE_DECODE) on the same inputs.
"""
import numpy as np
import pytest

from oracle import oracle
from oxidized_gpt_oss_b200 import abi, synth

pytestmark = pytest.mark.gpu
MAX_ABS = 2e-2
MEAN_REL = 1e-3


def _run(d, x_np, mode):
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    layer = MoELayer(d)
    x = torch.from_numpy(x_np.view(np.int16)).cuda()
    y = layer.forward(x, mode=mode)
    layer.ctx.sync()  # raises if a kernel reported a pipeline timeout
    idx, w, _ = layer.route(x)
    torch.cuda.synchronize()
    return layer, y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def _check(d, x, y, idx, w):
    W = oracle.Weights(d)
    y_ref = oracle.moe_forward_spec(W, x, idx=idx, wts=w, acc64=True)
    err = np.abs(y - y_ref)
    max_abs = float(err.max())
    mean_rel = float(err.sum() / max(np.abs(y_ref).sum(), 1e-30))
    assert np.all(np.isfinite(y))
    assert max_abs <= MAX_ABS, f"max abs error {max_abs}"
    assert mean_rel <= MEAN_REL, f"mean relative error {mean_rel}"
    return max_abs, mean_rel


@pytest.mark.parametrize("H,I,E,K,T", [
    (128, 128, 8, 4, 1),      # one k-step, one row tile of mlp2
    (192, 320, 16, 4, 5),     # K % 128 == 64 on both GEMMs: the overhanging tail box
    (256, 128, 4, 2, 8),      # every token on 2 of 4 experts: 8 slots per expert
    (384, 192, 8, 1, 7),      # top-1
    (2880, 2880, 32, 4, 8),   # gpt-oss-20b widths, the decode batch
])
def test_shapes(cuda_ctx, H, I, E, K, T):
    d = synth.moe_layer(seed=H + 3 * I + T, hidden=H, intermediate=I, n_experts=E, top_k=K)
    x = synth.activations(11, T, H)
    _, y, idx, w = _run(d, x, abi.OXG_MODE_MXF4)
    max_abs, mean_rel = _check(d, x, y, idx, w)
    print(f"mxf4 H={H} I={I} E={E} k={K} T={T}: max_abs={max_abs:.3e} mean_rel={mean_rel:.3e}")


def test_matches_decode_path(cuda_ctx):
    d = synth.moe_layer(seed=21, hidden=2880, intermediate=2880, n_experts=32, top_k=4)
    x = synth.activations(21, 8, 2880)
    _, y_mxf, idx_a, _ = _run(d, x, abi.OXG_MODE_MXF4)
    _, y_dec, idx_b, _ = _run(d, x, abi.OXG_MODE_DECODE)
    assert np.array_equal(idx_a, idx_b)
    scale = np.abs(y_dec).max()
    assert np.abs(y_mxf - y_dec).max() <= 1e-3 * scale


def test_wide_scales_and_activation_range(cuda_ctx):
    # weight scales far outside the f16-exact window of the prefill path and
    # tokens 2^+-20 apart: the per-block exponents absorb both
    d = synth.moe_layer(seed=31, hidden=256, intermediate=256, n_experts=8, top_k=4, scale_range=(90, 150))
    x = synth.activations(31, 6, 256)
    xf = synth.bf16_bits_to_f32(x).copy()
    xf[1] *= 2.0 ** 20
    xf[2] *= 2.0 ** -20
    xf[3, :64] *= 2.0 ** 12   # one block far above the rest of its row
    x = synth.f32_to_bf16_bits(xf)
    _, y, idx, w = _run(d, x, abi.OXG_MODE_MXF4)
    W = oracle.Weights(d)
    y_ref = oracle.moe_forward_spec(W, x, idx=idx, wts=w, acc64=True)
    rel = np.abs(y - y_ref).max(axis=1) / np.maximum(np.abs(y_ref).max(axis=1), 1e-30)
    assert np.all(rel < 1e-3), rel


def test_deterministic_and_auto_prefill_fallback(cuda_ctx):
    import torch
    d = synth.moe_layer(seed=41, hidden=512, intermediate=384, n_experts=16, top_k=4)
    x = synth.activations(41, 8, 512)
    layer, y1, _, _ = _run(d, x, abi.OXG_MODE_MXF4)
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    y2 = layer.forward(xt, mode=abi.OXG_MODE_MXF4).cpu().numpy()
    assert np.array_equal(y1, y2)
    # scales outside the f16-exact window: AUTO prefill takes the block-scaled GEMMs
    d = synth.moe_layer(seed=42, hidden=256, intermediate=256, n_experts=16, top_k=4, scale_range=(95, 145))
    x = synth.activations(42, 96, 256)
    layer, y3, idx, w = _run(d, x, abi.OXG_MODE_AUTO)
    layer.ctx.profile(True)
    layer.ctx.profile_reset()
    layer.forward(torch.from_numpy(x.view(np.int16)).cuda())
    launched = {n: layer.ctx.profile_read(n)[1] for n in ("mxf_gemm1", "mxf_gemm2", "moe_mlp1_prefill")}
    layer.ctx.profile(False)
    assert launched == {"mxf_gemm1": 1, "mxf_gemm2": 1, "moe_mlp1_prefill": 0}, launched
    # weights up to 6 * 2^18: outputs ~1e8, so the bar is relative here
    y_ref = oracle.moe_forward_spec(oracle.Weights(d), x, idx=idx, wts=w, acc64=True)
    rel = np.abs(y3 - y_ref).max(axis=1) / np.maximum(np.abs(y_ref).max(axis=1), 1e-30)
    assert np.all(rel < 1e-3), rel.max()
    assert np.abs(y3 - y_ref).sum() / np.abs(y_ref).sum() <= MEAN_REL


def test_unsupported_requests_are_refused(cuda_ctx):
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=51, hidden=128, intermediate=96, n_experts=8, top_k=4)  # I % 64 != 0
    layer = MoELayer(d)
    x = torch.from_numpy(synth.activations(51, 4, 128).view(np.int16)).cuda()
    with pytest.raises(abi.OxgError):
        layer.forward(x, mode=abi.OXG_MODE_MXF4)
    # an E8M0 scale of 255 (NaN as a block scale; +inf in the reference's dequantisation)
    d = synth.moe_layer(seed=52, hidden=128, intermediate=128, n_experts=8, top_k=4)
    d["w2_scales"] = d["w2_scales"].copy()
    d["w2_scales"][3, 5, 1] = 255
    layer = MoELayer(d)
    x = torch.from_numpy(synth.activations(52, 4, 128).view(np.int16)).cuda()
    with pytest.raises(abi.OxgError):
        layer.forward(x, mode=abi.OXG_MODE_MXF4)


@pytest.mark.parametrize("H,I,E,K,T", [
    (256, 256, 16, 4, 100),   # tensor-core router + scatter with padded positions
    (192, 320, 12, 4, 70),    # E % 16 != 0: single-CTA permute + E4M3 gather; K tails; partial weight tiles
    (512, 512, 32, 4, 300),   # ragged expert tiles
    (2880, 2880, 32, 4, 512),  # gpt-oss-20b widths
])
def test_prefill_shapes(cuda_ctx, H, I, E, K, T):
    d = synth.moe_layer(seed=7 * H + I + T, hidden=H, intermediate=I, n_experts=E, top_k=K)
    x = synth.activations(13, T, H)
    _, y, idx, w = _run(d, x, abi.OXG_MODE_MXF4)
    max_abs, mean_rel = _check(d, x, y, idx, w)
    print(f"mxf4 prefill H={H} I={I} E={E} k={K} T={T}: max_abs={max_abs:.3e} mean_rel={mean_rel:.3e}")


def test_prefill_matches_f16_path(cuda_ctx):
    d = synth.moe_layer(seed=61, hidden=2880, intermediate=2880, n_experts=32, top_k=4)
    x = synth.activations(61, 1024, 2880)
    _, y_mxf, idx_a, _ = _run(d, x, abi.OXG_MODE_MXF4)
    _, y_f16, idx_b, _ = _run(d, x, abi.OXG_MODE_PREFILL)
    assert np.array_equal(idx_a, idx_b)
    err = np.abs(y_mxf - y_f16)
    assert err.sum() / np.abs(y_f16).sum() <= 5e-4
