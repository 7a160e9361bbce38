"""Prefill path (tcgen05 grouped GEMMs) against the SPEC oracle.

Same tolerance as the decode tests: max |err| <= 2e-2 and
sum|err| / sum|ref| <= 1e-3 against the fp64-accumulating oracle, with the
GPU's routing fed to the oracle (routing itself is checked in
test_moe_gpu.py)."""
import numpy as np
import pytest

from oracle import oracle
from oxidized_gpt_oss_b200 import synth

pytestmark = pytest.mark.gpu
MAX_ABS = 2e-2
MEAN_REL = 1e-3


def _run(d, x_np, mode):
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    layer = MoELayer(d)
    x = torch.from_numpy(x_np.view(np.int16)).cuda()
    y = layer.forward(x, mode=mode)
    idx, w, _ = layer.route(x)
    layer.ctx.sync()
    torch.cuda.synchronize()
    return layer, y.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()


def _check(d, x, y, idx, w):
    y_ref = oracle.moe_forward_spec(oracle.Weights(d), x, idx=idx, wts=w, acc64=True)
    err = np.abs(y - y_ref)
    max_abs = float(err.max())
    mean_rel = float(err.sum() / np.abs(y_ref).sum())
    assert max_abs <= MAX_ABS, f"max abs error {max_abs}"
    assert mean_rel <= MEAN_REL, f"mean relative error {mean_rel}"
    return max_abs, mean_rel


@pytest.mark.parametrize("H,I,E,K,T", [
    (128, 192, 8, 4, 100),
    (256, 128, 16, 2, 70),
    (192, 320, 4, 4, 33),
])
def test_prefill_small(cuda_ctx, H, I, E, K, T):
    from oxidized_gpt_oss_b200 import abi
    d = synth.moe_layer(seed=H + T, hidden=H, intermediate=I, n_experts=E, top_k=K)
    x = synth.activations(T, T, H)
    _, y, idx, w = _run(d, x, abi.OXG_MODE_PREFILL)
    _check(d, x, y, idx, w)


def test_prefill_expert_beyond_one_token_tile(cuda_ctx):
    """A router bias that sends every token to expert 0: 300 slots for one
    expert, i.e. two token tiles (256 + 44), next to experts with 1-2 tokens."""
    from oxidized_gpt_oss_b200 import abi
    d = synth.moe_layer(seed=77, hidden=128, intermediate=128, n_experts=8, top_k=2)
    d["router_b"] = synth.f32_to_bf16_bits(np.array([50.0] + [0.0] * 7, np.float32))
    x = synth.activations(77, 300, 128)
    layer, y, idx, w = _run(d, x, abi.OXG_MODE_PREFILL)
    assert (idx[:, 0] == 0).all()
    _check(d, x, y, idx, w)


def test_prefill_gpt_oss_widths(cuda_ctx):
    """H = I = 2880, 32 experts, top-4, 256 tokens (1024 slots) — ~32 slots
    per expert on average."""
    from oxidized_gpt_oss_b200 import abi
    d = synth.moe_layer(seed=3)
    x = synth.activations(3, 256, 2880)
    _, y, idx, w = _run(d, x, abi.OXG_MODE_PREFILL)
    max_abs, mean_rel = _check(d, x, y, idx, w)
    print(f"prefill gpt-oss widths: max_abs={max_abs:.3e} mean_rel={mean_rel:.3e}")


def test_prefill_benchmark_shape_8192_tokens(cuda_ctx):
    """The benchmarked configuration itself: 8192 tokens through one
    gpt-oss-20b MoE block (the bench's layer, seed 0) on the default path
    (AUTO, which takes the tcgen05 grouped GEMMs here). Every expert gets
    ~1024 slots, i.e. 4-5 token tiles of 256, so tiles beyond the first of
    each expert are exercised. A seeded sample of 96 tokens (all k slots of
    each, spread over the whole batch and so over every token tile) is
    checked against the fp64 oracle; routing must equal the oracle's own
    top-k except at near-ties (k-th and (k+1)-th logits closer than 1e-4)."""
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=0)
    T, K = 8192, d["top_k"]
    x = synth.activations(4242, T, d["hidden"])
    layer = MoELayer(d)
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    y = layer.forward(xt).cpu().numpy()
    idx, w, logits = (a.cpu().numpy() for a in layer.route(xt))
    layer.ctx.sync()
    counts = np.bincount(idx.ravel(), minlength=d["n_experts"])
    assert counts.max() > 768, "some expert must span more than three 256-slot tiles"
    sample = np.sort(np.random.default_rng(8192).choice(T, 96, replace=False))
    W = oracle.Weights(d)
    ref_logits = oracle.router_logits(W, x[sample])
    assert np.max(np.abs(logits[sample] - ref_logits)) < 1e-4 * max(1.0, np.abs(ref_logits).max())
    ref_idx, _ = oracle.topk_softmax(ref_logits, K)
    srt = -np.sort(-ref_logits, axis=1)
    near_tie = (srt[:, K - 1] - srt[:, K]) < 1e-4
    same = np.all(idx[sample] == ref_idx, axis=1)
    assert np.all(same | near_tie), f"routing differs on tokens {sample[~(same | near_tie)]}"
    max_abs, mean_rel = _check(d, x[sample], y[sample], idx[sample], w[sample])
    layer.release()
    print(f"prefill 8192 tokens, 96 sampled: max_abs={max_abs:.3e} mean_rel={mean_rel:.3e}")


def test_prefill_matches_decode_path(cuda_ctx):
    """The two GPU paths (tcgen05 prefill, mma decode) on the same inputs."""
    import torch
    from oxidized_gpt_oss_b200 import abi
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=12, hidden=256, intermediate=256, n_experts=16, top_k=4)
    layer = MoELayer(d)
    x = torch.from_numpy(synth.activations(12, 200, 256).view(np.int16)).cuda()
    yp = layer.forward(x, mode=abi.OXG_MODE_PREFILL).clone()
    yd = layer.forward(x, mode=abi.OXG_MODE_DECODE).clone()
    layer.ctx.sync()
    err = (yp - yd).abs()
    assert err.max().item() <= MAX_ABS and (err.sum() / yd.abs().sum()).item() <= MEAN_REL


def test_prefill_refuses_scales_outside_f16_range(cuda_ctx):
    import torch
    from oxidized_gpt_oss_b200 import abi
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=5, hidden=128, intermediate=128, n_experts=4, top_k=2, scale_range=(110, 150))
    layer = MoELayer(d)
    x = torch.zeros((80, 128), dtype=torch.int16, device="cuda")
    with pytest.raises(abi.OxgError, match="prefill mode needs"):
        layer.forward(x, mode=abi.OXG_MODE_PREFILL)
    # AUTO falls back to the decode kernels, which take any scale
    y = layer.forward(x, mode=abi.OXG_MODE_AUTO)
    layer.ctx.sync()
    assert torch.isfinite(y).all()
