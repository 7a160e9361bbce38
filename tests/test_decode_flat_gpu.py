"""Decode expert kernels against the SPEC oracle: the flat split of the
weight chunks over the warps of the grid (tiles split between warps summed in
a fixed order) and, above 8 tokens, the grouped kernels that give every group
of at most 8 slots of an expert an equal share of the GPU.

Shapes cover: one to eight tokens at gpt-oss-20b widths; K with a trailing
narrow group (H = 96: three 32-blocks, I = 160: one full group and one of one
block); more warps in the grid than weight chunks (tiny layers); 128 active
experts (E = 256, k = 16), where the mlp2 kernel gives each expert one CTA.
Bar: max |err| <= 2e-2 and sum|err| / sum|ref| <= 1e-3 against the
fp64-accumulating oracle on the GPU's routing, and two forwards of the same
input are bit-identical (the split sums do not depend on timing)."""
import numpy as np
import pytest

from oracle import oracle
from oxidized_gpt_oss_b200 import synth

pytestmark = pytest.mark.gpu
MAX_ABS = 2e-2
MEAN_REL = 1e-3


@pytest.mark.parametrize("H,I,E,K,T", [
    (2880, 2880, 32, 4, 1),
    (2880, 2880, 32, 4, 2),
    (2880, 2880, 32, 4, 5),
    (2880, 2880, 32, 4, 8),
    (96, 160, 8, 4, 3),       # tail-only mlp1 groups, 1 full + 1 narrow mlp2 group
    (64, 64, 4, 2, 1),        # 8 + 4 tiles of one group: far more warps than chunks
    (256, 192, 256, 16, 8),   # 128 active experts
    (512, 1024, 16, 4, 7),    # 7 tokens on 16 experts: several experts with 2+ tokens
])
def test_flat_decode_against_oracle(cuda_ctx, H, I, E, K, T):
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=H + I + E + T, hidden=H, intermediate=I, n_experts=E, top_k=K)
    x = synth.activations(7 * T + E, T, H)
    layer = MoELayer(d)
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    y1 = layer.forward(xt).clone()
    y2 = layer.forward(xt).clone()
    idx, w, _ = layer.route(xt)
    layer.ctx.sync()
    assert torch.equal(y1, y2), "two forwards of the same tokens differ"
    y = y1.cpu().numpy()
    y_ref = oracle.moe_forward_spec(oracle.Weights(d), x, idx=idx.cpu().numpy(), wts=w.cpu().numpy(), acc64=True)
    err = np.abs(y - y_ref)
    max_abs, mean_rel = float(err.max()), float(err.sum() / max(np.abs(y_ref).sum(), 1e-30))
    assert np.all(np.isfinite(y))
    assert max_abs <= MAX_ABS, f"max abs error {max_abs}"
    assert mean_rel <= MEAN_REL, f"mean relative error {mean_rel}"
    layer.release()


@pytest.mark.parametrize("H,I,E,K,T,hot", [
    (2880, 2880, 32, 4, 64, 0.0),    # the batched-decode batch, roughly uniform loads
    (2880, 2880, 32, 4, 64, 1.1),    # Zipf-like skew: the busiest expert holds most tokens
    (2880, 2880, 32, 4, 24, 1.1),
    (256, 192, 8, 2, 40, 2.0),       # few experts, many tokens each: several groups per expert
    (96, 160, 16, 4, 17, 0.5),       # narrow trailing groups, a group of one slot
])
def test_grouped_decode_against_oracle(cuda_ctx, H, I, E, K, T, hot):
    """Above 8 tokens each expert's slots are cut into groups of at most 8
    and every group gets an equal share of the GPU (grouped mlp1 / mlp2
    kernels). A router bias of -hot * ln(rank) skews the loads as in the
    batched-decode benchmark."""
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=H + E + T, hidden=H, intermediate=I, n_experts=E, top_k=K)
    if hot:
        rank = np.random.default_rng(E + T).permutation(E) + 1
        b = oracle.np_bf16_to_f32(d["router_b"]) - hot * np.log(rank)
        d["router_b"] = oracle.np_f32_to_bf16(b.astype(np.float32))
    x = synth.activations(3 * T + E, T, H)
    layer = MoELayer(d)
    xt = torch.from_numpy(x.view(np.int16)).cuda()
    y1 = layer.forward(xt).clone()
    y2 = layer.forward(xt).clone()
    idx, w, _ = layer.route(xt)
    layer.ctx.sync()
    assert torch.equal(y1, y2), "two forwards of the same tokens differ"
    idx_np = idx.cpu().numpy()
    if hot >= 1.0:
        assert np.bincount(idx_np.ravel(), minlength=E).max() > 8, "the skew must give some expert > 8 slots"
    y_ref = oracle.moe_forward_spec(oracle.Weights(d), x, idx=idx_np, wts=w.cpu().numpy(), acc64=True)
    err = np.abs(y1.cpu().numpy() - y_ref)
    max_abs, mean_rel = float(err.max()), float(err.sum() / max(np.abs(y_ref).sum(), 1e-30))
    assert max_abs <= MAX_ABS, f"max abs error {max_abs}"
    assert mean_rel <= MEAN_REL, f"mean relative error {mean_rel}"
    layer.release()


def test_flat_decode_repeated_calls_reuse_counters(cuda_ctx):
    """Many forwards of changing batches on one layer: the arrival counters
    the kernels leave at zero must serve every later call (a counter left
    behind would make a split tile or a combined row go missing)."""
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=91, hidden=512, intermediate=512, n_experts=16, top_k=4)
    layer = MoELayer(d)
    for it, T in enumerate((1, 8, 3, 8, 1, 6, 2, 8, 4, 7, 40, 9, 64, 5)):
        x = synth.activations(500 + it, T, 512)
        xt = torch.from_numpy(x.view(np.int16)).cuda()
        y = layer.forward(xt)
        idx, w, _ = layer.route(xt)
        layer.ctx.sync()
        y_ref = oracle.moe_forward_spec(oracle.Weights(d), x, idx=idx.cpu().numpy(), wts=w.cpu().numpy(),
                                        acc64=True)
        err = np.abs(y.cpu().numpy() - y_ref)
        assert err.max() <= MAX_ABS, f"call {it} (T={T}): max abs error {err.max()}"
    layer.release()
