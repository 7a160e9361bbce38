"""The oracle, pinned: against the reference's own known-answer tests (restated
as committed fixtures), against an independent numpy restatement, and against
its committed small-layer fixture. CPU only."""
import json
import os

import numpy as np
import pytest

from oracle import oracle
from oxidized_gpt_oss_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def test_kat_4x64_dequant_bit_exact(oracle_lib):
    # src/mxfp4.rs:63-95 dequantizes_known_4x64_tensor
    kat = _load("mxfp4_kat_4x64.json")
    out = oracle.dequantize_mxfp4(np.array(kat["blocks"], np.uint8), np.array(kat["scales_bf16"], np.uint16),
                                  kat["rows"], kat["cols"])
    assert out.tolist() == kat["expected_bf16"]


def test_kat_pins_sign_and_negative_zero():
    kat = _load("mxfp4_kat_4x64.json")
    # code 8 is -0.0 (bf16 0x8000): element 8 of row 0 (nibble 8, scale 1)
    assert kat["expected_bf16"][8] == 0x8000
    assert kat["expected_bf16"][0] == 0x0000


def test_integration_sanity_2x32(oracle_lib):
    # tests/integration.rs:30-48 mxfp4_dequant_sanity
    g = _load("mxfp4_sanity_2x32.json")
    out = oracle.dequantize_mxfp4(np.array(g["blocks"], np.uint8), np.array(g["scales_bf16"], np.uint16),
                                  g["rows"], g["cols"])
    assert out.tolist() == g["expected_bf16"]
    vals = synth.bf16_bits_to_f32(out)
    assert abs(vals.mean()) < g["assert_abs_mean_lt"]
    assert vals.std() > g["assert_std_gt"]


def test_e8m0_table(oracle_lib):
    tab = _load("e8m0_table.json")["f32_bits"]
    L = oracle.lib()
    got = [np.float32(L.oxo_e8m0_to_f32(e)).view(np.uint32).item() for e in range(256)]
    assert got == tab
    # the bf16-bits adapter (e << 7) gives the same values
    adapted = synth.bf16_bits_to_f32((np.arange(256, dtype=np.uint16) << 7)).view(np.uint32).tolist()
    assert adapted == tab


def test_e8m0_dequant_equals_bf16_adapter(oracle_lib):
    rng = np.random.default_rng(3)
    rows, cols = 7, 96
    blocks = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    sc = rng.integers(0, 256, rows * cols // 32, dtype=np.uint8)
    a = oracle.dequantize_mxfp4_e8m0(blocks, sc, rows, cols)
    b = oracle.dequantize_mxfp4(blocks, sc.astype(np.uint16) << 7, rows, cols)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("rows,cols,nb,ns,msg", [
    (2, 48, 48, 2, "cols must be divisible by 32, got 48"),
    (2, 64, 63, 4, "blocks length mismatch: expected 64, got 63"),
    (2, 64, 64, 3, "scales length mismatch: expected 4, got 3"),
])
def test_dequant_shape_errors_mirror_reference(oracle_lib, rows, cols, nb, ns, msg):
    with pytest.raises(oracle.OracleShapeError, match=msg):
        oracle.dequantize_mxfp4(np.zeros(nb, np.uint8), np.zeros(ns, np.uint16), rows, cols)


def test_bf16_rounding_matches_numpy_restatement(oracle_lib):
    rng = np.random.default_rng(5)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 1e3,
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e-40, -1e-45, 3.4e38, 1.0 + 2 ** -8,
                                  1.0 + 3 * 2 ** -9], np.float32)])
    L = oracle.lib()
    got = np.array([L.oxo_f32_to_bf16(float(x)) for x in v], np.uint16)
    assert np.array_equal(got, oracle.np_f32_to_bf16(v))
    nan = L.oxo_f32_to_bf16(float("nan"))
    assert (nan & 0x7F80) == 0x7F80 and (nan & 0x7F) != 0


def test_f16_rounding_matches_numpy(oracle_lib):
    rng = np.random.default_rng(6)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 100,
                        (rng.standard_normal(5000) * 1e-5).astype(np.float32),
                        np.array([65504.0, 65520.0, 65519.99, 1e-8, 2 ** -24, 2 ** -25, 3 * 2 ** -26, -0.0,
                                  np.inf], np.float32)])
    L = oracle.lib()
    got = np.array([L.oxo_f32_to_f16(float(x)) for x in v], np.uint16)
    assert np.array_equal(got, v.astype(np.float16).view(np.uint16))
    back = np.array([L.oxo_f16_to_f32(int(h)) for h in got], np.float32)
    assert np.array_equal(back, got.view(np.float16).astype(np.float32))


def test_topk_ties_take_lower_index(oracle_lib):
    logits = np.array([[1.0, 3.0, 3.0, 2.0, 3.0, 0.5]], np.float32)
    idx, w = oracle.topk_softmax(logits, 4)
    assert idx.tolist() == [[1, 2, 4, 3]]
    assert np.isclose(w.sum(), 1.0)


def test_swiglu_clamped_definition(oracle_lib):
    g = np.array([-100.0, -1.0, 0.0, 1.0, 6.9, 7.0, 50.0, np.nan], np.float32)
    u = np.array([-100.0, -7.5, 0.0, 2.0, 7.5, -3.0, 1.0, 0.0], np.float32)
    out = oracle.swiglu_clamped(g, u, 1.702, 7.0)
    gc = np.minimum(g[:7], 7.0)
    uc = np.clip(u[:7], -7.0, 7.0)
    ref = gc / (1 + np.exp(-1.702 * gc)) * (uc + 1)
    assert np.allclose(out[:7], ref, rtol=1e-6, atol=1e-30)
    assert np.isnan(out[7])
    assert not np.any(np.isnan(out[:7]))


def test_spec_matches_numpy_restatement(oracle_lib):
    d = synth.moe_layer(seed=11, hidden=64, intermediate=96, n_experts=6, top_k=3)
    x = synth.activations(11, 9, 64)
    W = oracle.Weights(d)
    y = oracle.moe_forward_spec(W, x, acc64=True)
    y_np = oracle.np_moe_forward(d, x)
    assert np.max(np.abs(y - y_np)) < 1e-4 * max(1.0, np.abs(y_np).max())
    # the fp32-accumulating variant stays within the layer tolerance of the fp64 one
    y32 = oracle.moe_forward_spec(W, x, acc64=False)
    assert np.max(np.abs(y32 - y)) < 2e-2


def test_spec_small_fixture_regression(oracle_lib):
    f = np.load(os.path.join(GOLDEN, "moe_small_seed1.npz"))
    H, I, E, K = f["dims"].tolist()
    alpha, limit = f["act"].tolist()
    d = dict(hidden=H, intermediate=I, n_experts=E, top_k=K, alpha=alpha, limit=limit)
    for k in ("router_w", "router_b", "w1_blocks", "w1_scales", "b1", "w2_blocks", "w2_scales", "b2"):
        d[k] = f[k]
    W = oracle.Weights(d)
    y, slots = oracle.moe_forward_spec(W, f["x"], acc64=True, want_slots=True)
    assert np.array_equal(y, f["y"])
    assert np.array_equal(slots, f["slot_y"])
    idx, w = oracle.topk_softmax(oracle.router_logits(W, f["x"]), K)
    assert np.array_equal(idx, f["idx"])


def test_ref_faithful_runs_and_is_near_plain_semantics(oracle_lib):
    # REF-FAITHFUL differs from SPEC by design (f16 buffers, plain SiLU, no
    # router bias); check it is the reference's algorithm: with router bias
    # absent its routing equals SPEC's routing on bias-free weights.
    d = synth.moe_layer(seed=4, hidden=64, intermediate=64, n_experts=8, top_k=4, router_bias=False)
    x = synth.activations(4, 3, 64)
    W = oracle.Weights(d)
    y16 = oracle.moe_forward_ref_faithful(W, x)
    assert y16.shape == (3, 64) and y16.dtype == np.uint16
    assert np.all(np.isfinite(y16.view(np.float16).astype(np.float32)))


def test_synth_config0_shapes_and_ranges():
    d = synth.moe_layer(seed=0, hidden=128, intermediate=64, n_experts=4)
    assert d["w1_blocks"].shape == (4, 128, 64) and d["w1_scales"].shape == (4, 128, 4)
    assert d["w2_blocks"].shape == (4, 128, 32) and d["w2_scales"].shape == (4, 128, 2)
    assert d["w1_scales"].min() >= 118 and d["w1_scales"].max() <= 126
    assert synth.moe_bytes_per_expert() == 13_236_480
