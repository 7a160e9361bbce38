"""Checkpoint loader (oxidized_gpt_oss_b200/loader.py) on CPU.

Round trips through the reference's checkpoint naming (src/model.rs:145-412,
src/loader.rs:29-119): every packed tensor comes back bit-identical, gate and
up rows are re-interleaved into the mlp1 layout, scales stored as the
reference reads them (bf16 bit patterns, src/loader.rs:62) become the same
E8M0 bytes, a missing LM head ties to the embedding, and scales that are not
powers of two are refused.
"""
import os

import numpy as np
import pytest

from oxidized_gpt_oss_b200 import loader, synth

DIMS = dict(n_layers=2, hidden=64, n_heads=4, n_kv_heads=2, vocab=48, sliding_window=8, intermediate=96,
            n_experts=4, top_k=2)


def _model():
    return synth.model_weights(seed=9, **DIMS)


def _assert_same(a, b, path=""):
    if isinstance(a, dict):
        for k in a:
            if k == "dims":
                continue
            _assert_same(a[k], b[k], f"{path}.{k}")
    elif isinstance(a, list):
        for i, (x, y) in enumerate(zip(a, b)):
            _assert_same(x, y, f"{path}[{i}]")
    elif isinstance(a, np.ndarray):
        assert np.array_equal(np.asarray(b), a), path
    else:
        assert a == b, path


@pytest.mark.parametrize("bf16_scales", [False, True])
def test_round_trip_is_exact(tmp_path, bf16_scales):
    m = _model()
    loader.save_model_weights(str(tmp_path), m, scales_as_bf16=bf16_scales)
    got = loader.load_model_weights(str(tmp_path), m["dims"])
    _assert_same(m, got)
    # the interleave: mlp1 row 2r is gate row r, 2r + 1 is up row r
    ck = loader.ModelCheckpoint(str(tmp_path))
    g = ck.get("model.layers.1.mlp.experts.gate_proj.weight.blocks")
    assert np.array_equal(got["layers"][1]["moe"]["w1_blocks"][:, 0::2], g)


def test_tied_lm_head(tmp_path):
    m = _model()
    loader.save_model_weights(str(tmp_path), m)
    src = loader.read_safetensors(os.path.join(tmp_path, "model.safetensors"))
    t = {k: np.array(v) for k, v in src.items() if k != "lm_head.weight"}
    os.remove(os.path.join(tmp_path, "model.safetensors"))
    loader.write_safetensors(os.path.join(tmp_path, "model.safetensors"), t)
    got = loader.load_model_weights(str(tmp_path), m["dims"])
    assert np.array_equal(got["unembed"], m["embed"])


def test_scales_must_be_powers_of_two():
    good = synth.f32_to_bf16_bits(np.array([0.0, 0.5, 2.0 ** -20], np.float32))
    assert loader.e8m0_scales(good, "s").tolist() == [0, 126, 107]
    with pytest.raises(ValueError, match="powers of two"):
        loader.e8m0_scales(synth.f32_to_bf16_bits(np.array([1.5], np.float32)), "s")
    with pytest.raises(ValueError, match="powers of two"):
        loader.e8m0_scales(synth.f32_to_bf16_bits(np.array([-1.0], np.float32)), "s")


def test_missing_tensor_is_named(tmp_path):
    m = _model()
    loader.save_model_weights(str(tmp_path), m)
    src = loader.read_safetensors(os.path.join(tmp_path, "model.safetensors"))
    t = {k: np.array(v) for k, v in src.items() if "layers.1.mlp.experts.down_proj.weight.scales" not in k}
    os.remove(os.path.join(tmp_path, "model.safetensors"))
    loader.write_safetensors(os.path.join(tmp_path, "model.safetensors"), t)
    with pytest.raises(KeyError, match="down_proj.weight.scales"):
        loader.load_model_weights(str(tmp_path), m["dims"])
