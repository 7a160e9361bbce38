"""The full-decoder oracle (oracle/model_oracle.py) on CPU.

* Its vectorised attention equals a loop restatement of the reference's
  Attention::forward (src/model.rs:1022-1057) — causal order, GQA head
  mapping, the sliding window of `window` keys ending at the query — when no
  sink is given.
* Sinks only add to the softmax denominator; a very negative sink is no sink.
* Greedy selection breaks ties to the last index (src/sampler.rs:7-16).
* RoPE tables and the RMS norm, and a tiny model runs end to end.
"""
import numpy as np
import pytest

from oracle import model_oracle as mo
from oxidized_gpt_oss_b200 import synth


def _qkv(seed, T, nh, nkv, hd):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, nh * hd)).astype(np.float32)
    k = rng.standard_normal((T, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((T, nkv * hd)).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("window", [None, 1, 4])
def test_attention_matches_reference_loop(window):
    T, nh, nkv, hd = 11, 4, 2, 8
    q, k, v = _qkv(window or 0, T, nh, nkv, hd)
    ref = mo.reference_attention_loop(q, k, v, window, hd)
    got = mo.attention(q.reshape(T, nh, hd).astype(np.float64), k.reshape(T, nkv, hd).astype(np.float64),
                       v.reshape(T, nkv, hd).astype(np.float64), np.arange(T), window or 0, None,
                       1.0 / np.sqrt(hd))
    np.testing.assert_allclose(got.reshape(T, nh * hd), ref, rtol=2e-5, atol=2e-5)


def test_sink_only_joins_the_denominator():
    T, nh, nkv, hd = 7, 4, 2, 8
    q, k, v = (a.astype(np.float64) for a in _qkv(3, T, nh, nkv, hd))
    q, k, v = q.reshape(T, nh, hd), k.reshape(T, nkv, hd), v.reshape(T, nkv, hd)
    pos = np.arange(T)
    plain = mo.attention(q, k, v, pos, 0, None, 0.125)
    far = mo.attention(q, k, v, pos, 0, np.full(nh, -1e4), 0.125)
    np.testing.assert_allclose(far, plain, rtol=1e-12, atol=1e-12)
    sinks = np.array([0.5, -1.0, 2.0, 0.0])
    got = mo.attention(q, k, v, pos, 0, sinks, 0.125)
    for h in range(nh):
        kv = h // 2
        for t in range(T):
            s = (k[: t + 1, kv] @ q[t, h]) * 0.125
            mass = np.exp(s).sum()
            np.testing.assert_allclose(got[t, h], plain[t, h] * mass / (mass + np.exp(sinks[h])), rtol=1e-10)


def test_greedy_ties_to_last_index():
    assert mo.greedy(np.array([[1.0, 3.0, 3.0, 2.0]]))[0] == 2
    assert mo.greedy(np.array([[5.0, 1.0, 5.0]]))[0] == 2
    assert mo.greedy(np.array([[0.0, 1.0, -1.0]]))[0] == 1


def test_rope_tables_and_norm():
    cos, sin = mo.rope_tables(300, 150000.0)
    assert np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)
    np.testing.assert_allclose(cos ** 2 + sin ** 2, 1.0, atol=2e-7)
    # highest frequency pair turns by one radian per position
    np.testing.assert_allclose(cos[1, 0], np.cos(1.0), rtol=1e-7)
    x = np.full((1, 64), 3.0)
    g = synth.f32_to_bf16_bits(np.ones(64, dtype=np.float32))
    np.testing.assert_allclose(mo.rms_norm(x, g, 1e-5), 1.0, rtol=1e-2)


def test_tiny_model_runs_and_window_matters():
    m = synth.model_weights(seed=5, n_layers=2, hidden=64, n_heads=4, n_kv_heads=2, vocab=32,
                            sliding_window=3, intermediate=64, n_experts=4, top_k=2)
    toks = np.random.default_rng(0).integers(0, 32, 9)
    lg = mo.forward(m, toks, n_logits=3)
    assert lg.shape == (3, 32) and np.all(np.isfinite(lg))
    # a window covering the whole sequence is full attention
    m_full = dict(m, dims=dict(m["dims"], sliding_window=0))
    m_wide = dict(m, dims=dict(m["dims"], sliding_window=64))
    np.testing.assert_allclose(mo.forward(m_wide, toks, 3), mo.forward(m_full, toks, 3), rtol=1e-12)
    assert not np.allclose(mo.forward(m, toks, 3), mo.forward(m_full, toks, 3))
