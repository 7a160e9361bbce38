"""Standalone clamped SwiGLU kernel against the oracle."""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu


def test_swiglu_matches_oracle(cuda_ctx):
    import torch
    from oxidized_gpt_oss_b200.ffn import swiglu
    rng = np.random.default_rng(0)
    n = 100_003
    g = (rng.standard_normal(n) * 6).astype(np.float32)
    u = (rng.standard_normal(n) * 6).astype(np.float32)
    g[:6] = [-1e30, -90.0, 7.0, 7.5, np.inf, np.nan]
    u[:6] = [1.0, -8.0, 8.0, -np.inf, 0.0, 0.0]
    out = swiglu(torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()).cpu().numpy()
    ref = oracle.swiglu_clamped(g, u, 1.702, 7.0)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    assert np.allclose(out[fin], ref[fin], rtol=2e-6, atol=1e-30)
