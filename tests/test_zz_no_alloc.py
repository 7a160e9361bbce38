"""oxg_moe_forward_noalloc: the layer forward for callers that must not have the
library allocate device memory (runtimes that pre-reserve the whole GPU,
latency-critical loops that cannot absorb an allocation's synchronisation,
embedders that forbid foreign allocations). Its scratch is a fixed 4 MiB
array inside the library; its results must agree with oxg_moe_forward's within
the layer tolerance.

This file is collected last so that, if it fails, a run stopping at the first
failure has already run every other test. It creates its own context, so it
also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oxidized_gpt_oss_b200 import abi, synth

pytestmark = pytest.mark.gpu
MAX_ABS = 2e-2   # the layer tolerance every MoE parity test uses
MEAN_REL = 1e-3


def _noalloc(layer, x, out):
    lib = abi.load()
    return lib.oxg_moe_forward_noalloc(layer.ctx.handle, layer.layer, x.data_ptr(), x.shape[0],
                                       out.data_ptr())


def test_noalloc_matches_forward_on_two_calls_in_a_row():
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    layer = MoELayer(synth.moe_layer(seed=21))  # gpt-oss-20b shapes
    for seed, T in ((31, 8), (32, 5)):  # the second call reuses the array left by the first
        x = torch.from_numpy(synth.activations(seed, T, layer.hidden).view(np.int16)).cuda()
        ref = layer.forward(x)
        out = torch.full((T, layer.hidden), float("nan"), dtype=torch.float32, device="cuda")
        abi.check(_noalloc(layer, x, out), layer.ctx.handle)
        torch.cuda.synchronize()
        err = (out - ref).abs()
        assert torch.isfinite(out).all()
        assert err.max().item() <= MAX_ABS
        assert (err.sum() / ref.abs().sum()).item() <= MEAN_REL


def test_noalloc_refuses_an_expert_parallel_shard():
    """A layer uploaded as a shard (experts [8, 16) of 32) holds only those
    experts' weights; the call must refuse it before launching anything."""
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    d = synth.moe_layer(seed=23, hidden=256, intermediate=256, n_experts=32, top_k=4)
    layer = MoELayer(d, experts=(8, 8))
    x = torch.zeros((4, layer.hidden), dtype=torch.int16, device="cuda")
    out = torch.empty((4, layer.hidden), dtype=torch.float32, device="cuda")
    st = _noalloc(layer, x, out)
    assert st == abi.OXG_ERR_STATE
    msg = abi.load().oxg_last_error(layer.ctx.handle).decode()
    assert "holds experts [8, 16) only" in msg
    layer.release()


def test_noalloc_refuses_batches_beyond_its_array():
    import torch
    from oxidized_gpt_oss_b200.moe import MoELayer
    layer = MoELayer(synth.moe_layer(seed=22, hidden=2880, intermediate=2880, n_experts=4, top_k=4))
    T = 46
    x = torch.zeros((T, layer.hidden), dtype=torch.int16, device="cuda")
    out = torch.empty((T, layer.hidden), dtype=torch.float32, device="cuda")
    st = _noalloc(layer, x, out)
    assert st == abi.OXG_ERR_SHAPE
    msg = abi.load().oxg_last_error(layer.ctx.handle).decode()
    assert "enough for 45 tokens" in msg
