"""Expert-parallel orchestration on CPU: two gloo ranks, float64 numpy shards
(tests/ep_workers.py), against the oracle's single-process layer."""
import os
import pickle
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle
from oxidized_gpt_oss_b200 import ep, synth

import ep_workers


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_splits_and_ranges():
    c = np.array([[1, 2, 3, 4], [5, 6, 7, 8]])
    send, recv, seg = ep.splits(c, 2, 0)
    assert send == [3, 7] and recv == [3, 11] and seg.tolist() == [[1, 2], [5, 6]]
    send, recv, seg = ep.splits(c, 2, 1)
    assert send == [11, 15] and recv == [7, 15] and seg.tolist() == [[3, 4], [7, 8]]
    assert ep.shard_range(32, 4, 3) == (24, 8)
    with pytest.raises(ValueError):
        ep.shard_range(32, 3, 0)


@pytest.mark.parametrize("bias_rank0", [False, True])
def test_two_ranks_match_single_process(tmp_path, bias_rank0):
    layer_kw = dict(seed=21, hidden=64, intermediate=64, n_experts=8, top_k=4)
    tokens = (13, 20)
    mp.spawn(ep_workers.cpu_worker, args=(2, _port(), layer_kw, tokens, str(tmp_path), bias_rank0),
             nprocs=2, join=True)
    d = synth.moe_layer(**layer_kw)
    if bias_rank0:
        b = np.zeros(8, np.float32)
        b[:4] = 50.0
        d["router_b"] = synth.f32_to_bf16_bits(b)
    for r in range(2):
        with open(os.path.join(tmp_path, f"rank{r}.pkl"), "rb") as f:
            got = pickle.load(f)
        ref = oracle.np_moe_forward(d, got["x"])
        assert np.allclose(got["y"], ref, rtol=1e-5, atol=1e-6), np.abs(got["y"] - ref).max()
        if bias_rank0:  # nothing goes to rank 1's experts
            assert got["splits"][0][1] == 0


def test_rank_that_leaves_between_steps_is_reported(tmp_path):
    """Failure detection on the host: after one step together, rank 1 exits
    between steps; rank 0's next step raises from its first collective within
    the process group's timeout instead of hanging."""
    mp.spawn(ep_workers.cpu_leave_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    with open(os.path.join(tmp_path, "rank0.pkl"), "rb") as f:
        got = pickle.load(f)
    assert got["raised"] is not None, "the step with a departed rank did not fail"
    assert got["seconds"] < 30.0, got
