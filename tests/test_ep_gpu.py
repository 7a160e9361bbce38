"""Expert parallelism on 2 GPUs (NCCL): each rank's output through dispatch /
all-to-all / resident experts / all-to-all / combine equals, bit for bit, the
single-GPU forward of the full layer on the same tokens (every output row is
the same dot products in the same order)."""
import os
import pickle
import socket

import pytest
import torch
import torch.multiprocessing as mp

import ep_workers

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("layer_kw,tokens", [
    (dict(seed=31, hidden=256, intermediate=256, n_experts=16, top_k=4), (200, 90)),
    (dict(seed=32), (300, 257)),  # gpt-oss-20b widths, 32 experts split 16 + 16
])
def test_two_gpus_equal_single_gpu(tmp_path, layer_kw, tokens):
    mp.spawn(ep_workers.gpu_worker, args=(2, _port(), layer_kw, tokens, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        with open(os.path.join(tmp_path, f"rank{r}.pkl"), "rb") as f:
            got = pickle.load(f)
        assert got["equal"], f"rank {r}: max |ep - single| = {got['max_diff']}"


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
@pytest.mark.parametrize("layer_kw,tokens", [
    (dict(seed=31, hidden=256, intermediate=256, n_experts=16, top_k=4), (200, 90)),
    (dict(seed=33, hidden=256, intermediate=256, n_experts=16, top_k=4), (150, 0)),  # a rank with no tokens
    (dict(seed=32), (300, 257)),
])
def test_two_gpus_peer_memory_equal_single_gpu(tmp_path, layer_kw, tokens):
    mp.spawn(ep_workers.gpu_p2p_worker, args=(2, _port(), layer_kw, tokens, str(tmp_path)), nprocs=2,
             join=True)
    for r in range(2):
        with open(os.path.join(tmp_path, f"rank{r}.pkl"), "rb") as f:
            got = pickle.load(f)
        for it, (equal, diff) in enumerate(got["res"]):
            assert equal, f"rank {r} forward {it}: max |ep - single| = {diff}"
