"""Failure detection on the GPU without a GPU fault: a peer-memory expert-
parallel step whose other rank does not take part gives up after a short,
settable wait budget, reports OXG_ERR_TIMEOUT at the synchronisation, and the
context stays usable. Two processes; with one GPU they share it, and only rank
0 ever launches a kernel that waits (rank 1 connects, then waits on the host),
so no two waiting kernels run on one GPU."""
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


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_expert_parallel_wait_times_out_and_context_survives(tmp_path):
    from oxidized_gpt_oss_b200 import abi
    mp.spawn(ep_workers.gpu_timeout_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    with open(os.path.join(tmp_path, "rank0.pkl"), "rb") as f:
        got = pickle.load(f)
    assert got.get("first_step_equal", True), "the step both ranks took differs from the whole layer"
    assert got["status"] == abi.OXG_ERR_TIMEOUT, got
    assert "timed out" in got["message"], got
    assert got["seconds"] < 5.0, got  # three waits of 50 ms, not the ~2 s default
    assert got["usable_after"], "the context did not run the whole layer after the timeout"
