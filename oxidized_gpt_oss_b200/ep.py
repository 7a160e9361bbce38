"""Expert parallelism over one process per GPU.

The reference has no multi-device path: MoELayer::forward (src/moe.rs:16-100)
runs every expert in one process. Here the E experts of a layer are split into
N contiguous shards, one per rank, and every rank routes its own tokens:

1. ``dispatch``: route + sort the rank's T*k slots expert-major (so also
   destination-rank-major) and write their operand rows (f16 x * 2^-sigma with
   a per-row 2^sigma) — ``MoELayer.dispatch``;
2. exchange the per-expert counts (all-gather), then the rows and scales
   (all-to-all, variable splits): each rank receives, source by source, the
   rows of its own experts in expert order;
3. run the resident experts over them — ``MoELayer.experts``, which treats
   each (source, expert) run as a segment of the grouped GEMM, so nothing is
   re-sorted;
4. send the f32 output rows back (the reverse all-to-all); they land in the
   order step 1 wrote;
5. weighted top-k combine — ``MoELayer.combine``.

Each output row is the same dot products, in the same order, as on one GPU, so
the result is identical to ``MoELayer.forward`` on the full layer.

The collectives go through ``torch.distributed`` (NCCL between GPUs); the shard
object only needs ``dispatch``, ``experts``, ``combine``, ``n_experts``,
``expert_begin`` and ``expert_count``.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def shard_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous expert range (begin, count) of ``rank``; needs E % world == 0."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split evenly over {world} ranks")
    per = n_experts // world
    return rank * per, per


def splits(counts_all: np.ndarray, world: int, rank: int) -> tuple[list[int], list[int], np.ndarray]:
    """From the gathered per-expert counts [world, E] of every rank's dispatch:
    rows this rank sends to each rank, rows it receives from each rank, and the
    received segment table [world, E / world] (source-major, expert order)."""
    E = counts_all.shape[1]
    per = E // world
    by_dest = counts_all.reshape(world, world, per)  # [src, dest, expert within dest]
    send = by_dest[rank].sum(axis=1).astype(np.int64).tolist()
    seg = by_dest[:, rank, :]
    recv = seg.sum(axis=1).astype(np.int64).tolist()
    return send, recv, np.ascontiguousarray(seg, dtype=np.int32)


class ExpertParallelMoE:
    """One MoE layer split over the ranks of ``group`` (default: the world)."""

    def __init__(self, shard, group=None):
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        begin, count = shard_range(shard.n_experts, self.world, self.rank)
        if (shard.expert_begin, shard.expert_count) != (begin, count):
            raise ValueError(f"rank {self.rank} must hold experts [{begin}, {begin + count}), "
                             f"holds [{shard.expert_begin}, {shard.expert_begin + shard.expert_count})")
        self.last_splits = None

    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, out_split: list[int], in_split: list[int]):
        dist.all_to_all_single(out, inp, out_split, in_split, group=self.group)

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        T = hidden.shape[0]
        rows, scale, counts = self.shard.dispatch(hidden)
        gathered = [torch.empty_like(counts) for _ in range(self.world)]
        dist.all_gather(gathered, counts, group=self.group)
        counts_all = torch.stack(gathered).cpu().numpy()
        send, recv, seg = splits(counts_all, self.world, self.rank)
        self.last_splits = (send, recv)
        H = rows.shape[1]
        rows_in = rows.new_empty((sum(recv), H))
        scale_in = scale.new_empty((sum(recv),))
        self._exchange(rows_in, rows, recv, send)
        self._exchange(scale_in, scale, recv, send)
        y_in = self.shard.experts(rows_in, scale_in, seg)
        y_back = y_in.new_empty((rows.shape[0], y_in.shape[1]))
        self._exchange(y_back, y_in, send, recv)
        return self.shard.combine(y_back, T)

    __call__ = forward
