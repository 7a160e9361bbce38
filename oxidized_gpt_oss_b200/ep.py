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


class PeerExpertParallelMoE:
    """The same split with the exchange inside the library: rows and output
    rows are stored straight into the other GPUs' buffers (CUDA IPC mappings
    over NVLink), counts and completion flags too, so a forward needs no host
    round trip (``oxg_moe_forward_ep``). ``torch.distributed`` only carries
    the IPC handles once, at construction. Every rank must call ``forward``
    the same number of times; ``close`` on every rank when all are done."""

    def __init__(self, shard, max_tokens: int, group=None, max_recv_rows: int = 0, decode_tokens: int = 0):
        """decode_tokens: forwards of at most that many tokens (<= 64) process
        the received rows with the grouped decode kernels (within the layer
        tolerance of one GPU's forward, not bit for bit); the same value on
        every rank."""
        import ctypes
        from .mxfp4 import context
        self.shard = shard
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_tokens = int(max_tokens)
        c = context(shard.ctx)
        self._ctx = c
        handle = (ctypes.c_char * 64)()
        from . import abi
        abi.check(c.lib.oxg_ep_init(c.handle, shard.layer, self.rank, self.world, self.max_tokens,
                                    int(max_recv_rows), handle), c.handle)
        mine = bytes(handle)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        blob = (ctypes.c_char * (64 * self.world)).from_buffer_copy(b"".join(handles))
        abi.check(c.lib.oxg_ep_connect(c.handle, blob), c.handle)
        if decode_tokens:
            abi.check(c.lib.oxg_ep_set_decode_tokens(c.handle, int(decode_tokens)), c.handle)
        self._abi = abi

    def forward(self, hidden: torch.Tensor, out: torch.Tensor | None = None, shard=None) -> torch.Tensor:
        """shard: another layer's shard on the same context with the same
        shapes and expert range (the buffers depend only on those)."""
        from .mxfp4 import context
        shard = shard or self.shard
        x = hidden.contiguous()
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, shard.hidden), dtype=torch.float32, device=x.device)
        c = context(shard.ctx)
        self._abi.check(c.lib.oxg_moe_forward_ep(c.handle, shard.layer, x.data_ptr() if T else None, T,
                                                 out.data_ptr() if T else None), c.handle)
        return out

    def set_wait_budget(self, seconds: float) -> None:
        """Every wait of a forward on another rank's flag gives up after
        ``seconds`` (default ~2 s): a rank that skips a step, or stopped,
        then shows as OXG_ERR_TIMEOUT at the next synchronisation, with the
        context still usable."""
        self._abi.check(self._ctx.lib.oxg_ep_set_wait_budget(self._ctx.handle, float(seconds)), self._ctx.handle)

    def last_received(self) -> int:
        """Rows this rank received in the last forward (waits for it)."""
        import ctypes
        n = ctypes.c_longlong()
        self._abi.check(self._ctx.lib.oxg_ep_last_received(self._ctx.handle, ctypes.byref(n)), self._ctx.handle)
        return n.value

    __call__ = forward

    def close(self) -> None:
        """After every rank's last forward: synchronise, then unmap and free."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self._abi.check(self._ctx.lib.oxg_ep_close(self._ctx.handle), self._ctx.handle)
        dist.barrier(group=self.group)
