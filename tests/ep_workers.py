"""Worker processes for the expert-parallel tests (spawned, one per rank).

The CPU tests run the orchestrator over gloo with ``NumpyShard`` — the layer
computed in float64 numpy from the oracle's restatement — standing in for the
CUDA shard, so the collective plumbing (counts, splits, row exchange, return,
combine order) is checked without a GPU. The GPU worker runs the real shard
over NCCL and compares with the single-GPU forward."""
import datetime
import os
import pickle

import numpy as np
import torch
import torch.distributed as dist

from oracle import oracle
from oxidized_gpt_oss_b200 import ep, synth


class NumpyShard:
    """dispatch / experts / combine of one expert range, in float64."""

    def __init__(self, d, begin, count):
        self.d = d
        self.n_experts, self.top_k, self.hidden = d["n_experts"], d["top_k"], d["hidden"]
        self.expert_begin, self.expert_count = begin, count

    def dispatch(self, hidden):
        d, K = self.d, self.top_k
        x = oracle.np_bf16_to_f32(hidden.numpy().view(np.uint16)).astype(np.float64)
        logits = x @ oracle.np_bf16_to_f32(d["router_w"]).astype(np.float64).T
        if d.get("router_b") is not None:
            logits = logits + oracle.np_bf16_to_f32(d["router_b"]).astype(np.float64)
        idx = np.argsort(-logits, axis=1, kind="stable")[:, :K]
        top = np.take_along_axis(logits, idx, axis=1)
        ex = np.exp(top - top.max(axis=1, keepdims=True))
        self.wts = ex / ex.sum(axis=1, keepdims=True)
        self.idx = idx
        flat = idx.reshape(-1)
        order = np.argsort(flat, kind="stable")
        self.pos = np.empty_like(order)
        self.pos[order] = np.arange(order.size)
        rows = torch.from_numpy(np.ascontiguousarray(x[order // K]))
        scale = torch.ones(order.size, dtype=torch.float64)
        counts = torch.from_numpy(np.bincount(flat, minlength=self.n_experts).astype(np.int32))
        return rows, scale, counts

    def _expert(self, e, xr):
        d = self.d
        w1 = oracle.np_dequant_f32(d["w1_blocks"][e], d["w1_scales"][e]).astype(np.float64)
        w2 = oracle.np_dequant_f32(d["w2_blocks"][e], d["w2_scales"][e]).astype(np.float64)
        b1 = oracle.np_bf16_to_f32(d["b1"][e]).astype(np.float64)
        b2 = oracle.np_bf16_to_f32(d["b2"][e]).astype(np.float64)
        h1 = xr @ w1.T + b1
        g = np.minimum(h1[:, 0::2], d["limit"])
        u = np.clip(h1[:, 1::2], -d["limit"], d["limit"])
        h = g / (1.0 + np.exp(-d["alpha"] * g)) * (u + 1.0)
        return h @ w2.T + b2

    def experts(self, rows, scale, seg):
        x = rows.numpy() * scale.numpy()[:, None]
        out = np.zeros((x.shape[0], self.hidden))
        r = 0
        for s in range(seg.shape[0]):
            for el in range(self.expert_count):
                n = int(seg[s, el])
                if n:
                    out[r:r + n] = self._expert(self.expert_begin + el, x[r:r + n])
                r += n
        return torch.from_numpy(out)

    def combine(self, y_rows, T):
        y = y_rows.numpy()
        K = self.top_k
        out = np.zeros((T, self.hidden))
        for j in range(K):
            out += self.wts[:, j:j + 1] * y[self.pos[np.arange(T) * K + j]]
        return torch.from_numpy(out)


def _init(rank, world, port, backend):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))


def cpu_worker(rank, world, port, layer_kw, tokens, out_dir, bias_rank0):
    _init(rank, world, port, "gloo")
    try:
        d = synth.moe_layer(**layer_kw)
        if bias_rank0:  # every slot to rank 0's experts: empty splits elsewhere
            b = np.zeros(d["n_experts"], np.float32)
            b[: d["n_experts"] // world] = 50.0
            d["router_b"] = synth.f32_to_bf16_bits(b)
        begin, count = ep.shard_range(d["n_experts"], world, rank)
        moe = ep.ExpertParallelMoE(NumpyShard(d, begin, count))
        x = synth.activations(100 + rank, tokens[rank], d["hidden"])
        y = moe(torch.from_numpy(x.view(np.int16))).numpy()
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"x": x, "y": y, "splits": moe.last_splits}, f)
    finally:
        dist.destroy_process_group()


def gpu_worker(rank, world, port, layer_kw, tokens, out_dir):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    try:
        from oxidized_gpt_oss_b200.moe import MoELayer
        d = synth.moe_layer(**layer_kw)
        begin, count = ep.shard_range(d["n_experts"], world, rank)
        shard = MoELayer(d, experts=(begin, count))
        full = MoELayer(d)
        moe = ep.ExpertParallelMoE(shard)
        x = torch.from_numpy(synth.activations(100 + rank, tokens[rank], d["hidden"]).view(np.int16)).cuda()
        y_ep = moe(x).clone()
        y_full = full.forward(x).clone()
        torch.cuda.synchronize()
        dist.barrier()
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"equal": bool(torch.equal(y_ep, y_full)),
                         "max_diff": float((y_ep - y_full).abs().max()) if y_ep.numel() else 0.0,
                         "splits": moe.last_splits}, f)
    finally:
        dist.destroy_process_group()


def gpu_p2p_worker(rank, world, port, layer_kw, tokens, out_dir):
    """Peer-memory expert parallelism: two forwards (two epochs) per rank, each
    compared with the full layer's single-GPU forward."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    moe = None
    try:
        from oxidized_gpt_oss_b200.moe import MoELayer
        d = synth.moe_layer(**layer_kw)
        begin, count = ep.shard_range(d["n_experts"], world, rank)
        shard = MoELayer(d, experts=(begin, count))
        full = MoELayer(d)
        moe = ep.PeerExpertParallelMoE(shard, max_tokens=max(tokens))
        res = []
        for it in range(2):
            x = torch.from_numpy(synth.activations(100 * it + rank, tokens[rank], d["hidden"]).view(np.int16)).cuda()
            y_ep = moe(x).clone()
            y_full = full.forward(x).clone() if tokens[rank] else torch.empty_like(y_ep)
            torch.cuda.synchronize()
            shard.ctx.sync()
            res.append((bool(torch.equal(y_ep, y_full)),
                        float((y_ep - y_full).abs().max()) if y_ep.numel() else 0.0))
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"res": res}, f)
    finally:
        if moe is not None:
            moe.close()
        dist.destroy_process_group()


def gpu_model_ep_worker(rank, world, port, out_dir):
    """Batched decode of a 2-layer gpt-oss-architecture model (16 experts,
    vocab 4096) with the MoE blocks expert parallel (8 experts per GPU, rows
    over peer memory, decode steps received on the grouped kernels) against
    the same sequences with every expert on this GPU: three sequences per
    rank, four teacher-forced steps, logits compared."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    g = None
    try:
        from oxidized_gpt_oss_b200.model import GPTModel
        m = synth.model_weights(seed=9, n_layers=2, vocab=4096, n_experts=16)
        shard = ep.shard_range(16, world, rank)
        g = GPTModel(m, max_seq=256, max_tokens=128, max_batch=3, experts=shard)
        g.connect_expert_parallel()
        full = GPTModel(m, max_seq=256, max_tokens=128, max_batch=3)
        rng = np.random.default_rng(100 + rank)
        cur = torch.zeros(3, dtype=torch.int32, device="cuda")
        for sq, n in enumerate((40, 70, 20)):  # every rank runs the same steps
            ids = torch.from_numpy(rng.integers(0, 4096, n).astype(np.int32)).cuda()
            cur[sq:sq + 1].copy_(g.prefill_seq(sq, ids))
            full.prefill_seq(sq, ids)
        lg_ep = torch.empty((3, 4096), dtype=torch.float32, device="cuda")
        lg_full = torch.empty_like(lg_ep)
        diffs, agree = [], 0
        for _ in range(4):
            nx = g.step_batch(cur, logits=lg_ep)
            nf = full.step_batch(cur, logits=lg_full)
            torch.cuda.synchronize()
            g.sync()
            diffs.append(float((lg_ep - lg_full).abs().max()))
            agree += int((nx == nf).sum())
            cur = nx
        full.release()
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"diffs": diffs, "agree": agree}, f)
    finally:
        if g is not None:
            g.close_expert_parallel()
        dist.destroy_process_group()


def gpu_p2p_grouped_worker(rank, world, port, layer_kw, tokens, hot, out_dir):
    """Peer-memory expert parallelism with decode-sized batches received on
    the grouped decode kernels: two forwards per rank, each checked against
    the oracle on the full layer's routing of the same tokens. A router bias
    of -hot * ln(rank) skews the loads (segments of more than 8 rows)."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    moe = None
    try:
        from oxidized_gpt_oss_b200.moe import MoELayer
        d = synth.moe_layer(**layer_kw)
        E = d["n_experts"]
        if hot:
            rk = np.random.default_rng(E).permutation(E) + 1
            b = oracle.np_bf16_to_f32(d["router_b"]) - hot * np.log(rk)
            d["router_b"] = oracle.np_f32_to_bf16(b.astype(np.float32))
        begin, count = ep.shard_range(E, world, rank)
        shard = MoELayer(d, experts=(begin, count))
        full = MoELayer(d)
        moe = ep.PeerExpertParallelMoE(shard, max_tokens=max(tokens), decode_tokens=max(tokens))
        res = []
        for it in range(2):
            x = synth.activations(100 * it + rank, tokens[rank], d["hidden"])
            xt = torch.from_numpy(x.view(np.int16)).cuda()
            y_ep = moe(xt).clone()
            torch.cuda.synchronize()
            shard.ctx.sync()
            if tokens[rank] == 0:
                res.append((0.0, 0.0, 0))
                continue
            idx, w, _ = full.route(xt)
            full.ctx.sync()
            idx_np = idx.cpu().numpy()
            y_ref = oracle.moe_forward_spec(oracle.Weights(d), x, idx=idx_np, wts=w.cpu().numpy(), acc64=True)
            err = np.abs(y_ep.cpu().numpy() - y_ref)
            res.append((float(err.max()), float(err.sum() / max(np.abs(y_ref).sum(), 1e-30)),
                        int(np.bincount(idx_np.ravel(), minlength=E).max())))
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump({"res": res}, f)
    finally:
        if moe is not None:
            moe.close()
        dist.destroy_process_group()


def gpu_timeout_worker(rank, world, port, out_dir):
    """Failure detection without a GPU fault. Both ranks connect a peer-memory
    exchange (gloo carries the handles; with one GPU both processes share it
    and only rank 0 ever launches a kernel that waits). With two GPUs both
    first run one forward together. Then rank 1 skips a step: rank 0's
    forward waits on flags nothing sets, gives up after the 50 ms budget and
    reports OXG_ERR_TIMEOUT at the synchronisation; rank 0's context then
    still runs the whole layer."""
    import time
    n_dev = torch.cuda.device_count()
    torch.cuda.set_device(rank % n_dev)
    _init(rank, world, port, "gloo")
    moe = None
    out = {}
    try:
        from oxidized_gpt_oss_b200 import abi
        from oxidized_gpt_oss_b200.moe import MoELayer
        d = synth.moe_layer(seed=41, hidden=256, intermediate=256, n_experts=16, top_k=4)
        begin, count = ep.shard_range(16, world, rank)
        shard = MoELayer(d, experts=(begin, count))
        # 80 tokens per rank: above the small-batch path, so the whole layer on
        # one GPU takes the same router and expert kernels as the exchange and
        # the first step must match it bit for bit
        moe = ep.PeerExpertParallelMoE(shard, max_tokens=96)
        x = torch.from_numpy(synth.activations(300 + rank, 80, 256).view(np.int16)).cuda()
        full = MoELayer(d) if rank == 0 else None
        y_ref = full.forward(x).clone() if full else None
        if n_dev >= world:  # a good step on separate GPUs first
            y = moe(x).clone()
            shard.ctx.sync()
            out["first_step_equal"] = bool(torch.equal(y, y_ref)) if full else True
        dist.barrier()
        if rank == 0:
            moe.set_wait_budget(0.05)
            t0 = time.perf_counter()
            status = 0
            try:
                moe(x)
                shard.ctx.sync()
            except abi.OxgError as e:
                status = e.status
                out["message"] = e.message
            out["status"] = status
            out["seconds"] = time.perf_counter() - t0
            y2 = full.forward(x)
            full.ctx.sync()
            out["usable_after"] = bool(torch.equal(y2, y_ref))
        dist.barrier()  # rank 1 skipped the step: it waits here, on the host
    finally:
        if moe is not None:
            moe.close()
        with open(os.path.join(out_dir, f"rank{rank}.pkl"), "wb") as f:
            pickle.dump(out, f)
        dist.destroy_process_group()


def cpu_leave_worker(rank, world, port, out_dir):
    """A rank that leaves between steps: after one step together rank 1 exits
    (no collective in flight). Rank 0's next step fails in its first
    collective instead of hanging (the process group's 10 s timeout bounds it
    even where the backend does not notice the closed connection)."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    d = synth.moe_layer(seed=42, hidden=64, intermediate=64, n_experts=4, top_k=2)
    begin, count = ep.shard_range(4, world, rank)
    moe = ep.ExpertParallelMoE(NumpyShard(d, begin, count))
    x = torch.from_numpy(synth.activations(400 + rank, 5, 64).view(np.int16))
    moe(x)
    if rank == 1:
        return  # leaves between steps: the process exits
    out = {"raised": None}
    t0 = time.perf_counter()
    try:
        moe(x)
    except Exception as e:  # the backend's error for a lost peer or a timeout
        out["raised"] = type(e).__name__
    out["seconds"] = time.perf_counter() - t0
    with open(os.path.join(out_dir, "rank0.pkl"), "wb") as f:
        pickle.dump(out, f)
    try:
        dist.destroy_process_group()
    except Exception:
        pass
