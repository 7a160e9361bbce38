#!/usr/bin/env python
"""Benchmark of the MXFP4 MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload moe_prefill|moe_decode|dequant|model_decode|model_batch|tensor_peak]
                    [--tokens T] [--layers L]

Workloads (seeded synthetic inputs, random-init gpt-oss-20b shapes):
  moe_prefill (default) 8192 tokens per GPU through one MoE block on the
              tcgen05 grouped-GEMM path (router logits ~N(0, 1), so expert
              loads are roughly uniform). Metric: tokens/s; roofline: TFLOP/s
              of the gate/up GEMM against the measured dense 16-bit tensor
              peak, and beside it the dense MXFP4 (kind::mxf4) rate measured
              in the same run. On N GPUs the experts are split 32/N per GPU
              (expert parallel; rows exchanged over NVLink peer memory, or
              NCCL all-to-all with --ep nccl); on one GPU
              the line also carries a "decode" object (the moe_decode
              workload measured in the same process) and a "model_decode"
              object (the model_decode workload, 64 timed steps).
  moe_decode  one MoE block forward over T tokens (default 8: the 8-token
              gpt-oss-20b block — hidden 2880, 32 experts top-4, MXFP4
              weights with E8M0 scales in [118, 126], bf16 activations).
              Metric: tokens/s; roofline: HBM GB/s of the gate/up kernel.
              N > 1: independent replicas.
  model_decode greedy decode of the full 24-layer gpt-oss-20b architecture
              (random init), batch 1: a 2048-token prompt, then --steps
              one-token steps replayed from a captured CUDA graph. Metric:
              tokens/s; roofline: HBM GB/s of the slowest weight-streaming
              kernel; e2e through oxg_model_generate (host prompt in, host
              tokens out).
  dequant     standalone MXFP4 -> bf16 dequant of one layer's expert tensors
              (32x5760x2880 + 32x2880x2880, E8M0 in [110, 135]). Metric: GB/s
              of algorithmic traffic (423,014,400 B read + 1,592,524,800 B written).
  model_batch  64 sequences at KV length 8192 over the 24-layer model,
              Zipf-skewed expert loads, one batched greedy step per timed
              step (expert parallel over N GPUs under torchrun).
  tensor_peak  issue rate of tcgen05 kind::f16, kind::mxf8f6f4 (E2M1 x E4M3)
              and kind::mxf4 (E2M1 x E2M1) MMAs, one CTA per SM, from shared
              memory: the measured tensor denominators.

Steps cycle over L uploaded layers (default 4 x 424 MB of packed weights), so
inputs are larger than L2 and no step finds the previous step's weights
cached. N > 1 runs one process per GPU (torchrun); timing is max over ranks
and ``value`` is the whole-job aggregate.

``--impl reference`` times the reference's own CPU algorithm for the same
workload (the oracle's REF-FAITHFUL restatement: f16 buffers, per-call
weight conversion, sequential loops) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE tokens/s + HBM GB/s (decode), MXFP4 TFLOPS (prefill) at 1/2/4/8 B200"
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "ncu_traffic.json")
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


FALLBACK_TFLOPS = 1590.0


def tensor_peak():
    """Dense 16-bit tensor-core peak (burst figure: each kernel is timed alone)."""
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_TFLOPS, "fallback"


MMA_KINDS = (("f16", "tcgen05.mma.kind::f16, f16 x f16 -> f32, M128 N256 K16"),
             ("mxf8f6f4", "tcgen05.mma.kind::mxf8f6f4.block_scale, E2M1 x E4M3, UE8M0, M128 N256 K32"),
             ("mxf4", "tcgen05.mma.kind::mxf4.block_scale.block32, E2M1 x E2M1, UE8M0, M128 N256 K64"))


def mma_rates(ctx, iters: int = 65536, repeats: int = 3):
    """Measured tensor-core issue rate (TFLOP/s, best of `repeats`) of each
    instruction kind, one CTA per SM issuing back to back from shared memory."""
    return {name: max(ctx.mma_rate(k, iters) for _ in range(repeats)) for k, (name, _) in enumerate(MMA_KINDS)}


def ncu_traffic(kernel: str, key: str):
    """Per-launch DRAM bytes of `kernel` from the committed ncu summary, or None."""
    try:
        with open(TRAFFIC_PATH) as f:
            t = json.load(f)
        return t[kernel][key]
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.out or "").splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm, smax = float(f[1]), float(f[2])
            except ValueError:
                continue
            sms.append(sm)
            mx = smax
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sms)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


# --------------------------------------------------------------------------- helpers
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def max_over_ranks(v: float, ws: int) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws: int):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def emit(d: dict):
    print(json.dumps(d), flush=True)


# --------------------------------------------------------------------------- reference arm
def host_cpu():
    """(cores this process may run on, CPU model name) of the host."""
    try:
        cores = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        cores = os.cpu_count() or 1
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return cores, model


def ref_moe_rates(d, x_np, steps: int = 1):
    """The reference's MoE algorithm (the oracle's REF-FAITHFUL restatement of
    src/moe.rs:16-100 and src/model.rs:1088-1184: f16 buffers, per-call weight
    conversion, sequential loops) on this host, measured two ways with explicit
    thread counts (never inherited from OMP_NUM_THREADS, which torchrun sets
    to 1): one token on one thread (the reference is single-threaded), and one
    token per core on every core of the host. Returns tokens/s for both, the
    core count and the CPU model; the same at every GPU count."""
    from oracle import oracle
    cores, model = host_cpu()
    T = min(cores, x_np.shape[0])
    W = oracle.Weights(d)
    L = oracle.RefLayer(W, x_np[:T])
    L.forward(x_np[:1], nthreads=1)  # warm: page in the weights
    t0 = time.perf_counter()
    L.forward(x_np[:1], nthreads=1)
    one_s = time.perf_counter() - t0
    L.forward(x_np[:T], nthreads=T)
    t0 = time.perf_counter()
    for _ in range(max(steps, 1)):
        L.forward(x_np[:T], nthreads=T)
    all_s = (time.perf_counter() - t0) / max(steps, 1)
    L.close()
    return {"single_thread": 1.0 / one_s, "all_cores": T / all_s, "cores": T, "cpu_model": model,
            "single_thread_s_per_token": one_s, "all_cores_s_per_step": all_s}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle
    from oxidized_gpt_oss_b200 import synth
    threads, cpu_model = host_cpu()
    if args.workload == "dequant":
        (w1, s1, r1, c1), _ = synth.dequant_tensors(seed=0)
        rows = 5760 * 4  # bounded sample: 4 experts' mlp1 rows per step
        blocks = w1.reshape(-1, c1 // 2)[:rows]
        scales = s1.reshape(-1, c1 // 32)[:rows]
        per_step_bytes = rows * c1 // 2 + rows * c1 // 32 + rows * c1 * 2
        for _ in range(args.warmup):
            oracle.dequantize_mxfp4_e8m0(blocks, scales, rows, c1)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            oracle.dequantize_mxfp4_e8m0(blocks, scales, rows, c1)
        dt = time.perf_counter() - t0
        value = per_step_bytes * args.steps / dt / 1e9
        unit = "GB/s"
        sample = f"{rows} rows x {c1} cols of mlp1 per step ({per_step_bytes} B algorithmic)"
        config = dequant_config()
        threads = 1
    else:
        # bounded sample: one MoE block through the reference's algorithm,
        # timed on one thread and on every core of the host (explicit thread
        # counts: the same measurement at every GPU count)
        d = synth.moe_layer(seed=0)
        x = synth.activations(0, max(threads, 1), d["hidden"])
        n_rep = 2 if args.workload in ("moe_prefill", "moe_decode") else 1
        r = ref_moe_rates(d, x, steps=n_rep)
        threads = r["cores"]
        n_layers = synth.GPT_OSS_20B_MODEL["n_layers"]
        unit = "tokens/s"
        if args.workload == "model_decode":
            # one sequence decodes one token at a time, single-threaded, as the reference does
            value = r["single_thread"] / n_layers
            threads = 1
            sample = (f"one token through one MoE block on one thread ({r['single_thread_s_per_token']:.2f} s) "
                      f"x {n_layers} layers; attention and LM head not counted (an upper bound on its rate)")
            config = model_config(args, synth.GPT_OSS_20B_MODEL, args.prompt)
        elif args.workload == "model_batch":
            # independent sequences: one per host core, each decoding as the reference does
            value = r["all_cores"] / n_layers
            sample = (f"{r['cores']} sequences' tokens through one MoE block, one per core "
                      f"({r['all_cores_s_per_step']:.2f} s) x {n_layers} layers; attention and LM head "
                      f"not counted (an upper bound on its rate)")
            config = model_batch_config(args, synth.GPT_OSS_20B_MODEL)
        else:
            value = r["all_cores"]
            sample = (f"{r['cores']} of the workload's {args.tokens} tokens per step (one per core) through one "
                      f"MoE block, {n_rep} steps of {r['all_cores_s_per_step']:.2f} s")
            config = prefill_config(args, d, ws) if args.workload == "moe_prefill" else moe_config(args, d)
        dt = args.steps * (x.shape[0] / value if value > 0 else 0.0)
    cb = {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample,
          "cpu_model": cpu_model, "scope": "this host's cores, the same measurement at every GPU count"}
    if args.workload != "dequant":
        cb["single_thread_tokens_s"] = r["single_thread"]
        cb["all_cores_tokens_s"] = r["all_cores"]
    emit({"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": ws,
          "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / max(args.steps, 1) * 1e3,
          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
          "data": "synthetic", "config": config, "cpu_baseline": cb,
          "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})


def moe_config(args, d):
    """Workload description shared by both arms (so their configs compare equal)."""
    return {"workload": "moe_block_decode", "tokens_per_gpu": args.tokens, "hidden": d["hidden"],
            "intermediate": d["intermediate"], "experts": d["n_experts"], "top_k": d["top_k"],
            "weights": "mxfp4 e2m1 + e8m0[118,126]", "layers_cycled": args.layers,
            "l2": "inputs larger than L2: steps cycle over 4 layers x 424 MB of packed weights",
            "parallelism": "replicas" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "single"}


def prefill_config(args, d, ws):
    """The moe_prefill workload, shared by both arms."""
    return {"workload": "moe_prefill", "tokens_per_gpu": args.tokens, "hidden": d["hidden"],
            "intermediate": d["intermediate"], "experts": d["n_experts"], "top_k": d["top_k"],
            "weights": "mxfp4 e2m1 + e8m0[118,126]", "layers_cycled": args.layers,
            "l2": "inputs larger than L2 (424 MB of packed weights and 189 MB of slot activations per step)",
            "parallelism": (f"ep{ws} (experts 32/{ws} per GPU; " +
                            ("rows and output rows stored over NVLink peer memory by the library's kernels)"
                             if args.ep == "p2p" else "NCCL all-to-all)")) if ws > 1 else "single"}


def dequant_config():
    return {"workload": "dequant_layer", "elements": 32 * 5760 * 2880 + 32 * 2880 * 2880,
            "l2": "inputs larger than L2 (423 MB in, 1.59 GB out per step)"}


# --------------------------------------------------------------------------- our arm
def cpu_baseline_moe(d, x):
    """The reference's algorithm on this host (rank 0, one GPU): the headline
    value is one thread (the reference is single-threaded); the all-cores rate
    (what the reference arm reports) rides along."""
    r = ref_moe_rates(d, x, steps=1)
    return {"value": r["single_thread"], "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"one token through one MoE block on one thread (the reference's algorithm as written), "
                      f"{r['single_thread_s_per_token']:.2f} s",
            "all_cores": {"value": r["all_cores"], "cores": r["cores"],
                          "sample": f"{r['cores']} tokens, one per core, {r['all_cores_s_per_step']:.2f} s"},
            "cpu_model": r["cpu_model"]}


def oracle_parity(d, x_np, y, idx, w, logits, n_sample: int, seed: int):
    """Checks sampled rows of a GPU forward against the fp64 SPEC oracle (the
    checker; it runs beside the CPU baseline, outside every timed region):
    routing identical to the oracle's own top-k except at near-ties, and the
    layer bar max |err| <= 2e-2, sum|err| / sum|ref| <= 1e-3."""
    from oracle import oracle
    cores, _ = host_cpu()
    T, K = x_np.shape[0], d["top_k"]
    sample = np.sort(np.random.default_rng(seed).choice(T, min(n_sample, T), replace=False))
    W = oracle.Weights(d)
    ref_logits = oracle.router_logits(W, x_np[sample])
    ref_idx, _ = oracle.topk_softmax(ref_logits, K)
    srt = -np.sort(-ref_logits, axis=1)
    near_tie = (srt[:, K - 1] - srt[:, K]) < 1e-4
    same = np.all(idx[sample] == ref_idx, axis=1)
    y_ref = oracle.moe_forward_spec(W, x_np[sample], idx=idx[sample], wts=w[sample], acc64=True, nthreads=cores)
    err = np.abs(y[sample] - y_ref)
    max_abs = float(err.max())
    mean_rel = float(err.sum() / max(np.abs(y_ref).sum(), 1e-30))
    return {"oracle_sample_tokens": int(sample.size), "oracle_max_abs": max_abs, "oracle_mean_rel": mean_rel,
            "routing_matches_oracle": bool(np.all(same | near_tie)),
            "logits_max_abs_diff": float(np.abs(logits[sample] - ref_logits).max()),
            "within_bar": bool(max_abs <= 2e-2 and mean_rel <= 1e-3 and np.all(same | near_tie))}


def gpu_layers(args, d0, device):
    """Layer 0 from the numpy generator; the rest from a seeded torch generator
    on the device (same shapes and distributions)."""
    import torch
    layers = [d0]
    H, I, E = d0["hidden"], d0["intermediate"], d0["n_experts"]
    for li in range(1, args.layers):
        g = torch.Generator(device=device)
        g.manual_seed(1000 + li)
        def u8(shape, lo, hi):
            return torch.randint(lo, hi + 1, shape, generator=g, device=device, dtype=torch.int32).to(torch.uint8)
        def bf16(shape, std):
            return (torch.randn(shape, generator=g, device=device) * std).to(torch.bfloat16).view(torch.int16)
        layers.append(dict(d0, router_w=bf16((E, H), 0.02), router_b=bf16((E,), 0.01),
                           w1_blocks=u8((E, 2 * I, H // 2), 0, 255), w1_scales=u8((E, 2 * I, H // 32), 118, 126),
                           b1=bf16((E, 2 * I), 0.01), w2_blocks=u8((E, H, I // 2), 0, 255),
                           w2_scales=u8((E, H, I // 32), 118, 126), b2=bf16((E, H), 0.01)))
    return layers


def run_moe(args, ws, rank, local):
    import torch
    from oxidized_gpt_oss_b200 import abi, synth
    from oxidized_gpt_oss_b200.moe import MoELayer
    from oxidized_gpt_oss_b200.mxfp4 import context

    device = torch.device("cuda", local)
    T = args.tokens
    d0 = synth.moe_layer(seed=0)
    H, I, E, K = d0["hidden"], d0["intermediate"], d0["n_experts"], d0["top_k"]
    ctx = context(None)
    layers = [MoELayer(d, ctx=ctx, layer=i) for i, d in enumerate(gpu_layers(args, d0, device))]
    for L in layers:
        L.reserve(T)
    n_x = 16
    xs_np = [synth.activations(1000 * rank + i, T, H) for i in range(n_x)]
    xs = [torch.from_numpy(x.view(np.int16)).to(device) for x in xs_np]
    ys = [torch.empty((T, H), dtype=torch.float32, device=device) for _ in range(2)]

    mode = {"auto": abi.OXG_MODE_AUTO, "mxf4": abi.OXG_MODE_MXF4, "f16": abi.OXG_MODE_DECODE}[args.path]

    def step(i):
        layers[i % len(layers)].forward(xs[i % n_x], out=ys[i % 2], mode=mode)

    # distinct experts each step reads (routing is deterministic per (layer, x))
    distinct = {}
    for i in range(args.steps):
        key = (i % len(layers), i % n_x)
        if key not in distinct:
            idx, _, _ = layers[key[0]].route(xs[key[1]])
            distinct[key] = int(torch.unique(idx).numel())
    hits = sum(distinct[(i % len(layers), i % n_x)] for i in range(args.steps))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    launches0 = ctx.launches()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(ws)
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier(ws)
    ms = ev0.elapsed_time(ev1)
    launches = ctx.launches() - launches0
    # Second pass over the same steps with per-kernel CUDA events recorded by
    # the library around each of its launches (events between kernels cost
    # the chained launches their overlap, so the headline above runs without).
    ctx.profile(True)
    ctx.profile_reset()
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    names = ("route_small", "router_topk", "router_mma", "permute", "scatter", "moe_mlp1_decode",
             "moe_mlp2_decode", "mxf_mlp1", "mxf_mlp2", "combine")
    k_ms = {n: ctx.profile_read(n) for n in names}
    k_ms = {n: v for n, v in k_ms.items() if v[1] > 0}
    ctx.profile(False)
    ms_max = max_over_ranks(ms, ws)

    # roofline of the dominant kernel (mlp1: gate/up projection + SwiGLU).
    # Algorithmic bytes: the hit experts' codes, scales and biases once, x
    # once, and the intermediate h once each way (f32 on the mma.sync path,
    # four E4M3 terms on the block-scaled path).
    mxf = "mxf_mlp1" in k_ms
    k1, k2 = ("mxf_mlp1", "mxf_mlp2") if mxf else ("moe_mlp1_decode", "moe_mlp2_decode")
    h_bytes = T * K * I * 4  # f32, or four E4M3 terms
    mlp1_w = 2 * I * H // 2 + 2 * I * H // 32 + 2 * I * 2
    mlp2_w = H * I // 2 + H * I // 32 + H * 2
    mlp1_bytes = hits * mlp1_w + args.steps * (T * H * 2 + h_bytes)
    mlp2_bytes = hits * mlp2_w + args.steps * (h_bytes + T * K * H * 4)
    layer_bytes = mlp1_bytes + mlp2_bytes + args.steps * (E * H * 2 + T * H * 4)
    hbm, hbm_kind = peaks()
    m1_ms, m1_n = k_ms[k1]
    m2_ms, m2_n = k_ms[k2]
    achieved = mlp1_bytes / (m1_ms * 1e-3) / 1e9
    traffic = ncu_traffic(k1, f"T{T}")

    # end to end through the host-buffer API: pinned x in, y out, every step
    xh = [torch.from_numpy(x.view(np.int16)).pin_memory() for x in xs_np]
    yh = torch.empty((T, H), dtype=torch.float32).pin_memory()
    for i in range(args.warmup):
        layers[i % len(layers)].forward_host(xh[i % n_x], yh, mode=mode)
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        layers[i % len(layers)].forward_host(xh[i % n_x], yh, mode=mode)
    e2e_ms = (time.perf_counter() - t0) * 1e3
    barrier(ws)
    e2e_ms = max_over_ranks(e2e_ms, ws)

    out = {"metric": METRIC, "value": T * ws * args.steps / (ms_max * 1e-3), "unit": "tokens/s",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": ("mxfp4 weights (E2M1 + E8M0 into tcgen05 block-scaled MMA) x bf16 activations as "
                     "E4M3 terms (2 for x, 4 for h), f32 accumulate") if mxf else
                    "mxfp4 weights x bf16 activations (exact f16 MMA operands), f32 accumulate",
           "data": "synthetic", "config": moe_config(args, d0),
           "roofline": {"bound": "hbm", "kernel": k1, "achieved": achieved, "peak": hbm,
                        "peak_kind": hbm_kind, "unit": "GB/s", "frac": achieved / hbm,
                        "traffic": traffic,
                        "algorithmic_bytes_per_launch": mlp1_bytes / max(m1_n, 1),
                        "avg_launch_us": m1_ms / max(m1_n, 1) * 1e3,
                        "distinct_experts_per_step": hits / args.steps},
           "layer": {"hbm_gbs": layer_bytes / (ms * 1e-3) / 1e9, "frac": layer_bytes / (ms * 1e-3) / 1e9 / hbm,
                     "kernel_us_per_step": {n: v[0] / max(v[1], 1) * 1e3 for n, v in k_ms.items()},
                     "mlp2_gbs": mlp2_bytes / (m2_ms * 1e-3) / 1e9},
           "e2e": {"value": T * ws * args.steps / (e2e_ms * 1e-3), "unit": "tokens/s",
                   "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 4},
           "gpu_launches": launches,
           "clocks": clk.summary()}
    if rank == 0 and ws == 1:
        out["cpu_baseline"] = cpu_baseline_moe(d0, xs_np[0])
        # parity of the measured configuration: layer 0 on batch 0 against the oracle
        y0 = layers[0].forward(xs[0], mode=mode)
        idx0, w0, lg0 = layers[0].route(xs[0])
        ctx.sync()
        out["parity"] = oracle_parity(d0, xs_np[0], y0.cpu().numpy(), idx0.cpu().numpy(), w0.cpu().numpy(),
                                      lg0.cpu().numpy(), n_sample=T, seed=T)
    return out


def run_prefill(args, ws, rank, local):
    """8192 tokens per GPU through one gpt-oss-20b MoE layer on the tcgen05
    grouped-GEMM path (router logits ~N(0, 1): x ~N(0, 1), W_router ~N(0, 0.02)).
    On N GPUs the 32 experts are split 32/N per GPU (expert parallel): every
    rank routes its own 8192 tokens and the rows travel by NCCL all-to-all."""
    import torch
    from oxidized_gpt_oss_b200 import abi, ep, synth
    from oxidized_gpt_oss_b200.moe import MoELayer
    from oxidized_gpt_oss_b200.mxfp4 import context

    device = torch.device("cuda", local)
    T = args.tokens
    d0 = synth.moe_layer(seed=0)
    H, I, E, K = d0["hidden"], d0["intermediate"], d0["n_experts"], d0["top_k"]
    ctx = context(None)
    shard = ep.shard_range(E, ws, rank) if ws > 1 else None
    layers = [MoELayer(d, ctx=ctx, layer=i, experts=shard) for i, d in enumerate(gpu_layers(args, d0, device))]
    for L in layers:
        L.reserve(T)
    p2p = None
    eps = None
    if ws > 1 and args.ep == "p2p":
        p2p = ep.PeerExpertParallelMoE(layers[0], max_tokens=T)
    elif ws > 1:
        eps = [ep.ExpertParallelMoE(L) for L in layers]
    n_x = 2
    xs_np = [synth.activations(1000 * rank + i, T, H) for i in range(n_x)]
    xs = [torch.from_numpy(x.view(np.int16)).to(device) for x in xs_np]
    y = torch.empty((T, H), dtype=torch.float32, device=device)
    mode = {"auto": abi.OXG_MODE_AUTO, "mxf4": abi.OXG_MODE_MXF4, "f16": abi.OXG_MODE_PREFILL}[args.path]
    rows_done = [0]  # expert rows this rank computed (varies with the routing under EP)

    count_rows = [False]  # in the profiled pass: ask each step how many rows it received

    def step(i, x=None):
        x = xs[i % n_x] if x is None else x
        if p2p is not None:
            out = p2p.forward(x, out=y, shard=layers[i % len(layers)])
            if count_rows[0]:
                rows_done[0] += p2p.last_received()
            return out
        if eps is None:
            rows_done[0] += T * K
            return layers[i % len(layers)].forward(x, out=y, mode=mode)
        m = eps[i % len(eps)]
        out = m.forward(x)
        rows_done[0] += sum(m.last_splits[1])
        return out

    for i in range(args.warmup):
        step(i)
    ctx.sync()
    torch.cuda.synchronize()
    launches0 = ctx.launches()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(ws)
        torch.cuda.synchronize()
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier(ws)
    ms = ev0.elapsed_time(ev1)
    launches = ctx.launches() - launches0
    ctx.sync()
    ctx.profile(True)
    ctx.profile_reset()
    rows_done[0] = 0
    count_rows[0] = True
    for i in range(args.steps):
        step(i)
    torch.cuda.synchronize()
    count_rows[0] = False
    rows_profiled = rows_done[0]
    names = ("router_topk", "router_mma", "permute", "gather_f16", "scatter_gather", "moe_mlp1_prefill",
             "moe_mlp2_prefill", "scatter_e4m3", "gather_e4m3", "mxf_gemm1", "mxf_gemm2", "combine",
             "ep_counts", "ep_scatter", "ep_signal", "ep_segments")
    k_ms = {n: ctx.profile_read(n) for n in names}
    k_ms = {n: v for n, v in k_ms.items() if v[1] > 0}
    mxf = "mxf_gemm1" in k_ms
    k1, k2 = ("mxf_gemm1", "mxf_gemm2") if mxf else ("moe_mlp1_prefill", "moe_mlp2_prefill")
    ctx.profile(False)
    ms_max = max_over_ranks(ms, ws)

    # algorithmic FLOPs per expert row: GEMM1 2 * 2I * H, GEMM2 2 * H * I
    # (the f16 hi/lo split executes GEMM2 twice); rows = T*k per step on one
    # GPU, the rows this rank received under EP
    f1_row, f2_row = 2.0 * (2 * I) * H, 2.0 * H * I
    rows_per_step = rows_profiled / args.steps
    flop1, flop2 = f1_row * rows_per_step, f2_row * rows_per_step
    peak, peak_kind = tensor_peak()
    rates = mma_rates(ctx) if ws == 1 else None
    m1_ms, m1_n = k_ms[k1]
    m2_ms, m2_n = k_ms[k2]
    achieved = f1_row * rows_profiled / (m1_ms * 1e-3) / 1e12
    layer_tflops = (flop1 + flop2) * args.steps / (ms * 1e-3) / 1e12

    # end to end: host x (pinned) in, host y (pinned) out, every step
    xh = [torch.from_numpy(x.view(np.int16)).pin_memory() for x in xs_np]
    yh = torch.empty((T, H), dtype=torch.float32).pin_memory()
    if ws == 1:
        def e2e_step(i):
            layers[i % len(layers)].forward_host(xh[i % n_x], yh, mode=mode)
    else:
        x_dev = torch.empty((T, H), dtype=torch.int16, device=device)

        def e2e_step(i):
            x_dev.copy_(xh[i % n_x], non_blocking=True)
            yh.copy_(step(i, x_dev), non_blocking=True)
            torch.cuda.current_stream().synchronize()
    for i in range(min(args.warmup, 2)):
        e2e_step(i)
    barrier(ws)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        e2e_step(i)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3, ws)

    out = {"metric": METRIC, "value": T * ws * args.steps / (ms_max * 1e-3), "unit": "tokens/s",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": ("mxfp4 weights (E2M1 + E8M0 into tcgen05 block-scaled MMA) x bf16 activations as E4M3 "
                     "terms (2 for x, 4 for h), f32 accumulate") if mxf else
                    "mxfp4 weights x bf16 activations (exact f16 tcgen05 operands), f32 accumulate",
           "data": "synthetic",
           "config": prefill_config(args, d0, ws),
           "roofline": {"bound": "tensor", "kernel": k1, "achieved": achieved, "peak": peak,
                        "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": achieved / peak,
                        "traffic": ncu_traffic(k1, f"T{T}") if ws == 1 else None,
                        "algorithmic_flop_per_launch": flop1,
                        "flop_per_unit": f1_row, "unit_of_work": "expert row (token, slot)",
                        "avg_launch_us": m1_ms / max(m1_n, 1) * 1e3,
                        # the dense MXFP4 tensor rate measured in this run (kind::mxf4, E2M1 x E2M1)
                        "mxfp4_peak": rates["mxf4"] if rates else None,
                        "frac_of_mxfp4_peak": achieved / rates["mxf4"] if rates else None},
           "e2e": {"value": T * ws * args.steps / (e2e_ms * 1e-3), "unit": "tokens/s",
                   "h2d_bytes_per_step": T * H * 2, "d2h_bytes_per_step": T * H * 4},
           "gpu_launches": launches,
           "clocks": clk.summary(),
           "layer": {"tflops": layer_tflops, "frac": layer_tflops / peak,
                     "kernel_us_per_step": {n: round(v[0] / max(v[1], 1) * 1e3, 1) for n, v in k_ms.items()},
                     "mlp2_tflops": flop2 * m2_n / (m2_ms * 1e-3) / 1e12,
                     "expert_rows_per_step_rank0": rows_per_step}}

    # parity of the measured configuration, outside the timed regions
    if ws > 1:
        # every rank: the expert-parallel output of its 8192 tokens against a
        # forward of the same tokens with every expert of the layer on this GPU
        full = MoELayer(d0, ctx=ctx, layer=args.layers)
        full.reserve(T)
        y_ep = step(0, xs[0]).clone()
        y_one = full.forward(xs[0], mode=mode)
        ctx.sync()
        eq = bool(torch.equal(y_ep, y_one))
        diff = float((y_ep - y_one).abs().max().item())
        import torch.distributed as dist
        t = torch.tensor([0.0 if eq else 1.0, diff], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out["parity"] = {"ep_bit_exact": bool(t[0].item() == 0.0), "ep_max_abs_diff": float(t[1].item()),
                         "ranks_checked": ws, "tokens_per_rank": T,
                         "against": "the same tokens through oxg_moe_forward with all 32 experts on one GPU"}
        full.release()
    if p2p is not None:
        p2p.close()
    if rank == 0 and ws == 1:
        out["cpu_baseline"] = cpu_baseline_moe(d0, xs_np[0])
        y0 = layers[0].forward(xs[0], out=y, mode=mode)
        idx0, w0, lg0 = layers[0].route(xs[0])
        ctx.sync()
        out["parity"] = oracle_parity(d0, xs_np[0], y0.cpu().numpy(), idx0.cpu().numpy(), w0.cpu().numpy(),
                                      lg0.cpu().numpy(), n_sample=32, seed=T)
    return out


def run_tensor_peak(args, ws, rank, local):
    """Issue rate of the tensor-core instruction kinds the MoE kernels use
    (and the dense MXFP4 one), measured on this GPU: the denominators of the
    prefill GEMMs' tensor roofline beside the cuBLAS bf16 figure."""
    import torch
    from oxidized_gpt_oss_b200 import abi
    ctx = abi.Context(local)
    for k in range(len(MMA_KINDS)):  # warm-up
        ctx.mma_rate(k, 4096)
    with ClockSampler(local) as clk:
        barrier(ws)
        rates = mma_rates(ctx, iters=max(65536, args.steps * 4096), repeats=max(args.warmup, 3))
        barrier(ws)
    peak, peak_kind = tensor_peak()
    out = {"metric": "tensor-core issue rate (dense, back to back from shared memory)",
           "value": rates["mxf4"], "unit": "TFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "e2m1 x e2m1 (mxf4)",
           "data": "none (zero tiles in shared memory)",
           "config": {"workload": "tensor_peak", "ctas": "one per SM", "tile": "M128 N256, one accumulator"},
           "kinds": {name: {"tflops": rates[name], "instruction": what} for name, what in MMA_KINDS},
           "bf16_cublas_tflops": {"value": peak, "kind": peak_kind},
           "clocks": clk.summary(), "gpu_launches": None}
    ctx.close()
    return out


def run_dequant(args, ws, rank, local):
    import torch
    from oxidized_gpt_oss_b200 import synth
    from oxidized_gpt_oss_b200.mxfp4 import context, dequantize_mxfp4
    device = torch.device("cuda", local)
    (w1, s1, r1, c1), (w2, s2, r2, c2) = synth.dequant_tensors(seed=rank)
    tens = [(torch.from_numpy(w).to(device), torch.from_numpy(s).to(device), r, c)
            for w, s, r, c in ((w1, s1, r1, c1), (w2, s2, r2, c2))]
    outs = [torch.empty(r * c, dtype=torch.int16, device=device) for _, _, r, c in tens]
    read_b = sum(w.numel() + s.numel() for w, s, _, _ in tens)
    write_b = sum(o.numel() * 2 for o in outs)
    ctx = context(None)

    def step():
        for (b, s, r, c), o in zip(tens, outs):
            dequantize_mxfp4(b, s, r, c, ctx=ctx, out=o)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.profile(True)
    ctx.profile_reset()
    launches0 = ctx.launches()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier(ws)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier(ws)
    ms = max_over_ranks(ev0.elapsed_time(ev1), ws)
    k_ms, k_n = ctx.profile_read("dequant_mxfp4")
    launches = ctx.launches() - launches0
    ctx.profile(False)
    hbm, hbm_kind = peaks()
    total = (read_b + write_b) * args.steps
    achieved = total / (k_ms * 1e-3) / 1e9
    # e2e: host codes+scales in, bf16 out, every step
    hb = [(w.cpu().pin_memory(), s.cpu().pin_memory()) for w, s, _, _ in tens]
    ho = [torch.empty_like(o, device="cpu").pin_memory() for o in outs]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for (b, s), (db, ds, r, c), o, h in zip(hb, tens, outs, ho):
            db.copy_(b, non_blocking=True)
            ds.copy_(s, non_blocking=True)
            dequantize_mxfp4(db, ds, r, c, ctx=ctx, out=o)
            h.copy_(o, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, ws)
    out = {"metric": METRIC, "value": total * ws / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": ws,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8->bf16",
           "data": "synthetic",
           "config": dequant_config(),
           "roofline": {"bound": "hbm", "kernel": "dequant_mxfp4", "achieved": achieved, "peak": hbm,
                        "peak_kind": hbm_kind, "unit": "GB/s", "frac": achieved / hbm,
                        "traffic": ncu_traffic("dequant_mxfp4", "layer"),
                        "avg_launch_us": k_ms / max(k_n, 1) * 1e3},
           "e2e": {"value": total * ws / e2e_s / 1e9, "unit": "GB/s", "h2d_bytes_per_step": read_b,
                   "d2h_bytes_per_step": write_b},
           "gpu_launches": launches, "clocks": clk.summary()}
    if rank == 0 and ws == 1:
        from oracle import oracle
        rows = 5760 * 2
        t0 = time.perf_counter()
        oracle.dequantize_mxfp4_e8m0(w1.reshape(-1, c1 // 2)[:rows], s1.reshape(-1, c1 // 32)[:rows], rows, c1)
        dt = time.perf_counter() - t0
        nb = rows * c1 // 2 + rows * c1 // 32 + rows * c1 * 2
        out["cpu_baseline"] = {"value": nb / dt / 1e9, "unit": "GB/s", "cores": oracle.max_threads(),
                               "kind": "port", "sample": f"{rows} rows of mlp1 ({nb} B algorithmic), OpenMP"}
    return out


MODEL_KERNELS = ("embed_norm", "linear_qkv", "qkv_rope", "attention", "linear_o", "residual_norm", "route_small",
                 "moe_mlp1_decode", "moe_mlp2_decode", "lm_head", "argmax")


def model_config(args, d, prompt):
    return {"workload": "gpt_oss_20b_decode", "layers": d["n_layers"], "hidden": d["hidden"],
            "heads": f"{d['n_heads']}q/{d['n_kv_heads']}kv x {d['head_dim']}", "vocab": d["vocab"],
            "sliding_window": d["sliding_window"], "experts": d["n_experts"], "top_k": d["top_k"],
            "batch": 1, "prompt_tokens": prompt, "decode_steps": args.steps,
            "weights": "random init: attention/embeddings bf16, experts mxfp4 e2m1 + e8m0[118,126]",
            "l2": "inputs larger than L2: every step streams ~3.7 GB of weights",
            "parallelism": "replicas" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "single"}


def model_batch_config(args, d):
    """The model_batch workload (configuration 4), shared by both arms."""
    cfg = model_config(args, d, args.prompt)
    cfg.update(workload="gpt_oss_20b_batched_decode", batch=args.batch, kv_length=args.prompt,
               router=f"bias -{ZIPF_S} ln(rank) per layer (seeded rank permutation): Zipf-like expert loads",
               l2="inputs larger than L2: every step streams the weights of all hit experts and every KV run")
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws > 1:
        cfg["parallelism"] = (f"ep{ws}: experts {d['n_experts']}/{ws} per GPU, {args.batch // ws} sequences per "
                              f"GPU; per layer and step the rows and output rows cross NVLink peer memory")
    return cfg


def run_model(args, ws, rank, local):
    """Greedy decode of the full 24-layer gpt-oss-20b architecture, batch 1:
    a prompt of ``--prompt`` tokens, then ``--steps`` timed one-token steps
    (each: embedding, 24 x (attention + MoE block), LM head, argmax fed back on
    the device)."""
    import torch
    from oxidized_gpt_oss_b200 import synth
    from oxidized_gpt_oss_b200.model import GPTModel

    device = torch.device("cuda", local)
    over = {} if args.model_layers is None else {"n_layers": args.model_layers}
    m = synth.model_weights_device(seed=rank, device=device, **over)
    d = m["dims"]
    P = args.prompt
    max_seq = P + args.warmup + args.steps + 8
    g = GPTModel(m, max_seq=max_seq, max_tokens=min(P, 2048))
    del m
    torch.cuda.empty_cache()
    ctx = g.ctx
    rng = np.random.default_rng(1234 + rank)
    prompt = rng.integers(0, d["vocab"], P).astype(np.int32)
    prompt_dev = torch.from_numpy(prompt).to(device)
    first = torch.zeros(1, dtype=torch.int32, device=device)
    toks = torch.zeros(args.steps, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record(stream)
    g.forward_device(prompt_dev, 1, None, first)
    ev[1].record(stream)
    warm = g.decode(args.warmup).clone() if args.warmup else torch.zeros(0, dtype=torch.int32, device=device)
    torch.cuda.synchronize()
    g.sync()
    prefill_ms = ev[0].elapsed_time(ev[1])
    launches0 = ctx.launches()
    with ClockSampler(local) as clk:
        barrier(ws)
        torch.cuda.synchronize()
        ev[2].record(stream)
        g.decode(args.steps, out=toks)  # one eager step, then replays of the captured step
        ev[3].record(stream)
        torch.cuda.synchronize()
        barrier(ws)
    g.sync()
    ms = ev[2].elapsed_time(ev[3])
    launches = ctx.launches() - launches0
    ms_max = max_over_ranks(ms, ws)
    seq = np.concatenate([first.cpu().numpy(), warm.cpu().numpy(), toks.cpu().numpy()])

    # per-kernel device time: eager steps (library CUDA events around each
    # launch), each queued behind a GPU sleep so no host gap enters a bracket
    w0 = args.warmup
    g.reset_kv_cache()
    g.forward_device(prompt_dev, 1, None, first)
    cur = first.clone()
    nxt = torch.zeros(1, dtype=torch.int32, device=device)
    torch.cuda.synchronize()
    ctx.profile(True)
    ctx.profile_reset()
    n_prof = 8
    for i in range(n_prof):
        torch.cuda._sleep(40_000_000)
        g.forward_device(cur, 1, None, nxt)
        cur.copy_(nxt)
        torch.cuda.synchronize()
    k_ms = {n: ctx.profile_read(n) for n in MODEL_KERNELS}
    k_ms = {n: v for n, v in k_ms.items() if v[1] > 0}
    ctx.profile(False)
    same = int(cur.item()) == int(seq[n_prof]) if n_prof < seq.size else None

    # algorithmic HBM bytes of one step (weights streamed once, KV read once)
    H, V, L = d["hidden"], d["vocab"], d["n_layers"]
    nh, nkv, hd, W = d["n_heads"], d["n_kv_heads"], d["head_dim"], d["sliding_window"]
    Nq, Nkv = nh * hd, nkv * hd
    qkv_b = (Nq + 2 * Nkv) * H * 2
    o_b = H * Nq * 2
    mlp1_w = 2 * d["intermediate"] * H // 2 + 2 * d["intermediate"] * H // 32 + 2 * d["intermediate"] * 2
    mlp2_w = H * d["intermediate"] // 2 + H * d["intermediate"] // 32 + H * 2
    head_b = V * H * 2 + V * 4
    pos_mid = P + w0 + args.steps / 2
    kv_b = sum(2 * nkv * hd * 2 * (min(W, pos_mid) if (li % 2 == 0 and W) else pos_mid) for li in range(L))
    per_kernel_bytes = {"linear_qkv": L * qkv_b, "linear_o": L * o_b, "moe_mlp1_decode": L * d["top_k"] * mlp1_w,
                        "moe_mlp2_decode": L * d["top_k"] * mlp2_w, "lm_head": head_b, "attention": kv_b}
    step_bytes = sum(per_kernel_bytes.values()) + L * d["n_experts"] * H * 2
    hbm, hbm_kind = peaks()
    kern = {}
    for n, (t, cnt) in k_ms.items():
        per_step_ms = t / n_prof
        e = {"us_per_step": per_step_ms * 1e3, "launches_per_step": cnt / n_prof}
        if n in per_kernel_bytes:
            e["gbs"] = per_kernel_bytes[n] / (per_step_ms * 1e-3) / 1e9
        kern[n] = e
    dom = max((n for n in kern if n in per_kernel_bytes), key=lambda n: kern[n]["us_per_step"])
    dom_ms, dom_n = k_ms[dom]
    achieved = per_kernel_bytes[dom] * n_prof / (dom_ms * 1e-3) / 1e9

    # end to end through oxg_model_generate: host prompt in, host tokens out
    n_new = w0 + args.steps + 1
    g.generate(prompt[: min(P, 64)], 2)  # warm the call path
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out_tokens = g.generate(prompt, n_new)
    e2e_s = time.perf_counter() - t0
    e2e_same = out_tokens == seq.tolist()

    out = {"metric": METRIC, "value": ws * args.steps / (ms_max * 1e-3), "unit": "tokens/s",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16 activations and attention weights, mxfp4 experts, f32 accumulate",
           "data": "synthetic", "config": model_config(args, d, P),
           "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "peak_kind": hbm_kind,
                        "unit": "GB/s", "frac": achieved / hbm, "traffic": ncu_traffic(dom, "T1"),
                        "algorithmic_bytes_per_launch": per_kernel_bytes[dom] / max(dom_n / n_prof, 1),
                        "avg_launch_us": dom_ms / max(dom_n, 1) * 1e3},
           "step": {"hbm_gbs": step_bytes / (ms / args.steps * 1e-3) / 1e9,
                    "frac": step_bytes / (ms / args.steps * 1e-3) / 1e9 / hbm, "bytes": step_bytes,
                    "kernels": kern, "prefill_ms": prefill_ms, "prefill_tokens": P,
                    "eager_steps_match_graph_steps": same, "generate_matches_device_loop": e2e_same,
                    "kernel_times": "eager steps queued behind a GPU sleep, library CUDA events per launch"},
           "e2e": {"value": n_new / e2e_s, "unit": "tokens/s",
                   "what": f"oxg_model_generate: {P}-token host prompt, {n_new} greedy tokens to the host "
                           f"(prompt prefill included)",
                   "h2d_bytes_per_step": P * 4 / n_new, "d2h_bytes_per_step": 4},
           "gpu_launches": launches,
           "clocks": clk.summary()}
    if rank == 0 and ws == 1:
        out["cpu_baseline"] = cpu_baseline_model(d)
    g.release()
    return out


ZIPF_S = 1.1
BATCH_KERNELS = MODEL_KERNELS + ("router_topk", "permute", "combine", "router_mma", "ep_counts",
                                  "ep_scatter", "ep_segments", "moe_ep_decode", "ep_signal")


def zipf_router(m, s, seed):
    """Skews each layer's expert loads: adds -s ln(rank) to the router bias,
    ranks 1..E a seeded permutation per layer, so with router logits of about
    unit spread the experts are picked with Zipf-like frequencies (rank^-s)."""
    import torch
    rng = np.random.default_rng(seed)
    for lw in m["layers"]:
        mw = lw["moe"]
        rb = mw["router_b"]
        E = rb.numel()
        rank = np.empty(E)
        rank[rng.permutation(E)] = np.arange(1, E + 1)
        zb = torch.tensor(-s * np.log(rank), dtype=torch.float32, device=rb.device)
        mw["router_b"] = (rb.view(torch.bfloat16).float() + zb).to(torch.bfloat16).view(torch.int16)


def run_model_batch(args, ws, rank, local):
    """Batched greedy decode over the full 24-layer gpt-oss-20b architecture:
    ``--batch`` sequences, each with its own KV cache filled by a random
    ``--prompt``-token prompt, then ``--steps`` timed steps that each advance
    every sequence by one token (oxg_model_step_batch: one batch through the
    projections, MoE blocks and LM head; attention per sequence). Router
    biases skewed Zipf-like (s = 1.1) so the expert loads are imbalanced."""
    import torch
    from oxidized_gpt_oss_b200 import synth
    from oxidized_gpt_oss_b200.model import GPTModel

    device = torch.device("cuda", local)
    over = {} if args.model_layers is None else {"n_layers": args.model_layers}
    # one model on every rank (expert parallel over N > 1 GPUs: the same weights)
    m = synth.model_weights_device(seed=0, device=device, **over)
    zipf_router(m, ZIPF_S, 77)
    d = m["dims"]
    B, P = args.batch, args.prompt
    if B % ws:
        raise SystemExit(f"--batch {B} must be a multiple of the GPU count {ws}")
    Br = B // ws  # this rank's sequences
    chunk = 2048
    n_prof, n_e2e, n_par = 4, max(4, min(args.steps, 16)), 4
    max_seq = P + args.warmup + args.steps + n_prof + n_e2e + n_par + 8
    from oxidized_gpt_oss_b200 import ep
    shard = ep.shard_range(d["n_experts"], ws, rank) if ws > 1 else None
    g = GPTModel(m, max_seq=max_seq, max_tokens=min(chunk, max_seq), max_batch=Br, experts=shard)
    if ws > 1:
        g.connect_expert_parallel()
        # every expert on this GPU too, for the parity check of the same
        # sequences; and a control: the first half of them as a batch of Br / 2
        g_full = GPTModel(m, max_seq=max_seq, max_tokens=min(chunk, max_seq), max_batch=Br)
        g_half = GPTModel(m, max_seq=max_seq, max_tokens=min(chunk, max_seq), max_batch=max(Br // 2, 1))
    del m
    torch.cuda.empty_cache()
    ctx = g.ctx
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    cur = torch.zeros(Br, dtype=torch.int32, device=device)

    def prompts():
        rng = np.random.default_rng(4321 + rank)
        return [torch.from_numpy(rng.integers(0, d["vocab"], P).astype(np.int32)).to(device) for _ in range(Br)]

    ev[0].record(stream)
    for sq, prompt in enumerate(prompts()):
        for c0 in range(0, P, chunk):
            nx = g.prefill_seq(sq, prompt[c0:c0 + chunk])
        cur[sq:sq + 1].copy_(nx)
    ev[1].record(stream)
    torch.cuda.synchronize()
    g.sync()
    prefill_ms = ev[0].elapsed_time(ev[1])
    parity = None
    if ws > 1:
        # expert-parallel steps against every expert on this GPU, same
        # sequences, teacher-forced with the expert-parallel tokens (outside
        # every timed region). The decode kernels' split of each expert's
        # weights depends on how many groups of slots share the GPU, so the
        # two runs round differently; a random-init 24-layer model amplifies
        # that (a router near-tie flips an expert, an attention weight moves),
        # which the control measures on one GPU: the first Br / 2 sequences
        # stepped as a batch of Br / 2 against the same sequences in the batch
        # of Br. Routing agreement counts (layer, token) expert sets.
        hb = max(Br // 2, 1)
        for sq, prompt in enumerate(prompts()):
            for c0 in range(0, P, chunk):
                g_full.prefill_seq(sq, prompt[c0:c0 + chunk])
                if sq < hb:
                    g_half.prefill_seq(sq, prompt[c0:c0 + chunk])
        lg_ep = torch.empty((Br, d["vocab"]), dtype=torch.float32, device=device)
        lg_full = torch.empty_like(lg_ep)
        lg_half = torch.empty((hb, d["vocab"]), dtype=torch.float32, device=device)
        tap_ep, tap_full, tap_half = g.route_tap(Br), g_full.route_tap(Br), g_half.route_tap(hb)
        diff, same, diff_c, same_c, r_same, r_same_c, first = 0.0, 0, 0.0, 0, 0, 0, []
        for _ in range(n_par):
            nx_ep = g.step_batch(cur, logits=lg_ep)
            nx_full = g_full.step_batch(cur, logits=lg_full)
            nx_half = g_half.step_batch(cur[:hb], logits=lg_half)
            torch.cuda.synchronize()
            g.sync()
            d_step = (lg_ep - lg_full).abs().max(dim=1).values
            first.append(float(d_step.max().item()))
            diff = max(diff, first[-1])
            same += int((nx_ep == nx_full).sum().item())
            diff_c = max(diff_c, float((lg_full[:hb] - lg_half).abs().max().item()))
            same_c += int((nx_full[:hb] == nx_half).sum().item())
            sf = torch.sort(tap_full, dim=2).values
            r_same += int((torch.sort(tap_ep, dim=2).values == sf).all(dim=2).sum().item())
            r_same_c += int((torch.sort(tap_half, dim=2).values == sf[:, :hb]).all(dim=2).sum().item())
            cur = nx_ep
        for gm in (g, g_full, g_half):
            gm.route_tap(None)
        import torch.distributed as dist
        L_ = d["n_layers"]
        t = torch.tensor([diff, -same / (n_par * Br), diff_c, -same_c / (n_par * hb), -r_same / (n_par * Br * L_),
                          -r_same_c / (n_par * hb * L_), first[0]], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        v = t.tolist()
        for gm in (g_full, g_half):
            gm.release()
        del g_full, g_half
        torch.cuda.empty_cache()
        parity = {"steps_checked": n_par, "sequences_per_rank": Br,
                  "against": "the same sequences with every expert on one GPU, teacher-forced",
                  "max_logit_abs_diff": v[0], "first_step_max_logit_abs_diff": v[6],
                  "greedy_tokens_agree_min_over_ranks": -v[1], "routing_sets_agree_min_over_ranks": -v[4],
                  "control_one_gpu_batch_half_vs_full": {"max_logit_abs_diff": v[2],
                                                         "greedy_tokens_agree_min_over_ranks": -v[3],
                                                         "routing_sets_agree_min_over_ranks": -v[5]},
                  "moe_block": "tests/test_ep_gpu.py checks the expert-parallel decode block against the oracle"}
    for _ in range(args.warmup):
        cur = g.step_batch(cur)
    torch.cuda.synchronize()
    g.sync()
    launches0 = ctx.launches()
    with ClockSampler(local) as clk:
        barrier(ws)
        torch.cuda.synchronize()
        ev[2].record(stream)
        for _ in range(args.steps):
            cur = g.step_batch(cur)
        ev[3].record(stream)
        torch.cuda.synchronize()
        barrier(ws)
    g.sync()
    ms = ev[2].elapsed_time(ev[3])
    launches = ctx.launches() - launches0
    ms_max = max_over_ranks(ms, ws)

    # per-kernel device time: steps queued behind a GPU sleep, library CUDA
    # events per launch; the routing of the last one gives the experts hit
    tap = g.route_tap(Br)
    ctx.profile(True)
    ctx.profile_reset()
    for _ in range(n_prof):
        torch.cuda._sleep(40_000_000)
        cur = g.step_batch(cur)
        torch.cuda.synchronize()
    k_ms = {n: ctx.profile_read(n) for n in BATCH_KERNELS}
    k_ms = {n: v for n, v in k_ms.items() if v[1] > 0}
    ctx.profile(False)
    if ws > 1:  # every rank's routing: the experts hit anywhere, and on this GPU
        import torch.distributed as dist
        allr = [torch.empty_like(tap) for _ in range(ws)]
        dist.all_gather(allr, tap.contiguous())
        routes = torch.cat([a.reshape(a.shape[0], -1) for a in allr], dim=1).cpu().numpy()  # [L, B * k]
    else:
        routes = tap.cpu().numpy().reshape(tap.shape[0], -1)
    g.route_tap(None)
    L, E = d["n_layers"], d["n_experts"]
    loads = np.stack([np.bincount(routes[li], minlength=E) for li in range(L)])
    hit = (loads > 0).sum(axis=1)
    e0, ne = shard if shard is not None else (0, E)
    hit_here = (loads[:, e0:e0 + ne] > 0).sum(axis=1)  # experts this GPU streams per layer

    H, V = d["hidden"], d["vocab"]
    nh, nkv, hd, W = d["n_heads"], d["n_kv_heads"], d["head_dim"], d["sliding_window"]
    Nq, Nkv = nh * hd, nkv * hd
    qkv_b = (Nq + 2 * Nkv) * H * 2
    o_b = H * Nq * 2
    mlp1_w = 2 * d["intermediate"] * H // 2 + 2 * d["intermediate"] * H // 32 + 2 * d["intermediate"] * 2
    mlp2_w = H * d["intermediate"] // 2 + H * d["intermediate"] // 32 + H * 2
    head_b = V * H * 2 + Br * V * 4
    pos_mid = P + n_par + args.warmup + args.steps / 2
    kv_b = Br * sum(2 * nkv * hd * 2 * (min(W, pos_mid) if (li % 2 == 0 and W) else pos_mid) for li in range(L))
    per_kernel_bytes = {"linear_qkv": L * qkv_b, "linear_o": L * o_b, "lm_head": head_b, "attention": kv_b}
    if ws > 1:
        per_kernel_bytes["moe_ep_decode"] = int(hit_here.sum()) * (mlp1_w + mlp2_w)
    else:
        per_kernel_bytes["moe_mlp1_decode"] = int(hit.sum()) * mlp1_w
        per_kernel_bytes["moe_mlp2_decode"] = int(hit.sum()) * mlp2_w
    step_bytes = sum(per_kernel_bytes.values()) + L * E * H * 2
    hbm, hbm_kind = peaks()
    kern = {}
    for n, (t, cnt) in k_ms.items():
        per_step_ms = t / n_prof
        e = {"us_per_step": per_step_ms * 1e3, "launches_per_step": cnt / n_prof}
        if n in per_kernel_bytes:
            e["gbs"] = per_kernel_bytes[n] / (per_step_ms * 1e-3) / 1e9
        kern[n] = e
    dom = max((n for n in kern if n in per_kernel_bytes), key=lambda n: kern[n]["us_per_step"])
    dom_ms, dom_n = k_ms[dom]
    achieved = per_kernel_bytes[dom] * n_prof / (dom_ms * 1e-3) / 1e9

    # end to end through the public API: each step's tokens from pinned host
    # memory, the greedy tokens back to pinned host memory
    host_tok = torch.empty(Br, dtype=torch.int32, pin_memory=True)
    host_tok.copy_(cur)
    torch.cuda.synchronize()
    barrier(ws)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        nx = g.step_batch(host_tok.to(device, non_blocking=True))
        host_tok.copy_(nx)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, ws)

    cfg = model_batch_config(args, d)
    out = {"metric": METRIC, "value": ws * Br * args.steps / (ms_max * 1e-3), "unit": "tokens/s",
           "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "bf16 activations and attention weights, mxfp4 experts, f32 accumulate",
           "data": "synthetic", "config": cfg,
           "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "peak_kind": hbm_kind,
                        "unit": "GB/s", "frac": achieved / hbm, "traffic": None,
                        "algorithmic_bytes_per_launch": per_kernel_bytes[dom] / max(dom_n / n_prof, 1),
                        "avg_launch_us": dom_ms / max(dom_n, 1) * 1e3},
           "step": {"hbm_gbs": step_bytes / (ms / args.steps * 1e-3) / 1e9,
                    "frac": step_bytes / (ms / args.steps * 1e-3) / 1e9 / hbm, "bytes": step_bytes,
                    "kernels": kern, "prefill_ms": prefill_ms, "prefill_tokens": Br * P,
                    "experts_hit_per_layer": float(hit.mean()),
                    "experts_streamed_per_layer_this_gpu": float(hit_here.mean()),
                    "max_expert_load_over_mean": float((loads.max(axis=1) / loads.mean(axis=1)).mean()),
                    "kernel_times": "steps queued behind a GPU sleep, library CUDA events per launch"},
           "e2e": {"value": ws * Br * n_e2e / e2e_s, "unit": "tokens/s",
                   "what": f"oxg_model_step_batch x {n_e2e}: {Br} tokens per GPU from pinned host memory in, "
                           f"{Br} greedy tokens to pinned host memory out per step",
                   "h2d_bytes_per_step": Br * 4, "d2h_bytes_per_step": Br * 4},
           "gpu_launches": launches,
           "clocks": clk.summary()}
    if parity is not None:
        out["parity"] = parity
    if ws > 1:
        g.close_expert_parallel()
    if rank == 0 and ws == 1:
        cb = cpu_baseline_model(d)
        cb["sample"] += "; the reference decodes one sequence at a time, so its rate does not grow with the batch"
        out["cpu_baseline"] = cb
    g.release()
    return out


def cpu_baseline_model(d):
    """The reference's algorithm for one decode token through one MoE block
    (REF-FAITHFUL oracle, single thread), scaled to the model's layers;
    attention and the LM head are left out, so this bounds the reference's
    CPU decode rate from above."""
    from oxidized_gpt_oss_b200 import synth
    d0 = synth.moe_layer(seed=0)
    x = synth.activations(0, 1, d0["hidden"])
    cores, _ = host_cpu()
    b = cpu_baseline_moe(d0, synth.activations(0, cores, d0["hidden"]))
    n = d["n_layers"]
    return {"value": b["value"] / n, "unit": "tokens/s", "cores": 1, "kind": "port",
            "sample": f"one token through one MoE block (the reference's algorithm, single thread, "
                      f"{1.0 / b['value']:.2f} s) x {n} layers; attention and LM head not counted",
            "all_cores": {"value": b["all_cores"]["value"] / n, "cores": b["all_cores"]["cores"],
                          "sample": "one sequence per core, each as above"},
            "cpu_model": b["cpu_model"]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["moe_decode", "moe_prefill", "dequant", "model_decode", "model_batch",
                                           "tensor_peak"],
                    default="moe_prefill")
    ap.add_argument("--prompt", type=int, default=None,
                    help="model_decode: prompt tokens (default 2048); model_batch: KV length per sequence (8192)")
    ap.add_argument("--batch", type=int, default=64, help="model_batch: concurrent sequences")
    ap.add_argument("--model-layers", type=int, default=None, help="model_decode: layers (default 24)")
    ap.add_argument("--no-decode", action="store_true",
                    help="moe_prefill on one GPU: skip the decode measurement added to the line")
    ap.add_argument("--no-model", action="store_true",
                    help="moe_prefill on one GPU: skip the 24-layer decoder measurement added to the line")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per GPU (default 8 for moe_decode, 8192 for moe_prefill)")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--path", choices=["auto", "mxf4", "f16"], default="auto",
                    help="expert kernels on one GPU: the library's choice, the block-scaled tcgen05 kernels "
                         "(E2M1 straight into the tensor cores), or the f16-operand kernels (tcgen05 GEMMs for "
                         "prefill, mma.sync for decode)")
    ap.add_argument("--ep", choices=["p2p", "nccl"], default="p2p",
                    help="moe_prefill on N > 1 GPUs: exchange over peer memory in the library's kernels "
                         "(default) or by NCCL all-to-all")
    args = ap.parse_args()
    if args.tokens is None:
        args.tokens = 8192 if args.workload == "moe_prefill" else 8
    if args.prompt is None:
        args.prompt = 8192 if args.workload == "model_batch" else 2048
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        run = {"dequant": run_dequant, "moe_prefill": run_prefill, "moe_decode": run_moe,
               "model_decode": run_model, "model_batch": run_model_batch,
               "tensor_peak": run_tensor_peak}[args.workload]
        out = run(args, ws, rank, local)
        def brief(r):
            # the figures a reader of the line needs, kept short so that the
            # end of the line (decode last) survives a truncated log tail
            rf = r.get("roofline", {})
            b = {"value": r["value"], "unit": r["unit"], "ms_per_step": r["ms_per_step"], "steps": r["steps"],
                 "roofline": {k: rf.get(k) for k in ("kernel", "achieved", "peak", "unit", "frac", "traffic",
                                                      "avg_launch_us", "algorithmic_bytes_per_launch")},
                 "e2e": r.get("e2e"), "gpu_launches": r.get("gpu_launches")}
            for k in ("parity", "cpu_baseline"):
                if k in r:
                    b[k] = r[k]
            return b

        if args.workload == "moe_prefill" and ws == 1 and not args.no_model:
            # configuration 2: the full 24-layer decoder, batch 1, greedy decode
            margs = argparse.Namespace(**vars(args))
            margs.steps, margs.warmup = 64, 4
            md = run_model(margs, ws, rank, local)
            out["model_decode"] = brief(md)
            st = md.get("step", {})
            out["model_decode"]["step"] = {k: st.get(k) for k in ("hbm_gbs", "frac", "eager_steps_match_graph_steps",
                                                                  "generate_matches_device_loop")}
            out["model_decode"]["kernel_us_per_step"] = {n: round(v["us_per_step"], 1)
                                                         for n, v in st.get("kernels", {}).items()}
        if args.workload == "moe_prefill" and ws == 1 and not args.no_decode:
            # the metric's decode half (tokens/s and HBM GB/s at 8 tokens), same process; last in the line
            dargs = argparse.Namespace(**vars(args))
            dargs.tokens, dargs.steps, dargs.warmup = 8, max(args.steps, 20), max(args.warmup, 5)
            dec = run_moe(dargs, ws, rank, local)
            out["decode"] = brief(dec)
            out["decode"]["layer_frac"] = dec["layer"]["frac"]
            out["decode"]["kernel_us_per_step"] = {n: round(v, 1) for n, v in dec["layer"]["kernel_us_per_step"].items()}
        if rank == 0:
            emit(out)
    finally:
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
