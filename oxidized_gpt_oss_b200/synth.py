"""Seeded synthetic MoE-layer inputs (random-init gpt-oss-20b-shaped weights).

No checkpoints or datasets are used anywhere: every workload is generated here
from a seed with the distributions the benchmark configurations name.

* ``moe_layer(seed, ...)`` — one MoE block: router Linear H->E (bf16 weights
  ~N(0, 0.02), bias ~N(0, 0.01)), E experts with mlp1 [2I, H] (gate/up rows
  interleaved: even rows gate, odd rows up) and mlp2 [H, I] in MXFP4 (packed
  E2M1 codes uniform over all 16 codes, one E8M0 scale per 32-element block
  uniform in ``scale_range``), bf16 biases ~N(0, 0.01).
* ``activations(seed, T, H)`` — bf16 ~N(0, 1) hidden states [T, H].
* ``dequant_tensors(seed, ...)`` — the standalone dequant workload.

bf16 values are returned as uint16 bit patterns (round-to-nearest-even).
"""
from __future__ import annotations

import numpy as np

GPT_OSS_20B = dict(hidden=2880, intermediate=2880, n_experts=32, top_k=4, alpha=1.702, limit=7.0)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _normal_bf16(rng: np.random.Generator, shape, std: float) -> np.ndarray:
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))


def moe_layer(seed: int = 0, hidden: int = 2880, intermediate: int = 2880, n_experts: int = 32,
              top_k: int = 4, alpha: float = 1.702, limit: float = 7.0,
              scale_range=(118, 126), router_bias: bool = True) -> dict:
    if hidden % 32 or intermediate % 32:
        raise ValueError("hidden and intermediate must be multiples of the 32-element block")
    rng = np.random.default_rng(seed)
    H, I, E = hidden, intermediate, n_experts
    lo, hi = scale_range
    d = dict(hidden=H, intermediate=I, n_experts=E, top_k=top_k, alpha=alpha, limit=limit)
    d["router_w"] = _normal_bf16(rng, (E, H), 0.02)
    d["router_b"] = _normal_bf16(rng, (E,), 0.01) if router_bias else None
    d["w1_blocks"] = rng.integers(0, 256, size=(E, 2 * I, H // 2), dtype=np.uint8)
    d["w1_scales"] = rng.integers(lo, hi + 1, size=(E, 2 * I, H // 32), dtype=np.uint8)
    d["b1"] = _normal_bf16(rng, (E, 2 * I), 0.01)
    d["w2_blocks"] = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    d["w2_scales"] = rng.integers(lo, hi + 1, size=(E, H, I // 32), dtype=np.uint8)
    d["b2"] = _normal_bf16(rng, (E, H), 0.01)
    return d


def activations(seed: int, T: int, H: int) -> np.ndarray:
    rng = np.random.default_rng(seed + 0x5EED)
    return _normal_bf16(rng, (T, H), 1.0)


def dequant_tensors(seed: int = 0, n_experts: int = 32, hidden: int = 2880, intermediate: int = 2880,
                    scale_range=(110, 135)):
    """The standalone dequant workload: one layer's mlp1 [E, 2I, H] and mlp2 [E, H, I]."""
    rng = np.random.default_rng(seed)
    lo, hi = scale_range
    E, H, I = n_experts, hidden, intermediate
    w1 = rng.integers(0, 256, size=(E, 2 * I, H // 2), dtype=np.uint8)
    s1 = rng.integers(lo, hi + 1, size=(E, 2 * I, H // 32), dtype=np.uint8)
    w2 = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    s2 = rng.integers(lo, hi + 1, size=(E, H, I // 32), dtype=np.uint8)
    return (w1, s1, E * 2 * I, H), (w2, s2, E * H, I)


def moe_bytes_per_expert(hidden: int = 2880, intermediate: int = 2880) -> int:
    """Algorithmic HBM bytes one expert's weights cost a decode step."""
    H, I = hidden, intermediate
    return (2 * I * H // 2 + 2 * I * H // 32 + H * I // 2 + H * I // 32) + (2 * I + H) * 2


# ---------------------------------------------------------------------------
# Full decoder (gpt-oss-20b architecture, random init)
# ---------------------------------------------------------------------------
GPT_OSS_20B_MODEL = dict(n_layers=24, hidden=2880, n_heads=64, n_kv_heads=8, head_dim=64, vocab=201088,
                         sliding_window=128, rope_theta=150000.0, rms_eps=1e-5, intermediate=2880,
                         n_experts=32, top_k=4, alpha=1.702, limit=7.0)

_ATTN_KEYS = ("attn_norm", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "bo", "sinks", "mlp_norm")


def model_weights(seed: int = 0, **over) -> dict:
    """Random-init weights of a gpt-oss-architecture decoder (numpy, host).

    Distributions: embedding bf16 ~N(0, 1); LM head ~N(0, 0.02); RMS-norm
    weights 1 + N(0, 0.02); q/k/v/o weights ~N(0, 0.02), biases ~N(0, 0.01);
    sink logits ~N(0, 1); each layer's MoE block as ``moe_layer`` (seed
    seed * 1000 + 1 + layer). ``over`` overrides fields of
    ``GPT_OSS_20B_MODEL`` (e.g. fewer layers or a smaller vocab for tests).
    """
    d = dict(GPT_OSS_20B_MODEL)
    d.update(over)
    rng = np.random.default_rng(seed)
    H, V, nh, nkv, hd = d["hidden"], d["vocab"], d["n_heads"], d["n_kv_heads"], d["head_dim"]
    m = dict(dims=d)
    m["embed"] = _normal_bf16(rng, (V, H), 1.0)
    m["unembed"] = _normal_bf16(rng, (V, H), 0.02)
    m["final_norm"] = f32_to_bf16_bits(1.0 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.02))
    layers = []
    for layer in range(d["n_layers"]):
        a = {}
        a["attn_norm"] = f32_to_bf16_bits(1.0 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.02))
        a["wq"] = _normal_bf16(rng, (nh * hd, H), 0.02)
        a["wk"] = _normal_bf16(rng, (nkv * hd, H), 0.02)
        a["wv"] = _normal_bf16(rng, (nkv * hd, H), 0.02)
        a["bq"] = _normal_bf16(rng, (nh * hd,), 0.01)
        a["bk"] = _normal_bf16(rng, (nkv * hd,), 0.01)
        a["bv"] = _normal_bf16(rng, (nkv * hd,), 0.01)
        a["wo"] = _normal_bf16(rng, (H, nh * hd), 0.02)
        a["bo"] = _normal_bf16(rng, (H,), 0.01)
        a["sinks"] = _normal_bf16(rng, (nh,), 1.0)
        a["mlp_norm"] = f32_to_bf16_bits(1.0 + rng.standard_normal(H, dtype=np.float32) * np.float32(0.02))
        a["moe"] = moe_layer(seed * 1000 + 1 + layer, hidden=H, intermediate=d["intermediate"],
                             n_experts=d["n_experts"], top_k=d["top_k"], alpha=d["alpha"], limit=d["limit"])
        layers.append(a)
    m["layers"] = layers
    return m


def model_weights_device(seed: int = 0, device="cuda", **over) -> dict:
    """The same architecture and distributions as ``model_weights``, drawn on
    the GPU with torch's generator (a different stream of random numbers) —
    for full-size benchmarks, where drawing ~13 GB on the host would dominate
    the set-up time. bf16 tensors are returned as int16 bit patterns."""
    import torch

    d = dict(GPT_OSS_20B_MODEL)
    d.update(over)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, V, nh, nkv, hd = d["hidden"], d["vocab"], d["n_heads"], d["n_kv_heads"], d["head_dim"]
    I, E = d["intermediate"], d["n_experts"]

    def normal(shape, std, mean=0.0):
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std + mean
        return t.to(torch.bfloat16).view(torch.int16)

    def codes(shape):
        return torch.randint(0, 256, shape, generator=g, device=device, dtype=torch.int32).to(torch.uint8)

    def scales(shape, lo=118, hi=126):
        return torch.randint(lo, hi + 1, shape, generator=g, device=device, dtype=torch.int32).to(torch.uint8)

    m = dict(dims=d)
    m["embed"] = normal((V, H), 1.0)
    m["unembed"] = normal((V, H), 0.02)
    m["final_norm"] = normal((H,), 0.02, 1.0)
    layers = []
    for _ in range(d["n_layers"]):
        a = dict(attn_norm=normal((H,), 0.02, 1.0), wq=normal((nh * hd, H), 0.02), wk=normal((nkv * hd, H), 0.02),
                 wv=normal((nkv * hd, H), 0.02), bq=normal((nh * hd,), 0.01), bk=normal((nkv * hd,), 0.01),
                 bv=normal((nkv * hd,), 0.01), wo=normal((H, nh * hd), 0.02), bo=normal((H,), 0.01),
                 sinks=normal((nh,), 1.0), mlp_norm=normal((H,), 0.02, 1.0))
        a["moe"] = dict(hidden=H, intermediate=I, n_experts=E, top_k=d["top_k"], alpha=d["alpha"], limit=d["limit"],
                        router_w=normal((E, H), 0.02), router_b=normal((E,), 0.01),
                        w1_blocks=codes((E, 2 * I, H // 2)), w1_scales=scales((E, 2 * I, H // 32)),
                        b1=normal((E, 2 * I), 0.01), w2_blocks=codes((E, H, I // 2)),
                        w2_scales=scales((E, H, I // 32)), b2=normal((E, H), 0.01))
        layers.append(a)
    m["layers"] = layers
    return m
