"""CPU restatement of the full gpt-oss-architecture decoder (float64 numpy).

TEST INFRASTRUCTURE ONLY: this module is the checker of the library's
oxg_model_* path. Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU
legs may import it.

Reference files followed (cipher-rc5/oxidized_gpt_oss):
  * GPTModel::forward: src/model.rs:713-741 (embed -> layers -> final norm ->
    LM head of the last token, :800-844)
  * TransformerLayer::forward: src/model.rs:848-887 (norm, attention,
    residual, norm, MoE, residual)
  * RMS norm: src/backend/metal_stub.rs:109-157 (x * 1/sqrt(mean(x^2) + eps)
    * gamma + beta; beta is zero for gpt-oss)
  * Attention::forward: src/model.rs:899-1084 (q/k/v projections + bias,
    GQA head -> kv head = head / (nh / nkv), keys max(0, t+1-window) .. t,
    scale 1/sqrt(head_dim), softmax, o projection + bias)
  * greedy choice: src/sampler.rs:7-16 (ties to the last maximal index)
  * MoE block: oracle.np_moe_forward (src/moe.rs:16-100 with the SPEC rules)
Where the reference is incomplete, gpt-oss's definitions apply (the reference
applies no RoPE and has no sinks): RoPE on the two halves of every head with
angle pos * theta^(-2i/64) (cos/sin evaluated in float64 and rounded to f32,
the tables the library builds), and one sink logit per head that joins the
softmax denominator only. Activations are rounded to bf16 where the library's
operands are bf16: the normed inputs of every matrix product, q/k/v after
RoPE (the KV cache) and the attention output.
"""
from __future__ import annotations

import numpy as np

from . import oracle as _o

bf16 = _o.np_bf16_to_f32


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float -> nearest bf16 (ties to even, via f32) -> float64."""
    return bf16(_o.np_f32_to_bf16(np.asarray(x, dtype=np.float32))).astype(np.float64)


def rope_tables(max_seq: int, theta: float, head_dim: int = 64):
    i = np.arange(head_dim // 2, dtype=np.float64)
    inv = np.power(float(np.float32(theta)), -2.0 * i / head_dim)
    ang = np.arange(max_seq, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32).astype(np.float64), np.sin(ang).astype(np.float32).astype(np.float64)


def rms_norm(x: np.ndarray, gamma_bf16: np.ndarray, eps: float) -> np.ndarray:
    """bf16(x / sqrt(mean(x^2) + eps) * gamma) for rows of x (float64)."""
    x32 = np.asarray(x, dtype=np.float32).astype(np.float64)
    ms = np.mean(x32 * x32, axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(ms + float(np.float32(eps)))
    return round_bf16(x32 * inv * bf16(gamma_bf16).astype(np.float64))


def apply_rope(x: np.ndarray, pos: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x [T, heads, 64]; rotates (x[:32], x[32:]) by the position's angles."""
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    x1, x2 = x[..., :32], x[..., 32:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, qpos: np.ndarray, window: int,
              sinks: np.ndarray | None, scale: float) -> np.ndarray:
    """q [T, nh, 64] at positions qpos; k, v [P, nkv, 64] for positions 0..P-1.
    Returns [T, nh, 64]: per query, keys max(0, p+1-window) .. p (all keys <= p
    when window == 0), softmax over the scores and the head's sink."""
    T, nh, _ = q.shape
    P, nkv, _ = k.shape
    G = nh // nkv
    out = np.zeros_like(q)
    keys = np.arange(P)
    for h in range(nh):
        kv = h // G
        s = (q[:, h, :] @ k[:, kv, :].T) * scale  # [T, P]
        mask = keys[None, :] <= qpos[:, None]
        if window > 0:
            mask &= keys[None, :] > (qpos[:, None] - window)
        s = np.where(mask, s, -np.inf)
        m = s.max(axis=1, keepdims=True)
        if sinks is not None:
            m = np.maximum(m, sinks[h])
        p = np.exp(s - m)
        den = p.sum(axis=1, keepdims=True)
        if sinks is not None:
            den = den + np.exp(sinks[h] - m)
        out[:, h, :] = (p @ v[:, kv, :]) / den
    return out


def reference_attention_loop(q: np.ndarray, k: np.ndarray, v: np.ndarray, window: int | None,
                             head_dim: int) -> np.ndarray:
    """The reference's per-head loop as written (src/model.rs:1022-1057), for
    a prefill of T tokens from position 0: q [T, nh*hd], k/v [T, nkv*hd]
    float arrays, returns the context [T, nh*hd]. Pure Python loops: small
    cases only."""
    T = q.shape[0]
    nh = q.shape[1] // head_dim
    nkv = k.shape[1] // head_dim
    groups = nh // nkv
    scale = np.float32(1.0) / np.sqrt(np.float32(head_dim))
    ctx = np.zeros((T, nh * head_dim), dtype=np.float32)
    for head in range(nh):
        kvh = head // groups
        for target in range(T):
            qs = q[target, head * head_dim:(head + 1) * head_dim].astype(np.float32)
            start = max(target + 1 - window, 0) if window else 0
            scores = []
            for source in range(start, target + 1):
                ks = k[source, kvh * head_dim:(kvh + 1) * head_dim].astype(np.float32)
                dot = np.float32(0.0)
                for i in range(head_dim):
                    dot = np.float32(dot + qs[i] * ks[i])
                scores.append(np.float32(dot * scale))
            sc = np.array(scores, dtype=np.float32)
            mx = sc.max()
            ex = np.exp(sc - mx).astype(np.float32)
            tot = ex.sum(dtype=np.float32)
            w = ex / tot if tot > 0 else np.full_like(ex, 1.0 / len(ex))
            o = np.zeros(head_dim, dtype=np.float32)
            for j, source in enumerate(range(start, target + 1)):
                vs = v[source, kvh * head_dim:(kvh + 1) * head_dim].astype(np.float32)
                o = (o + w[j] * vs).astype(np.float32)
            ctx[target, head * head_dim:(head + 1) * head_dim] = o
    return ctx


def routing_excess(route_logits: np.ndarray, idx: np.ndarray) -> np.ndarray:
    """Per token: how far the chosen experts ``idx`` [T, k] fall short of the
    top-k of ``route_logits`` [T, E] — the largest logit left out minus the
    smallest chosen (0 when idx is a top-k set)."""
    rl = np.asarray(route_logits)
    chosen = np.take_along_axis(rl, np.asarray(idx, dtype=np.int64), axis=1)
    mask = np.zeros(rl.shape, bool)
    np.put_along_axis(mask, np.asarray(idx, dtype=np.int64), True, axis=1)
    left = np.where(mask, -np.inf, rl).max(axis=1)
    return np.maximum(left - chosen.min(axis=1), 0.0)


def greedy(logits: np.ndarray) -> np.ndarray:
    """Argmax per row, ties to the last maximal index (src/sampler.rs:7-16)."""
    lg = np.asarray(logits)
    V = lg.shape[-1]
    return (V - 1 - np.argmax(lg[..., ::-1], axis=-1)).astype(np.int64)


def forward(m: dict, tokens, n_logits: int = 1, return_hidden: bool = False, route_gaps: list | None = None,
            routes=None, route_logits: list | None = None):
    """Full forward of ``tokens`` from position 0 -> float64 logits of the
    last ``n_logits`` tokens [n_logits, V] (and the final residual stream).
    ``route_gaps``, when a list, receives per layer the gap between each
    token's k-th and (k+1)-th router logits (a tie that rounding differences
    in the bf16 activations can decide either way). ``routes``, when given,
    holds per layer the expert ids [T, k] to use instead of the oracle's own
    top-k (the routing the library chose, from its routing tap); their
    weights are the softmax of the oracle's router logits at those ids.
    ``route_logits``, when a list, receives per layer the router logits [T, E]."""
    d = m["dims"]
    toks = np.asarray(tokens, dtype=np.int64)
    T = toks.size
    H, nh, nkv, hd = d["hidden"], d["n_heads"], d["n_kv_heads"], d["head_dim"]
    eps, W = d["rms_eps"], d["sliding_window"]
    cos, sin = rope_tables(T, d["rope_theta"], hd)
    pos = np.arange(T)
    scale = 1.0 / np.sqrt(float(hd))
    res = bf16(m["embed"][toks]).astype(np.float64)
    for layer, a in enumerate(m["layers"]):
        xn = rms_norm(res, a["attn_norm"], eps)
        q = xn @ bf16(a["wq"]).astype(np.float64).T
        k = xn @ bf16(a["wk"]).astype(np.float64).T
        v = xn @ bf16(a["wv"]).astype(np.float64).T
        if a.get("bq") is not None:
            q = q + bf16(a["bq"])
        if a.get("bk") is not None:
            k = k + bf16(a["bk"])
        if a.get("bv") is not None:
            v = v + bf16(a["bv"])
        q = round_bf16(apply_rope(q.reshape(T, nh, hd), pos, cos, sin))
        k = round_bf16(apply_rope(k.reshape(T, nkv, hd), pos, cos, sin))
        v = round_bf16(v.reshape(T, nkv, hd))
        sinks = bf16(a["sinks"]).astype(np.float64) if a.get("sinks") is not None else None
        window = W if layer % 2 == 0 else 0
        ctx = round_bf16(attention(q, k, v, pos, window, sinks, scale).reshape(T, nh * hd))
        o = ctx @ bf16(a["wo"]).astype(np.float64).T
        if a.get("bo") is not None:
            o = o + bf16(a["bo"])
        res = res + o
        xn2 = rms_norm(res, a["mlp_norm"], eps)
        if route_gaps is not None:
            mw = a["moe"]
            rl = xn2 @ bf16(mw["router_w"]).astype(np.float64).T
            if mw.get("router_b") is not None:
                rl = rl + bf16(mw["router_b"])
            srt = -np.sort(-rl, axis=1)
            kk = mw["top_k"]
            route_gaps.append(srt[:, kk - 1] - srt[:, kk] if kk < srt.shape[1] else np.full(T, np.inf))
        x2 = _o.np_f32_to_bf16(xn2.astype(np.float32))
        mw = a["moe"]
        rl = bf16(x2).astype(np.float64) @ bf16(mw["router_w"]).astype(np.float64).T
        if mw.get("router_b") is not None:
            rl = rl + bf16(mw["router_b"])
        if route_logits is not None:
            route_logits.append(rl)
        if routes is not None:
            idx = np.asarray(routes[layer], dtype=np.int64)
            top = np.take_along_axis(rl, idx, axis=1)
            ex = np.exp(top - top.max(axis=1, keepdims=True))
            y = _o.np_moe_forward(mw, x2, idx=idx, wts=ex / ex.sum(axis=1, keepdims=True))
        else:
            y = _o.np_moe_forward(a["moe"], x2)
        res = res + y.astype(np.float64)
    last = res[T - n_logits:]
    xf = rms_norm(last, m["final_norm"], eps)
    logits = xf @ bf16(m["unembed"]).astype(np.float64).T
    return (logits, res) if return_hidden else logits
