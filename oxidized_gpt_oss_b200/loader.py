"""Checkpoint loader — mirror of ModelCheckpoint (src/loader.rs:29-119) and
the layer assembly of GPTModel::load_from_safetensors (src/model.rs:98-412),
without the bf16 materialisation.

The reference reads every ``<base>.blocks`` / ``<base>.scales`` pair,
dequantises it to bf16 on the host (src/loader.rs:42-73) and keeps the result
under ``<base>``. Here the pairs stay packed: ``load_model_weights`` returns
the dict that ``GPTModel`` and ``MoELayer`` upload as is (E2M1 codes and E8M0
scales go to HBM unchanged), so a 20b checkpoint's experts occupy 12.7 GB on
the device instead of 47 GB of bf16.

Tensor names are the reference's (src/model.rs:145-412):
``model.embed_tokens.weight``, ``model.norm.weight``, ``lm_head.weight``
(absent: tied to the embedding), and per layer ``model.layers.{i}.``
``input_layernorm.weight``, ``post_attention_layernorm.weight``,
``self_attn.{q,k,v,o}_proj.{weight,bias}``, ``self_attn.sinks``,
``mlp.router.{weight,bias}`` and ``mlp.experts.{gate,up,down}_proj.{weight,bias}``
with the weights as ``.weight.blocks`` [E, rows, cols/2] uint8 and
``.weight.scales`` [E, rows, cols/32]. The reference reads the scales as u16
(src/loader.rs:62); both forms are accepted: uint8 E8M0 bytes, or bf16 bit
patterns, which must then be exact powers of two (bits = e << 7) or zero.
Gate and up rows are interleaved into the gpt-oss mlp1 layout (even rows
gate, odd rows up).
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

_DTYPES = {"U8": np.uint8, "I8": np.int8, "BF16": np.uint16, "F16": np.float16, "F32": np.float32,
           "I32": np.int32, "I64": np.int64, "U16": np.uint16}


def read_safetensors(path: str) -> dict:
    """name -> read-only numpy view (memory-mapped) of one .safetensors file;
    bf16 tensors come back as uint16 bit patterns."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    base = 8 + n
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = _DTYPES.get(info["dtype"])
        if dt is None:
            raise ValueError(f"unsupported tensor dtype in conversion: {info['dtype']} ({name})")
        a, b = info["data_offsets"]
        out[name] = mm[base + a:base + b].view(dt).reshape(info["shape"])
    return out


def write_safetensors(path: str, tensors: dict) -> None:
    """The inverse (uint16 arrays are written as BF16): used to build test checkpoints."""
    names = {np.dtype(np.uint8): "U8", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32",
             np.dtype(np.int32): "I32", np.dtype(np.float16): "F16"}
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        header[name] = {"dtype": names[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a)
        off += a.nbytes
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for a in blobs:
            f.write(a.tobytes())


class ModelCheckpoint:
    """Every tensor of a checkpoint directory (``model.safetensors.index.json``
    weight map, else every ``*.safetensors`` file), memory-mapped."""

    def __init__(self, model_dir: str):
        idx = os.path.join(model_dir, "model.safetensors.index.json")
        files = []
        if os.path.exists(idx):
            with open(idx) as f:
                files = sorted(set(json.load(f)["weight_map"].values()))
        else:
            files = sorted(p for p in os.listdir(model_dir) if p.endswith(".safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files in {model_dir}")
        self.tensors = {}
        for fn in files:
            self.tensors.update(read_safetensors(os.path.join(model_dir, fn)))

    def get(self, name: str) -> np.ndarray:
        if name not in self.tensors:
            raise KeyError(f"tensor {name} not found in checkpoint")
        return self.tensors[name]

    def get_optional(self, name: str):
        return self.tensors.get(name)


def e8m0_scales(scales: np.ndarray, name: str) -> np.ndarray:
    """Scales as E8M0 bytes: uint8 as stored, or bf16 bits that are exact
    powers of two 2^(e-127) (bits = e << 7) or zero (bits = 0)."""
    s = np.asarray(scales)
    if s.dtype == np.uint8:
        return s
    if s.dtype != np.uint16:
        raise ValueError(f"{name}: scales must be uint8 E8M0 or bf16, got {s.dtype}")
    if np.any(s & 0x807F):
        raise ValueError(f"{name}: bf16 scales must be powers of two (sign 0, mantissa 0)")
    return (s >> 7).astype(np.uint8)


def _packed(ck: ModelCheckpoint, base: str):
    return ck.get(base + ".blocks"), e8m0_scales(ck.get(base + ".scales"), base + ".scales")


def load_model_weights(model_dir: str, dims: dict) -> dict:
    """The checkpoint as the weight dict of ``synth.model_weights`` (packed
    MXFP4 experts), for ``GPTModel(weights)``. ``dims`` gives the
    architecture (``synth.GPT_OSS_20B_MODEL`` for gpt-oss-20b)."""
    ck = ModelCheckpoint(model_dir)
    d = dict(dims)
    m = dict(dims=d)
    m["embed"] = ck.get("model.embed_tokens.weight")
    lm = ck.get_optional("lm_head.weight")
    m["unembed"] = lm if lm is not None else m["embed"]
    m["final_norm"] = ck.get("model.norm.weight")
    layers = []
    for i in range(d["n_layers"]):
        p = f"model.layers.{i}"
        a = {"attn_norm": ck.get(f"{p}.input_layernorm.weight"),
             "mlp_norm": ck.get(f"{p}.post_attention_layernorm.weight"),
             "sinks": ck.get_optional(f"{p}.self_attn.sinks")}
        for n in ("q", "k", "v", "o"):
            a[f"w{n}"] = ck.get(f"{p}.self_attn.{n}_proj.weight")
            a[f"b{n}"] = ck.get_optional(f"{p}.self_attn.{n}_proj.bias")
        gq, gs = _packed(ck, f"{p}.mlp.experts.gate_proj.weight")
        uq, us = _packed(ck, f"{p}.mlp.experts.up_proj.weight")
        dq, ds = _packed(ck, f"{p}.mlp.experts.down_proj.weight")
        E, I = gq.shape[0], gq.shape[1]
        w1q = np.empty((E, 2 * I, gq.shape[2]), np.uint8)
        w1q[:, 0::2], w1q[:, 1::2] = gq, uq
        w1s = np.empty((E, 2 * I, gs.shape[2]), np.uint8)
        w1s[:, 0::2], w1s[:, 1::2] = gs, us
        gb = ck.get_optional(f"{p}.mlp.experts.gate_proj.bias")
        ub = ck.get_optional(f"{p}.mlp.experts.up_proj.bias")
        b1 = np.zeros((E, 2 * I), np.uint16)
        if gb is not None:
            b1[:, 0::2] = gb
        if ub is not None:
            b1[:, 1::2] = ub
        db = ck.get_optional(f"{p}.mlp.experts.down_proj.bias")
        a["moe"] = dict(hidden=d["hidden"], intermediate=I, n_experts=E, top_k=d["top_k"], alpha=d["alpha"],
                        limit=d["limit"], router_w=ck.get(f"{p}.mlp.router.weight"),
                        router_b=ck.get_optional(f"{p}.mlp.router.bias"), w1_blocks=w1q, w1_scales=w1s, b1=b1,
                        w2_blocks=dq, w2_scales=ds,
                        b2=db if db is not None else np.zeros((E, d["hidden"]), np.uint16))
        layers.append(a)
    m["layers"] = layers
    return m


def save_model_weights(model_dir: str, m: dict, scales_as_bf16: bool = False) -> None:
    """Writes a weight dict in the reference's checkpoint naming (one file):
    the inverse of ``load_model_weights``, for tests and tools."""
    os.makedirs(model_dir, exist_ok=True)
    t = {"model.embed_tokens.weight": m["embed"], "lm_head.weight": m["unembed"], "model.norm.weight": m["final_norm"]}
    for i, a in enumerate(m["layers"]):
        p = f"model.layers.{i}"
        t[f"{p}.input_layernorm.weight"] = a["attn_norm"]
        t[f"{p}.post_attention_layernorm.weight"] = a["mlp_norm"]
        if a.get("sinks") is not None:
            t[f"{p}.self_attn.sinks"] = a["sinks"]
        for n in ("q", "k", "v", "o"):
            t[f"{p}.self_attn.{n}_proj.weight"] = a[f"w{n}"]
            if a.get(f"b{n}") is not None:
                t[f"{p}.self_attn.{n}_proj.bias"] = a[f"b{n}"]
        mw = a["moe"]
        t[f"{p}.mlp.router.weight"] = mw["router_w"]
        if mw.get("router_b") is not None:
            t[f"{p}.mlp.router.bias"] = mw["router_b"]
        sc = (lambda s: (s.astype(np.uint16) << 7)) if scales_as_bf16 else (lambda s: s)
        for n, rows in (("gate", slice(0, None, 2)), ("up", slice(1, None, 2))):
            t[f"{p}.mlp.experts.{n}_proj.weight.blocks"] = mw["w1_blocks"][:, rows]
            t[f"{p}.mlp.experts.{n}_proj.weight.scales"] = sc(mw["w1_scales"][:, rows])
            t[f"{p}.mlp.experts.{n}_proj.bias"] = mw["b1"][:, rows]
        t[f"{p}.mlp.experts.down_proj.weight.blocks"] = mw["w2_blocks"]
        t[f"{p}.mlp.experts.down_proj.weight.scales"] = sc(mw["w2_scales"])
        t[f"{p}.mlp.experts.down_proj.bias"] = mw["b2"]
    write_safetensors(os.path.join(model_dir, "model.safetensors"), t)
