"""Generates the committed golden fixtures in this directory.

The reference (a Rust crate) cannot be built or imported here, so its
known-answer tests are restated from their own definitions:

* ``mxfp4_kat_4x64.json`` — src/mxfp4.rs:63-95 ``dequantizes_known_4x64_tensor``:
  nibbles ``i % 16`` packed low-nibble-first, bf16 scales
  ``[1, 2, 0.5, 1.5, 0.25, 4, 3, 0.75]`` (one per 32-block, row-major), and the
  expected output of the test's own formula ``bf16(sign * TABLE[n & 7] * scale)``.
* ``mxfp4_sanity_2x32.json`` — tests/integration.rs:30-48 ``mxfp4_dequant_sanity``:
  blocks ``0x21``, scale ``bf16(0.1)``; the test asserts |mean| < 1 and std > 0.
  The exact per-element expectation (same formula) is stored beside it.
* ``e8m0_table.json`` — F8E8M0::to_f32 (src/dtype.rs:245-252) for all 256
  codes, as f32 bit patterns: 0 -> 0.0, e -> 2^(e-127), 255 -> powi(2, 128) = inf.
* ``moe_small_seed1.npz`` — a small seeded MoE layer (H=96, I=160, E=8, k=4,
  T=7) with the SPEC oracle's fp64-accumulated output, routing and per-slot
  expert outputs; cross-checked here against the independent numpy
  restatement before it is written. This pins the oracle against regressions;
  the reference has no MoE fixture of its own.

Run from the repository root: ``python tests/golden/make_golden.py``.
"""
from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from oxidized_gpt_oss_b200 import synth  # noqa: E402

TABLE = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def bf16_bits(v: float) -> int:
    return int(synth.f32_to_bf16_bits(np.array([v], dtype=np.float32))[0])


def kat_4x64() -> dict:
    rows, cols = 4, 64
    nibbles = [i % 16 for i in range(rows * cols)]
    blocks = [(nibbles[2 * i] & 0x0F) | ((nibbles[2 * i + 1] & 0x0F) << 4) for i in range(rows * cols // 2)]
    scales_f32 = [1.0, 2.0, 0.5, 1.5, 0.25, 4.0, 3.0, 0.75]
    scales = [bf16_bits(v) for v in scales_f32]
    expected = []
    for row in range(rows):
        for col in range(cols):
            n = nibbles[row * cols + col]
            sign = -1.0 if n & 0b1000 else 1.0
            base = TABLE[n & 0b0111]
            scale = scales_f32[row * (cols // 32) + col // 32]
            prod = np.float32(sign) * np.float32(base) * np.float32(scale)
            expected.append(bf16_bits(float(prod)))
    return dict(source="src/mxfp4.rs:63-95", rows=rows, cols=cols, blocks=blocks, scales_bf16=scales,
                expected_bf16=expected)


def sanity_2x32() -> dict:
    rows, cols = 2, 32
    blocks = [0x21] * (rows * cols // 2)
    scale = bf16_bits(0.1)
    scale_f32 = float(synth.bf16_bits_to_f32(np.array([scale], dtype=np.uint16))[0])
    expected = []
    for i in range(rows * cols):
        n = (0x21 & 0x0F) if i % 2 == 0 else (0x21 >> 4)
        expected.append(bf16_bits(float(np.float32(TABLE[n]) * np.float32(scale_f32))))
    return dict(source="tests/integration.rs:30-48", rows=rows, cols=cols, blocks=blocks,
                scales_bf16=[scale] * (rows * (cols // 32)), expected_bf16=expected,
                assert_abs_mean_lt=1.0, assert_std_gt=0.0)


def e8m0_table() -> dict:
    bits = []
    for e in range(256):
        if e == 0:
            v = 0.0
        elif e == 255:
            v = float("inf")
        else:
            v = 2.0 ** (e - 127)
        bits.append(struct.unpack("<I", struct.pack("<f", v))[0])
    return dict(source="src/dtype.rs:245-252", f32_bits=bits)


def moe_small() -> dict:
    d = synth.moe_layer(seed=1, hidden=96, intermediate=160, n_experts=8, top_k=4)
    x = synth.activations(1, 7, 96)
    W = oracle.Weights(d)
    y, slots = oracle.moe_forward_spec(W, x, acc64=True, want_slots=True)
    logits = oracle.router_logits(W, x)
    idx, wts = oracle.topk_softmax(logits, 4)
    y_np = oracle.np_moe_forward(d, x)
    err = float(np.max(np.abs(y - y_np)))
    assert err < 1e-3, f"C oracle and numpy restatement disagree: {err}"
    out = {k: v for k, v in d.items() if isinstance(v, np.ndarray)}
    out.update(x=x, y=y, slot_y=slots, idx=idx, wts=wts, logits=logits,
               dims=np.array([d["hidden"], d["intermediate"], d["n_experts"], d["top_k"]], dtype=np.int32),
               act=np.array([d["alpha"], d["limit"]], dtype=np.float32))
    return out


def main() -> None:
    oracle.build()
    with open(os.path.join(HERE, "mxfp4_kat_4x64.json"), "w") as f:
        json.dump(kat_4x64(), f)
    with open(os.path.join(HERE, "mxfp4_sanity_2x32.json"), "w") as f:
        json.dump(sanity_2x32(), f)
    with open(os.path.join(HERE, "e8m0_table.json"), "w") as f:
        json.dump(e8m0_table(), f)
    np.savez_compressed(os.path.join(HERE, "moe_small_seed1.npz"), **moe_small())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
