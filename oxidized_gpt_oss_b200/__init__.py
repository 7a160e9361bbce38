"""oxidized_gpt_oss_b200 — B200-native (sm_100a) MXFP4 mixture-of-experts hot path.

The compute lives in ``liboxg_b200.so`` (hand-written CUDA for sm_100a behind a
C ABI declared in ``include/oxg_b200.h``). This package is the Python mirror of
the reference runner's hot-path interface (cipher-rc5/oxidized_gpt_oss):

* ``mxfp4.dequantize_mxfp4``  — src/mxfp4.rs:15
* ``ffn.swiglu``              — src/ffn.rs:5 (clamped gpt-oss form)
* ``moe.MoELayer.forward``    — src/moe.rs:16

It holds no fallback: every call goes through the CUDA library, and loading
fails loudly when the library or a GPU is missing.
"""
__all__ = ["abi", "mxfp4", "ffn", "moe", "synth"]
