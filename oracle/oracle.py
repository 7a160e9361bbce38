"""Python access to the CPU oracle (liboxg_oracle.so) plus an independent numpy
restatement used to cross-check it.

TEST INFRASTRUCTURE ONLY: this module is the checker. Only tests/,
``__graft_entry__.smoke()`` and bench.py's CPU legs (``cpu_baseline`` and
``--impl reference``) may import it.

Reference files followed (cipher-rc5/oxidized_gpt_oss):
  * dequant: src/mxfp4.rs:7-54 (E2M1 table :7, decode_e2m1 :9-13, nibble order :39-44)
  * E8M0 scale: src/dtype.rs:245-252 (0 -> 0.0, else 2^(e-127))
  * router matmul: src/utils.rs:34-89 (A*B^T, B stored [out, in])
  * top-k + softmax: src/moe.rs:51-73, src/utils.rs:91-111
  * expert MLP: src/model.rs:1088-1184; combine: src/moe.rs:76-99
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboxg_oracle.so")
_lib = None


def build() -> str:
    """Compile the C oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_SZ = ctypes.c_size_t


class MoEWeights(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int),
        ("intermediate", ctypes.c_int),
        ("n_experts", ctypes.c_int),
        ("top_k", ctypes.c_int),
        ("alpha", ctypes.c_float),
        ("limit", ctypes.c_float),
        ("router_w", _P),
        ("router_b", _P),
        ("w1_blocks", _P),
        ("w1_scales", _P),
        ("b1", _P),
        ("w2_blocks", _P),
        ("w2_scales", _P),
        ("b2", _P),
    ]


def _declare(L: ctypes.CDLL) -> None:
    L.oxo_f32_to_bf16.argtypes = [ctypes.c_float]
    L.oxo_f32_to_bf16.restype = ctypes.c_uint16
    L.oxo_bf16_to_f32.argtypes = [ctypes.c_uint16]
    L.oxo_bf16_to_f32.restype = ctypes.c_float
    L.oxo_f32_to_f16.argtypes = [ctypes.c_float]
    L.oxo_f32_to_f16.restype = ctypes.c_uint16
    L.oxo_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.oxo_f16_to_f32.restype = ctypes.c_float
    L.oxo_e8m0_to_f32.argtypes = [ctypes.c_uint8]
    L.oxo_e8m0_to_f32.restype = ctypes.c_float
    L.oxo_decode_e2m1.argtypes = [ctypes.c_uint8]
    L.oxo_decode_e2m1.restype = ctypes.c_float
    for name in ("oxo_dequantize_mxfp4", "oxo_dequantize_mxfp4_e8m0"):
        f = getattr(L, name)
        f.argtypes = [_P, _SZ, _P, _SZ, _SZ, _SZ, _P, ctypes.c_char_p, _SZ]
        f.restype = ctypes.c_int
    L.oxo_router_logits.argtypes = [ctypes.POINTER(MoEWeights), _P, ctypes.c_int, _P]
    L.oxo_router_logits.restype = None
    L.oxo_topk_softmax.argtypes = [_P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P]
    L.oxo_topk_softmax.restype = None
    L.oxo_swiglu_clamped.argtypes = [_P, _P, _SZ, ctypes.c_float, ctypes.c_float, _P]
    L.oxo_swiglu_clamped.restype = None
    L.oxo_swiglu_plain.argtypes = [_P, _P, _SZ, _P]
    L.oxo_swiglu_plain.restype = None
    L.oxo_moe_forward_spec.argtypes = [ctypes.POINTER(MoEWeights), _P, ctypes.c_int, _P, _P, _P, _P,
                                       ctypes.c_int, ctypes.c_int]
    L.oxo_moe_forward_spec.restype = ctypes.c_int
    L.oxo_moe_forward_ref_faithful.argtypes = [ctypes.POINTER(MoEWeights), _P, ctypes.c_int, _P,
                                               ctypes.c_int]
    L.oxo_moe_forward_ref_faithful.restype = ctypes.c_int
    L.oxo_max_threads.argtypes = []
    L.oxo_max_threads.restype = ctypes.c_int
    L.oxo_ref_prepare.argtypes = [ctypes.POINTER(MoEWeights), _P, ctypes.c_int]
    L.oxo_ref_prepare.restype = ctypes.c_void_p
    L.oxo_ref_forward.argtypes = [ctypes.c_void_p, _P, ctypes.c_int, _P, ctypes.c_int]
    L.oxo_ref_forward.restype = ctypes.c_int
    L.oxo_ref_free.argtypes = [ctypes.c_void_p]
    L.oxo_ref_free.restype = None


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


class OracleShapeError(ValueError):
    """Raised where the reference panics on a shape assert (src/mxfp4.rs:16-33)."""


# ---------------------------------------------------------------- dequant
def dequantize_mxfp4(blocks: np.ndarray, scales_bf16: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """dequantize_mxfp4(blocks, scales_u16, rows, cols) -> bf16 bits (src/mxfp4.rs:15)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    scales_bf16 = np.ascontiguousarray(scales_bf16, dtype=np.uint16).reshape(-1)
    out = np.empty(rows * cols, dtype=np.uint16)
    err = ctypes.create_string_buffer(256)
    rc = lib().oxo_dequantize_mxfp4(_ptr(blocks), blocks.size, _ptr(scales_bf16), scales_bf16.size,
                                    rows, cols, _ptr(out), err, 256)
    if rc:
        raise OracleShapeError(err.value.decode())
    return out


def dequantize_mxfp4_e8m0(blocks: np.ndarray, scales_e8m0: np.ndarray, rows: int, cols: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    scales_e8m0 = np.ascontiguousarray(scales_e8m0, dtype=np.uint8).reshape(-1)
    out = np.empty(rows * cols, dtype=np.uint16)
    err = ctypes.create_string_buffer(256)
    rc = lib().oxo_dequantize_mxfp4_e8m0(_ptr(blocks), blocks.size, _ptr(scales_e8m0), scales_e8m0.size,
                                         rows, cols, _ptr(out), err, 256)
    if rc:
        raise OracleShapeError(err.value.decode())
    return out


# ---------------------------------------------------------------- MoE
class Weights:
    """Holds numpy arrays for one MoE layer and the ctypes view of them."""

    def __init__(self, d: dict):
        self.d = d
        self.hidden = int(d["hidden"])
        self.intermediate = int(d["intermediate"])
        self.n_experts = int(d["n_experts"])
        self.top_k = int(d["top_k"])
        self.alpha = float(d["alpha"])
        self.limit = float(d["limit"])
        self.arrays = {k: np.ascontiguousarray(d[k]) for k in
                       ("router_w", "router_b", "w1_blocks", "w1_scales", "b1", "w2_blocks", "w2_scales", "b2")
                       if d.get(k) is not None}
        self.c = MoEWeights(self.hidden, self.intermediate, self.n_experts, self.top_k, self.alpha,
                            self.limit,
                            *[_ptr(self.arrays.get(k)) for k in ("router_w", "router_b", "w1_blocks",
                                                                 "w1_scales", "b1", "w2_blocks",
                                                                 "w2_scales", "b2")])


def router_logits(W: Weights, x_bf16: np.ndarray) -> np.ndarray:
    T = x_bf16.shape[0]
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    out = np.empty((T, W.n_experts), dtype=np.float32)
    lib().oxo_router_logits(ctypes.byref(W.c), _ptr(x), T, _ptr(out))
    return out


def topk_softmax(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    idx = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    lib().oxo_topk_softmax(_ptr(logits), T, E, k, _ptr(idx), _ptr(w))
    return idx, w


def swiglu_clamped(gate: np.ndarray, up: np.ndarray, alpha: float = 1.702, limit: float = 7.0) -> np.ndarray:
    g = np.ascontiguousarray(gate, dtype=np.float32).reshape(-1)
    u = np.ascontiguousarray(up, dtype=np.float32).reshape(-1)
    out = np.empty_like(g)
    lib().oxo_swiglu_clamped(_ptr(g), _ptr(u), g.size, alpha, limit, _ptr(out))
    return out.reshape(np.shape(gate))


def swiglu_plain(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate, dtype=np.float32).reshape(-1)
    u = np.ascontiguousarray(up, dtype=np.float32).reshape(-1)
    out = np.empty_like(g)
    lib().oxo_swiglu_plain(_ptr(g), _ptr(u), g.size, _ptr(out))
    return out.reshape(np.shape(gate))


def moe_forward_spec(W: Weights, x_bf16: np.ndarray, idx=None, wts=None, acc64: bool = True,
                     nthreads: int = 0, want_slots: bool = False):
    """SPEC MoE forward -> y fp32 [T, H] (and per-slot expert outputs if asked)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T = x.shape[0]
    y = np.empty((T, W.hidden), dtype=np.float32)
    slots = np.empty((T * W.top_k, W.hidden), dtype=np.float32) if want_slots else None
    idx_a = None if idx is None else np.ascontiguousarray(idx, dtype=np.int32)
    w_a = None if wts is None else np.ascontiguousarray(wts, dtype=np.float32)
    rc = lib().oxo_moe_forward_spec(ctypes.byref(W.c), _ptr(x), T, _ptr(idx_a), _ptr(w_a), _ptr(y),
                                    _ptr(slots), int(acc64), int(nthreads))
    if rc:
        raise RuntimeError(f"oxo_moe_forward_spec failed: {rc}")
    return (y, slots) if want_slots else y


def moe_forward_ref_faithful(W: Weights, x_bf16: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """REF-FAITHFUL MoE forward -> f16 bits [T, H]."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    T = x.shape[0]
    y = np.empty((T, W.hidden), dtype=np.uint16)
    rc = lib().oxo_moe_forward_ref_faithful(ctypes.byref(W.c), _ptr(x), T, _ptr(y), int(nthreads))
    if rc:
        raise RuntimeError(f"oxo_moe_forward_ref_faithful failed: {rc}")
    return y


def max_threads() -> int:
    return int(lib().oxo_max_threads())


class RefLayer:
    """REF-FAITHFUL layer split at the reference's load/forward boundary."""

    def __init__(self, W: Weights, x_bf16: np.ndarray):
        self.W = W  # keeps the weight arrays alive
        x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
        self.h = lib().oxo_ref_prepare(ctypes.byref(W.c), _ptr(x), x.shape[0])
        if not self.h:
            raise RuntimeError("oxo_ref_prepare failed")

    def forward(self, x_bf16: np.ndarray, nthreads: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
        y = np.empty((x.shape[0], self.W.hidden), dtype=np.uint16)
        rc = lib().oxo_ref_forward(self.h, _ptr(x), x.shape[0], _ptr(y), int(nthreads))
        if rc:
            raise RuntimeError(f"oxo_ref_forward failed: {rc}")
        return y

    def close(self) -> None:
        if self.h:
            lib().oxo_ref_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


# ---------------------------------------------------------------- numpy restatement
# An independent vectorised restatement, used only to cross-check the C oracle.
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0],
                dtype=np.float32)


def np_f32_to_bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def np_bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def np_e8m0_to_f32(s: np.ndarray) -> np.ndarray:
    return np_bf16_to_f32(np.asarray(s, dtype=np.uint16) << 7)


def np_decode_codes(blocks: np.ndarray) -> np.ndarray:
    """Packed bytes [..., n] -> E2M1 values [..., 2n]; low nibble is the even element."""
    b = np.asarray(blocks, dtype=np.uint8)
    out = np.empty(b.shape[:-1] + (b.shape[-1] * 2,), dtype=np.float32)
    out[..., 0::2] = E2M1[b & 0x0F]
    out[..., 1::2] = E2M1[b >> 4]
    return out


def np_dequant_f32(blocks: np.ndarray, scales_e8m0: np.ndarray) -> np.ndarray:
    """[..., rows, cols/2] codes + [..., rows, cols/32] E8M0 -> exact f32 values."""
    v = np_decode_codes(blocks)
    s = np_e8m0_to_f32(scales_e8m0)
    return (v.reshape(v.shape[:-1] + (-1, 32)) * s[..., None]).reshape(v.shape)


def np_moe_forward(d: dict, x_bf16: np.ndarray, idx=None, wts=None) -> np.ndarray:
    """fp64 numpy restatement of the SPEC layer (small shapes only)."""
    H, I, E, K = d["hidden"], d["intermediate"], d["n_experts"], d["top_k"]
    x = np_bf16_to_f32(x_bf16).astype(np.float64)
    if idx is None:
        rw = np_bf16_to_f32(d["router_w"]).astype(np.float64)
        logits = x @ rw.T
        if d.get("router_b") is not None:
            logits = logits + np_bf16_to_f32(d["router_b"]).astype(np.float64)
        order = np.argsort(-logits, axis=1, kind="stable")
        idx = order[:, :K]
        top = np.take_along_axis(logits, idx, axis=1)
        ex = np.exp(top - top.max(axis=1, keepdims=True))
        wts = ex / ex.sum(axis=1, keepdims=True)
    y = np.zeros((x.shape[0], H), dtype=np.float64)
    alpha, limit = d["alpha"], d["limit"]
    for e in np.unique(idx):
        w1 = np_dequant_f32(d["w1_blocks"][e], d["w1_scales"][e]).astype(np.float64)
        w2 = np_dequant_f32(d["w2_blocks"][e], d["w2_scales"][e]).astype(np.float64)
        b1 = np_bf16_to_f32(d["b1"][e]).astype(np.float64)
        b2 = np_bf16_to_f32(d["b2"][e]).astype(np.float64)
        t_sel, j_sel = np.nonzero(idx == e)
        h1 = x[t_sel] @ w1.T + b1
        g = np.minimum(h1[:, 0::2], limit)
        u = np.clip(h1[:, 1::2], -limit, limit)
        h = g / (1.0 + np.exp(-alpha * g)) * (u + 1.0)
        ye = h @ w2.T + b2
        y[t_sel] += np.asarray(wts)[t_sel, j_sel][:, None] * ye
    return y.astype(np.float32)
