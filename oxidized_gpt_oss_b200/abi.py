"""ctypes binding of liboxg_b200.so (the C ABI in include/oxg_b200.h).

This is the binding a host runner writes against the library (a Rust runner
declares the same functions in an ``extern "C"`` block). Loading fails loudly
if the library has not been built: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
import re

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "liboxg_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(_PKG), "include", "oxg_b200.h")

OXG_OK = 0
OXG_ERR_INVALID_ARG = -1
OXG_ERR_SHAPE = -2
OXG_ERR_CUDA = -3
OXG_ERR_NCCL = -4
OXG_ERR_TIMEOUT = -5
OXG_ERR_STATE = -6
OXG_ERR_UNSUPPORTED = -7
OXG_ERR_OOM = -8

OXG_SCALE_E8M0 = 0
OXG_SCALE_BF16 = 1
OXG_MODE_AUTO = 0
OXG_MODE_DECODE = 1
OXG_MODE_PREFILL = 2
OXG_MODE_MXF4 = 3
OXG_PRECISION_PARITY = 0


class OxgError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status
        self.message = message


class MoeDims(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("intermediate", ctypes.c_int), ("n_experts", ctypes.c_int),
                ("top_k", ctypes.c_int), ("swiglu_alpha", ctypes.c_float), ("swiglu_limit", ctypes.c_float)]


class MoeWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("router_w", "router_b", "w1_blocks", "w1_scales", "b1",
                                               "w2_blocks", "w2_scales", "b2")]


class ModelDims(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("vocab", ctypes.c_int),
                ("sliding_window", ctypes.c_int), ("max_seq", ctypes.c_int), ("max_tokens", ctypes.c_int),
                ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float), ("max_batch", ctypes.c_int),
                ("kv_pages", ctypes.c_int)]


class AttnWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("attn_norm", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "bo",
                                               "sinks", "mlp_norm")]


_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_CTX = ctypes.c_void_p

# name -> (restype, argtypes)
SIGNATURES = {
    "oxg_abi_version": (_I, []),
    "oxg_status_string": (ctypes.c_char_p, [_I]),
    "oxg_ctx_create": (_I, [_I, ctypes.POINTER(ctypes.c_void_p)]),
    "oxg_ctx_destroy": (_I, [_CTX]),
    "oxg_last_error": (ctypes.c_char_p, [_CTX]),
    "oxg_ctx_set_stream": (_I, [_CTX, _P]),
    "oxg_ctx_get_stream": (_P, [_CTX]),
    "oxg_ctx_set_host_chunk": (_I, [_CTX, _I]),
    "oxg_sync": (_I, [_CTX]),
    "oxg_dequant_mxfp4": (_I, [_CTX, _P, _SZ, _P, _SZ, _I, _SZ, _SZ, _P]),
    "oxg_swiglu": (_I, [_CTX, _P, _P, _SZ, ctypes.c_float, ctypes.c_float, _P]),
    "oxg_moe_upload": (_I, [_CTX, _I, ctypes.POINTER(MoeDims), ctypes.POINTER(MoeWeights)]),
    "oxg_moe_release": (_I, [_CTX, _I]),
    "oxg_moe_reserve": (_I, [_CTX, _I, _I]),
    "oxg_moe_forward": (_I, [_CTX, _I, _P, _I, _P, _I, _I]),
    "oxg_moe_forward_host": (_I, [_CTX, _I, _P, _I, _P, _I, _I]),
    "oxg_moe_route": (_I, [_CTX, _I, _P, _I, _P, _P, _P]),
    "oxg_moe_last_counts": (_I, [_CTX, _P, _I]),
    "oxg_moe_forward_noalloc": (_I, [_CTX, _I, _P, _I, _P]),
    "oxg_moe_upload_shard": (_I, [_CTX, _I, ctypes.POINTER(MoeDims), ctypes.POINTER(MoeWeights), _I, _I]),
    "oxg_moe_dispatch": (_I, [_CTX, _I, _P, _I, _P, _P, _P]),
    "oxg_moe_experts": (_I, [_CTX, _I, _P, _P, _I, _P, _P]),
    "oxg_moe_combine": (_I, [_CTX, _I, _P, _I, _P]),
    "oxg_ep_init": (_I, [_CTX, _I, _I, _I, _I, ctypes.c_longlong, _P]),
    "oxg_ep_connect": (_I, [_CTX, _P]),
    "oxg_moe_forward_ep": (_I, [_CTX, _I, _P, _I, _P]),
    "oxg_ep_close": (_I, [_CTX]),
    "oxg_ep_set_decode_tokens": (_I, [_CTX, _I]),
    "oxg_ep_set_wait_budget": (_I, [_CTX, ctypes.c_double]),
    "oxg_ep_last_received": (_I, [_CTX, ctypes.POINTER(ctypes.c_longlong)]),
    "oxg_model_init": (_I, [_CTX, ctypes.POINTER(ModelDims)]),
    "oxg_model_reset_seq": (_I, [_CTX, _I]),
    "oxg_model_kv_pages": (_I, [_CTX, ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "oxg_model_upload_embeddings": (_I, [_CTX, _P, _P, _P]),
    "oxg_model_upload_attention": (_I, [_CTX, _I, ctypes.POINTER(AttnWeights)]),
    "oxg_model_reset": (_I, [_CTX]),
    "oxg_model_position": (_I, [_CTX, ctypes.POINTER(ctypes.c_int)]),
    "oxg_model_forward": (_I, [_CTX, _P, _I, _I, _P, _P]),
    "oxg_model_generate": (_I, [_CTX, _P, _I, _I, _P]),
    "oxg_model_decode": (_I, [_CTX, _I, _P]),
    "oxg_model_route_tap": (_I, [_CTX, _P, _I]),
    "oxg_model_prefill_seq": (_I, [_CTX, _I, _P, _I, _P]),
    "oxg_model_step_batch": (_I, [_CTX, _I, _P, _P, _P]),
    "oxg_model_release": (_I, [_CTX]),
    "oxg_profile_enable": (_I, [_CTX, _I]),
    "oxg_profile_read": (_I, [_CTX, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                              ctypes.POINTER(ctypes.c_int)]),
    "oxg_profile_reset": (_I, [_CTX]),
    "oxg_measure_mma_rate": (_I, [_CTX, _I, _I, ctypes.POINTER(ctypes.c_double)]),
    "oxg_kernel_launches": (_I, [_CTX, ctypes.POINTER(ctypes.c_longlong)]),
}

_lib = None


def header_symbols(path: str = HEADER_PATH) -> list[str]:
    """Every function the public header declares."""
    with open(path) as f:
        text = f.read()
    return re.findall(r"OXG_API\s+[^;(]*?\b(oxg_[a-z0-9_]+)\s*\(", text)


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library (once) and declare every signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise OSError(f"{path} is missing: build it with __graft_entry__.build() "
                      f"(make -C oxidized_gpt_oss_b200/csrc)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, ctx=None) -> None:
    if status != OXG_OK:
        lib = load()
        msg = lib.oxg_last_error(ctx)
        raise OxgError(status, msg.decode() if msg else lib.oxg_status_string(status).decode())


class Context:
    """Owns an oxg_ctx (device + stream + scratch + uploaded layers)."""

    def __init__(self, device: int = 0, stream=None):
        self.lib = load()
        h = ctypes.c_void_p()
        check(self.lib.oxg_ctx_create(device, ctypes.byref(h)), None)
        self.handle = h
        self.device = device
        if stream is not None:
            self.set_stream(stream)

    def set_stream(self, stream) -> None:
        """stream: a torch.cuda.Stream or a raw cudaStream_t int (0 / None:
        CUDA's legacy default stream, which is torch's default stream)."""
        raw = getattr(stream, "cuda_stream", stream)
        check(self.lib.oxg_ctx_set_stream(self.handle, raw or None), self.handle)

    def sync(self) -> None:
        check(self.lib.oxg_sync(self.handle), self.handle)

    def set_host_chunk(self, tokens: int) -> None:
        """Tokens per chunk of host-buffer forwards (0: automatic, < 0: off)."""
        check(self.lib.oxg_ctx_set_host_chunk(self.handle, int(tokens)), self.handle)

    def profile(self, on: bool = True) -> None:
        check(self.lib.oxg_profile_enable(self.handle, int(on)), self.handle)

    def profile_reset(self) -> None:
        check(self.lib.oxg_profile_reset(self.handle), self.handle)

    def profile_read(self, name: str) -> tuple[float, int]:
        """(total device ms, launches) of kernel `name` since the last reset."""
        ms = ctypes.c_double()
        n = ctypes.c_int()
        check(self.lib.oxg_profile_read(self.handle, name.encode(), ctypes.byref(ms), ctypes.byref(n)),
              self.handle)
        return ms.value, n.value

    def mma_rate(self, kind: int, iters: int = 65536) -> float:
        """TFLOP/s of one tensor-core instruction kind issued back to back on
        every SM (0 kind::f16, 1 kind::mxf8f6f4 E2M1 x E4M3, 2 kind::mxf4)."""
        v = ctypes.c_double()
        check(self.lib.oxg_measure_mma_rate(self.handle, int(kind), int(iters), ctypes.byref(v)), self.handle)
        return v.value

    def launches(self) -> int:
        n = ctypes.c_longlong()
        check(self.lib.oxg_kernel_launches(self.handle, ctypes.byref(n)), self.handle)
        return n.value

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.oxg_ctx_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
