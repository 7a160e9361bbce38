"""The C-ABI library loads and exports every symbol include/oxg_b200.h declares.
CPU only: nothing here launches GPU work."""
import ctypes
import subprocess

import pytest

from oxidized_gpt_oss_b200 import abi


def test_header_declares_the_entry_points():
    syms = abi.header_symbols()
    assert len(syms) == len(set(syms))
    for required in ("oxg_ctx_create", "oxg_dequant_mxfp4", "oxg_moe_upload", "oxg_moe_forward",
                     "oxg_moe_forward_host", "oxg_swiglu", "oxg_moe_route"):
        assert required in syms


def test_library_exports_every_header_symbol():
    lib = abi.load()
    out = subprocess.run(["nm", "-D", "--defined-only", abi.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for s in abi.header_symbols():
        assert s in exported, f"{s} declared in the header but not exported"
        assert hasattr(lib, s)
    # only the declared API is exported (kernels and helpers stay hidden)
    assert {s for s in exported if s.startswith("oxg_")} == set(abi.header_symbols())


def test_binding_covers_the_header():
    assert set(abi.SIGNATURES) == set(abi.header_symbols())


def test_version_and_status_strings():
    lib = abi.load()
    assert lib.oxg_abi_version() == 1
    assert lib.oxg_status_string(0) == b"ok"
    assert lib.oxg_status_string(abi.OXG_ERR_SHAPE) == b"shape mismatch"


def test_null_context_is_an_error_not_a_crash():
    lib = abi.load()
    st = lib.oxg_sync(None)
    assert st == abi.OXG_ERR_INVALID_ARG
    assert lib.oxg_last_error(None) == b"ctx is NULL"
    st = lib.oxg_dequant_mxfp4(None, None, 0, None, 0, 0, 0, 0, None)
    assert st == abi.OXG_ERR_INVALID_ARG


def test_ctx_create_without_gpu_reports_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = abi.load()
    h = ctypes.c_void_p()
    st = lib.oxg_ctx_create(0, ctypes.byref(h))
    assert st != abi.OXG_OK
    assert not h.value
    assert lib.oxg_last_error(None)


def test_package_fails_loudly_when_library_missing(tmp_path):
    with pytest.raises(OSError, match="missing"):
        abi._lib_backup = abi._lib
        try:
            abi._lib = None
            abi.load(str(tmp_path / "nope.so"))
        finally:
            abi._lib = abi._lib_backup
