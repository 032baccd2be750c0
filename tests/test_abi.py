"""The C-ABI library: loads without a GPU and exports every symbol the header
declares (no compute calls here)."""
import ctypes
import os
import subprocess

import pytest


def test_library_exports_every_header_symbol(sdg):
    L = sdg.lib()
    syms = sdg.header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/sdg.h but not exported"


def test_library_has_no_driver_link_dependency(sdg):
    # static CUDA runtime, driver resolved lazily: loads on a CPU-only host
    out = subprocess.run(["ldd", sdg.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out and "libcudart.so" not in out


def test_status_codes_match_header(sdg):
    txt = open(sdg.HEADER).read()
    for code, name in sdg.STATUS.items():
        assert f"{name} = {code}" in txt


def test_null_engine_is_rejected(sdg):
    L = sdg.lib()
    assert L.sdg_prepare(None) == 7          # SDG_ERR_NOT_INIT
    assert L.sdg_release(None) == 7
    assert "null engine" in sdg.last_error()


def test_bad_op_arguments_are_rejected_without_gpu(sdg):
    L = sdg.lib()
    assert L.sdg_linear(None, 1, 1, None, None, 1, None, 0, None, None, 0, None, None) == 2   # SDG_ERR_ARG
    assert L.sdg_conv2d(None, None, 1, 8, 8, 64, 0, None, None, 64, 5, 1, None, None, 0, None, None, None, 0, None,
                        None) == 2


def test_init_without_device_fails_cleanly(sdg):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    h = ctypes.c_void_p()
    rc = sdg.lib().sdg_init(0, None, ctypes.byref(h))
    assert rc == 1 and not h.value           # SDG_ERR_CUDA, no engine
