"""The C-ABI boundary without a GPU: libchatcuda.so loads, exports every
function include/chatcuda.h declares, the ctypes binding covers exactly that
set, and calls fail with a status (never an abort) when no device is present."""
import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "chatcuda.h")


def declared() -> set[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"\b(cw_[a-z0-9_]+)\s*\(", src))


def test_header_declares_the_surface():
    names = declared()
    for must in ["cw_ctx_create", "cw_storage", "cw_empty", "cw_copy", "cw_read", "cw_q4_gemv",
                 "cw_attention", "cw_rmsnorm", "cw_rmsnorm_unit", "cw_rope", "cw_swiglu",
                 "cw_geglu", "cw_argmax", "cw_add", "cw_q4_0_gemv", "cw_model_load_gguf",
                 "cw_generate", "cw_begin_profile", "cw_report_profile"]:
        assert must in names, must


def test_library_exports_every_declared_symbol():
    from chat_wgpu_b200 import _lib
    lib = _lib.load()
    missing = [n for n in sorted(declared()) if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (cw_[a-z0-9_]+)$", out, flags=re.M))
    assert declared() <= exported, sorted(declared() - exported)


def test_binding_matches_header():
    from chat_wgpu_b200 import _lib
    assert set(_lib.SIGNATURES) == declared()


def test_no_device_is_a_status_not_an_abort():
    from chat_wgpu_b200 import _lib
    lib = _lib.load()
    h = C.c_void_p()
    rc = lib.cw_ctx_create(0, C.byref(h))
    if rc == 0:
        lib.cw_ctx_destroy(h)
        pytest.skip("a CUDA device is present")
    assert rc == 8  # CW_ERR_NO_DEVICE
    assert lib.cw_last_error()
    assert lib.cw_abi_version() == 1


def test_null_arguments_rejected():
    from chat_wgpu_b200 import _lib
    lib = _lib.load()
    assert lib.cw_ctx_create(0, None) == 1
    assert lib.cw_storage(None, None, 0, None) == 1
    assert b"bad arguments" in lib.cw_last_error()
    # the split k-quant / Q8_0 GEMV entry points: a status, before any device work
    for fn in ("cw_q6_k_split", "cw_q8_0_split"):
        assert getattr(lib, fn)(None, 0, 256, 256, None) == 1, fn
        assert b"bad arguments" in lib.cw_last_error()
    for fn in ("cw_q6_k_gemv", "cw_q8_0_gemv"):
        assert getattr(lib, fn)(None, 0, 0, 256, 16, None) == 1, fn
        assert b"bad arguments" in lib.cw_last_error()
    assert lib.cw_kquant_gemv(None, 0, 0, 12, 256, 16, None) == 1


def test_product_does_not_link_the_oracle():
    from chat_wgpu_b200 import _lib
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "cworacle" not in out
    for root, _, files in os.walk(os.path.join(ROOT, "chat_wgpu_b200")):
        for f in files:
            if f.endswith((".py", ".cu", ".cpp", ".h", ".cuh")):
                txt = open(os.path.join(root, f)).read()
                assert "oracle" not in txt.replace("oracle.", "").lower() or f == "__init__.py", f
