"""ctypes binding of libchatcuda.so (declarations in include/chatcuda.h).

The library is the only compute path: if it is missing or fails to load,
importing anything that needs it raises.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libchatcuda.so")

CW_OK = 0
STATUS_NAMES = {
    0: "CW_OK", 1: "CW_ERR_INVALID_ARG", 2: "CW_ERR_CUDA", 3: "CW_ERR_OOM",
    4: "CW_ERR_NOT_FOUND", 5: "CW_ERR_UNSUPPORTED", 6: "CW_ERR_TIMEOUT",
    7: "CW_ERR_FORMAT", 8: "CW_ERR_NO_DEVICE",
}


class CwError(RuntimeError):
    """A libchatcuda call returned a non-zero cw_status."""

    def __init__(self, status: int, func: str, msg: str):
        self.status = status
        super().__init__(f"{func}: {STATUS_NAMES.get(status, status)}: {msg}")


class ProfileRow(C.Structure):
    _fields_ = [("kernel", C.c_char * 32), ("passes", C.c_uint32), ("total_ms", C.c_double)]


class ModelInfo(C.Structure):
    _fields_ = [
        ("dim", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
        ("n_kv", C.c_uint32), ("head_dim", C.c_uint32), ("hidden", C.c_uint32),
        ("vocab", C.c_uint32), ("eps", C.c_float), ("rope_theta", C.c_float),
        ("norm_kind", C.c_uint32), ("activation", C.c_uint32), ("qk_norm", C.c_uint32),
        ("qkv_bias", C.c_uint32), ("post_norms", C.c_uint32), ("sliding_window", C.c_uint32),
        ("attn_softcap", C.c_float), ("final_softcap", C.c_float), ("embed_scale", C.c_float),
        ("weight_bytes", C.c_uint64), ("arch", C.c_char * 16),
    ]


_vp = C.c_void_p
_sz = C.c_size_t
_buf = C.c_uint64
_pbuf = C.POINTER(C.c_uint64)
_f = C.c_float

# name -> argtypes (all return int cw_status unless listed in _RESTYPE)
SIGNATURES = {
    "cw_last_error": [],
    "cw_abi_version": [],
    "cw_ctx_create": [C.c_int, C.POINTER(_vp)],
    "cw_ctx_destroy": [_vp],
    "cw_ctx_backend": [_vp, C.c_char_p, _sz],
    "cw_ctx_device": [_vp, C.POINTER(C.c_int)],
    "cw_ctx_stream": [_vp, C.POINTER(_vp)],
    "cw_ctx_set_pdl": [_vp, C.c_int],
    "cw_storage": [_vp, _vp, _sz, _pbuf],
    "cw_storage_u32": [_vp, _vp, _sz, _pbuf],
    "cw_storage_bytes": [_vp, _vp, _sz, _pbuf],
    "cw_empty": [_vp, _sz, _pbuf],
    "cw_empty_persistent": [_vp, _sz, _pbuf],
    "cw_buf_release": [_vp, _buf],
    "cw_buf_nbytes": [_vp, _buf, C.POINTER(_sz)],
    "cw_buf_device_ptr": [_vp, _buf, C.POINTER(_vp)],
    "cw_copy": [_vp, _buf, _sz, _buf, _sz, _sz],
    "cw_write": [_vp, _buf, _sz, _vp, _sz],
    "cw_read": [_vp, _buf, _vp, _sz],
    "cw_read_u32": [_vp, _buf, _vp, _sz],
    "cw_flush": [_vp],
    "cw_sync": [_vp],
    "cw_reset_frame": [_vp],
    "cw_clear_cache": [_vp],
    "cw_begin_profile": [_vp],
    "cw_report_profile": [_vp, C.POINTER(ProfileRow), _sz, C.POINTER(_sz)],
    "cw_q4_gemv": [_vp, _buf, _buf, _buf, _sz, _sz, _pbuf],
    "cw_q4_quantize": [_vp, _buf, _sz, _sz, _pbuf, _pbuf],
    "cw_attention": [_vp, _buf, _buf, _buf, _sz, _sz, _sz, _sz, _pbuf],
    "cw_attention_ext": [_vp, _buf, _buf, _buf, _sz, _sz, _sz, _sz, _f, C.c_uint32, _pbuf],
    "cw_add": [_vp, _buf, _buf, _sz, _pbuf],
    "cw_rmsnorm": [_vp, _buf, _buf, _sz, _sz, _f, _pbuf],
    "cw_rmsnorm_unit": [_vp, _buf, _buf, _sz, _sz, _f, _pbuf],
    "cw_rope": [_vp, _buf, _sz, _sz, _sz, _f, _pbuf],
    "cw_swiglu": [_vp, _buf, _buf, _sz, _pbuf],
    "cw_geglu": [_vp, _buf, _buf, _sz, _pbuf],
    "cw_argmax": [_vp, _buf, _sz, _pbuf],
    "cw_attention_noalloc": [C.c_int, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz],
    "cw_q4_0_upload": [_vp, _vp, _sz, _sz, _pbuf],
    "cw_q4_0_pack": [_vp, _buf, _sz, _sz, _pbuf],
    "cw_q4_0_gemv": [_vp, _buf, _buf, _sz, _sz, _pbuf],
    "cw_q4_0_dequant": [_vp, _buf, _sz, _sz, _pbuf],
    "cw_q4_0_gemm": [_vp, _buf, _buf, _sz, _sz, _sz, _pbuf],
    "cw_kquant_gemv": [_vp, _buf, _buf, C.c_int, _sz, _sz, _pbuf],
    "cw_kquant_dequant": [_vp, _buf, C.c_int, _sz, _sz, _pbuf],
    "cw_q6_k_split": [_vp, _buf, _sz, _sz, _pbuf],
    "cw_q6_k_gemv": [_vp, _buf, _buf, _sz, _sz, _pbuf],
    "cw_q8_0_split": [_vp, _buf, _sz, _sz, _pbuf],
    "cw_q8_0_gemv": [_vp, _buf, _buf, _sz, _sz, _pbuf],
    "cw_q4_0_gemv_bench": [_vp, _buf, C.POINTER(C.c_uint64), _sz, _sz, _sz, _sz,
                           C.POINTER(C.c_double)],
    "cw_model_load_gguf": [_vp, C.c_char_p, C.POINTER(_vp)],
    "cw_model_free": [_vp],
    "cw_model_get_info": [_vp, C.POINTER(ModelInfo)],
    "cw_tp_unique_id": [_vp, _sz],
    "cw_model_load_gguf_tp": [_vp, C.c_char_p, C.c_int, C.c_int, _vp, C.POINTER(_vp)],
    "cw_model_tp_info": [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_uint32),
                         C.POINTER(C.c_uint32)],
    "cw_session_create": [_vp, _sz, C.POINTER(_vp)],
    "cw_session_free": [_vp],
    "cw_session_begin": [_vp, _vp, _sz],
    "cw_session_run": [_vp, _sz, C.POINTER(_sz)],
    "cw_session_prefill": [_vp, C.POINTER(_sz)],
    "cw_session_set_prefill_chunk": [_vp, _sz],
    "cw_gguf_inspect": [C.c_char_p, C.POINTER(_sz), C.POINTER(C.c_uint64)],
    "cw_session_set_sampling": [_vp, C.c_float, C.c_uint32, C.c_float, C.c_uint64],
    "cw_session_set_eos": [_vp, _vp, _sz],
    "cw_session_stopped": [_vp, C.POINTER(C.c_int)],
    "cw_session_add_tap": [_vp, C.c_char_p, C.c_uint32, _sz],
    "cw_group_create": [C.POINTER(_vp), _sz, C.POINTER(_vp)],
    "cw_group_free": [_vp],
    "cw_group_run": [_vp, _sz],
    "cw_group_run_timed": [_vp, _sz, C.POINTER(C.c_double)],
    "cw_group_set_streaming": [_vp, C.c_int, C.POINTER(C.c_int)],
    "cw_session_clear_taps": [_vp],
    "cw_session_read_tap": [_vp, C.c_char_p, C.c_uint32, _sz, _vp, _sz],
    "cw_sample": [_vp, _buf, _sz, C.c_float, C.c_uint32, C.c_float, C.c_uint64, C.c_uint64, _pbuf],
    "cw_session_read_kv": [_vp, C.c_uint32, _sz, _vp, _vp],
    "cw_session_tokens": [_vp, _vp, _sz, C.POINTER(_sz)],
    "cw_session_logits": [_vp, _vp, _sz],
    "cw_session_pos": [_vp, C.POINTER(_sz)],
    "cw_session_hidden": [_vp, _vp, _sz],
    "cw_session_set_graph": [_vp, C.c_int],
    "cw_session_set_persistent": [_vp, C.c_int],
    "cw_session_inject_stall": [_vp, C.c_uint32],
    "cw_session_tp_handle": [_vp, _vp, _sz],
    "cw_session_tp_attach": [_vp, _vp, _sz],
    "cw_session_persistent": [_vp, C.POINTER(C.c_int)],
    "cw_session_step": [_vp, C.c_uint32, C.POINTER(C.c_uint32)],
    "cw_session_run_timed": [_vp, _sz, C.POINTER(C.c_double)],
    "cw_session_launches": [_vp, C.POINTER(_sz), C.POINTER(_sz)],
    "cw_session_profile": [_vp, _sz, C.POINTER(ProfileRow), _sz, C.POINTER(_sz)],
    "cw_generate": [_vp, _vp, _sz, _sz, _vp],
}
_RESTYPE = {"cw_last_error": C.c_char_p}

_lock = threading.Lock()
_lib = None


def load(path: str | None = None):
    """Load libchatcuda.so (built in-tree by chat_wgpu_b200/csrc/Makefile)."""
    global _lib
    with _lock:
        if _lib is None:
            p = path or LIB_PATH
            if not os.path.exists(p):
                raise ImportError(
                    f"{p} is missing: build it with `make -C chat_wgpu_b200/csrc` "
                    "(there is no CPU fallback)")
            L = C.CDLL(p)
            for name, args in SIGNATURES.items():
                fn = getattr(L, name)
                fn.argtypes = args
                fn.restype = _RESTYPE.get(name, C.c_int)
            _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call `name` and raise CwError on a non-zero status."""
    L = load()
    rc = getattr(L, name)(*args)
    if rc != CW_OK:
        msg = L.cw_last_error()
        raise CwError(rc, name, msg.decode(errors="replace") if msg else "")


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
