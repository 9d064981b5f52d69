"""ctypes binding of the CPU oracle (oracle/libcworacle.so).

TEST INFRASTRUCTURE ONLY: this module is the checker the CUDA path is compared
against.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
--impl reference legs import it; the product package never does.

Each wrapper names the reference file:line its C function restates (paths in
the chat-wgpu source tree); see cw_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcworacle.so")
_lock = threading.Lock()
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build(force: bool = False) -> str:
    """Compile the oracle with oracle/Makefile (gcc, no GPU needed)."""
    src = os.path.join(HERE, "cw_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = C.CDLL(LIB_PATH)
            sig = {
                "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
                "orc_bf16_to_f32": (C.c_float, [C.c_uint16]),
                "orc_dequant_f16": (None, [_u8p, _sz, _f32p]),
                "orc_dequant_q8_0": (None, [_u8p, _sz, _f32p]),
                "orc_dequant_q4_0": (None, [_u8p, _sz, _f32p]),
                "orc_dequant_q4_1": (None, [_u8p, _sz, _f32p]),
                "orc_dequant_q6_k": (None, [_u8p, _sz, _f32p]),
                "orc_dequant_q4_k": (None, [_u8p, _sz, _f32p]),
                "orc_dequant_q5_k": (None, [_u8p, _sz, _f32p]),
                "orc_quantize_q4_0": (None, [_f32p, _sz, _sz, _f32p, _u32p]),
                "orc_q4_gemv": (None, [_f32p, _f32p, _u32p, _sz, _sz, _f32p]),
                "orc_q4_0_gemv": (None, [_f32p, _u8p, _sz, _sz, _f32p]),
                "orc_matmul": (None, [_f32p, _f32p, _sz, _sz, _sz, _f32p]),
                "orc_rmsnorm": (None, [_f32p, _f32p, _sz, _sz, C.c_float, C.c_int, _f32p]),
                "orc_rope": (None, [_f32p, _sz, _sz, C.c_uint32, C.c_float, _f32p]),
                "orc_attention": (None, [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _f32p]),
                "orc_attention_ext": (None, [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz,
                                             C.c_float, C.c_uint32, _f32p]),
                "orc_add": (None, [_f32p, _f32p, _sz, _f32p]),
                "orc_swiglu": (None, [_f32p, _f32p, _sz, _f32p]),
                "orc_geglu": (None, [_f32p, _f32p, _sz, _f32p]),
                "orc_argmax": (C.c_uint32, [_f32p, _sz]),
                "orc_model_open": (C.c_void_p, [C.c_char_p, C.c_char_p, _sz]),
                "orc_model_close": (None, [C.c_void_p]),
                "orc_model_dims": (None, [C.c_void_p, _u32p]),
                "orc_generate": (C.c_int, [C.c_void_p, _u32p, _sz, _sz, _u32p, C.c_void_p]),
                "orc_model_reset": (C.c_int, [C.c_void_p, _sz]),
                "orc_model_step": (C.c_int, [C.c_void_p, C.c_uint32, _sz, C.c_void_p, C.c_void_p]),
                "orc_model_set_tap": (C.c_int, [C.c_void_p, C.c_long]),
                "orc_model_get_tap": (C.c_int, [C.c_void_p, _f32p, _f32p, _f32p]),
                "orc_set_threads": (None, [C.c_int]),
                "orc_get_threads": (C.c_int, []),
            }
            for name, (res, args) in sig.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def get_threads() -> int:
    return int(lib().orc_get_threads())


# --- dequantisation: src/loader/dequant.rs --------------------------------
def f16_to_f32(h: int) -> float:
    """src/loader/dequant.rs:9-21"""
    return float(lib().orc_f16_to_f32(int(h)))


def bf16_to_f32(h: int) -> float:
    """src/loader/dequant.rs:23-25"""
    return float(lib().orc_bf16_to_f32(int(h)))


def _deq(fn, raw, n):
    out = np.empty(n, dtype=np.float32)
    getattr(lib(), fn)(np.ascontiguousarray(np.frombuffer(bytes(raw), dtype=np.uint8)
                                            if not isinstance(raw, np.ndarray) else raw.view(np.uint8).ravel()),
                       n, out)
    return out


def dequant_q4_0(raw, n: int) -> np.ndarray:
    """src/loader/dequant.rs:62-78"""
    return _deq("orc_dequant_q4_0", raw, n)


def dequant_q8_0(raw, n: int) -> np.ndarray:
    """src/loader/dequant.rs:46-58"""
    return _deq("orc_dequant_q8_0", raw, n)


def dequant_q4_1(raw, n: int) -> np.ndarray:
    """src/loader/dequant.rs:82-97"""
    return _deq("orc_dequant_q4_1", raw, n)


def dequant_q6_k(raw, n: int) -> np.ndarray:
    """src/loader/dequant.rs:102-131"""
    return _deq("orc_dequant_q6_k", raw, n)


def dequant_q4_k(raw, n: int) -> np.ndarray:
    """ggml block_q4_K (not in the reference; ROADMAP.md:52-53)"""
    return _deq("orc_dequant_q4_k", raw, n)


def dequant_q5_k(raw, n: int) -> np.ndarray:
    """ggml block_q5_K (not in the reference; ROADMAP.md:52-53)"""
    return _deq("orc_dequant_q5_k", raw, n)


def dequant_f16(raw, n: int) -> np.ndarray:
    """src/loader/dequant.rs:37-39"""
    return _deq("orc_dequant_f16", raw, n)


# --- q4 --------------------------------------------------------------------
def quantize_q4_0(w: np.ndarray, out_f: int, in_f: int):
    """src/kernels/q4.rs:37-60 -> (scales f32[out*in/32], quants u32[out*in/8])."""
    s = np.empty(out_f * in_f // 32, dtype=np.float32)
    q = np.empty(out_f * in_f // 8, dtype=np.uint32)
    lib().orc_quantize_q4_0(_f32(w).ravel(), out_f, in_f, s, q)
    return s, q


def q4_gemv(x, scales, quants, in_f: int, out_f: int) -> np.ndarray:
    """src/main.rs:133-150"""
    y = np.empty(out_f, dtype=np.float32)
    lib().orc_q4_gemv(_f32(x), _f32(scales), np.ascontiguousarray(quants, dtype=np.uint32), in_f, out_f, y)
    return y


def q4_0_gemv(x, blocks: np.ndarray, in_f: int, out_f: int) -> np.ndarray:
    """dequant.rs:62-78 + matmul.wgsl:43-50 over a GGUF Q4_0 [out_f, in_f] weight."""
    y = np.empty(out_f, dtype=np.float32)
    lib().orc_q4_0_gemv(_f32(x), np.ascontiguousarray(blocks, dtype=np.uint8).ravel(), in_f, out_f, y)
    return y


def matmul(a, b, m: int, k: int, n: int) -> np.ndarray:
    """examples/bench/src/lib.rs:221-233"""
    c = np.empty(m * n, dtype=np.float32)
    lib().orc_matmul(_f32(a).ravel(), _f32(b).ravel(), m, k, n, c)
    return c


# --- ops -------------------------------------------------------------------
def rmsnorm(x, w, rows: int, dim: int, eps: float, unit: bool = False) -> np.ndarray:
    """src/kernels/norm.wgsl:20-56"""
    y = np.empty(rows * dim, dtype=np.float32)
    lib().orc_rmsnorm(_f32(x).ravel(), _f32(w).ravel(), rows, dim, eps, 1 if unit else 0, y)
    return y


def rope(x, rows: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    """src/kernels/rope.wgsl:25-34"""
    y = np.empty(rows * head_dim, dtype=np.float32)
    lib().orc_rope(_f32(x).ravel(), rows, head_dim, pos, theta, y)
    return y


def attention(q, k, v, n_heads: int, n_kv: int, seq: int, head_dim: int,
              softcap: float = 0.0, window: int = 0) -> np.ndarray:
    """src/kernels/attention.wgsl:23-96 (softcap/window: restated Gemma-2)."""
    out = np.empty(n_heads * head_dim, dtype=np.float32)
    lib().orc_attention_ext(_f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel(), n_heads, n_kv, seq,
                            head_dim, softcap, window, out)
    return out


def add(a, b) -> np.ndarray:
    """src/kernels/ewise.wgsl:9-13"""
    a, b = _f32(a).ravel(), _f32(b).ravel()
    c = np.empty_like(a)
    lib().orc_add(a, b, a.size, c)
    return c


def swiglu(g, u) -> np.ndarray:
    """src/kernels/glu.wgsl:25,33-36"""
    g, u = _f32(g).ravel(), _f32(u).ravel()
    o = np.empty_like(g)
    lib().orc_swiglu(g, u, g.size, o)
    return o


def geglu(g, u) -> np.ndarray:
    """src/kernels/glu.wgsl:27-30,38-42"""
    g, u = _f32(g).ravel(), _f32(u).ravel()
    o = np.empty_like(g)
    lib().orc_geglu(g, u, g.size, o)
    return o


def argmax(logits) -> int:
    """src/kernels/argmax.wgsl:18-55"""
    l = _f32(logits).ravel()
    return int(lib().orc_argmax(l, l.size))


_MASK64 = (1 << 64) - 1


def _splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & _MASK64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & _MASK64
    return x ^ (x >> 31)


def sample(logits, temperature: float, top_k: int = 0, top_p: float = 1.0, seed: int = 0,
           draw: int = 0):
    """Temperature / top-k / top-p draw.  The reference has no sampler (its
    decode is greedy, src/wasm.rs:57,63; sampling is on ROADMAP.md:56-57), so
    this restates the rules the CUDA path documents (include/chatcuda.h,
    cw_session_set_sampling) with numpy: w = exp((l - max) / T) in f32,
    masses floor(w * 2^40), top-k by value threshold (ties kept), nucleus by
    mass threshold (ties kept), draw target = floor(u53 * Z / 2^53) with
    u53 = splitmix64(seed ^ (draw+1) * 0x9E3779B97F4A7C15) >> 11, token =
    first index whose inclusive prefix mass exceeds the target.
    Returns (token, detail) where detail holds the kept masses, Z and target
    so a caller can judge draws that sit at a rounding boundary."""
    l = np.asarray(logits, dtype=np.float32).ravel()
    amax = argmax(l)
    if not temperature > 0 or np.isnan(l[amax]):
        return amax, None
    ok = ~np.isnan(l)
    if 0 < top_k < l.size:
        kth = np.sort(l[ok])[::-1][min(top_k, int(ok.sum())) - 1]
        ok &= l >= kth
    w = np.zeros(l.size, np.float32)
    w[ok] = np.exp((l[ok] - l[amax]) * np.float32(1.0 / np.float32(temperature)),
                   dtype=np.float32)
    m = np.floor(w.astype(np.float64) * 2.0 ** 40).astype(np.uint64)
    if top_p < 1.0:
        total = int(m.sum(dtype=np.uint64))
        need = max(1, int(float(top_p) * float(total)))
        order = np.argsort(-w, kind="stable")
        cum = np.cumsum(m[order].astype(object))
        j = int(np.searchsorted(np.array(cum, dtype=np.float64), need, side="left"))
        tau = w[order[min(j, l.size - 1)]]
        m[w < tau] = 0
    Z = int(m.sum(dtype=np.uint64))
    u53 = _splitmix64(seed ^ (((draw + 1) * 0x9E3779B97F4A7C15) & _MASK64)) >> 11
    target = (u53 * Z) >> 53
    incl = np.cumsum(m.astype(np.uint64))
    tok = int(np.searchsorted(incl, target, side="right")) if Z else amax
    return tok, {"mass": m, "Z": Z, "target": target, "incl": incl}


# --- model -----------------------------------------------------------------
class Model:
    """GGUF-backed model: src/model/qwen3.rs (+ restated gemma2 family)."""

    def __init__(self, path: str):
        err = C.create_string_buffer(512)
        self._h = lib().orc_model_open(path.encode(), err, 512)
        if not self._h:
            raise RuntimeError(f"oracle model open failed: {err.value.decode()}")
        d = np.zeros(7, dtype=np.uint32)
        lib().orc_model_dims(self._h, d)
        (self.dim, self.n_layers, self.n_heads, self.n_kv, self.head_dim,
         self.hidden, self.vocab) = (int(v) for v in d)

    def close(self):
        if self._h:
            lib().orc_model_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate(self, prompt, max_new: int, want_logits: bool = False):
        """src/model/mod.rs:57-125 (max_new == 0 still yields one token)."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        n_out = max(int(max_new), 1)
        toks = np.zeros(n_out, dtype=np.uint32)
        logits = np.zeros((n_out, self.vocab), dtype=np.float32) if want_logits else None
        rc = lib().orc_generate(self._h, p, p.size, int(max_new), toks,
                                logits.ctypes.data if logits is not None else None)
        if rc != 0:
            raise RuntimeError("oracle generate failed")
        return (toks, logits) if want_logits else toks

    def reset(self, max_seq: int):
        if lib().orc_model_reset(self._h, int(max_seq)) != 0:
            raise RuntimeError("oracle reset failed")

    def set_tap(self, layer: int) -> None:
        """Hook::tap (src/model/mod.rs:155-165) for `layer` (-1 = off)."""
        if lib().orc_model_set_tap(self._h, int(layer)) != 0:
            raise RuntimeError("oracle set_tap failed")

    def tap(self) -> dict:
        """The last step's tapped vectors: q, post_attn, layer_out."""
        q = np.zeros(self.n_heads * self.head_dim, np.float32)
        pa = np.zeros(self.dim, np.float32)
        lo = np.zeros(self.dim, np.float32)
        if lib().orc_model_get_tap(self._h, q, pa, lo) != 0:
            raise RuntimeError("no tap set")
        return {"q": q, "post_attn": pa, "layer_out": lo}

    def step(self, token: int, pos: int, want_logits: bool = True):
        hidden = np.zeros(self.dim, dtype=np.float32)
        logits = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        rc = lib().orc_model_step(self._h, int(token), int(pos), hidden.ctypes.data,
                                  logits.ctypes.data if logits is not None else None)
        if rc != 0:
            raise RuntimeError("oracle step failed")
        return hidden, logits
