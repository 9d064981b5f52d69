"""Writes the golden fixtures under tests/golden/.

reference_kats.json
    The known-answer tests of chat-wgpu's own test suite, transcribed with
    their source lines: the dequantisation unit tests of
    src/loader/dequant.rs:133-200, the GGUF parse test of
    src/loader/gguf.rs:219-251 and the closed-form GPU checks of the verify
    harness src/main.rs:53-161 (inputs and expected outputs, abs tol 1e-3 as
    src/main.rs:268-273).

q4_gemv_256x512.npz
    The q4 GEMV check of src/main.rs:123-152 rebuilt from its own recipe:
    x = fill(0x1234, 256), w = fill(0x5678, 512*256) with the reference's
    LCG (src/main.rs:257-266), re-quantised by quantize_q4_0
    (src/kernels/q4.rs:37-60) and reduced by the CPU dequant-and-dot of
    src/main.rs:133-150.  Everything here is restated in numpy float32 scalar
    arithmetic (one rounding per operation, like Rust's f32), independently
    of the C oracle, and the script checks the two agree bit for bit.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
F = np.float32


def lcg_fill(seed: int, n: int) -> np.ndarray:
    """src/main.rs:257-266: s = s*6364136223846793005 + 1442695040888963407
    (wrapping u64), value = ((s >> 33) as f32 / u32::MAX as f32 - 0.5) * 0.2."""
    s = (seed | 1) & 0xFFFFFFFFFFFFFFFF
    out = np.empty(n, dtype=np.float32)
    umax = F(4294967295.0)
    for i in range(n):
        s = (s * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
        out[i] = (F(s >> 33) / umax - F(0.5)) * F(0.2)
    return out


def quantize_q4_0_np(w: np.ndarray, out_f: int, in_f: int):
    """src/kernels/q4.rs:37-60 in float32 scalar arithmetic."""
    nb = in_f // 32
    scales = np.zeros(out_f * nb, dtype=np.float32)
    quants = np.zeros(out_f * in_f // 8, dtype=np.uint32)
    for o in range(out_f):
        for b in range(nb):
            blk = w[o * in_f + b * 32: o * in_f + b * 32 + 32]
            absmax = F(np.max(np.abs(blk)))
            d = absmax / F(8.0)
            inv = F(1.0) / d if d != 0 else F(0.0)
            scales[o * nb + b] = d
            for wd in range(4):
                word = 0
                for n in range(8):
                    v = blk[wd * 8 + n]
                    r = np.round(F(v * inv))  # numpy rounds half to even ...
                    t = F(v * inv)
                    if abs(t - np.trunc(t)) == F(0.5):  # ... Rust rounds half away from zero
                        r = np.trunc(t) + np.sign(t)
                    q = min(max(int(r) + 8, 0), 15)
                    word |= q << (n * 4)
                quants[o * (in_f // 8) + b * 4 + wd] = word
    return scales, quants


def q4_gemv_np(x, scales, quants, in_f, out_f):
    """src/main.rs:133-150, float32 scalar arithmetic in the same order."""
    nb = in_f // 32
    y = np.zeros(out_f, dtype=np.float32)
    for o in range(out_f):
        s = F(0.0)
        for b in range(nb):
            d = scales[o * nb + b]
            for wd in range(4):
                word = int(quants[o * (in_f // 8) + b * 4 + wd])
                for n in range(8):
                    q = (word >> (n * 4)) & 0xF
                    k = b * 32 + wd * 8 + n
                    s = F(s + F(F(d * F(F(q) - F(8.0))) * x[k]))
        y[o] = s
    return y


def reference_kats() -> dict:
    q4_0_block = [0x00, 0x3C] + [8 | (15 << 4)] * 16
    q8_0_block = [0x00, 0x38] + list(range(32))
    q4_1_block = [0x00, 0x3C, 0x00, 0x38] + [0x00 | (15 << 4)] * 16
    q6k = [0] * 210
    for i in range(192, 208):
        q6k[i] = 1
    q6k[208], q6k[209] = 0x00, 0x3C
    # src/loader/gguf.rs:219-251 minimal file
    g = bytearray(b"GGUF" + struct.pack("<IQQ", 3, 1, 1))
    key = b"qwen3.block_count"
    g += struct.pack("<Q", len(key)) + key + struct.pack("<II", 4, 28)
    nm = b"output_norm.weight"
    g += struct.pack("<Q", len(nm)) + nm + struct.pack("<IQIQ", 1, 4, 0, 0)
    while len(g) % 32:
        g.append(0)
    g += struct.pack("<4f", 1.0, 2.0, 3.0, 4.0)
    return {
        "source": "chat-wgpu test suite (paths relative to its repository)",
        "f16_to_f32": {"cite": "src/loader/dequant.rs:137-142",
                       "cases": [[0x3C00, 1.0], [0xC000, -2.0], [0x0000, 0.0]]},
        "bf16_to_f32": {"cite": "src/loader/dequant.rs:145-148",
                        "cases": [[0x3F80, 1.0], [0xC000, -2.0]]},
        "q8_0": {"cite": "src/loader/dequant.rs:151-161", "block": q8_0_block,
                 "expect": {"0": 0.0, "1": 0.5, "10": 5.0}},
        "q4_1": {"cite": "src/loader/dequant.rs:164-173", "block": q4_1_block,
                 "expect": {"0": 0.5, "16": 15.5}},
        "q6_k": {"cite": "src/loader/dequant.rs:176-188", "block": q6k,
                 "expect": {"0": -32.0, "255": -32.0}},
        "q4_0": {"cite": "src/loader/dequant.rs:190-200", "block": q4_0_block,
                 "expect": {"0": 0.0, "16": 7.0}},
        "gguf_minimal": {"cite": "src/loader/gguf.rs:219-251", "bytes_hex": bytes(g).hex(),
                         "meta": {"qwen3.block_count": 28},
                         "tensor": {"name": "output_norm.weight", "values": [1.0, 2.0, 3.0, 4.0]}},
        "verify_tol_abs": {"cite": "src/main.rs:268-273", "value": 1e-3},
        "rmsnorm_plain": {"cite": "src/main.rs:61-67", "rows": 4, "dim": 1024, "eps": 1e-6,
                          "x": 1.0, "w": 1.0, "expect": "1/sqrt(1+eps)"},
        "rmsnorm_unit": {"cite": "src/main.rs:69-75", "rows": 4, "dim": 1024, "eps": 1e-6,
                         "x": 1.0, "w": 1.0, "expect": "2/sqrt(1+eps)"},
        "swiglu": {"cite": "src/main.rs:77-82", "n": 4096, "g": 1.5, "u": -0.7,
                   "expect": "g/(1+exp(-g))*u"},
        "geglu": {"cite": "src/main.rs:84-91", "n": 4096, "g": 1.5, "u": -0.7, "c": 0.79788456,
                  "expect": "0.5*g*(1+tanh(c*(g+0.044715*g^3)))*u"},
        "rope_pos0": {"cite": "src/main.rs:93-98", "rows": 16, "head_dim": 128, "theta": 10000.0,
                      "x": "((i % 23) - 11) * 0.07", "expect": "identity"},
        "attention_single_key": {"cite": "src/main.rs:100-118", "n_heads": 4, "n_kv": 2,
                                 "head_dim": 16, "q": "i*0.01", "k": 0.5,
                                 "v": "((i % 9) - 4) * 0.1", "expect": "V[h / (n_heads/n_kv)]"},
        "ewise_add": {"cite": "src/main.rs:154-161", "n": 1000, "a": "i", "b": "-i*0.5",
                      "expect": "i - i*0.5"},
        "q4_gemv": {"cite": "src/main.rs:120-152", "in_f": 256, "out_f": 512,
                    "x_seed": 0x1234, "w_seed": 0x5678, "fixture": "q4_gemv_256x512.npz"},
    }


def main():
    kats = reference_kats()
    with open(os.path.join(HERE, "reference_kats.json"), "w") as f:
        json.dump(kats, f, indent=1)
    in_f, out_f = 256, 512
    x = lcg_fill(0x1234, in_f)
    w = lcg_fill(0x5678, out_f * in_f)
    scales, quants = quantize_q4_0_np(w, out_f, in_f)
    y = q4_gemv_np(x, scales, quants, in_f, out_f)
    # cross-check against the C oracle (same recipe, independent code)
    sys.path.insert(0, ROOT)
    from oracle import oracle
    s2, q2 = oracle.quantize_q4_0(w, out_f, in_f)
    assert np.array_equal(s2, scales) and np.array_equal(q2, quants), "oracle quantiser differs"
    y2 = oracle.q4_gemv(x, scales, quants, in_f, out_f)
    assert np.array_equal(y2.view(np.uint32), y.view(np.uint32)), "oracle q4 gemv differs"
    np.savez_compressed(os.path.join(HERE, "q4_gemv_256x512.npz"), x=x, scales=scales,
                        quants=quants, y=y)
    print("wrote reference_kats.json and q4_gemv_256x512.npz")


if __name__ == "__main__":
    main()
