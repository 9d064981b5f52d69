"""Pins the CPU oracle to chat-wgpu's own known-answer tests
(tests/golden/reference_kats.json, transcribed from src/loader/dequant.rs,
src/loader/gguf.rs and the verify harness src/main.rs) and to the LCG-seeded
q4 GEMV fixture rebuilt from src/main.rs:120-152."""
import json
import math
import os

import numpy as np
import pytest

from conftest import GOLDEN

KATS = json.load(open(os.path.join(GOLDEN, "reference_kats.json")))
TOL = KATS["verify_tol_abs"]["value"]


def test_f16_kats(orc):
    for h, v in KATS["f16_to_f32"]["cases"]:
        assert orc.f16_to_f32(h) == v


def test_f16_exhaustive_against_numpy(orc):
    # every f16 bit pattern: exact decode incl. subnormals/inf (dequant.rs:9-21)
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    raw = bits.view(np.uint8)
    got = orc.dequant_f16(raw, 65536)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))


def test_bf16_kats(orc):
    for h, v in KATS["bf16_to_f32"]["cases"]:
        assert orc.bf16_to_f32(h) == v


@pytest.mark.parametrize("name,fn,n", [("q8_0", "dequant_q8_0", 32), ("q4_1", "dequant_q4_1", 32),
                                       ("q6_k", "dequant_q6_k", 256), ("q4_0", "dequant_q4_0", 32)])
def test_block_kats(orc, name, fn, n):
    k = KATS[name]
    out = getattr(orc, fn)(np.array(k["block"], dtype=np.uint8), n)
    for idx, v in k["expect"].items():
        assert out[int(idx)] == v, (name, idx, out[int(idx)], v)


def test_q4_0_layout_semantics(orc):
    # low nibble -> element j, high nibble -> element j+16, value d*(q-8)
    rng = np.random.default_rng(3)
    blocks = np.zeros((64, 18), dtype=np.uint8)
    d = rng.uniform(0.002, 0.02, 64).astype(np.float16)
    blocks[:, :2] = d.view(np.uint8).reshape(64, 2)
    blocks[:, 2:] = rng.integers(0, 256, (64, 16), dtype=np.uint8)
    out = orc.dequant_q4_0(blocks.ravel(), 64 * 32).reshape(64, 32)
    lo = (blocks[:, 2:] & 0xF).astype(np.int32) - 8
    hi = (blocks[:, 2:] >> 4).astype(np.int32) - 8
    df = d.astype(np.float32)[:, None]
    assert np.array_equal(out[:, :16], df * lo.astype(np.float32))
    assert np.array_equal(out[:, 16:], df * hi.astype(np.float32))


def test_q4_gemv_fixture(orc):
    """src/main.rs:120-152: quantize_q4_0 of the LCG weights + dequant-and-dot."""
    import make_golden as mg  # noqa: E402  (tests/golden on sys.path below)
    z = np.load(os.path.join(GOLDEN, "q4_gemv_256x512.npz"))
    w = mg.lcg_fill(0x5678, 512 * 256)
    assert np.array_equal(mg.lcg_fill(0x1234, 256), z["x"])
    s, q = orc.quantize_q4_0(w, 512, 256)
    assert np.array_equal(s, z["scales"]) and np.array_equal(q, z["quants"])
    y = orc.q4_gemv(z["x"], z["scales"], z["quants"], 256, 512)
    assert np.array_equal(y.view(np.uint32), z["y"].view(np.uint32))
    # and the dense-mode path on the dequantised weights agrees within 1e-3
    deq = np.zeros(512 * 256, np.float32)
    nb = 256 // 32
    for o in range(512):
        for b in range(nb):
            dd = z["scales"][o * nb + b]
            for wd in range(4):
                word = int(z["quants"][o * 32 + b * 4 + wd])
                for n in range(8):
                    deq[o * 256 + b * 32 + wd * 8 + n] = dd * (((word >> (4 * n)) & 15) - 8)
    ref = deq.reshape(512, 256).astype(np.float64) @ z["x"].astype(np.float64)
    assert np.max(np.abs(y - ref)) < TOL


def test_quantize_rounding_edges(orc):
    # exact .5 ties round away from zero (Rust f32::round), all-zero block -> d=0, q=8
    w = np.zeros(64, np.float32)
    w[:32] = np.array([8.0, -8.0, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5] + [0.0] * 24, np.float32)
    s, q = orc.quantize_q4_0(w, 1, 64)
    assert s[0] == 1.0 and s[1] == 0.0
    nib = [(int(q[i // 8]) >> (4 * (i % 8))) & 15 for i in range(64)]
    assert nib[:8] == [15, 0, 9, 7, 10, 6, 11, 5]  # 8->clamp 15, -8->0, .5->1, -.5->-1 ...
    assert all(v == 8 for v in nib[32:])


def test_closed_form_kats(orc):
    eps = 1e-6
    y = orc.rmsnorm(np.ones(4 * 1024), np.ones(1024), 4, 1024, eps)
    assert np.max(np.abs(y - 1 / math.sqrt(1 + eps))) < TOL
    y = orc.rmsnorm(np.ones(4 * 1024), np.ones(1024), 4, 1024, eps, unit=True)
    assert np.max(np.abs(y - 2 / math.sqrt(1 + eps))) < TOL
    g, u = 1.5, -0.7
    out = orc.swiglu(np.full(4096, g), np.full(4096, u))
    assert np.max(np.abs(out - g / (1 + math.exp(-g)) * u)) < TOL
    c = 0.79788456
    out = orc.geglu(np.full(4096, g), np.full(4096, u))
    assert np.max(np.abs(out - 0.5 * g * (1 + math.tanh(c * (g + 0.044715 * g ** 3))) * u)) < TOL
    x = ((np.arange(16 * 128) % 23) - 11) * 0.07
    assert np.max(np.abs(orc.rope(x, 16, 128, 0, 10000.0) - x)) < TOL
    nh, nkv, hd = 4, 2, 16
    q = np.arange(nh * hd) * 0.01
    v = ((np.arange(nkv * hd) % 9) - 4) * 0.1
    out = orc.attention(q, np.full(nkv * hd, 0.5), v, nh, nkv, 1, hd)
    exp = np.concatenate([v[(h // (nh // nkv)) * hd:(h // (nh // nkv) + 1) * hd] for h in range(nh)])
    assert np.max(np.abs(out - exp)) < TOL
    a = np.arange(1000, dtype=np.float32)
    assert np.max(np.abs(orc.add(a, -a * 0.5) - (a - a * 0.5))) < TOL


def test_argmax_tie_rules(orc):
    x = np.array([1.0, 3.0, 3.0, -1.0], np.float32)
    assert orc.argmax(x) == 1  # lowest index on ties (argmax.wgsl:26,43)
    assert orc.argmax(np.array([np.nan, 2.0, np.nan], np.float32)) == 1
    assert orc.argmax(np.full(5, -np.inf, np.float32)) == 0
    assert orc.argmax(np.array([-0.0, 0.0], np.float32)) == 0


def test_attention_lanes_vs_softmax(orc):
    rng = np.random.default_rng(0)
    nh, nkv, hd, seq = 8, 2, 64, 77
    q = rng.normal(size=nh * hd)
    k = rng.normal(size=seq * nkv * hd)
    v = rng.normal(size=seq * nkv * hd)
    out = orc.attention(q, k, v, nh, nkv, seq, hd).reshape(nh, hd)
    K = k.reshape(seq, nkv, hd)
    V = v.reshape(seq, nkv, hd)
    for h in range(nh):
        g = h // (nh // nkv)
        s = (K[:, g, :] @ q[h * hd:(h + 1) * hd]) * hd ** -0.5
        p = np.exp(s - s.max())
        ref = (p[:, None] * V[:, g, :]).sum(0) / p.sum()
        assert np.max(np.abs(out[h] - ref)) < 1e-4


def test_attention_window_softcap(orc):
    rng = np.random.default_rng(1)
    nh, nkv, hd, seq, win, cap = 4, 2, 32, 50, 20, 5.0
    q, k, v = rng.normal(size=nh * hd), rng.normal(size=seq * nkv * hd), rng.normal(size=seq * nkv * hd)
    out = orc.attention(q, k, v, nh, nkv, seq, hd, softcap=cap, window=win).reshape(nh, hd)
    K, V = k.reshape(seq, nkv, hd), v.reshape(seq, nkv, hd)
    for h in range(nh):
        g = h // (nh // nkv)
        s = (K[seq - win:, g, :] @ q[h * hd:(h + 1) * hd]) * hd ** -0.5
        s = cap * np.tanh(s / cap)
        p = np.exp(s - s.max())
        ref = (p[:, None] * V[seq - win:, g, :]).sum(0) / p.sum()
        assert np.max(np.abs(out[h] - ref)) < 1e-4


def test_gguf_minimal_kat(orc, tmp_path):
    """src/loader/gguf.rs:219-251 through the Python reader and the writer."""
    from chat_wgpu_b200.gguf import GgufReader, GgufWriter, GGML_F32
    raw = bytes.fromhex(KATS["gguf_minimal"]["bytes_hex"])
    p = tmp_path / "min.gguf"
    p.write_bytes(raw)
    r = GgufReader(str(p))
    assert r.meta["qwen3.block_count"] == 28
    assert list(r.vector_f32("output_norm.weight")) == [1.0, 2.0, 3.0, 4.0]
    r.close()
    w = GgufWriter()
    w.meta["qwen3.block_count"] = 28
    w.add("output_norm.weight", GGML_F32, (4,), np.array([1, 2, 3, 4], np.float32))
    w.meta["general.alignment"] = 32
    q = tmp_path / "w.gguf"
    w.write(str(q))
    r2 = GgufReader(str(q))
    assert list(r2.vector_f32("output_norm.weight")) == [1.0, 2.0, 3.0, 4.0]
    r2.close()


import sys  # noqa: E402
sys.path.insert(0, GOLDEN)


def test_oracle_q4_k_q5_k_by_construction(orc):
    """Q4_K / Q5_K (ggml block layout, not in the reference): a block with
    d = 1, dmin = 0.5, 6-bit (scale, min) pairs (3, 2) for sub-blocks 0-3 and
    (5, 4) for 4-7, nibbles lo = 1, hi = 2 (and for Q5_K every fifth bit set
    on sub-block 0 only) dequantises to (d*sc)*q - dmin*m."""
    b = np.zeros(176, np.uint8)
    b[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    b[2:4] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    b[4:8], b[8:12], b[12:16] = 3, 2, 5 | (4 << 4)
    q4 = b[:144].copy()
    q4[16:] = 0x21
    y = orc.dequant_q4_k(q4, 256)
    assert (y[0], y[32], y[128], y[160]) == (2.0, 5.0, 3.0, 8.0)
    q5 = b.copy()
    q5[16:48] = 0x01            # fifth bit of sub-block 0 (chunk 0, low nibbles)
    q5[48:] = 0x21
    y5 = orc.dequant_q5_k(q5, 256)
    assert y5[0] == 3 * 17 - 1 and y5[32] == 5.0 and y5[64] == 3 * 1 - 1
