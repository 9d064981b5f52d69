"""Per-op parity of the CUDA kernels (through the C-ABI, via the Python
mirror of the reference's op wrappers) against the CPU oracle and the
reference's known-answer tests.

Tolerances: integer/byte work (quantise, pack, dequantise, argmax) is
bit-exact; floating-point ops must agree within 1e-3 relative (rel_err in
conftest.py), the north-star's gate; the reference's own verify checks use
1e-3 absolute (src/main.rs:268-273) and are applied as such."""
import json
import math
import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu
REL = 1e-3
KATS = json.load(open(os.path.join(GOLDEN, "reference_kats.json")))


def q4_0_blocks(rng, rows, in_f, zero_frac=0.0):
    nb = rows * (in_f // 32)
    b = np.empty((nb, 18), np.uint8)
    d = rng.uniform(0.002, 0.02, nb).astype(np.float16)
    if zero_frac:
        d[rng.random(nb) < zero_frac] = 0
    b[:, :2] = d.view(np.uint8).reshape(nb, 2)
    b[:, 2:] = rng.integers(0, 256, (nb, 16), dtype=np.uint8)
    return b


# ---------------------------------------------------------------- verify KATs
def test_verify_kats(ctx):
    """The closed-form checks of the reference's verify harness, src/main.rs:61-161."""
    from chat_wgpu_b200.kernels import activation, attention, norm, rope
    eps = 1e-6
    ones = ctx.storage(np.ones(4 * 1024))
    w1 = ctx.storage(np.ones(1024))
    y = ctx.read(norm.rmsnorm(ctx, ones, w1, 4, 1024, eps), 4096)
    assert np.max(np.abs(y - 1 / math.sqrt(1 + eps))) < 1e-3
    y = ctx.read(norm.rmsnorm_unit(ctx, ones, w1, 4, 1024, eps), 4096)
    assert np.max(np.abs(y - 2 / math.sqrt(1 + eps))) < 1e-3
    g, u = 1.5, -0.7
    G, U = ctx.storage(np.full(4096, g)), ctx.storage(np.full(4096, u))
    y = ctx.read(activation.swiglu(ctx, G, U, 4096), 4096)
    assert np.max(np.abs(y - g / (1 + math.exp(-g)) * u)) < 1e-3
    c = 0.79788456
    y = ctx.read(activation.geglu(ctx, G, U, 4096), 4096)
    assert np.max(np.abs(y - 0.5 * g * (1 + math.tanh(c * (g + 0.044715 * g ** 3))) * u)) < 1e-3
    x = ((np.arange(16 * 128) % 23) - 11) * 0.07
    y = ctx.read(rope.rope(ctx, ctx.storage(x), 16, 128, 0, 10000.0), 16 * 128)
    assert np.max(np.abs(y - x)) < 1e-3
    nh, nkv, hd = 4, 2, 16
    q = np.arange(nh * hd) * 0.01
    v = ((np.arange(nkv * hd) % 9) - 4) * 0.1
    out = ctx.read(attention.attention(ctx, ctx.storage(q), ctx.storage(np.full(nkv * hd, 0.5)),
                                       ctx.storage(v), nh, nkv, 1, hd), nh * hd)
    exp = np.concatenate([v[(h // 2) * hd:(h // 2 + 1) * hd] for h in range(nh)])
    assert np.max(np.abs(out - exp)) < 1e-3
    a = np.arange(1000, dtype=np.float32)
    y = ctx.read(attention.add(ctx, ctx.storage(a), ctx.storage(-a * 0.5), 1000), 1000)
    assert np.max(np.abs(y - (a - a * 0.5))) < 1e-3


def test_q4_gemv_reference_fixture(ctx):
    """q4::gemv on the LCG fixture of src/main.rs:120-152 (crate layout)."""
    from chat_wgpu_b200.kernels import q4
    z = np.load(os.path.join(GOLDEN, "q4_gemv_256x512.npz"))
    y = ctx.read(q4.gemv(ctx, ctx.storage(z["x"]), ctx.storage(z["scales"]),
                         ctx.storage_u32(z["quants"]), 256, 512), 512)
    assert np.max(np.abs(y - z["y"])) < 1e-3
    assert rel_err(y, z["y"]) < REL


# ---------------------------------------------------------------- q4 family
def test_quantize_bit_exact(ctx, orc):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(11)
    for out_f, in_f in [(1, 32), (7, 64), (512, 256), (300, 1024)]:
        w = rng.normal(0, 0.05, out_f * in_f).astype(np.float32)
        w[:32] = 0.0  # an all-zero block
        if w.size >= 64:
            w[32] = 8.0  # block max 8 -> d = 1, so the values below are exact .5 ties
            w[40:48] = np.float32(0.5) * (1 + 2 * (np.arange(8) % 4)) * np.where(np.arange(8) % 2, -1, 1)
        s_ref, q_ref = orc.quantize_q4_0(w, out_f, in_f)
        sb, qb = q4.quantize_q4_0(ctx, ctx.storage(w), out_f, in_f)
        s = ctx.read(sb, s_ref.size)
        q = ctx.read_u32(qb, q_ref.size)
        assert np.array_equal(s.view(np.uint32), s_ref.view(np.uint32))
        assert np.array_equal(q, q_ref)


@pytest.mark.parametrize("in_f,out_f", [(256, 512), (32, 1), (64, 7), (1024, 3072), (3072, 1024),
                                        (2048, 1000)])
def test_q4_gemv_crate_layout(ctx, orc, in_f, out_f):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(in_f * 7 + out_f)
    w = rng.normal(0, 0.05, out_f * in_f).astype(np.float32)
    x = rng.normal(0, 1, in_f).astype(np.float32)
    s, q = orc.quantize_q4_0(w, out_f, in_f)
    y_ref = orc.q4_gemv(x, s, q, in_f, out_f)
    y = ctx.read(q4.gemv(ctx, ctx.storage(x), ctx.storage(s), ctx.storage_u32(q), in_f, out_f), out_f)
    assert rel_err(y, y_ref) < REL


def test_q4_0_pack_dequant_bit_exact(ctx, orc):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(5)
    for rows, in_f in [(1, 32), (13, 96), (256, 1024)]:
        blocks = q4_0_blocks(rng, rows, in_f, zero_frac=0.1)
        # special scales: subnormal, -0, max f16
        dd = blocks[:, :2].copy().view(np.float16).ravel()
        k = min(3, dd.size)
        dd[:k] = np.array([6e-8, -0.0, 65504.0], np.float16)[:k]
        blocks[:, :2] = dd.view(np.uint8).reshape(-1, 2)
        ref = orc.dequant_q4_0(blocks.ravel(), rows * in_f)
        w = q4.q4_0_upload(ctx, blocks, rows, in_f)
        got = ctx.read(q4.q4_0_dequant(ctx, w, rows, in_f), rows * in_f)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        # device-side pack of device-resident GGUF blocks gives the same weight
        w2 = q4.q4_0_pack(ctx, ctx.storage_bytes(blocks), rows, in_f)
        got2 = ctx.read(q4.q4_0_dequant(ctx, w2, rows, in_f), rows * in_f)
        assert np.array_equal(got2.view(np.uint32), ref.view(np.uint32))


SWEEP = [(1024, 2048), (1024, 3072), (3072, 1024), (2048, 6144), (6144, 2048), (2560, 9728),
         (9728, 2560), (4096, 12288), (12288, 4096), (1024, 151936)]


@pytest.mark.parametrize("in_f,out_f", SWEEP + [(32, 1), (64, 3), (96, 17), (256, 513)])
def test_q4_0_gemv_vs_oracle(ctx, orc, in_f, out_f):
    """GGUF Q4_0 GEMV over the benchmark shape sweep and ragged edge shapes."""
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(in_f + 3 * out_f)
    blocks = q4_0_blocks(rng, out_f, in_f, zero_frac=0.01)
    x = rng.normal(0, 1, in_f).astype(np.float32)
    y_ref = orc.q4_0_gemv(x, blocks, in_f, out_f)
    w = q4.q4_0_upload(ctx, blocks, out_f, in_f)
    y = ctx.read(q4.q4_0_gemv(ctx, ctx.storage(x), w, in_f, out_f), out_f)
    assert rel_err(y, y_ref) < REL
    w.release()


def test_q4_0_gemv_activation_edges(ctx, orc):
    """x with zero blocks, huge dynamic range and large magnitudes: the error stays at
    f32-accumulation grade relative to sum_k |w_k x_k|.  (Subnormal activations are
    not gated: their products are implementation-defined in the reference too,
    where WGSL may flush subnormals to zero.)"""
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(9)
    in_f, out_f = 512, 300
    blocks = q4_0_blocks(rng, out_f, in_f)
    w = q4.q4_0_upload(ctx, blocks, out_f, in_f)
    xs = [np.zeros(in_f, np.float32),
          np.concatenate([np.zeros(32), rng.normal(0, 1, in_f - 32)]).astype(np.float32),
          (rng.normal(0, 1, in_f) * np.exp(rng.uniform(-20, 20, in_f))).astype(np.float32),
          rng.normal(0, 1e4, in_f).astype(np.float32)]
    for x in xs:
        y_ref = orc.q4_0_gemv(x, blocks, in_f, out_f)
        y = ctx.read(q4.q4_0_gemv(ctx, ctx.storage(x), w, in_f, out_f), out_f)
        # absolute floor relative to the sum of |terms| for cancellation-heavy rows
        deq = orc.dequant_q4_0(blocks.ravel(), in_f * out_f).reshape(out_f, in_f)
        scale = np.abs(deq) @ np.abs(x).astype(np.float64) + 1e-30
        assert np.max(np.abs(y - y_ref) / scale) < 1e-4


def test_q4_0_gemv_rejects_bad_shapes(ctx):
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(1)
    w = q4.q4_0_upload(ctx, q4_0_blocks(rng, 4, 64), 4, 64)
    with pytest.raises(CwError):
        q4.q4_0_gemv(ctx, ctx.storage(np.ones(64)), w, 64, 5)   # wrong rows
    with pytest.raises(CwError):
        q4.q4_0_gemv(ctx, ctx.storage(np.ones(16)), w, 64, 4)   # x too short
    with pytest.raises(CwError):
        q4.gemv(ctx, ctx.storage(np.ones(40)), ctx.storage(np.ones(4)), ctx.storage_u32(np.ones(20)),
                40, 4)  # in_f not a multiple of 32


# ---------------------------------------------------------------- other ops
@pytest.mark.parametrize("rows,dim", [(1, 1024), (16, 128), (8, 128), (1, 2304), (3, 100)])
def test_rmsnorm(ctx, orc, rows, dim):
    from chat_wgpu_b200.kernels import norm
    rng = np.random.default_rng(rows * dim)
    x = rng.normal(0, 3, rows * dim).astype(np.float32)
    w = rng.normal(1, 0.02, dim).astype(np.float32)
    for unit, fn in [(False, norm.rmsnorm), (True, norm.rmsnorm_unit)]:
        y = ctx.read(fn(ctx, ctx.storage(x), ctx.storage(w), rows, dim, 1e-6), rows * dim)
        assert rel_err(y, orc.rmsnorm(x, w, rows, dim, 1e-6, unit)) < REL


@pytest.mark.parametrize("pos,theta", [(0, 1e6), (1, 1e6), (383, 1e6), (4607, 1e6), (767, 1e4)])
def test_rope(ctx, orc, pos, theta):
    from chat_wgpu_b200.kernels import rope
    rng = np.random.default_rng(pos)
    for rows, hd in [(16, 128), (8, 256)]:
        x = rng.normal(0, 1, rows * hd).astype(np.float32)
        y = ctx.read(rope.rope(ctx, ctx.storage(x), rows, hd, pos, theta), rows * hd)
        assert rel_err(y, orc.rope(x, rows, hd, pos, theta)) < REL


@pytest.mark.parametrize("nh,nkv,hd,seq", [(4, 2, 16, 1), (16, 8, 128, 1), (16, 8, 128, 7),
                                           (16, 8, 128, 384), (32, 8, 128, 4608), (8, 4, 256, 768),
                                           (4, 4, 64, 1000), (8, 1, 128, 300), (2, 2, 40, 33)])
def test_attention(ctx, orc, nh, nkv, hd, seq):
    from chat_wgpu_b200.kernels import attention
    rng = np.random.default_rng(seq + hd)
    q = rng.normal(0, 1, nh * hd).astype(np.float32)
    k = rng.normal(0, 1, seq * nkv * hd).astype(np.float32)
    v = rng.normal(0, 1, seq * nkv * hd).astype(np.float32)
    out = ctx.read(attention.attention(ctx, ctx.storage(q), ctx.storage(k), ctx.storage(v), nh, nkv,
                                       seq, hd), nh * hd)
    assert rel_err(out, orc.attention(q, k, v, nh, nkv, seq, hd)) < REL


@pytest.mark.parametrize("seq,window,cap", [(100, 40, 50.0), (768, 4096, 50.0), (600, 128, 0.0)])
def test_attention_softcap_window(ctx, orc, seq, window, cap):
    from chat_wgpu_b200.kernels import attention
    rng = np.random.default_rng(seq)
    nh, nkv, hd = 8, 4, 256
    q = rng.normal(0, 3, nh * hd).astype(np.float32)
    k = rng.normal(0, 1, seq * nkv * hd).astype(np.float32)
    v = rng.normal(0, 1, seq * nkv * hd).astype(np.float32)
    out = ctx.read(attention.attention(ctx, ctx.storage(q), ctx.storage(k), ctx.storage(v), nh, nkv,
                                       seq, hd, softcap=cap, window=window), nh * hd)
    assert rel_err(out, orc.attention(q, k, v, nh, nkv, seq, hd, softcap=cap, window=window)) < REL


def test_add_glu(ctx, orc):
    from chat_wgpu_b200.kernels import activation, attention
    rng = np.random.default_rng(2)
    for n in [1, 1000, 3072, 12288]:
        a = rng.normal(0, 4, n).astype(np.float32)
        b = rng.normal(0, 4, n).astype(np.float32)
        A, B = ctx.storage(a), ctx.storage(b)
        assert np.array_equal(ctx.read(attention.add(ctx, A, B, n), n), orc.add(a, b))
        assert rel_err(ctx.read(activation.swiglu(ctx, A, B, n), n), orc.swiglu(a, b)) < REL
        assert rel_err(ctx.read(activation.geglu(ctx, A, B, n), n), orc.geglu(a, b)) < REL


def test_argmax(ctx, orc):
    from chat_wgpu_b200.kernels import argmax
    rng = np.random.default_rng(4)
    cases = [rng.normal(size=151936).astype(np.float32),
             np.array([1.0, 3.0, 3.0, -1.0], np.float32),
             np.array([np.nan, 2.0, np.nan], np.float32),
             np.full(5, -np.inf, np.float32),
             np.array([-0.0, 0.0, -0.0], np.float32),
             np.full(256000, 7.0, np.float32)]
    big = rng.normal(size=256000).astype(np.float32)
    big[[1000, 200000]] = 99.0  # tie far apart -> lowest index
    cases.append(big)
    for x in cases:
        got = int(ctx.read_u32(argmax.argmax(ctx, ctx.storage(x), x.size), 1)[0])
        assert got == orc.argmax(x), (x[:4], got)


def test_arena_and_profiler(ctx):
    """empty() slots repeat per frame (context.rs:207-227); report_profile rows."""
    from chat_wgpu_b200.kernels import attention
    ctx.clear_cache()
    a = ctx.storage(np.ones(64))
    ctx.reset_frame()
    h1 = attention.add(ctx, a, a, 64).handle
    ctx.reset_frame()
    h2 = attention.add(ctx, a, a, 64).handle
    assert h1 == h2
    ctx.begin_profile()
    for _ in range(3):
        ctx.reset_frame()
        attention.add(ctx, a, a, 64)
    ctx.sync()
    rows = ctx.report_profile()
    assert rows and rows[0][0] == "ewise_add" and rows[0][1] == 3
