"""GGUF k-quant GEMV and dequantisation (cw_kquant_*) against the oracle.

Q6_K is the reference's own format (src/loader/dequant.rs:102-131, KAT
q6_k_zero_quants at :175-188); Q4_K / Q5_K are restated from ggml's
published layout (the reference lists them on ROADMAP.md:52-53).  Gates:
dequantisation bit-exact; GEMV within the north-star's 1e-3 relative."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
REL = 1e-3
Q4_K, Q5_K, Q6_K = 12, 13, 14
BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}


def kq_blocks(rng, qtype, rows, in_f):
    nb = rows * (in_f // 256)
    b = rng.integers(0, 256, (nb, BYTES[qtype]), dtype=np.uint8)
    if qtype == Q6_K:
        b[:, 192:208] = rng.integers(-64, 64, (nb, 16)).astype(np.int8).view(np.uint8)
        b[:, 208:210] = rng.uniform(5e-4, 2e-3, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    else:
        b[:, 0:2] = rng.uniform(1e-3, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
        b[:, 2:4] = rng.uniform(0, 1e-2, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b


def _deq(orc, qtype, raw, n):
    return {Q4_K: orc.dequant_q4_k, Q5_K: orc.dequant_q5_k, Q6_K: orc.dequant_q6_k}[qtype](raw, n)


@pytest.mark.parametrize("qtype", [Q4_K, Q5_K, Q6_K])
def test_kquant_dequant_bit_exact(ctx, orc, qtype):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(qtype)
    rows, in_f = 37, 1024
    raw = kq_blocks(rng, qtype, rows, in_f)
    w = ctx.storage_bytes(raw.ravel())
    got = ctx.read(q4.kquant_dequant(ctx, w, qtype, rows, in_f), rows * in_f)
    ref = _deq(orc, qtype, raw.ravel(), rows * in_f)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q6_k_reference_kat(ctx, orc):
    """dequant.rs:175-188: all quants 0, int8 scales 1, d = 1 -> every value -32."""
    from chat_wgpu_b200.kernels import q4
    b = np.zeros(210, np.uint8)
    b[192:208] = 1
    b[208], b[209] = 0x00, 0x3C
    w = ctx.storage_bytes(b)
    got = ctx.read(q4.kquant_dequant(ctx, w, Q6_K, 1, 256), 256)
    assert got[0] == -32.0 and got[255] == -32.0 and np.all(got == -32.0)
    assert np.array_equal(orc.dequant_q6_k(b, 256), got)


SHAPES = [(1024, 2048), (1024, 3072), (3072, 1024), (2048, 6144), (6144, 2048), (2560, 9728),
          (9728, 2560), (4096, 12288), (12288, 4096), (256, 1), (512, 77)]


@pytest.mark.parametrize("qtype", [Q4_K, Q5_K, Q6_K])
@pytest.mark.parametrize("in_f,out_f", SHAPES)
def test_kquant_gemv_vs_oracle(ctx, orc, qtype, in_f, out_f):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(in_f + 7 * out_f + qtype)
    raw = kq_blocks(rng, qtype, out_f, in_f)
    x = rng.normal(0, 1, in_f).astype(np.float32)
    w = ctx.storage_bytes(raw.ravel())
    y = ctx.read(q4.kquant_gemv(ctx, ctx.storage(x), w, qtype, in_f, out_f), out_f)
    W = _deq(orc, qtype, raw.ravel(), out_f * in_f).reshape(out_f, in_f).astype(np.float64)
    assert rel_err(y, W @ x.astype(np.float64)) < REL
    w.release()


@pytest.mark.parametrize("in_f,out_f", SHAPES)
def test_q6_k_split_gemv_vs_oracle(ctx, orc, in_f, out_f):
    """The streaming GEMV over the aligned Q6_K split (the decode step's form)
    against the oracle's dequant_q6_k product and the per-row kernel."""
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(3 * in_f + out_f)
    raw = kq_blocks(rng, Q6_K, out_f, in_f)
    x = rng.normal(0, 1, in_f).astype(np.float32)
    w = ctx.storage_bytes(raw.ravel())
    ws = q4.q6_k_split(ctx, w, out_f, in_f)
    xb = ctx.storage(x)
    W = orc.dequant_q6_k(raw.ravel(), out_f * in_f).reshape(out_f, in_f).astype(np.float64)
    y = ctx.read(q4.q6_k_gemv(ctx, xb, ws, in_f, out_f), out_f)
    assert rel_err(y, W @ x.astype(np.float64)) < REL
    # the per-row kernel over the raw blocks agrees too
    y2 = ctx.read(q4.kquant_gemv(ctx, xb, w, Q6_K, in_f, out_f), out_f)
    assert rel_err(y, y2.astype(np.float64)) < REL
    with pytest.raises(CwError):  # a raw weight is not a split one
        q4.q6_k_gemv(ctx, xb, w, in_f, out_f)
    ws.release()
    w.release()


def test_q6_k_gemv_refuses_unaligned_chunks(ctx):
    """in_f = 6400: 25 super-blocks per row, 4 rows per chunk -> a chunk's d
    values would start 8 bytes off a 16-byte boundary; refused, not run."""
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(5)
    raw = kq_blocks(rng, Q6_K, 8, 6400)
    w = ctx.storage_bytes(raw.ravel())
    ws = q4.q6_k_split(ctx, w, 8, 6400)
    with pytest.raises(CwError):
        q4.q6_k_gemv(ctx, ctx.storage(np.ones(6400, np.float32)), ws, 6400, 8)
    ws.release()
    w.release()


def test_kquant_rejects_bad_shapes(ctx):
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.kernels import q4
    w = ctx.storage_bytes(np.zeros(144 * 4, np.uint8))
    x = ctx.storage(np.ones(512, np.float32))
    with pytest.raises(CwError):
        q4.kquant_gemv(ctx, x, w, Q4_K, 500, 2)    # in_f not a multiple of 256
    with pytest.raises(CwError):
        q4.kquant_gemv(ctx, x, w, Q4_K, 512, 3)    # weight too short
    with pytest.raises(CwError):
        q4.kquant_gemv(ctx, x, w, 7, 512, 2)       # unknown type
