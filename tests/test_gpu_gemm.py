"""The tcgen05 prefill GEMM (cw_q4_0_gemm) against the CPU oracle.

Every output row must equal the reference's GEMV of the same activation row
(q4.wgsl:40-73 semantics, oracle orc_q4_0_gemv) within the north-star's 1e-3
relative gate; the weights are dequantised bit-exactly by the oracle and the
product is formed in f64 for the larger cases.  Shapes: the benchmark's prefill
sweep (the projection shapes at 128 and 512 rows), ragged M/N/K edges (a
partial 128-row tile, N not a multiple of the 128-wide tile, K with a
trailing half 64-wide K step) and activation extremes."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_ops import q4_0_blocks

pytestmark = pytest.mark.gpu
REL = 1e-3


def _ref(orc, x, blocks, rows, in_f, out_f):
    if rows <= 8:
        return np.stack([orc.q4_0_gemv(x[r], blocks, in_f, out_f) for r in range(rows)])
    w = orc.dequant_q4_0(blocks.ravel(), out_f * in_f).reshape(out_f, in_f).astype(np.float64)
    return (x.astype(np.float64) @ w.T)


def _run(ctx, orc, rows, in_f, out_f, seed, scale=1.0, zero_frac=0.01):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(seed)
    blocks = q4_0_blocks(rng, out_f, in_f, zero_frac=zero_frac)
    x = (rng.normal(0, 1, (rows, in_f)) * scale).astype(np.float32)
    w = q4.q4_0_upload(ctx, blocks, out_f, in_f)
    y = ctx.read(q4.q4_0_gemm(ctx, ctx.storage(x.ravel()), w, rows, in_f, out_f),
                 rows * out_f).reshape(rows, out_f)
    w.release()
    return y, _ref(orc, x, blocks, rows, in_f, out_f)


PREFILL = [(1024, 2048), (1024, 3072), (3072, 1024), (2048, 6144), (6144, 2048), (2560, 9728),
           (9728, 2560), (4096, 12288), (12288, 4096)]


@pytest.mark.parametrize("rows", [128, 512])
@pytest.mark.parametrize("in_f,out_f", PREFILL)
def test_gemm_prefill_sweep(ctx, orc, rows, in_f, out_f):
    y, ref = _run(ctx, orc, rows, in_f, out_f, seed=rows + in_f + 7 * out_f)
    for r in range(rows):
        assert rel_err(y[r], ref[r]) < REL, r


@pytest.mark.parametrize("rows,in_f,out_f", [(1, 1024, 3072), (3, 64, 128), (7, 96, 200),
                                              (130, 1024, 3072), (129, 160, 129),
                                              (256, 32, 1), (200, 2304, 2048)])
def test_gemm_ragged(ctx, orc, rows, in_f, out_f):
    y, ref = _run(ctx, orc, rows, in_f, out_f, seed=rows * 31 + in_f + out_f)
    for r in range(rows):
        assert rel_err(y[r], ref[r]) < REL, r


@pytest.mark.parametrize("scale", [1e-3, 30.0, 3000.0])
def test_gemm_activation_range(ctx, orc, scale):
    """Tiny and large activations keep both f16 halves in range."""
    y, ref = _run(ctx, orc, 64, 1024, 512, seed=11, scale=scale)
    for r in range(64):
        assert rel_err(y[r], ref[r]) < REL, r


def test_gemm_rejects_bad_shapes(ctx):
    from chat_wgpu_b200 import _lib
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(0)
    w = q4.q4_0_upload(ctx, q4_0_blocks(rng, 8, 64), 8, 64)
    x = ctx.storage(np.ones(4 * 64, np.float32))
    with pytest.raises(_lib.CwError):
        q4.q4_0_gemm(ctx, x, w, 4, 64, 9)     # wrong rows of W
    with pytest.raises(_lib.CwError):
        q4.q4_0_gemm(ctx, x, w, 5, 64, 8)     # x too short
    w.release()
