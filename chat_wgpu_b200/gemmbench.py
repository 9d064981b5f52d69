"""Prefill Q4_0 GEMM microbenchmark (cw_q4_0_gemm on the tcgen05 tensor
cores): per shape and row count, device time of each phase from the context
profiler (CUDA events around the launches) and the achieved TFLOP/s.

Algorithmic work is 2*M*N*K flops (the product the reference's token-by-
token GEMVs would form); the kernel itself issues three f16 MMAs per K step
(the hi/lo operand split), so its tensor-pipe work is 3x that.

    python -m chat_wgpu_b200.gemmbench                # prefill sweep, M = 128, 512
    python -m chat_wgpu_b200.gemmbench --rows 4096 --json
    python -m chat_wgpu_b200.gemmbench --rows 4096 --shape 4096 12288 --iters 2
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from .context import GpuContext
from .gguf import random_q4_0_blocks
from .kernels import q4

SHAPES = [(1024, 2048), (1024, 3072), (3072, 1024), (2048, 6144), (6144, 2048), (2560, 9728),
          (9728, 2560), (4096, 12288), (12288, 4096)]


def bench(ctx: GpuContext, rows: int, in_f: int, out_f: int, iters: int = 10, seed: int = 0):
    rng = np.random.default_rng(seed)
    w = q4.q4_0_upload(ctx, random_q4_0_blocks(rng, out_f, in_f), out_f, in_f)
    x = ctx.storage(rng.normal(0, 1, rows * in_f).astype(np.float32))
    for _ in range(3):
        q4.q4_0_gemm(ctx, x, w, rows, in_f, out_f)
        ctx.reset_frame()
    ctx.sync()
    ctx.begin_profile()
    for _ in range(iters):
        q4.q4_0_gemm(ctx, x, w, rows, in_f, out_f)
        ctx.reset_frame()
    rep = {name: ms / count for name, count, ms in ctx.report_profile()}
    w.release()
    x.release()
    flops = 2.0 * rows * in_f * out_f
    mma_ms = rep.get("q4_gemm.mma", float("nan"))
    return {"rows": rows, "in_f": in_f, "out_f": out_f,
            "us_total": 1e3 * rep.get("q4_gemm", float("nan")),
            "us_split_x": 1e3 * rep.get("q4_gemm.split_x", float("nan")),
            "us_prep_w": 1e3 * rep.get("q4_gemm.prep_w", float("nan")),
            "us_mma": 1e3 * mma_ms,
            "tflops_mma": flops / (mma_ms * 1e-3) / 1e12,
            "tflops_pipe": 3 * flops / (mma_ms * 1e-3) / 1e12,
            "tflops_total": flops / (rep.get("q4_gemm", float("nan")) * 1e-3) / 1e12}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--rows", type=int, nargs="*", default=[128, 512])
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--shape", type=int, nargs=2, metavar=("K", "N"),
                    help="one (in_f, out_f) shape instead of the sweep")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    shapes = [tuple(a.shape)] if a.shape else SHAPES
    ctx = GpuContext(0)
    out = []
    for rows in a.rows:
        for in_f, out_f in shapes:
            r = bench(ctx, rows, in_f, out_f, a.iters)
            out.append(r)
            if not a.json:
                print(f"M={rows:5d} K={in_f:6d} N={out_f:6d}  total {r['us_total']:9.1f} us  "
                      f"split_x {r['us_split_x']:7.1f}  prep_w {r['us_prep_w']:7.1f}  "
                      f"mma {r['us_mma']:9.1f} us  {r['tflops_mma']:7.1f} TFLOP/s "
                      f"(pipe {r['tflops_pipe']:7.1f})", flush=True)
    if a.json:
        print(json.dumps(out))
    ctx.close()


if __name__ == "__main__":
    main()
