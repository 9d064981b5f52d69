"""Q4_0 GEMV microbenchmark -- the B200 counterpart of chat-wgpu's
examples/q4bench.rs: µs per launch and achieved HBM GB/s per projection
shape, kernel only (no model).

Each shape cycles through enough distinct weight copies (> 4x the L2 size)
that every launch streams its weight from HBM; the launches are replayed as
one CUDA graph and timed with CUDA events (cw_q4_0_gemv_bench).

    python -m chat_wgpu_b200.q4bench            # Qwen3 projection shape sweep
    python -m chat_wgpu_b200.q4bench --json
"""
from __future__ import annotations

import argparse
import ctypes as C
import json

import numpy as np

from . import _lib
from .context import GpuContext
from .gguf import random_q4_0_blocks
from .kernels import q4

# (in_f, out_f): Qwen3 0.6B/1.7B/4B/8B projections and LM heads
SHAPES = [(1024, 2048), (1024, 3072), (3072, 1024), (2048, 6144), (6144, 2048), (2560, 9728),
          (9728, 2560), (4096, 12288), (12288, 4096), (1024, 151936), (2048, 151936),
          (2560, 151936), (4096, 151936)]


def algorithmic_bytes(in_f: int, out_f: int) -> int:
    """N*K/32*18 (Q4_0 blocks) + 4K (x) + 4N (y)."""
    return out_f * (in_f // 32) * 18 + 4 * in_f + 4 * out_f


def bench_shape(ctx: GpuContext, in_f: int, out_f: int, iters: int = 200, seed: int = 0,
                l2_bytes: int = 126 << 20) -> dict:
    rng = np.random.default_rng(seed)
    wbytes = out_f * (in_f // 32) * 18
    n_w = max(2, min(512, -(-4 * l2_bytes // wbytes)))  # > 4x L2 (3.2x for K=1024, N=2048)
    blocks = random_q4_0_blocks(rng, out_f, in_f)
    ws = [q4.q4_0_upload(ctx, blocks, out_f, in_f) for _ in range(n_w)]
    x = ctx.storage(rng.normal(0, 1, in_f).astype(np.float32))
    arr = (C.c_uint64 * n_w)(*[w.handle for w in ws])
    us = C.c_double()
    iters = max(iters, n_w)
    _lib.call("cw_q4_0_gemv_bench", ctx.handle, x.handle, arr, n_w, in_f, out_f, iters, C.byref(us))
    for w in ws:
        w.release()
    nbytes = algorithmic_bytes(in_f, out_f)
    return {"in_f": in_f, "out_f": out_f, "us": us.value, "bytes": nbytes,
            "gbs": nbytes / (us.value * 1e-6) / 1e9, "copies": n_w}


KQ_TYPES = {"q4_k": (12, 144), "q5_k": (13, 176), "q6_k": (14, 210), "q8_0": (8, 272)}


def bench_kquant(ctx: GpuContext, qname: str, in_f: int, out_f: int, iters: int = 50,
                 seed: int = 0, l2_bytes: int = 126 << 20) -> dict:
    """k-quant GEMV (cw_kquant_gemv; Q6_K / Q8_0: cw_q6_k_gemv / cw_q8_0_gemv
    over the aligned split the model's decode step reads): device time per
    launch from the context
    profiler, cycling through copies that exceed 4x L2."""
    qtype, bb = KQ_TYPES[qname]
    rng = np.random.default_rng(seed)
    nb = out_f * (in_f // 256)
    wbytes = nb * bb
    raw = rng.integers(0, 256, nb * bb, dtype=np.uint8).reshape(nb, bb)
    if qtype == 8:  # 8 Q8_0 blocks of 34 bytes per 256 weights: every block's d
        for j in range(8):
            raw[:, 34 * j:34 * j + 2] = (rng.uniform(1e-3, 1e-2, nb).astype(np.float16)
                                         .view(np.uint8).reshape(nb, 2))
    else:
        off = 208 if qtype == 14 else 0
        raw[:, off:off + 2] = (rng.uniform(1e-3, 1e-2, nb).astype(np.float16)
                               .view(np.uint8).reshape(nb, 2))
    n_w = max(2, min(64, -(-4 * l2_bytes // wbytes)))
    ws = [ctx.storage_bytes(raw.ravel()) for _ in range(n_w)]
    if qtype in (8, 14):  # the split planes the decode projections stream
        sp, gv = (q4.q6_k_split, q4.q6_k_gemv) if qtype == 14 else (q4.q8_0_split, q4.q8_0_gemv)
        split = [sp(ctx, w, out_f, in_f) for w in ws]
        for w in ws:
            w.release()
        ws = split

        def gemv(w):
            return gv(ctx, x, w, in_f, out_f)
    else:
        def gemv(w):
            return q4.kquant_gemv(ctx, x, w, qtype, in_f, out_f)
    x = ctx.storage(rng.normal(0, 1, in_f).astype(np.float32))
    for w in ws[:2]:
        gemv(w)
        ctx.reset_frame()
    ctx.sync()
    ctx.begin_profile()
    for i in range(max(iters, n_w)):
        gemv(ws[i % n_w])
        ctx.reset_frame()
    rep = {name: ms / c for name, c, ms in ctx.report_profile()}
    for w in ws:
        w.release()
    us = 1e3 * rep["kquant_gemv"]
    nbytes = wbytes + 4 * in_f + 4 * out_f
    return {"type": qname, "in_f": in_f, "out_f": out_f, "us": us, "bytes": nbytes,
            "gbs": nbytes / (us * 1e-6) / 1e9}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--iters", type=int, default=200)
    ap.add_argument("--shape", default=None, help="one shape as IN_FxOUT_F, e.g. 1024x151936")
    ap.add_argument("--kquant", choices=sorted(KQ_TYPES), default=None,
                    help="time the k-quant GEMV of this type instead of Q4_0")
    args = ap.parse_args()
    shapes = SHAPES
    if args.shape:
        k, n = (int(v) for v in args.shape.lower().split("x"))
        shapes = [(k, n)]
    ctx = GpuContext(0)
    if args.kquant:
        rows = [bench_kquant(ctx, args.kquant, k, n) for k, n in shapes if k % 256 == 0]
    else:
        rows = [bench_shape(ctx, k, n, args.iters) for k, n in shapes]
    if args.json:
        print(json.dumps(rows))
    else:
        print(f"{'shape (in->out)':<18} {'us/pass':>9} {'GB/s':>9} {'bytes':>11}")
        for r in rows:
            print(f"{r['in_f']:>6}->{r['out_f']:<10} {r['us']:>9.2f} {r['gbs']:>9.1f} {r['bytes']:>11}")
    ctx.close()


if __name__ == "__main__":
    main()
