"""Batched-prefill timing: per-stage device time of cw_session_prefill (CUDA
events from the context profiler), prefill tokens/s, and the tensor-core
GEMMs' achieved TFLOP/s.

    python -m chat_wgpu_b200.prefillprof [--model qwen3-0.6b] [--prompt-len 128] [--reps 3]

Algorithmic GEMM work per prompt row is 2 * (sum of the projection sizes) of
every layer but the last, plus the last layer's QKV projection (prefill
stops there, see cw_prefill.cu); the GEMM kernel's tensor-pipe work is 3x
that (f16 hi/lo operand split)."""
from __future__ import annotations

import argparse

import numpy as np


def gemm_flops_per_row(info: dict) -> float:
    dim, hd, nh, nkv, hid = (info[k] for k in ("dim", "head_dim", "n_heads", "n_kv", "hidden"))
    qd, kvd = nh * hd, nkv * hd
    qkv = (qd + 2 * kvd) * dim
    layer = qkv + dim * qd + 2 * hid * dim + dim * hid
    return 2.0 * (layer * (info["n_layers"] - 1) + qkv)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    from . import gguf
    from .context import GpuContext
    from .model import Model, Session

    path = gguf.cached_model(a.model, seed=a.seed)
    ctx = GpuContext(0)
    m = Model(ctx, path)
    s = Session(m, a.prompt_len + 8)
    prompt = np.random.default_rng(a.seed + 1).integers(0, m.vocab_size, a.prompt_len)
    prompt = prompt.astype(np.uint32)
    s.begin(prompt)
    s.prefill()  # warm-up: scratch allocation, tensor maps, module load
    ctx.sync()
    ctx.begin_profile()
    for _ in range(a.reps):
        s.begin(prompt)
        s.prefill()
    rows = ctx.report_profile()
    agg = {}
    for name, count, ms in rows:
        if name.startswith("prefill."):
            c, t = agg.get(name, (0, 0.0))
            agg[name] = (c + count, t + ms)
    total = sum(t for _, t in agg.values()) / a.reps
    n = a.prompt_len - 1
    gemm_ms = agg.get("prefill.gemm", (0, float("nan")))[1] / a.reps
    fl = gemm_flops_per_row(m.info) * n
    print(f"{a.model}: prefill of {n} positions: {total:.3f} ms device time, "
          f"{n / total * 1e3:.0f} tok/s; GEMMs {gemm_ms:.3f} ms = {fl / gemm_ms / 1e9:.1f} "
          f"TFLOP/s algorithmic ({3 * fl / gemm_ms / 1e9:.1f} tensor-pipe)")
    print(f"{'stage':20s} {'launches':>9s} {'ms/prefill':>11s} {'share':>7s}")
    for name, (count, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        print(f"{name:20s} {count // a.reps:9d} {t / a.reps:11.3f} {t / a.reps / total:7.1%}")
    s.close()
    m.close()
    ctx.close()


if __name__ == "__main__":
    main()
