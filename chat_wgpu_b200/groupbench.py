"""Co-batched decode throughput (cw_group_*): B sessions of one model stepped
together, each after its own prompt (batched prefill), timed with CUDA events
over `--steps` group steps.

    python -m chat_wgpu_b200.groupbench [--model qwen3-0.6b] [--sessions 1 8 32]
                                        [--prompt-len 128] [--steps 32]

tok/s counts every session's produced token (B per step)."""
from __future__ import annotations

import argparse
import json

import numpy as np


def bench(model, B: int, prompt_len: int, steps: int, warmup: int = 3, seed: int = 0,
          profile: int = 0, streaming=None) -> dict:
    """streaming: None = the group's default projection path, True / False =
    streaming GEMVs / tensor-core GEMMs."""
    from .model import Session, SessionGroup
    rng = np.random.default_rng(seed + B)
    ss = []
    for _ in range(B):
        s = Session(model, prompt_len + warmup + steps + 4)
        s.begin(rng.integers(0, model.vocab_size, prompt_len).astype(np.uint32))
        s.prefill()
        ss.append(s)
    g = SessionGroup(ss)
    if streaming is not None:
        g.set_streaming(streaming)
    path = {1: "streaming GEMVs, integer-MMA products", 2: "streaming GEMVs, dp4a products",
            0: "tensor-core GEMMs"}[g.path]
    g.run(1 + warmup)  # the last prompt token (first produced token) + warm-up steps
    ms = g.run_timed(steps)
    produced = [len(s.tokens()) for s in ss]
    stages = None
    if profile:  # direct launches with an event pair per stage (not the timed graph)
        ctx = model.ctx
        ctx.sync()
        ctx.begin_profile()
        g.run(profile)
        stages = {}
        for name, count, t in ctx.report_profile():
            c0, t0 = stages.get(name, (0, 0.0))
            stages[name] = (c0 + count, t0 + t)
        stages = {k: (c // profile, t / profile) for k, (c, t) in stages.items()}
    g.close()
    for s in ss:
        s.close()
    assert all(p == 1 + warmup + steps for p in produced), produced
    return {"sessions": B, "steps": steps, "ms_per_step": ms / steps, "stages": stages,
            "path": path,
            "tok_s": B * steps / (ms / 1e3),
            "positions": f"{prompt_len + warmup}..{prompt_len + warmup + steps - 1}"}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--sessions", type=int, nargs="*", default=[1, 8, 32])
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--profile", type=int, default=0, metavar="STEPS",
                    help="also print a per-stage breakdown over STEPS direct-launch steps")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--path", choices=["auto", "streaming", "dp4a", "gemm"], default="auto",
                    help="projection path of the group step")
    a = ap.parse_args(argv)
    streaming = {"auto": None, "streaming": 1, "dp4a": 2, "gemm": 0}[a.path]
    from . import gguf
    from .context import GpuContext
    from .model import Model
    ctx = GpuContext(0)
    m = Model(ctx, gguf.cached_model(a.model))
    out = []
    for B in a.sessions:
        r = bench(m, B, a.prompt_len, a.steps, profile=a.profile, streaming=streaming)
        out.append(r)
        if not a.json:
            print(f"{a.model}: {B:4d} sessions  {r['ms_per_step']:.3f} ms/step  "
                  f"{r['tok_s']:9.0f} tok/s  (positions {r['positions']}, {r['path']})",
                  flush=True)
            for name, (c, t) in sorted((r["stages"] or {}).items(), key=lambda kv: -kv[1][1]):
                print(f"    {name:20s} {c:5d} launches/step  {t:8.3f} ms/step")
    if a.json:
        print(json.dumps(out))
    m.close()
    ctx.close()


if __name__ == "__main__":
    main()
