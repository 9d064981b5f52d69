"""Per-stage device-time breakdown of the decode step (the reference's
WGPU_PROFILE report, src/model/mod.rs:74-88, src/profile.rs:86-117).

    python -m chat_wgpu_b200.stepprof [--model qwen3-0.6b] [--prompt-len 128]
                                      [--steps 16] [--path auto|split|per-stage]

Runs the prompt, a few warm-up decode steps, times `--steps` decode steps
with CUDA events, then prints Session.profile(): for the persistent step,
per stage the span from its first CTA's start to its last CTA's end, the
grid-barrier gaps and the layer timeline (in-kernel %globaltimer stamps);
for the per-stage path, CUDA-event time per kernel."""
from __future__ import annotations

import argparse

import numpy as np


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--steps", type=int, default=16)
    ap.add_argument("--path", choices=["auto", "split", "per-stage"], default="auto")
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    from . import gguf
    from .context import GpuContext
    from .model import Model, Session

    path = gguf.cached_model(a.model, seed=a.seed)
    ctx = GpuContext(0)
    m = Model(ctx, path)
    s = Session(m, a.prompt_len + 3 * a.steps + 8)
    if a.path != "auto":
        s.set_persistent({"split": "split", "per-stage": False}[a.path])
    rng = np.random.default_rng(a.seed + 1)
    s.begin(rng.integers(0, m.vocab_size, a.prompt_len).astype(np.uint32))
    s.run(a.prompt_len - 1 + 4)
    ms = s.run_timed(a.steps)
    print(f"{a.model}: {ms / a.steps:.4f} ms/step over {a.steps} steps "
          f"({'persistent' if s.persistent else 'per-stage kernels'})")
    rows = s.profile(a.steps)
    timeline = [r for r in rows if "@" in r[0]]
    print(f"{'stage':28s} {'count':>6s} {'us each':>9s} {'us/step':>9s}")
    for name, count, total in sorted((r for r in rows if "@" not in r[0]), key=lambda r: -r[2]):
        print(f"{name:28s} {count:6d} {1000 * total / count:9.3f} {1000 * total / a.steps:9.2f}")
    if timeline:  # persistent step: mean offsets within a layer
        print("layer timeline (us from the first start of the layer's QKV stage; mean)")
        for name, count, total in sorted(timeline, key=lambda r: r[2] / r[1]):
            print(f"  {name:26s} {1000 * total / count:9.3f}")
    s.close()
    m.close()
    ctx.close()


if __name__ == "__main__":
    main()
