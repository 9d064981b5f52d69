"""Tensor-parallel decode latency (cw_model_load_gguf_tp): one process per GPU
under torchrun, each holding 1/N of the heads, FFN columns and LM-head rows;
the O / down partial sums and the argmax are all-reduced over NCCL inside
each step (captured in the step's CUDA graph).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m chat_wgpu_b200.tpbench [--model qwen3-8b] [--steps 64] [--check]

Rank 0 makes the NCCL id and shares it over a gloo group (host only); the
timed region is `--steps` greedy decode steps timed with CUDA events on each
rank, reported as the max over ranks.  `--check` also decodes the same prompt
on one GPU with the whole model and counts the tokens on which the streams
agree."""
from __future__ import annotations

import argparse
import json
import os

import numpy as np


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--check", action="store_true")
    a = ap.parse_args(argv)
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(minutes=10))
    from . import gguf
    from .context import GpuContext
    from .model import Model, Session, tp_unique_id
    if rank == 0:
        path = gguf.cached_model(a.model)  # written once, before the others read it
    dist.barrier()
    path = gguf.cached_model(a.model)
    ctx = GpuContext(local)
    box = [tp_unique_id() if rank == 0 and world > 1 else None]
    dist.broadcast_object_list(box, src=0)
    m = Model(ctx, path, tp=(rank, world, box[0] or bytes(128)))
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, m.vocab_size, a.prompt_len).astype(np.uint32)
    n_new = 1 + a.warmup + a.steps
    s = Session(m, a.prompt_len + n_new)
    s.begin(prompt)
    s.run(a.prompt_len - 1 + 1 + a.warmup)
    ms = s.run_timed(a.steps)
    toks = s.tokens()
    t = torch.tensor([ms], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    agree = None
    s.close()
    m.close()
    if a.check and rank == 0:
        full = Model(ctx, path)
        r = Session(full, a.prompt_len + n_new)
        r.begin(prompt)
        r.run(a.prompt_len - 1 + n_new)
        ref = r.tokens()
        agree = int(np.argmin(np.append(ref == toks, False)))
        r.close()
        full.close()
    if rank == 0:
        print(json.dumps({"model": a.model, "tp": world, "steps": a.steps,
                          "ms_per_token": ms / a.steps, "tok_s": a.steps / (ms / 1e3),
                          "positions": f"{a.prompt_len + a.warmup}..{a.prompt_len + n_new - 2}",
                          "tokens_agreeing_with_1gpu": agree, "of": len(toks)}), flush=True)
    ctx.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
