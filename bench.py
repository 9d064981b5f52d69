#!/usr/bin/env python
"""Decode throughput of the B200 build of chat-wgpu's batch-1 decode loop.

Workload (benchmark config 3, the one the headline metric is quoted on): Qwen3-0.6B
shape, random-init GGUF Q4_0 weights (seeded; there are no real checkpoints
on this machine), a 128-token uniform-random prompt, then greedy decode at
batch 1 with an f32 KV cache.  One "step" is one decode token: embed ->
28 layers -> lm_head -> argmax -> next input, as one CUDA-graph replay.

  value     decode tok/s (all ranks), device-timed with CUDA events around K
            back-to-back steps whose inputs live in HBM (weights 335 MB > L2)
  e2e       the same through Session.step(): per token a 4-byte H2D copy of
            the input token from pinned memory and a 4-byte D2H read of the
            produced token (the reference's ctx.read per token, mod.rs:103)
  roofline  the dominant kernel from a per-kernel CUDA-event profile pass
  cpu_baseline  the oracle port on the host cores (bounded sample)

Multi-GPU: one process per GPU, one independent model replica and session
per rank (sessions shard with no collective; weak scaling).  torch.distributed
is used only for the barrier and the max-over-ranks of the timings.

`--impl reference` times the reference's CPU implementation of this path
(the oracle port: the Rust/wgpu reference cannot be built here) on the same
config, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s/GPU, Qwen3 Q4_0 bs=1; Q4 GEMV HBM GB/s vs 8 TB/s peak"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--sessions", type=int, default=8,
                    help="co-batched sessions per GPU for the sessions_per_gpu figure (1 = skip)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--per-stage", action="store_true",
                    help="time the one-kernel-per-stage step instead of the persistent one")
    ap.add_argument("--profile-steps", type=int, default=8,
                    help="decode steps of the per-kernel profile pass (at least 1)")
    ap.add_argument("--no-gemv", action="store_true",
                    help="skip the Q4_0 GEMV shape sweep (the metric's second half)")
    ap.add_argument("--tp-model", default="qwen3-8b",
                    help="model of the tensor-parallel record when N > 1 ('' = skip)")
    ap.add_argument("--tp-steps", type=int, default=64)
    return ap.parse_args()


# ---------------------------------------------------------------- plumbing
class Dist:
    """One process per GPU (torchrun env).  The process group carries only the
    barrier and the max-over-ranks of the timings: sessions are independent
    replicas (no data-path collective).  Backend: NCCL on the GPU box; gloo
    (CW_DIST_BACKEND=gloo or no CUDA) for the CPU tests of this plumbing."""

    def __init__(self, backend: str | None = None):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False
        self.device = "cpu"
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            backend = backend or os.environ.get("CW_DIST_BACKEND") or (
                "nccl" if torch.cuda.is_available() else "gloo")
            timeout = datetime.timedelta(seconds=600)
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                self.device = f"cuda:{self.local}"
                dist.init_process_group("nccl", timeout=timeout,
                                        device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(backend, timeout=timeout)
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        import torch.distributed as dist
        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def allgather_bytes(self, data: bytes) -> list:
        """Every rank's bytes, in rank order."""
        if not self.pg:
            return [data]
        import torch.distributed as dist
        out = [None] * self.world
        dist.all_gather_object(out, data)
        return out

    def bcast_bytes(self, data):
        """Rank 0's bytes on every rank."""
        if not self.pg:
            return data
        import torch.distributed as dist
        box = [data]
        dist.broadcast_object_list(box, src=0)
        return box[0]

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()
            self.pg = False


def replica_rate(steps: int, world: int, seconds_max: float) -> float:
    """Whole-job tokens/s of `world` replicas that each ran `steps` tokens, the
    slowest in seconds_max (weak scaling: per-GPU work fixed as N grows)."""
    return steps * world / seconds_max


def physical_gpu(local: int) -> str:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids):
            return ids[local]
    return str(local)


class Clocks:
    """nvidia-smi sampling during the timed region (clocks + throttle reasons)."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: str):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", self.gpu],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax.append(float(p[2]))
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# DRAM bytes (read + write) per launch of the dominant kernel from one ncu
# capture of this bench's workload (profiles/decode_step_persistent_qwen3_0.6b.md:
# dram throughput x duration of the decode launch at position 130).
NCU_TRAFFIC = {("qwen3-0.6b", "decode_step"): 369.4e6}
NCU_TRAFFIC_SRC = "ncu, one decode_step launch at position 130 (profiles/decode_step_persistent_qwen3_0.6b.md)"


def measured_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# ---------------------------------------------------------------- bytes model
def kernel_bytes(info: dict, pos: float) -> dict:
    """Algorithmic HBM bytes per launch of each decode kernel at position pos:
    Q4_0 weights 18 B per 32 weights, f32 activations in/out, f32 KV cache
    reads of pos+1 rows per layer plus the new row's write."""
    dim, L, nh, nkv, hd, hid, V = (info[k] for k in ("dim", "n_layers", "n_heads", "n_kv",
                                                     "head_dim", "hidden", "vocab"))
    qd, kvd = nh * hd, nkv * hd
    q4 = lambda rows, k: rows * (k // 32) * 18  # noqa: E731
    return {
        "attn_in": q4(qd + 2 * kvd, dim) + 4 * dim * 2 + 4 * (qd + 2 * kvd),
        "attention": 4 * (2 * (pos + 1) * kvd + qd + 2 * kvd + qd),
        "attn_out": q4(dim, qd) + 4 * qd + 8 * dim,
        "ffn_in": q4(2 * hid, dim) + 4 * dim * 2 + 4 * hid,
        "ffn_out": q4(dim, hid) + 4 * hid + 8 * dim,
        "lm_head": q4(V, dim) + 4 * dim * 2 + 4 * V,
        "embed": 18 * (dim // 32) + 4 * dim,
        "finalize": 64,
    }


def step_bytes(info: dict, pos: float) -> float:
    kb = kernel_bytes(info, pos)
    L = info["n_layers"]
    return (L * (kb["attn_in"] + kb["attention"] + kb["attn_out"] + kb["ffn_in"] + kb["ffn_out"])
            + kb["lm_head"] + kb["embed"] + kb["finalize"])


def launch_bytes(info: dict, pos: float) -> dict:
    """kernel_bytes plus the persistent kernel, whose one launch is the step,
    and its fused stages (the same algorithmic bytes, regrouped)."""
    kb = kernel_bytes(info, pos)
    kb["decode_step"] = step_bytes(info, pos)
    kb["ffn"] = kb["ffn_in"] + kb["ffn_out"]                # gate/up + SwiGLU + down
    kb["attention_o"] = kb["attention"] + kb["attn_out"]  # attention + O projection
    return kb


# ---------------------------------------------------------------- CPU legs
REL = 1e-3  # the north star's tolerance (relative to the largest |logit|)


def host_threads() -> int:
    """Every host core this process may run on (torchrun exports
    OMP_NUM_THREADS=1, which the oracle would otherwise inherit)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_leg(path: str, prompt, gpu_tokens, budget_s: float = 10.0, single_s: float = 4.0):
    """The oracle port on the host cores, teacher-forced on the GPU's greedy
    stream: after the prompt, step i feeds the GPU's token i-1 and checks that
    the GPU's token i is the oracle's argmax, or within REL of its top logit
    (a near-tie the tolerance leaves open).  Times the decode steps on all
    host threads (at most budget_s, at least 4 steps), then a few more on one
    thread (the reference's scalar loops, src/main.rs:133-150)."""
    from oracle import oracle as orc
    threads = host_threads()
    orc.set_threads(threads)
    m = orc.Model(path)
    n = len(gpu_tokens)
    m.reset(len(prompt) + n + 8)
    tok = int(prompt[0])
    for pos in range(len(prompt) - 1):
        m.step(tok, pos, want_logits=False)
        tok = int(prompt[pos + 1])
    pos = len(prompt) - 1
    compared = mismatch = near_tie = 0
    t0 = time.perf_counter()
    for i in range(n):
        _, logits = m.step(tok, pos, want_logits=True)
        g = int(gpu_tokens[i])
        r = orc.argmax(logits)
        top = float(logits[r])
        tol = REL * max(float(np.max(np.abs(logits))), 1e-30)
        if g != r:
            if top - float(logits[g]) <= tol:
                near_tie += 1
            else:
                mismatch += 1
        compared += 1
        tok = g
        pos += 1
        if compared >= 4 and time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    multi = {"value": compared / dt, "cores": threads, "steps": compared, "seconds": dt}
    # single thread: the next positions, fed the GPU's tokens while they last
    orc.set_threads(1)
    t1 = time.perf_counter()
    k = 0
    while k < 2 or (time.perf_counter() - t1 < single_s and k < 64):
        m.step(tok, pos, want_logits=True)
        tok = int(gpu_tokens[compared + k]) if compared + k < n else 0
        pos += 1
        k += 1
    ds = time.perf_counter() - t1
    orc.set_threads(threads)
    m.close()
    single = {"value": k / ds, "cores": 1, "steps": k, "seconds": ds}
    parity = {"steps_compared": compared, "clear_gap_mismatches": mismatch, "near_ties": near_tie,
              "ok": mismatch == 0, "rule": f"GPU token == oracle argmax, or within {REL} x max|logit| "
              "of its top logit; the oracle is teacher-forced on the GPU stream"}
    return multi, single, parity


def cpu_gemv_sweep(threads: int, budget_s: float = 12.0) -> dict:
    """The GEMV sweep on the host: the oracle's Q4_0 dequant-dot
    (orc_q4_0_gemv, dequant.rs:62-78 + matmul.wgsl:43-50) per shape, on all
    host threads (repeated for at least 0.1 s) and on one thread (once).  All
    shapes view one buffer of random blocks sized for the largest."""
    from oracle import oracle as orc
    from chat_wgpu_b200 import gguf
    from chat_wgpu_b200.q4bench import SHAPES, algorithmic_bytes
    kmax, nmax = max(SHAPES, key=lambda s: s[0] * s[1])
    blocks = gguf.random_q4_0_blocks(np.random.default_rng(5), nmax, kmax).ravel()
    rows = []
    t_all = time.perf_counter()
    for k, n in SHAPES:
        if time.perf_counter() - t_all > budget_s:
            break
        w = blocks[: n * (k // 32) * 18]
        x = np.random.default_rng(k + n).normal(0, 1, k).astype(np.float32)
        b = algorithmic_bytes(k, n)
        orc.set_threads(threads)
        orc.q4_0_gemv(x, w, k, n)  # warm
        reps, t0 = 0, time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < 0.1:
            orc.q4_0_gemv(x, w, k, n)
            reps += 1
        multi = (time.perf_counter() - t0) / reps
        orc.set_threads(1)
        t1 = time.perf_counter()
        orc.q4_0_gemv(x, w, k, n)
        one = time.perf_counter() - t1
        rows.append({"in_f": k, "out_f": n, "us": round(multi * 1e6, 1),
                     "gbs": round(b / multi / 1e9, 2), "us_1thread": round(one * 1e6, 1),
                     "gbs_1thread": round(b / one / 1e9, 3)})
    orc.set_threads(threads)
    return {"kind": "port", "cores": threads, "unit": "us per call, GB/s (same algorithmic bytes)",
            "shapes": rows}


def gemv_sweep(ctx, peak_gbs: float) -> list:
    """The metric's second half: Q4_0 GEMV (cw_q4_0_gemv) per shape, config 1
    (1024 -> 3072) and the Qwen3 projection sweep with the four LM heads.
    Each shape's launches rotate through distinct weight copies totalling
    more than 3x the L2 size, replayed as one CUDA graph, timed with events."""
    from chat_wgpu_b200.q4bench import SHAPES, bench_shape
    rows = []
    for k, n in SHAPES:
        r = bench_shape(ctx, k, n)
        rows.append({"in_f": k, "out_f": n, "us": round(r["us"], 3), "gbs": round(r["gbs"], 1),
                     "frac": round(r["gbs"] / peak_gbs, 4), "bytes": r["bytes"],
                     "copies": r["copies"]})
    return rows


def tp_leg(args, dist, ctx) -> dict:
    """N > 1: the tensor-parallel record.  The --tp-model GGUF split over the
    job's N GPUs (cw_model_load_gguf_tp, one rank per GPU), greedy decode on
    the per-stage step with the O / down all-reduces and the argmax over
    NVLink peer memory (Session.tp_attach), then over NCCL; ms/token timed
    with CUDA events on every rank, max over ranks.  Rank 0 then decodes the
    same prompt with the whole model on its GPU (the persistent step) and
    counts the leading tokens on which the streams agree."""
    from chat_wgpu_b200 import gguf
    from chat_wgpu_b200.model import Model, Session, tp_unique_id
    name = args.tp_model
    if dist.rank == 0:
        gguf.cached_model(name, seed=args.seed)  # written once, before the others read it
    dist.barrier()
    path = gguf.cached_model(name, seed=args.seed)
    uid = dist.bcast_bytes(tp_unique_id() if dist.rank == 0 else None)
    m = Model(ctx, path, tp=(dist.rank, dist.world, uid))
    vocab = gguf.CONFIGS[name]["vocab"]
    P, W, K = 32, 4, args.tp_steps
    prompt = np.random.default_rng(args.seed + 2).integers(0, vocab, P).astype(np.uint32)
    out = {"model": name, "tp": dist.world, "steps": K, "warmup": W,
           "positions": f"{P - 1 + W}..{P - 2 + W + K}"}
    toks = None
    for mode in ("p2p", "nccl"):
        s = Session(m, P + W + K + 2)
        if mode == "p2p":
            s.tp_attach_p2p(dist.allgather_bytes)
        s.begin(prompt)
        s.run(P - 1 + W)
        dist.barrier()
        ms = dist.max(s.run_timed(K))
        t = s.tokens()
        dist.barrier()  # every rank done stepping before any frees its exchange area
        s.close()
        out[mode] = {"ms_per_token": ms / K, "tok_s": K / (ms / 1e3)}
        if mode == "p2p":
            toks = t
    out["path"] = ("per-stage kernels in a CUDA graph; p2p: each all-reduce one kernel of "
                   "8-byte value+epoch NVLink peer stores and a rank-order sum (cw_tp_p2p.cu); "
                   "nccl: ncclAllReduce nodes")
    m.close()
    if dist.rank == 0:
        full = Model(ctx, path)
        r = Session(full, P + W + K + 2)
        r.begin(prompt)
        r.run(P - 1 + W)
        ms1 = r.run_timed(K)
        ref = r.tokens()
        r.close()
        full.close()
        out["single_gpu"] = {"ms_per_token": ms1 / K, "path": "persistent step, whole model"}
        same = np.append(ref == toks, False)
        out["tokens_agreeing_with_1gpu"] = int(np.argmin(same))
        out["of"] = int(len(toks))
    dist.barrier()
    return out


def run_reference(args):
    """--impl reference: the oracle port on all host cores, same config; rank 0
    only (no process group, no device)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    from chat_wgpu_b200 import gguf
    path = gguf.cached_model(args.model, seed=args.seed)
    cfg = gguf.CONFIGS[args.model]
    rng = np.random.default_rng(args.seed + 1)
    prompt = rng.integers(0, cfg["vocab"], args.prompt_len).astype(np.uint32)
    from oracle import oracle as orc
    orc.set_threads(host_threads())
    m = orc.Model(path)
    m.reset(args.prompt_len + args.warmup + args.steps + 1)
    tok = int(prompt[0])
    for pos in range(args.prompt_len - 1):
        m.step(tok, pos, want_logits=False)
        tok = int(prompt[pos + 1])
    pos = args.prompt_len - 1
    for _ in range(args.warmup):
        _, lg = m.step(tok, pos)
        tok = orc.argmax(lg)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, lg = m.step(tok, pos)
        tok = orc.argmax(lg)
        pos += 1
    dt = time.perf_counter() - t0
    cores = orc.get_threads()
    m.close()
    value = args.steps / dt
    sample = (f"{args.steps} decode steps at positions {args.prompt_len - 1 + args.warmup}.."
              f"{pos - 1} of {args.model} (prompt {args.prompt_len}), oracle port, {cores} threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random-init Q4_0 GGUF, uniform-random prompt)",
        "config": {"workload": f"{args.model} greedy decode, bs=1, prompt {args.prompt_len}",
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the Rust/wgpu reference cannot be built or run here (no cargo, no graphics "
                "stack); this arm is the C restatement of its CPU path",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- main arm
def run_cuda(args, dist):
    from chat_wgpu_b200 import gguf
    from chat_wgpu_b200.context import GpuContext
    from chat_wgpu_b200.model import Model, Session

    cfg = gguf.CONFIGS[args.model]
    if dist.rank == 0:
        path = gguf.cached_model(args.model, seed=args.seed)
    dist.barrier()
    path = gguf.cached_model(args.model, seed=args.seed)
    ctx = GpuContext(dist.local)
    model = Model(ctx, path)
    info = model.info
    rng = np.random.default_rng(args.seed + 1)
    prompt = rng.integers(0, cfg["vocab"], args.prompt_len).astype(np.uint32)
    P, W, K = args.prompt_len, args.warmup, args.steps
    max_seq = P + W + K + args.profile_steps + 4

    # ---- device-timed decode: K graph replays, inputs resident in HBM
    s = Session(model, max_seq)
    if args.per_stage:
        s.set_persistent(False)
    persistent = s.persistent
    s.begin(prompt)
    s.run(P - 1)                     # prompt positions (no lm_head)
    s.run(W)                         # warm-up decode steps
    ctx.sync()
    dist.barrier()
    clk = Clocks(physical_gpu(dist.local))
    clk.start()
    time.sleep(0.3)
    ms = s.run_timed(K)
    clocks = clk.stop()
    ms_max = dist.max(ms)
    toks = s.tokens()
    assert toks.size == W + K, (toks.size, W + K)
    value = replica_rate(K, dist.world, ms_max / 1000.0)
    pos_lo, pos_hi = P - 1 + W, P - 1 + W + K - 1
    mean_pos = 0.5 * (pos_lo + pos_hi)
    _, launches_decode = s.launches()

    # ---- per-kernel profile: the step as a graph with an event pair per kernel
    prof = s.profile(max(1, args.profile_steps))
    s.close()

    # ---- the other step path on the same positions, for the record
    other = None
    if persistent:
        so = Session(model, max_seq)
        so.set_persistent(False)
        so.begin(prompt)
        so.run(P - 1 + W)
        ms_o = dist.max(so.run_timed(K))
        other = {"path": "per-stage kernels", "ms_per_step": ms_o / K,
                 "launches_per_step": so.launches()[1]}
        so.close()

    # ---- batched prefill of the same prompt (tcgen05 GEMMs), device time from
    # the context profiler's event pairs around each prefill launch
    prefill = None
    if P > 1:
        from chat_wgpu_b200.prefillprof import gemm_flops_per_row
        s3 = Session(model, max_seq)
        s3.begin(prompt)
        s3.prefill()                 # warm-up: scratch, tensor maps
        ctx.sync()
        reps = 3
        ctx.begin_profile()
        for _ in range(reps):
            s3.begin(prompt)
            s3.prefill()
        agg = {}
        for name, count, t in ctx.report_profile():
            if name.startswith("prefill."):
                agg[name] = agg.get(name, 0.0) + t
        s3.close()
        pf_ms = sum(agg.values()) / reps
        gemm_ms = agg.get("prefill.gemm", float("nan")) / reps
        fl = gemm_flops_per_row(info) * (P - 1)
        pk = measured_peaks()
        prefill = {"positions": P - 1, "ms": pf_ms, "tok_s": (P - 1) / pf_ms * 1e3,
                   "gemm_ms": gemm_ms, "gemm_tflops": fl / gemm_ms / 1e9,
                   "gemm_pipe_tflops": 3 * fl / gemm_ms / 1e9,
                   "gemm_pipe_frac": 3 * fl / gemm_ms / 1e9 / pk["bf16_tflops"],
                   "stage_ms": {k: round(v / reps, 4) for k, v in agg.items()},
                   "note": "GEMMs issue three f16 MMAs per K step (hi/lo operand split); "
                           "pipe_frac is against measured burst bf16 TFLOP/s"}

    # ---- co-batched: 8 independent sessions per GPU stepped together
    # (config 3's scaling setup), each after its own prompt
    group = None
    if args.sessions > 1:
        from chat_wgpu_b200.groupbench import bench as group_bench
        r = group_bench(model, args.sessions, P, K, warmup=W, seed=args.seed)
        t_max = dist.max(r["ms_per_step"] * K / 1000.0)  # seconds, slowest rank
        group = {"sessions_per_gpu": args.sessions,
                 "tok_s": replica_rate(K * args.sessions, dist.world, t_max),
                 "unit": "tok/s (all GPUs, all sessions)", "ms_per_step": t_max * 1e3 / K,
                 "positions": r["positions"],
                 "path": f"SessionGroup: one pass over the weights per step ({r['path']})"}
        if r["path"].startswith("streaming"):  # the other projection path, for the record
            r2 = group_bench(model, args.sessions, P, K, warmup=W, seed=args.seed,
                             streaming=False)
            t2 = dist.max(r2["ms_per_step"] * K / 1000.0)
            group["other_path"] = {"path": r2["path"], "ms_per_step": t2 * 1e3 / K,
                                   "tok_s": replica_rate(K * args.sessions, dist.world, t2)}

    # ---- e2e: public per-token API with host round trips
    s2 = Session(model, max_seq)
    s2.begin(prompt)
    s2.run(P - 1)
    tok = Session.TOKEN_DEVICE
    for _ in range(W):
        tok = s2.step(tok)
    dist.barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        tok = s2.step(tok)
    e2e_s = time.perf_counter() - t0
    e2e_max = dist.max(e2e_s)
    toks2 = s2.tokens()
    s2.close()
    e2e_value = replica_rate(K, dist.world, e2e_max)
    same_stream = bool(np.array_equal(toks, toks2))

    # ---- roofline of the dominant kernel
    peaks = measured_peaks()
    kb = launch_bytes(info, mean_pos + args.profile_steps / 2)
    rows = {name: (n, t) for name, n, t in prof}
    dom = max(((n, c, t) for n, (c, t) in rows.items() if n in kb), key=lambda r: r[2])
    dom_name, dom_count, dom_ms = dom
    dom_bytes = kb[dom_name]
    achieved = dom_bytes / (dom_ms / dom_count / 1000.0) / 1e9
    per_kernel = {n: {"launches": c, "ms": round(t, 4),
                      "gbs": round(kb[n] / (t / c / 1000.0) / 1e9, 1) if n in kb else None}
                  for n, (c, t) in rows.items()}
    sb = step_bytes(info, mean_pos)
    step_gbs = sb / (ms_max / K / 1000.0) / 1e9

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": dist.world, "steps": K,
        "warmup": W, "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (Q4_0 weights, f32 accumulation)",
        "data": "synthetic (seeded random-init Q4_0 GGUF, uniform-random prompt)",
        "config": {"workload": f"{args.model} greedy decode, bs=1, prompt {P}, timed decode "
                               f"positions {pos_lo}..{pos_hi}",
                   "parallelism": f"replicas x{dist.world} (one session per GPU)",
                   "l2": "inputs larger than L2 (335 MB of weights per step)",
                   "weight_bytes": int(info["weight_bytes"])},
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4, "same_tokens_as_device_loop": same_stream},
        "gpu_launches": int(K * launches_decode),
        "step_path": "persistent (one cooperative launch per token)" if persistent
                     else "per-stage kernels in a CUDA graph",
        "other_path": other,
        "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved,
                     "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                     "traffic": NCU_TRAFFIC.get((args.model, dom_name)),
                     "traffic_src": NCU_TRAFFIC_SRC if (args.model, dom_name) in NCU_TRAFFIC
                     else None,
                     "peak_src": peaks["src"],
                     "bytes_per_launch": int(dom_bytes)},
        "step_roofline": {"bytes_per_step": int(sb), "achieved_gbs": step_gbs,
                          "frac": step_gbs / peaks["hbm_gbs"],
                          "roofline_tok_s": peaks["hbm_gbs"] * 1e9 / sb},
        "kernels": per_kernel,
        "prefill": prefill,
        "sessions_per_gpu": group,
        "clocks": clocks,
    }
    if dist.rank == 0 and not args.no_gemv:
        line["gemv"] = {"unit": "us per launch, GB/s (algorithmic bytes N*K/32*18 + 4K + 4N)",
                        "peak_gbs": peaks["hbm_gbs"], "peak_src": peaks["src"],
                        "shapes": gemv_sweep(ctx, peaks["hbm_gbs"])}
    dist.barrier()
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        multi, single, parity = oracle_leg(path, prompt, toks)
        n = multi["steps"]
        line["cpu_baseline"] = {
            "value": multi["value"], "unit": "tok/s", "cores": multi["cores"], "kind": "port",
            "sample": f"{n} decode steps at positions {P - 1}..{P - 2 + n} after the same "
                      f"{P}-token prompt of {args.model} ({multi['seconds']:.1f} s timed), oracle "
                      f"port on {multi['cores']} host threads, fed the GPU's tokens",
            "single_thread": {"value": single["value"], "unit": "tok/s", "cores": 1,
                              "sample": f"{single['steps']} further decode steps on one thread "
                                        f"({single['seconds']:.1f} s)"},
            "nproc": os.cpu_count()}
        if not args.no_gemv:
            line["cpu_baseline"]["gemv"] = cpu_gemv_sweep(multi["cores"])
        line["parity"] = parity
    model.close()
    if dist.world > 1 and args.tp_model:
        line["tp"] = tp_leg(args, dist, ctx)
    ctx.close()
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    dist = Dist()
    try:
        run_cuda(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
