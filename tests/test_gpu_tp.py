"""Tensor-parallel decode over 2, 4 and 8 GPUs (cw_model_load_gguf_tp): one
process per GPU, each holding 1/world of the heads, FFN columns and LM-head
rows, with the O / down partial sums and the argmax all-reduced over NCCL or
over NVLink peer memory (Session.tp_attach).  The
greedy stream must match the single-GPU stream and the oracle (same gates as
test_gpu_model: tokens until the first ambiguous step, logits within 1e-3
relative), the ranks must agree on every token, a stop token must end every rank's
stream at the same place, and the calls a tensor-parallel model does not
support must fail cleanly."""
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import rel_err
from test_gpu_model import REL, compare_streams, session_stream

pytestmark = pytest.mark.gpu

WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tp_worker.py")
NAMES = ["small-qwen3", "tiny-qwen2", "tiny-gemma2", "small-qwen3-q6k", "tp8-qwen3"]


def n_gpus():
    import torch
    return torch.cuda.device_count()


@pytest.fixture(scope="module")
def tp_models(tmp_path_factory):
    from chat_wgpu_b200 import gguf
    d = tmp_path_factory.mktemp("tp_models")
    return {n: gguf.synth_model(str(d / f"{n}.gguf"), gguf.CONFIGS[n], seed=13) for n in NAMES}


def run_ranks(path, prompt, n_new, world, out_dir, p2p=False):
    from chat_wgpu_b200.model import tp_unique_id
    uid = tp_unique_id().hex()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    outs = [os.path.join(out_dir, f"rank{r}.npz") for r in range(world)]
    extra = []
    if p2p:
        d = os.path.join(out_dir, "p2p")
        os.makedirs(d, exist_ok=True)
        extra = [d]
    procs = [subprocess.Popen([sys.executable, WORKER, str(r), str(world), path, uid,
                               ",".join(str(int(t)) for t in prompt), str(n_new), outs[r]] + extra,
                              env=env)
             for r in range(world)]
    try:
        for p in procs:
            p.wait(timeout=300)
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
                p.wait()
    assert all(p.returncode == 0 for p in procs), [p.returncode for p in procs]
    return [dict(np.load(o)) for o in outs]


@pytest.mark.parametrize("mode", ["nccl", "p2p"])
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("name", NAMES)
def test_tp_matches_single_gpu_and_oracle(ctx, orc, tp_models, name, world, mode, tmp_path):
    """TP = world over NCCL or over NVLink peer memory (Session.tp_attach)."""
    if n_gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    from chat_wgpu_b200 import gguf
    cfg = gguf.CONFIGS[name]
    if (cfg["n_kv"] % world or cfg["hidden"] % (32 * world) or cfg["vocab"] % world
            or (cfg["n_heads"] * cfg["head_dim"]) % (32 * world)):
        pytest.skip(f"{name} does not split {world} ways")
    from chat_wgpu_b200.model import Model
    path = tp_models[name]
    om = orc.Model(path)
    prompt = (np.array([3, 17, 5, 9, 250, 1, 77, 12, 40], np.uint32) % om.vocab).astype(np.uint32)
    n_new = 16
    ranks = run_ranks(path, prompt, n_new, world, str(tmp_path), p2p=mode == "p2p")
    # every rank produced the same tokens; the logits slices tile the vocabulary
    for r in ranks[1:]:
        assert np.array_equal(ranks[0]["toks"], r["toks"])
    # with the 4th token as a stop token, the stream ends before its first occurrence
    first = int(np.argmax(ranks[0]["toks"] == ranks[0]["toks"][3]))
    for r in ranks:
        assert bool(r["eos_stopped"])
        assert np.array_equal(r["eos_toks"], ranks[0]["toks"][:first])
    vocab = int(ranks[0]["vocab"])
    assert vocab == om.vocab
    logits = np.zeros((n_new, vocab), np.float32)
    cover = np.zeros(vocab, np.int32)
    for r in ranks:
        off, n = int(r["vocab_offset"]), r["logits"].shape[1]
        logits[:, off:off + n] = r["logits"]
        cover[off:off + n] += 1
    assert np.all(cover == 1)
    toks = ranks[0]["toks"]
    # single GPU, same file
    m = Model(ctx, path)
    s_toks, s_logits = session_stream(m, prompt, n_new)
    for i in range(n_new):
        assert rel_err(logits[i], s_logits[i]) < REL, i
        if toks[i] != s_toks[i]:
            break
    m.close()
    ref_toks, ref_logits = om.generate(prompt, n_new, want_logits=True)
    assert compare_streams(toks, ref_toks, ref_logits, logits) >= 1
    om.close()


def test_tp_world1_is_the_plain_model(ctx, tp_models):
    """world 1 loads the whole model (no communicator)."""
    from chat_wgpu_b200.model import Model, tp_unique_id
    path = tp_models["small-qwen3"]
    a = Model(ctx, path, tp=(0, 1, bytes(128)))
    b = Model(ctx, path)
    assert (a.tp_world, a.vocab_offset, a.vocab_local) == (1, 0, b.vocab_size)
    assert a.info == b.info
    a.close()
    b.close()
    assert len(tp_unique_id()) == 128
