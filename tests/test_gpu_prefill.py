"""Batched prefill (cw_session_prefill: the prompt's projections as tcgen05
GEMMs) against the CPU oracle and against the token-by-token steps.

The reference has no prefill: its prompt runs one token at a time
(src/model/mod.rs:78-83).  Gates: the KV cache rows prefill writes equal the
token-by-token rows within 1e-3 relative (rel_err in conftest.py); the
logits and greedy stream that follow match the oracle's like the plain
session's do (test_gpu_model.compare_streams)."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_model import compare_streams, models  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu
REL = 1e-3


def _stream(model, prompt, max_new, prefill, persistent=None, chunk=0):
    from chat_wgpu_b200.model import Session
    s = Session(model, len(prompt) + max_new)
    if persistent is not None:
        s.set_persistent(persistent)
    s.set_prefill_chunk(chunk)
    s.begin(prompt)
    if prefill:
        assert s.prefill() == len(prompt) - 1
    else:
        s.run(len(prompt) - 1)
    kv = [s.read_kv(li, len(prompt) - 1) for li in range(model.info["n_layers"])]
    logits = []
    for _ in range(max_new):
        s.run(1)
        logits.append(s.logits())
    toks = s.tokens()
    s.close()
    return toks, np.stack(logits), kv


def _kv_close(kv_a, kv_b):
    for li, ((ka, va), (kb, vb)) in enumerate(zip(kv_a, kv_b)):
        for name, a, b in (("k", ka, kb), ("v", va, vb)):
            for g in range(a.shape[0]):
                for p in range(a.shape[1]):
                    assert rel_err(a[g, p], b[g, p]) < REL, f"layer {li} {name} head {g} pos {p}"


@pytest.mark.parametrize("name", ["tiny-qwen3", "small-qwen3", "tiny-gemma2", "tiny-qwen2"])
def test_prefill_vs_oracle(ctx, orc, models, name):  # noqa: F811
    from chat_wgpu_b200.model import Model
    om = orc.Model(models[name])
    rng = np.random.default_rng(17)
    prompt = rng.integers(0, om.vocab, 40).astype(np.uint32)
    ref_toks, ref_logits = om.generate(prompt, 16, want_logits=True)
    m = Model(ctx, models[name])
    toks, logits, kv = _stream(m, prompt, 16, prefill=True)
    assert compare_streams(toks, ref_toks, ref_logits, logits) >= 4
    _, _, kv_ref = _stream(m, prompt, 1, prefill=False)
    _kv_close(kv, kv_ref)
    m.close()
    om.close()


@pytest.mark.parametrize("chunk", [7, 128, 4096])
def test_prefill_chunks_long_prompt(ctx, models, chunk):  # noqa: F811
    """A 300-token prompt in several chunks (the later chunks attend over
    cache rows the earlier ones wrote) equals the token-by-token steps; one
    299-row chunk takes the long-chunk GEMM path (split weights)."""
    from chat_wgpu_b200.model import Model
    m = Model(ctx, models["small-qwen3"])
    prompt = np.random.default_rng(3).integers(0, m.info["vocab"], 300).astype(np.uint32)
    t1, l1, kv1 = _stream(m, prompt, 8, prefill=True, chunk=chunk)
    t2, l2, kv2 = _stream(m, prompt, 8, prefill=False)
    _kv_close(kv1, kv2)
    for i in range(len(l1)):
        assert rel_err(l1[i], l2[i]) < REL, i
    assert t1[0] == t2[0]
    m.close()


def test_prefill_sliding_window_gemma(ctx, orc, models):  # noqa: F811
    """Prompt far longer than the gemma2 test window (6): the windowed layers
    see only the last 6 keys in prefill exactly as in decode."""
    from chat_wgpu_b200.model import Model
    m = Model(ctx, models["tiny-gemma2"])
    prompt = np.random.default_rng(5).integers(0, m.info["vocab"], 90).astype(np.uint32)
    t1, l1, kv1 = _stream(m, prompt, 6, prefill=True)
    t2, l2, kv2 = _stream(m, prompt, 6, prefill=False)
    _kv_close(kv1, kv2)
    for i in range(len(l1)):
        assert rel_err(l1[i], l2[i]) < REL, i
    m.close()


def test_prefill_edges(ctx, models):  # noqa: F811
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["tiny-qwen3"])
    s = Session(m, 32)
    s.begin(np.array([3], np.uint32))
    assert s.prefill() == 0           # a one-token prompt has nothing to batch
    s.run(2)
    assert len(s.tokens()) == 2
    s.begin(np.array([3, 4, 5, 6], np.uint32))
    s.run(1)                          # position 0 by a step ...
    assert s.prefill() == 2           # ... then positions 1, 2 batched
    assert s.prefill() == 0           # nothing left but the last prompt token
    s.run(3)
    assert len(s.tokens()) == 3
    s.close()
    m.close()


def test_prefill_persistent_step_follows(ctx, models):  # noqa: F811
    """The persistent decode step continues from a prefilled cache."""
    from chat_wgpu_b200.model import Model
    m = Model(ctx, models["small-qwen3"])
    prompt = np.random.default_rng(9).integers(0, m.info["vocab"], 64).astype(np.uint32)
    t1, l1, _ = _stream(m, prompt, 8, prefill=True, persistent=True)
    t2, l2, _ = _stream(m, prompt, 8, prefill=False, persistent=False)
    for i in range(len(l1)):
        assert rel_err(l1[i], l2[i]) < REL, i
    m.close()
