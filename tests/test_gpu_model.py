"""Decode-loop parity: the fused CUDA-graph session, cw_generate and the
op-by-op composition against the CPU oracle's model (src/model/qwen3.rs +
src/model/mod.rs restated), on seeded random-init GGUF checkpoints.

Gates (north star): logits within 1e-3 relative (rel_err in conftest.py);
greedy tokens identical at every step until the first step whose oracle
top-2 logit gap is within that tolerance (after it the sequences may
legitimately diverge and are no longer compared)."""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
REL = 1e-3


def gap_ok(logits_ref: np.ndarray) -> bool:
    """True when the oracle's top-2 gap exceeds the tolerance, i.e. the argmax
    is decided beyond rounding noise."""
    top2 = np.partition(logits_ref, -2)[-2:]
    scale = max(float(np.max(np.abs(logits_ref))), 1e-30)
    return float(top2[1] - top2[0]) > REL * scale


def compare_streams(got_toks, ref_toks, ref_logits, got_logits=None):
    """Tokens must match until the first ambiguous step; logits compared on the
    shared prefix.  Returns the number of steps compared."""
    n = 0
    for i, (g, r) in enumerate(zip(got_toks, ref_toks)):
        if got_logits is not None:
            assert rel_err(got_logits[i], ref_logits[i]) < REL, f"logits differ at step {i}"
        if g != r:
            assert not gap_ok(ref_logits[i]), f"token {i}: got {g}, oracle {r} with a clear top-2 gap"
            return n
        n += 1
        if not gap_ok(ref_logits[i]):
            return n  # ambiguous step: later steps may diverge legitimately
    return n


def session_stream(model, prompt, max_new, use_graph=True, persistent=None):
    from chat_wgpu_b200.model import Session
    s = Session(model, len(prompt) + max_new)
    s.set_graph(use_graph)
    if persistent is not None:
        s.set_persistent(persistent)
    s.begin(prompt)
    s.run(len(prompt) - 1)  # prompt positions (no lm_head)
    logits = []
    for _ in range(max_new):
        s.run(1)
        logits.append(s.logits())
    toks = s.tokens()
    s.close()
    return toks, np.stack(logits)


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    from chat_wgpu_b200 import gguf
    d = tmp_path_factory.mktemp("gpu_models")
    out = {}
    for name, seed in [("tiny-qwen3", 7), ("small-qwen3", 2), ("tiny-gemma2", 3), ("tiny-qwen2", 5),
                       ("wide-ffn-qwen3", 9), ("odd-qwen3", 4)]:
        out[name] = gguf.synth_model(str(d / f"{name}.gguf"), gguf.CONFIGS[name], seed=seed)
    return out


# families the persistent one-launch step covers (the others always use the
# per-stage kernels), and where it is the default (the post-norm family runs
# it on request: its per-stage path is faster at Gemma-2-2B)
PERSISTENT = {"tiny-qwen3": False, "small-qwen3": True, "tiny-gemma2": True, "tiny-qwen2": True,
              "wide-ffn-qwen3": True, "odd-qwen3": True}
DEFAULT_PERSISTENT = dict(PERSISTENT, **{"tiny-gemma2": False})


@pytest.mark.parametrize("persistent", [False, True], ids=["per-stage", "persistent"])
@pytest.mark.parametrize("name", ["tiny-qwen3", "small-qwen3", "tiny-gemma2", "tiny-qwen2",
                                  "wide-ffn-qwen3", "odd-qwen3"])
def test_fused_session_vs_oracle(ctx, orc, models, name, persistent):
    from chat_wgpu_b200.model import Model
    if persistent and not PERSISTENT[name]:
        pytest.skip("family not covered by the persistent step")
    path = models[name]
    om = orc.Model(path)
    prompt = np.array([1, 5, 9, 2, 77, 3, 41, 8, 100, 6][: 4 if name == "tiny-qwen3" else 10],
                      np.uint32) % om.vocab
    max_new = 24
    ref_toks, ref_logits = om.generate(prompt, max_new, want_logits=True)
    m = Model(ctx, path)
    toks, logits = session_stream(m, prompt, max_new, persistent=persistent)
    n = compare_streams(toks, ref_toks, ref_logits, logits)
    assert n >= 4, f"only {n} steps compared"
    m.close()
    om.close()


def test_graph_equals_direct_launch(ctx, models):
    from chat_wgpu_b200.model import Model
    m = Model(ctx, models["small-qwen3"])
    prompt = np.array([3, 1, 4, 1, 5], np.uint32)
    t1, l1 = session_stream(m, prompt, 12, use_graph=True)
    t2, l2 = session_stream(m, prompt, 12, use_graph=False)
    assert np.array_equal(t1, t2)
    assert np.array_equal(l1.view(np.uint32), l2.view(np.uint32))
    m.close()


@pytest.mark.parametrize("name", ["tiny-qwen3", "small-qwen3", "tiny-gemma2", "tiny-qwen2"])
def test_persistent_default_and_coverage(ctx, models, name):
    """The persistent step is the default where the family is covered (but
    the post-norm family); asking for it where it is not covered fails loudly;
    one launch per step when it is used."""
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models[name])
    s = Session(m, 16)
    assert s.persistent == DEFAULT_PERSISTENT[name]
    if PERSISTENT[name]:
        s.set_persistent(True)
        assert s.persistent
        assert s.launches() == (1, 1)
        s.set_persistent(False)
        assert not s.persistent and s.launches()[1] > 1
        s.set_persistent(True)
        assert s.persistent
    else:
        with pytest.raises(CwError):
            s.set_persistent(True)
        assert not s.persistent
    s.close()
    m.close()


@pytest.mark.parametrize("n_prompt", [40, 200, 300, 600])
def test_persistent_equals_per_stage_long(ctx, orc, models, n_prompt):
    """Long prompts and 40 generated tokens on small-qwen3: the attention
    stage runs with one key split (40), several (200: 4 and 300: 5-6 splits,
    merged per head by the O-projection stage) and more than it defers (600:
    10 splits, combined inside the attention stage).  Persistent and
    per-stage paths both within tolerance of the oracle; persistent graph ==
    direct, bit-exact."""
    mode = True
    from chat_wgpu_b200.model import Model
    path = models["small-qwen3"]
    om = orc.Model(path)
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, om.vocab, n_prompt).astype(np.uint32)
    ref_toks, ref_logits = om.generate(prompt, 40, want_logits=True)
    m = Model(ctx, path)
    tp, lp = session_stream(m, prompt, 40, persistent=mode)
    ts, ls = session_stream(m, prompt, 40, persistent=False)
    assert compare_streams(tp, ref_toks, ref_logits, lp) >= 4
    assert compare_streams(ts, ref_toks, ref_logits, ls) >= 4
    td, ld = session_stream(m, prompt, 40, use_graph=False, persistent=mode)
    assert np.array_equal(tp, td)
    assert np.array_equal(lp.view(np.uint32), ld.view(np.uint32))
    m.close()
    om.close()


@pytest.mark.parametrize("n_prompt", [12, 150])
def test_persistent_gemma2_hd256(ctx, orc, tmp_path, n_prompt):
    """The post-norm step variant at Gemma-2 head and residual shapes
    (head_dim 256, dim 2304, GQA 4/2): UnitShift gains, GeGLU, soft-caps 5 and
    8, an 80-key window on even layers (150-token prompt: windowed layers read
    2-3 key splits, global layers 5), an odd layer count.  Persistent and
    per-stage paths both within tolerance of the oracle; graph == direct,
    bit-exact."""
    from chat_wgpu_b200 import gguf
    from chat_wgpu_b200.model import Model
    path = gguf.synth_model(str(tmp_path / "mid-gemma2.gguf"), gguf.CONFIGS["mid-gemma2"], seed=6)
    om = orc.Model(path)
    rng = np.random.default_rng(n_prompt)
    prompt = rng.integers(0, om.vocab, n_prompt).astype(np.uint32)
    ref_toks, ref_logits = om.generate(prompt, 24, want_logits=True)
    m = Model(ctx, path)
    tp, lp = session_stream(m, prompt, 24, persistent=True)
    ts, ls = session_stream(m, prompt, 24, persistent=False)
    assert compare_streams(tp, ref_toks, ref_logits, lp) >= 4
    assert compare_streams(ts, ref_toks, ref_logits, ls) >= 4
    td, ld = session_stream(m, prompt, 24, use_graph=False, persistent=True)
    assert np.array_equal(tp, td)
    assert np.array_equal(lp.view(np.uint32), ld.view(np.uint32))
    m.close()
    om.close()


def test_generate_api_matches_session(ctx, orc, models):
    """cw_generate (host read per token, mod.rs:103) == device-side session;
    max_new == 0 yields one token like the reference's post-push check."""
    from chat_wgpu_b200.model import Model, generate
    m = Model(ctx, models["tiny-qwen3"])
    prompt = np.array([9, 8, 7], np.uint32)
    toks, _ = session_stream(m, prompt, 10)
    assert np.array_equal(generate(m, prompt, 10), toks)
    assert generate(m, prompt, 0).size == 1
    assert generate(m, prompt, 0)[0] == toks[0]
    om = orc.Model(models["tiny-qwen3"])
    assert om.generate(prompt, 0).size == 1
    om.close()
    m.close()


def test_op_by_op_composition_vs_oracle(ctx, orc, models):
    """The reference's composition (qwen3.rs:139-191) through the per-op C-ABI."""
    from chat_wgpu_b200.model import OpByOpQwen3, generate_op_by_op
    path = models["tiny-qwen3"]
    mm = OpByOpQwen3(ctx, path)
    prompt = np.array([1, 5, 9, 2], np.uint32)
    toks, logits = generate_op_by_op(ctx, mm, prompt, 12, want_logits=True)
    om = orc.Model(path)
    ref_toks, ref_logits = om.generate(prompt, 12, want_logits=True)
    assert compare_streams(toks, ref_toks, ref_logits, logits) >= 4
    om.close()


def test_session_limits(ctx, models):
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["tiny-qwen3"])
    s = Session(m, 4)
    with pytest.raises(CwError):
        s.begin(np.array([1, 2, 3, 4, 5], np.uint32))  # longer than max_seq
    with pytest.raises(CwError):
        s.begin(np.array([1, 999], np.uint32))  # outside the vocabulary
    s.begin(np.array([1, 2], np.uint32))
    s.run(4)
    with pytest.raises(CwError):
        s.run(1)  # position 4 == max_seq
    assert s.pos == 4
    s.close()
    m.close()
