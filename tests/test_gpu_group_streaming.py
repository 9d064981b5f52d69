"""The co-batched step's streaming path (cw_mgemv.cu): groups of up to 8
sessions of a pre-norm family run every projection as one streaming GEMV
over all rows.  Each session must still behave exactly as it would alone:
logits within 1e-3 relative of the tensor-core group path, of its own
single-session step and of the oracle, and the same greedy tokens."""
import numpy as np
import pytest

from test_gpu_model import REL, compare_streams, models  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).astype(np.uint32) for n in lens]


def _run_group(m, prompts, steps, streaming, max_seq=64):
    from chat_wgpu_b200.model import Session, SessionGroup
    ss = [Session(m, max_seq) for _ in prompts]
    for s, p in zip(ss, prompts):
        s.begin(p)
    g = SessionGroup(ss)
    if g.path != int(streaming):
        g.set_streaming(streaming)
    assert g.path == int(streaming)
    logits = [[] for _ in ss]
    for _ in range(steps):
        g.run(1)
        for i, s in enumerate(ss):
            logits[i].append(s.logits())
    toks = [s.tokens() for s in ss]
    g.close()
    for s in ss:
        s.close()
    return toks, [np.stack(x) for x in logits]


def test_streaming_chosen(ctx, models):  # noqa: F811
    """Pre-norm families with 256-multiple widths and <= 8 sessions stream;
    the others (and larger groups) keep the tensor-core GEMMs."""
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session, SessionGroup
    for name, n, want in [("small-qwen3", 8, True), ("tiny-qwen2", 3, True),
                          ("small-qwen3", 9, False), ("tiny-qwen3", 2, False),
                          ("tiny-gemma2", 2, False)]:
        m = Model(ctx, models[name])
        ss = [Session(m, 8) for _ in range(n)]
        g = SessionGroup(ss)
        assert g.streaming == want, (name, n)
        if not want:
            with pytest.raises(CwError):
                g.set_streaming(True)
        g.close()
        for s in ss:
            s.close()
        m.close()


@pytest.mark.parametrize("name,lens", [
    ("small-qwen3", [3, 9, 5, 12, 1, 7, 2, 4]),  # 8 sessions: one set of 8 per CTA
    ("tiny-qwen2", [4, 1, 6]),                   # 3 sessions: sets of 4, qkv bias, untied head
])
def test_streaming_matches_gemm_path_and_oracle(ctx, orc, models, name, lens):  # noqa: F811
    from chat_wgpu_b200.model import Model
    m = Model(ctx, models[name])
    prompts = _prompts(m.info["vocab"], lens, 23)
    max_new = 8
    steps = max(lens) - 1 + max_new
    t_s, l_s = _run_group(m, prompts, steps, 1)  # integer-MMA products
    t_d, l_d = _run_group(m, prompts, steps, 2)  # dp4a products
    t_g, l_g = _run_group(m, prompts, steps, 0)  # tensor-core GEMMs
    om = orc.Model(models[name])
    for i, p in enumerate(prompts):
        first = len(p) - 1
        # the MMA and dp4a products are the same integers: equal tokens, and
        # logits equal up to the order of the per-block float additions
        assert np.array_equal(t_s[i], t_d[i]), i
        assert compare_streams(t_s[i][:max_new], t_d[i][:max_new], l_d[i][first:first + max_new],
                               l_s[i][first:first + max_new]) >= 3, i
        # the streaming and tensor-core paths agree (until a near tie)
        assert compare_streams(t_s[i][:max_new], t_g[i][:max_new], l_g[i][first:first + max_new],
                               l_s[i][first:first + max_new]) >= 3, i
        # and the streaming path follows the oracle's stream
        ref_toks, ref_logits = om.generate(p, max_new, want_logits=True)
        assert compare_streams(t_s[i][:max_new], ref_toks, ref_logits,
                               l_s[i][first:first + max_new]) >= 3, i
    om.close()
    m.close()


def test_streaming_8b_layer_shapes(ctx):
    """Qwen3-8B layer and head shapes (K = 4096 over 8 sessions per CTA, the
    12288-wide down projection over two sets of 4): every session's logits
    within 1e-3 relative of its own single-session steps, same tokens."""
    from chat_wgpu_b200 import gguf
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, gguf.cached_model("qwen3-8b-2l", seed=0))
    prompts = _prompts(m.info["vocab"], [5, 2, 7, 3, 4, 6, 1, 8], 31)
    steps = 12
    t_s, l_s = _run_group(m, prompts, steps, 1, max_seq=32)
    for i, p in enumerate(prompts):
        s = Session(m, 32)
        s.set_persistent(False)
        s.begin(p)
        solo = []
        for _ in range(steps):
            s.run(1)
            solo.append(s.logits())
        toks = s.tokens()
        s.close()
        first = len(p) - 1
        assert compare_streams(t_s[i], toks, np.stack(solo[first:]), l_s[i][first:]) >= 1, i
    m.close()


def test_streaming_qwen3_0_6b_eight_sessions(ctx):
    """Benchmark config 3's scaling setup: 8 sessions of the bench's
    Qwen3-0.6B checkpoint stepped as one group (the streaming path, integer
    MMA products), each session's logits within 1e-3 relative of its own
    single-session persistent step and the same greedy tokens."""
    from chat_wgpu_b200 import gguf
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, gguf.cached_model("qwen3-0.6b", seed=0))
    prompts = _prompts(m.info["vocab"], [24, 9, 31, 16, 5, 40, 12, 20], 41)
    steps = 48
    t_s, l_s = _run_group(m, prompts, steps, 1, max_seq=96)
    for i, p in enumerate(prompts):
        s = Session(m, 96)
        s.begin(p)
        solo = []
        for _ in range(steps):
            s.run(1)
            solo.append(s.logits())
        toks = s.tokens()
        s.close()
        first = len(p) - 1
        assert compare_streams(t_s[i], toks, np.stack(solo[first:]), l_s[i][first:]) >= 3, i
    m.close()
