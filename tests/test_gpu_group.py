"""Co-batched decode (cw_group_*): several sessions stepped together with one
pass over the weights per step.  Every session must behave exactly like it
would alone: its logits within 1e-3 relative of the oracle's and its greedy
stream identical until the first ambiguous step (test_gpu_model gates); its
sampling draws and stop tokens as in its own step."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_model import REL, compare_streams, models  # noqa: F401  (fixture)
from test_gpu_sample import _draw_ok

pytestmark = pytest.mark.gpu


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, n).astype(np.uint32) for n in lens]


@pytest.mark.parametrize("name", ["tiny-qwen3", "small-qwen3", "tiny-gemma2", "tiny-qwen2"])
def test_group_vs_oracle(ctx, orc, models, name):  # noqa: F811
    from chat_wgpu_b200.model import Model, Session, SessionGroup
    m = Model(ctx, models[name])
    om = orc.Model(models[name])
    lens = [3, 9, 5, 12, 1]  # mixed: some sessions still in their prompt while others decode
    prompts = _prompts(om.vocab, lens, 11)
    max_new = 10
    ss = [Session(m, 40) for _ in prompts]
    for s, p in zip(ss, prompts):
        s.begin(p)
    g = SessionGroup(ss)
    total = max(lens) - 1 + max_new
    logits = [[] for _ in ss]
    for step in range(total):
        g.run(1)
        for i, (s, p) in enumerate(zip(ss, prompts)):
            if len(p) - 1 <= step < len(p) - 1 + max_new:
                logits[i].append(s.logits())
    for i, (s, p) in enumerate(zip(ss, prompts)):
        ref_toks, ref_logits = om.generate(p, max_new, want_logits=True)
        toks = s.tokens()[:max_new]
        assert compare_streams(toks, ref_toks, ref_logits, np.stack(logits[i])) >= 3, i
    g.close()
    for s in ss:
        s.close()
    m.close()
    om.close()


def test_group_sampling_eos_prefill(ctx, orc, models):  # noqa: F811
    from chat_wgpu_b200.model import Model, Session, SessionGroup
    m = Model(ctx, models["small-qwen3"])
    prompts = _prompts(m.info["vocab"], [20, 6, 6], 5)
    # reference greedy stream of session 2, to pick a stop token it will meet
    r = Session(m, 64)
    r.begin(prompts[2])
    r.run(5 + 12)
    greedy2 = r.tokens()
    r.close()
    stop = int(greedy2[3])
    first = int(np.argmax(greedy2 == stop))
    ss = [Session(m, 64) for _ in prompts]
    ss[1].set_sampling(0.8, 40, 0.9, seed=77)
    ss[2].set_eos([stop])
    for s, p in zip(ss, prompts):
        s.begin(p)
    assert ss[0].prefill() == 19  # a prefilled session joins at its last prompt token
    g = SessionGroup(ss)
    logits1 = []
    for step in range(17):
        g.run(1)
        if step >= 5:
            logits1.append(ss[1].logits())
    t1 = ss[1].tokens()
    assert len(t1) == 12
    for i, (t, lg) in enumerate(zip(t1, logits1)):
        assert _draw_ok(int(t), lg, 0.8, 40, 0.9, 77, i, orc), i
    assert ss[2].stopped and np.array_equal(ss[2].tokens(), greedy2[:first])
    # session 0 equals its own single-session continuation
    solo = Session(m, 64)
    solo.begin(prompts[0])
    solo.prefill()
    solo.run(17)
    a, b = ss[0].tokens(), solo.tokens()
    assert a[0] == b[0] and len(a) == len(b) == 17
    g.close()
    for s in ss + [solo]:
        s.close()
    m.close()


def test_group_errors(ctx, models):  # noqa: F811
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session, SessionGroup
    m = Model(ctx, models["tiny-qwen3"])
    m2 = Model(ctx, models["tiny-qwen2"])
    a, b, c = Session(m, 8), Session(m, 8), Session(m2, 8)
    with pytest.raises(CwError):
        SessionGroup([a, c])          # different models
    with pytest.raises(CwError):
        SessionGroup([a, a])          # duplicate
    g = SessionGroup([a, b])
    with pytest.raises(CwError):
        g.run(1)                      # sessions have not begun
    a.begin(np.array([1, 2], np.uint32))
    b.begin(np.array([3], np.uint32))
    g.run(8)
    with pytest.raises(CwError):
        g.run(1)                      # full
    g.close()
    for s in (a, b, c):
        s.close()
    m.close()
    m2.close()
