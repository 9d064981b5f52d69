"""Sampling and stop tokens on the device (cw_sample, cw_session_set_sampling,
cw_session_set_eos) against the oracle's restatement (oracle.sample).

The reference decodes greedily and stops its chat loop on EOS ids before
emitting them (src/wasm.rs:48-51,99-101); temperature / top-k / top-p are on
its roadmap only (ROADMAP.md:56-57), so the oracle restates the documented
rules.  A draw is exact in fixed point except for expf's last-bit rounding,
so a GPU token that differs from the oracle's must sit on a mass boundary:
the target lies within a relative 1e-5 of the oracle's cumulative mass at
that token's edge."""
import numpy as np
import pytest

from test_gpu_model import models  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu


def _draw_ok(got, logits, T, k, p, seed, draw, orc):
    ref, d = orc.sample(logits, T, k, p, seed=seed, draw=draw)
    if got == ref:
        return True
    if d is None:
        return False
    tol = max(1, int(1e-5 * d["Z"]))
    incl = d["incl"].astype(np.int64)
    lo = int(incl[got - 1]) if got > 0 else 0
    hi = int(incl[got])
    # the GPU token's interval [lo, hi) must (nearly) contain the target, and
    # the oracle's own token must be adjacent across that boundary
    return lo - tol <= d["target"] < hi + tol


CASES = [(0.0, 0, 1.0), (1.0, 0, 1.0), (0.7, 40, 1.0), (1.0, 0, 0.9), (1.5, 64, 0.8),
         (0.3, 0, 0.5), (2.0, 1, 1.0), (1.0, 0, 0.0)]


@pytest.mark.parametrize("n", [1000, 151936])
@pytest.mark.parametrize("T,k,p", CASES)
def test_sample_op_vs_oracle(ctx, orc, n, T, k, p):
    from chat_wgpu_b200.kernels.argmax import sample
    rng = np.random.default_rng(n + int(100 * T) + k)
    logits = rng.normal(0, 3, n).astype(np.float32)
    buf = ctx.storage(logits)
    for draw in range(12):
        got = int(ctx.read_u32(sample(ctx, buf, n, T, k, p, seed=42, draw=draw), 1)[0])
        assert _draw_ok(got, logits, T, k, p, 42, draw, orc), (draw, got)
        ctx.reset_frame()


def test_sample_edges(ctx, orc):
    from chat_wgpu_b200.kernels.argmax import sample
    # ties at the max with T = 0 -> lowest index; NaN never drawn
    l = np.array([1.0, 5.0, np.nan, 5.0, -np.inf, 2.0], np.float32)
    b = ctx.storage(l)
    assert int(ctx.read_u32(sample(ctx, b, 6, 0.0), 1)[0]) == 1
    seen = set()
    for d in range(64):
        t = int(ctx.read_u32(sample(ctx, b, 6, 1.0, seed=3, draw=d), 1)[0])
        assert t in (0, 1, 3, 5)
        seen.add(t)
        ctx.reset_frame()
    assert {1, 3} <= seen
    # top_k = 1 keeps the tied maxima (1 and 3) only; without a tie it is greedy
    for d in range(16):
        assert int(ctx.read_u32(sample(ctx, b, 6, 5.0, top_k=1, seed=9, draw=d), 1)[0]) in (1, 3)
        ctx.reset_frame()
    b2 = ctx.storage(np.array([1.0, 5.0, np.nan, 4.0, -np.inf, 2.0], np.float32))
    for d in range(8):
        assert int(ctx.read_u32(sample(ctx, b2, 6, 5.0, top_k=1, seed=9, draw=d), 1)[0]) == 1
        ctx.reset_frame()


def test_sample_distribution(ctx, orc):
    """Empirical frequencies of 3000 draws follow softmax(l / T)."""
    from chat_wgpu_b200.kernels.argmax import sample
    rng = np.random.default_rng(1)
    l = rng.normal(0, 1, 50).astype(np.float32)
    b = ctx.storage(l)
    T = 1.5
    cnt = np.zeros(50)
    for d in range(3000):
        cnt[int(ctx.read_u32(sample(ctx, b, 50, T, seed=7, draw=d), 1)[0])] += 1
        ctx.reset_frame()
    p = np.exp((l - l.max()) / T)
    p /= p.sum()
    assert np.abs(cnt / 3000 - p).max() < 0.03


@pytest.mark.parametrize("persistent", [False, True])
def test_session_sampling_matches_oracle_on_its_logits(ctx, orc, models, persistent):  # noqa: F811
    """Inside the decode step: each produced token is the oracle's draw on the
    step's own logits with draw index = tokens produced before it."""
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["small-qwen3"])
    s = Session(m, 64)
    s.set_persistent(persistent)
    T, k, p, seed = 0.9, 50, 0.95, 1234
    s.set_sampling(T, k, p, seed)
    prompt = np.array([5, 9, 2, 77, 3], np.uint32)
    s.begin(prompt)
    s.run(len(prompt) - 1)
    logits = []
    for _ in range(16):
        s.run(1)
        logits.append(s.logits())
    toks = s.tokens()
    assert len(toks) == 16
    for i, (t, lg) in enumerate(zip(toks, logits)):
        assert _draw_ok(int(t), lg, T, k, p, seed, i, orc), i
    # the greedy stream differs: sampling really happened
    s.set_sampling(0.0)
    s.begin(prompt)
    s.run(len(prompt) - 1 + 16)
    assert not np.array_equal(s.tokens(), toks)
    s.close()
    m.close()


@pytest.mark.parametrize("persistent", [False, True])
def test_session_eos_stops(ctx, models, persistent):  # noqa: F811
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["small-qwen3"])
    s = Session(m, 64)
    s.set_persistent(persistent)
    prompt = np.array([1, 2, 3], np.uint32)
    s.begin(prompt)
    s.run(2 + 10)
    greedy = s.tokens()
    stop = int(greedy[4])
    first = int(np.argmax(greedy == stop))  # first occurrence of the stop token
    s.set_eos([stop])
    s.begin(prompt)
    produced = 0
    n = s.run(2)
    produced += s.run(10)
    assert produced == first and np.array_equal(s.tokens(), greedy[:first]) and n == 0
    assert s.stopped
    assert s.run(3) == 0 and len(s.tokens()) == first
    # the per-token API returns the stop token once, then nothing
    s.begin(prompt)
    assert not s.stopped
    out = [s.step(Session.TOKEN_DEVICE) for _ in range(2 + first + 3)]
    dec = out[2:]
    assert dec[:first] == list(greedy[:first]) and dec[first] == stop
    assert all(t == Session.TOKEN_DEVICE for t in dec[first + 1:])
    assert len(s.tokens()) == first
    s.set_eos([])
    s.begin(prompt)
    s.run(12)
    assert np.array_equal(s.tokens(), greedy)
    s.close()
    m.close()
