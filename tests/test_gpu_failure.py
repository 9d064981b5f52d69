"""The timeout path of the persistent step, exercised without a GPU fault.

Every device-side wait of the step (grid barriers, the attention-done
counters, the polls of the tagged QKV words, the weight ring's mbarriers)
is bounded by %globaltimer and reports through the
context's status word.  cw_session_inject_stall makes the next step's first
grid barrier wait for a count no CTA reaches; the step must give up after the
injected limit, every CTA must leave (draining its bulk copies), the next
synchronising call must fail with CW_ERR_TIMEOUT, and the context must then
run a clean session whose stream is identical to one that never stalled."""
import numpy as np
import pytest

from test_gpu_model import models, session_stream  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu
CW_ERR_TIMEOUT = 6


def test_injected_stall_times_out_and_context_recovers(ctx, models):  # noqa: F811
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["small-qwen3"])
    prompt = np.array([3, 1, 4, 1, 5, 9, 2, 6], np.uint32)
    ref_toks, ref_logits = session_stream(m, prompt, 6)

    s = Session(m, 32)
    assert s.persistent
    s.begin(prompt)
    s.run(3)
    s.inject_stall(200)  # 200 us
    s.run(1)
    with pytest.raises(CwError) as e:
        s.tokens()
    assert e.value.status == CW_ERR_TIMEOUT, e.value
    # the context still works: restart the session, the stream is unchanged
    s.begin(prompt)
    s.run(len(prompt) - 1)
    got = []
    for _ in range(6):
        s.run(1)
        got.append(s.logits())
    toks = s.tokens()
    assert np.array_equal(toks, ref_toks)
    assert np.array_equal(np.stack(got).view(np.uint32), ref_logits.view(np.uint32))
    s.close()
    # and a second session on the same context as well
    t2, l2 = session_stream(m, prompt, 6)
    assert np.array_equal(t2, ref_toks)
    m.close()


def test_inject_stall_needs_the_persistent_step(ctx, models):  # noqa: F811
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["tiny-qwen3"])  # the per-stage kernels only
    s = Session(m, 16)
    with pytest.raises(CwError):
        s.inject_stall(100)
    s.close()
    m.close()
