"""Models whose projections are GGUF k-quants (Q4_K / Q5_K / Q6_K blocks kept
raw in HBM), in the mixes of Q4_K_M-style files: q/k/v of different types
(three weights over one qkv vector), Q6_K down projections, Q4_K token
embedding and LM head, and a Q5_K variant with biases; and Q4_0 projections
under a Q5_K token embedding shared with the head (batched prefill
included).  The reference has no k-quant projections (ROADMAP.md:52-53);
the oracle dequantises ggml's published block layouts
(pinned by test_oracle_kat) and runs the same forward.  Gates as for the
Q4_0 models (test_gpu_model): tokens until the first ambiguous step, logits
within 1e-3 relative.  The paths that take Q4_0 only refuse these models."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_model import REL, compare_streams, session_stream

pytestmark = pytest.mark.gpu

NAMES = ["small-qwen3-q4km", "tiny-qwen2-q5k", "small-qwen3-q5k-embed"]


@pytest.fixture(scope="module")
def kq_models(tmp_path_factory):
    from chat_wgpu_b200 import gguf
    d = tmp_path_factory.mktemp("kq_models")
    return {n: gguf.synth_model(str(d / f"{n}.gguf"), gguf.CONFIGS[n], seed=17) for n in NAMES}


@pytest.mark.parametrize("use_graph", [True, False], ids=["graph", "direct"])
@pytest.mark.parametrize("name", NAMES)
def test_kquant_projections_vs_oracle(ctx, orc, kq_models, name, use_graph):
    from chat_wgpu_b200.model import Model
    om = orc.Model(kq_models[name])
    prompt = np.array([1, 5, 9, 2, 77, 3, 41, 8], np.uint32) % om.vocab
    ref_toks, ref_logits = om.generate(prompt, 16, want_logits=True)
    m = Model(ctx, kq_models[name])
    toks, logits = session_stream(m, prompt, 16, use_graph=use_graph)
    assert compare_streams(toks, ref_toks, ref_logits, logits) >= 1
    same = 0  # every step on which the streams still agree
    while same < len(toks) and toks[same] == ref_toks[same]:
        assert rel_err(logits[same], ref_logits[same]) < REL, same
        same += 1
    assert same >= 4
    m.close()
    om.close()


def test_kquant_model_refuses_q4_0_only_paths(ctx, kq_models):
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session, SessionGroup
    m = Model(ctx, kq_models["small-qwen3-q4km"])
    s = Session(m, 32)
    assert not s.persistent
    with pytest.raises(CwError):
        s.set_persistent(True)
    s.begin(np.arange(1, 9, dtype=np.uint32))
    with pytest.raises(CwError):
        s.prefill()
    with pytest.raises(CwError):
        SessionGroup([s])
    s.close()
    m.close()


def test_kquant_embedding_with_prefill(ctx, orc, kq_models):
    """Q4_0 projections: the tensor-core prefill runs under a Q5_K embedding."""
    from chat_wgpu_b200.model import Model, Session
    path = kq_models["small-qwen3-q5k-embed"]
    om = orc.Model(path)
    prompt = np.random.default_rng(3).integers(0, om.vocab, 24).astype(np.uint32)
    ref_toks, ref_logits = om.generate(prompt, 8, want_logits=True)
    m = Model(ctx, path)
    s = Session(m, 40)
    s.begin(prompt)
    assert s.prefill() == len(prompt) - 1
    logits = []
    for _ in range(8):
        s.run(1)
        logits.append(s.logits())
    assert compare_streams(s.tokens(), ref_toks, ref_logits, np.stack(logits)) >= 1
    s.close()
    m.close()
    om.close()
