"""Hook taps (Hook::tap, src/model/mod.rs:155-165) against the oracle's taps.

The reference's forward hands its hook "q" after QK-norm + RoPE
(src/model/qwen3.rs:165), "post_attn" after the attention residual (:180)
and "layer_out" after the FFN residual (:188).  The session records them in
device rings as part of the captured step (and in batched prefill); every
recorded vector must match the oracle's within 1e-3 relative."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_model import models  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu
REL = 1e-3
NAMES = ("q", "post_attn", "layer_out")


def _oracle_taps(orc, path, seq, layer):
    om = orc.Model(path)
    om.reset(len(seq) + 1)
    om.set_tap(layer)
    out = []
    for pos, tok in enumerate(seq):
        om.step(int(tok), pos, want_logits=False)
        out.append(om.tap())
    om.close()
    return out


@pytest.mark.parametrize("name", ["tiny-qwen3", "small-qwen3", "tiny-gemma2", "tiny-qwen2"])
@pytest.mark.parametrize("where", ["first", "last"])
def test_taps_per_step(ctx, orc, models, name, where):  # noqa: F811
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models[name])
    layer = 0 if where == "first" else m.info["n_layers"] - 1
    seq = np.random.default_rng(3).integers(0, m.info["vocab"], 14).astype(np.uint32)
    ref = _oracle_taps(orc, models[name], seq, layer)
    s = Session(m, 32)
    for n in NAMES:
        s.add_tap(n, layer, 16)
    assert s.launches()[0] > 1  # taps run the per-stage kernels
    s.begin(seq[:6])
    for pos, tok in enumerate(seq):
        s.step(int(tok))  # the same input token at every position as the oracle
    for pos in range(len(seq)):
        for n in NAMES:
            assert rel_err(s.read_tap(n, layer, pos), ref[pos][n]) < REL, (n, pos)
    s.clear_taps()
    if name == "small-qwen3":
        assert s.persistent and s.launches() == (1, 1)
    s.close()
    m.close()


@pytest.mark.parametrize("name", ["small-qwen3", "tiny-gemma2"])
def test_taps_in_prefill(ctx, orc, models, name):  # noqa: F811
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models[name])
    L = m.info["n_layers"]
    prompt = np.random.default_rng(4).integers(0, m.info["vocab"], 24).astype(np.uint32)
    for layer in (1, L - 1):
        ref = _oracle_taps(orc, models[name], prompt, layer)
        s = Session(m, 32)
        for n in NAMES:
            s.add_tap(n, layer, 32)
        s.begin(prompt)
        assert s.prefill() == len(prompt) - 1
        s.run(1)  # the last prompt token through the step
        for pos in range(len(prompt)):
            for n in NAMES:
                assert rel_err(s.read_tap(n, layer, pos), ref[pos][n]) < REL, (layer, n, pos)
        s.close()
    m.close()


def test_tap_ring_and_errors(ctx, models):  # noqa: F811
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session
    m = Model(ctx, models["tiny-qwen3"])
    s = Session(m, 32)
    s.add_tap("layer_out", 1, 4)
    with pytest.raises(CwError):
        s.add_tap("layer_out", 1, 4)     # twice
    with pytest.raises(CwError):
        s.add_tap("k", 0, 4)             # unknown name
    with pytest.raises(CwError):
        s.add_tap("q", 9, 4)             # no such layer
    s.begin(np.array([1, 2, 3], np.uint32))
    s.run(10)
    assert s.read_tap("layer_out", 1, 9).shape == (m.info["dim"],)
    with pytest.raises(CwError):
        s.read_tap("layer_out", 1, 5)    # overwritten: the ring holds positions 6..9
    with pytest.raises(CwError):
        s.read_tap("layer_out", 1, 10)   # not run yet
    s.close()
    m.close()
