"""Projections, embeddings and LM heads of the other GGUF types the
reference's loader takes (tensor_f32, src/loader/gguf.rs:109-121: F32, F16,
Q4_1, Q8_0, dequantised by dequant.rs:9-21, 46-58, 82-97) plus BF16
(dequant_bf16, dequant.rs:41-43), kept raw in HBM and read by the per-stage
GEMVs 256 weights at a time.

  * dequantisation (cw_kquant_dequant) bit-exact against the oracle's
    restatement of dequant.rs for every type;
  * the GEMV (cw_kquant_gemv) within 1e-3 relative of the oracle's dense
    dot (the reference's Proj::Dense, src/model/layers.rs:103-117: f32
    weights, sequential f32 dot, src/kernels/matmul.wgsl); Q8_0 also through
    the streaming GEMV over its split planes (cw_q8_0_split / cw_q8_0_gemv),
    the form the model's decode projections use;
  * whole models against the oracle's forward: a mix of F16 / Q8_0 / Q4_1 /
    F32 projections (q/k/v of different types), a Q8_0 embedding and an
    F16 untied head; an all-F32 qwen2 model with q/k/v biases (the
    reference's dense path over an f32 file); BF16 projections under an F16
    tied embedding.  Gates as for the Q4_0 models (test_gpu_model)."""
import numpy as np
import pytest

from conftest import rel_err
from test_gpu_model import REL, compare_streams, session_stream

pytestmark = pytest.mark.gpu

TYPES = {"f32": 0, "f16": 1, "q4_1": 3, "q8_0": 8, "bf16": 30}
NAMES = ["small-qwen3-mixed", "tiny-qwen2-f32", "small-qwen3-bf16"]


def _raw(kind, rng, rows, in_f):
    from chat_wgpu_b200 import gguf
    if kind == "q8_0":
        return gguf.random_q8_0_blocks(rng, rows, in_f).ravel()
    if kind == "q4_1":
        return gguf.random_q4_1_blocks(rng, rows, in_f).ravel()
    return np.ascontiguousarray(gguf.random_dense(rng, rows, in_f, kind)).view(np.uint8).ravel()


def _oracle_dequant(orc, kind, raw, n):
    """The oracle's restatement of dequant.rs for `kind`."""
    if kind == "f32":
        return raw.view(np.float32).copy()
    if kind == "bf16":
        return np.array([orc.bf16_to_f32(int(v)) for v in raw.view(np.uint16)], np.float32)
    fn = {"f16": "orc_dequant_f16", "q8_0": "orc_dequant_q8_0", "q4_1": "orc_dequant_q4_1"}[kind]
    return orc._deq(fn, raw, n)


@pytest.mark.parametrize("kind", sorted(TYPES))
def test_dequant_bit_exact(ctx, orc, kind):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(TYPES[kind] + 3)
    rows, in_f = 24, 512 if kind != "bf16" else 256
    raw = _raw(kind, rng, rows, in_f)
    got = ctx.read(q4.kquant_dequant(ctx, ctx.storage_bytes(raw), TYPES[kind], rows, in_f),
                   rows * in_f)
    ref = _oracle_dequant(orc, kind, raw, rows * in_f)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), kind


@pytest.mark.parametrize("kind", sorted(TYPES))
@pytest.mark.parametrize("in_f,out_f", [(256, 64), (1024, 3072), (4096, 512)])
def test_gemv_vs_dense_oracle(ctx, orc, kind, in_f, out_f):
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(in_f + out_f + TYPES[kind])
    raw = _raw(kind, rng, out_f, in_f)
    x = rng.normal(0, 1, in_f).astype(np.float32)
    got = ctx.read(q4.kquant_gemv(ctx, ctx.storage(x), ctx.storage_bytes(raw), TYPES[kind], in_f,
                                  out_f), out_f)
    w = _oracle_dequant(orc, kind, raw, out_f * in_f).reshape(out_f, in_f)
    ref = (w.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)  # exact-grade dot
    assert rel_err(got, ref) < REL, (kind, rel_err(got, ref))


@pytest.mark.parametrize("in_f,out_f", [(256, 64), (1024, 3072), (4096, 512), (3072, 77)])
def test_q8_0_split_gemv_vs_dense_oracle(ctx, orc, in_f, out_f):
    """The streaming GEMV over the Q8_0 code/scale planes (the decode step's
    form) against the oracle's dense product and the per-row kernel."""
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.kernels import q4
    rng = np.random.default_rng(5 * in_f + out_f)
    raw = _raw("q8_0", rng, out_f, in_f)
    x = rng.normal(0, 1, in_f).astype(np.float32)
    w = ctx.storage_bytes(raw)
    ws = q4.q8_0_split(ctx, w, out_f, in_f)
    xb = ctx.storage(x)
    got = ctx.read(q4.q8_0_gemv(ctx, xb, ws, in_f, out_f), out_f)
    wd = _oracle_dequant(orc, "q8_0", raw, out_f * in_f).reshape(out_f, in_f)
    ref = (wd.astype(np.float64) @ x.astype(np.float64)).astype(np.float32)
    assert rel_err(got, ref) < REL, rel_err(got, ref)
    row = ctx.read(q4.kquant_gemv(ctx, xb, w, TYPES["q8_0"], in_f, out_f), out_f)
    assert rel_err(got, row) < REL
    with pytest.raises(CwError):  # a raw weight is not a split one
        q4.q8_0_gemv(ctx, xb, w, in_f, out_f)
    ws.release()
    w.release()


@pytest.fixture(scope="module")
def dt_models(tmp_path_factory):
    from chat_wgpu_b200 import gguf
    d = tmp_path_factory.mktemp("dtype_models")
    return {n: gguf.synth_model(str(d / f"{n}.gguf"), gguf.CONFIGS[n], seed=23) for n in NAMES}


@pytest.mark.parametrize("use_graph", [True, False], ids=["graph", "direct"])
@pytest.mark.parametrize("name", NAMES)
def test_dtype_models_vs_oracle(ctx, orc, dt_models, name, use_graph):
    from chat_wgpu_b200.model import Model
    om = orc.Model(dt_models[name])
    prompt = np.array([1, 5, 9, 2, 77, 3, 41, 8], np.uint32) % om.vocab
    ref_toks, ref_logits = om.generate(prompt, 16, want_logits=True)
    m = Model(ctx, dt_models[name])
    toks, logits = session_stream(m, prompt, 16, use_graph=use_graph)
    assert compare_streams(toks, ref_toks, ref_logits, logits) >= 1
    same = 0
    while same < len(toks) and toks[same] == ref_toks[same]:
        assert rel_err(logits[same], ref_logits[same]) < REL, same
        same += 1
    assert same >= 4
    m.close()
    om.close()


def test_dtype_model_refuses_q4_0_only_paths(ctx, dt_models):
    """The persistent step, batched prefill and session groups take Q4_0
    projections: these models run the per-stage kernels and those calls fail
    with a status."""
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.model import Model, Session, SessionGroup
    m = Model(ctx, dt_models["small-qwen3-mixed"])
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
