"""Host side of the k-quant model files (no GPU): the synthetic Q4_K_M-style
and Q5_K writers produce the per-tensor types and block sizes of ggml's
layouts, the weights they encode centre near zero at the Q4_0 files' scale,
and the oracle reads and runs them (its dequantisation of the blocks is
pinned in test_oracle_kat)."""
import numpy as np
import pytest

from chat_wgpu_b200 import gguf


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("kq_cpu")
    return {n: gguf.synth_model(str(d / f"{n}.gguf"), gguf.CONFIGS[n], seed=5)
            for n in ("small-qwen3-q4km", "tiny-qwen2-q5k")}


def test_tensor_types_and_sizes(files):
    r = gguf.GgufReader(files["small-qwen3-q4km"])
    want = {"token_embd.weight": gguf.GGML_Q4_K, "output.weight": gguf.GGML_Q4_K,
            "blk.0.attn_q.weight": gguf.GGML_Q4_K, "blk.0.attn_k.weight": gguf.GGML_Q4_K,
            "blk.0.attn_v.weight": gguf.GGML_Q6_K, "blk.0.attn_output.weight": gguf.GGML_Q4_K,
            "blk.0.ffn_gate.weight": gguf.GGML_Q4_K, "blk.0.ffn_up.weight": gguf.GGML_Q4_K,
            "blk.0.ffn_down.weight": gguf.GGML_Q6_K}
    size = {gguf.GGML_Q4_K: 144, gguf.GGML_Q5_K: 176, gguf.GGML_Q6_K: 210}
    for name, t in want.items():
        tt, dims, raw = r.tensor(name)
        assert tt == t, name
        assert len(raw) == int(np.prod(dims)) // 256 * size[t], name
    r.close()
    r = gguf.GgufReader(files["tiny-qwen2-q5k"])
    assert r.tensor("blk.1.ffn_down.weight")[0] == gguf.GGML_Q5_K
    assert r.tensor("token_embd.weight")[0] == gguf.GGML_Q4_0
    r.close()


@pytest.mark.parametrize("five", [False, True], ids=["q4_k", "q5_k"])
def test_random_blocks_centre_near_zero(orc, five):
    rng = np.random.default_rng(0)
    b = gguf.random_q45_k_blocks(rng, 64, 1024, five)
    w = (orc.dequant_q5_k if five else orc.dequant_q4_k)(b.tobytes(), 64 * 1024)
    assert abs(float(np.mean(w))) < 0.01
    assert 0.005 < float(np.std(w)) < 0.1


def test_oracle_runs_kquant_models(orc, files):
    for name, path in files.items():
        om = orc.Model(path)
        prompt = np.array([1, 5, 9, 2], np.uint32) % om.vocab
        t1, l1 = om.generate(prompt, 3, want_logits=True)
        om.close()
        om = orc.Model(path)
        t2 = om.generate(prompt, 3)
        om.close()
        assert np.array_equal(t1, t2)
        assert np.all(np.isfinite(l1))
