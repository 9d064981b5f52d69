"""Shared fixtures.  Tests that need a B200 carry @pytest.mark.gpu; the rest
run on CPU (oracle, host logic, ABI surface, gloo multi-rank)."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA sm_100 device (B200)")
    config.addinivalue_line("markers", "slow: long-running (full-size model)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def ctx():
    from chat_wgpu_b200.context import GpuContext
    c = GpuContext(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def tiny_gguf(tmp_path_factory):
    from chat_wgpu_b200 import gguf
    d = tmp_path_factory.mktemp("models")
    return gguf.synth_model(str(d / "tiny-qwen3.gguf"), gguf.CONFIGS["tiny-qwen3"], seed=7)


def rel_err(got, ref):
    """Max |got-ref| / max(|ref|, 0.1*rms(ref)).

    The north-star gate is 1e-3 relative.  Outputs that sit near zero (a dot
    product whose terms cancel) cannot be held to a pure relative bound by
    any two f32 implementations that sum in different orders: the rounding
    noise of a K-term f32 sum is ~sqrt(K)*2^-24 of the typical output, i.e.
    ~5e-6*rms at K = 6144.  The floor 0.1*rms(ref) therefore allows near-zero
    outputs an absolute error of 1e-4*rms -- twenty times that noise, and
    two orders of magnitude below what a wrong row, block or scale produces."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    den = np.maximum(np.abs(ref), max(0.1 * rms, 1e-30))
    return float(np.max(np.abs(got - ref) / den)) if ref.size else 0.0
