"""cw_attention_noalloc: the attention entry point for callers that cannot
allocate device memory (their own pool owns the device, or their process
allocator must not see new blocks).  It must give the same result as
cw_attention while keeping its split scratch in the library's static device
array.

This file sorts last so that a run stopping at the first failure has run
every other test; it also passes on its own in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _call_noalloc(ctx, q, k, v, out, nh, nkv, seq, hd):
    from chat_wgpu_b200 import _lib
    stream = C.c_void_p()
    _lib.call("cw_ctx_stream", ctx.handle, C.byref(stream))
    _lib.call("cw_attention_noalloc", ctx.device, stream, q.device_ptr, k.device_ptr, v.device_ptr,
              out.device_ptr, nh, nkv, seq, hd)
    ctx.sync()


@pytest.mark.parametrize("nh,nkv,hd,seq", [(16, 8, 128, 384), (32, 8, 128, 4608), (8, 4, 256, 700),
                                           (4, 2, 16, 1)])
def test_noalloc_matches_attention_twice(nh, nkv, hd, seq):
    from chat_wgpu_b200.context import GpuContext
    from chat_wgpu_b200.kernels import attention
    ctx = GpuContext(0)
    rng = np.random.default_rng(seq + nh)
    out = ctx.empty_persistent(nh * hd)
    for call in range(2):  # two calls in a row share (and must reset) the scratch
        q = rng.normal(0, 1, nh * hd).astype(np.float32)
        k = rng.normal(0, 1, seq * nkv * hd).astype(np.float32)
        v = rng.normal(0, 1, seq * nkv * hd).astype(np.float32)
        Q, K, V = ctx.storage(q), ctx.storage(k), ctx.storage(v)
        ref = ctx.read(attention.attention(ctx, Q, K, V, nh, nkv, seq, hd), nh * hd)
        _call_noalloc(ctx, Q, K, V, out, nh, nkv, seq, hd)
        got = ctx.read(out, nh * hd)
        assert rel_err(got, ref) < 1e-3, (call, rel_err(got, ref))
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), call
    ctx.close()


def test_noalloc_rejects_oversize():
    from chat_wgpu_b200 import CwError
    from chat_wgpu_b200.context import GpuContext
    ctx = GpuContext(0)
    nh, nkv, hd, seq = 64, 8, 256, 8192  # partials larger than the static scratch
    q = ctx.empty_persistent(nh * hd)
    kv = ctx.empty_persistent(seq * nkv * hd)
    out = ctx.empty_persistent(nh * hd)
    with pytest.raises(CwError) as e:
        _call_noalloc(ctx, q, kv, kv, out, nh, nkv, seq, hd)
    assert e.value.status == 1 and "static scratch" in str(e.value)
    ctx.close()
