"""attention::attention and attention::add (chat-wgpu src/kernels/attention.rs)."""
from ..context import Buffer
from ._util import op


def attention(ctx, q: Buffer, k: Buffer, v: Buffer, n_heads: int, n_kv_heads: int, seq: int,
              head_dim: int, softcap: float = 0.0, window: int = 0) -> Buffer:
    """attention.rs:7-38; softcap/window are the family extensions (0 = off)."""
    if softcap or window:
        return op(ctx, "cw_attention_ext", q.handle, k.handle, v.handle, int(n_heads),
                  int(n_kv_heads), int(seq), int(head_dim), float(softcap), int(window))
    return op(ctx, "cw_attention", q.handle, k.handle, v.handle, int(n_heads), int(n_kv_heads),
              int(seq), int(head_dim))


def add(ctx, a: Buffer, b: Buffer, n: int) -> Buffer:
    """attention.rs:40-51: the residual connection c = a + b."""
    return op(ctx, "cw_add", a.handle, b.handle, int(n))
