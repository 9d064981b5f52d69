"""argmax::argmax (chat-wgpu src/kernels/argmax.rs)."""
from ..context import Buffer
from ._util import op


def argmax(ctx, logits: Buffer, n: int) -> Buffer:
    """Index of the max logit as a 1-element u32 buffer; ties -> lowest index.
    Read it with ctx.read_u32(buf, 1)."""
    return op(ctx, "cw_argmax", logits.handle, int(n))


def sample(ctx, logits: Buffer, n: int, temperature: float, top_k: int = 0, top_p: float = 1.0,
           seed: int = 0, draw: int = 0) -> Buffer:
    """One temperature / top-k / top-p draw (the rules of
    Session.set_sampling) as a 1-element u32 buffer; temperature 0 = argmax."""
    return op(ctx, "cw_sample", logits.handle, int(n), float(temperature), int(top_k),
              float(top_p), int(seed) & (2**64 - 1), int(draw) & (2**64 - 1))
