"""argmax::argmax (chat-wgpu src/kernels/argmax.rs)."""
from ..context import Buffer
from ._util import op


def argmax(ctx, logits: Buffer, n: int) -> Buffer:
    """Index of the max logit as a 1-element u32 buffer; ties -> lowest index.
    Read it with ctx.read_u32(buf, 1)."""
    return op(ctx, "cw_argmax", logits.handle, int(n))
