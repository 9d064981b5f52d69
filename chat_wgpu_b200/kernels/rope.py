"""rope::rope (chat-wgpu src/kernels/rope.rs)."""
from ..context import Buffer
from ._util import op


def rope(ctx, x: Buffer, rows: int, head_dim: int, pos: int, theta: float) -> Buffer:
    """Rotate-half RoPE of rows x head_dim at position pos (rope.rs:8-27)."""
    return op(ctx, "cw_rope", x.handle, int(rows), int(head_dim), int(pos), float(theta))
