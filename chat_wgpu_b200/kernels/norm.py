"""norm::rmsnorm / norm::rmsnorm_unit (chat-wgpu src/kernels/norm.rs)."""
from ..context import Buffer
from ._util import op


def rmsnorm(ctx, x: Buffer, w: Buffer, rows: int, dim: int, eps: float) -> Buffer:
    """y = x / rms * w (norm.rs:25-29)."""
    return op(ctx, "cw_rmsnorm", x.handle, w.handle, int(rows), int(dim), float(eps))


def rmsnorm_unit(ctx, x: Buffer, w: Buffer, rows: int, dim: int, eps: float) -> Buffer:
    """y = x / rms * (1 + w) (norm.rs:31-35)."""
    return op(ctx, "cw_rmsnorm_unit", x.handle, w.handle, int(rows), int(dim), float(eps))
