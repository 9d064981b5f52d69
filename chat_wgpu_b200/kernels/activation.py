"""Gated activations (chat-wgpu src/kernels/activation.rs:42-48)."""
from ..context import Buffer
from ._util import op


def swiglu(ctx, gate: Buffer, up: Buffer, n: int) -> Buffer:
    """silu(gate) * up."""
    return op(ctx, "cw_swiglu", gate.handle, up.handle, int(n))


def geglu(ctx, gate: Buffer, up: Buffer, n: int) -> Buffer:
    """gelu_tanh(gate) * up."""
    return op(ctx, "cw_geglu", gate.handle, up.handle, int(n))
