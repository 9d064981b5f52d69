"""Per-op host wrappers, one module per reference module in chat-wgpu
src/kernels/ (q4, attention, norm, rope, activation, argmax).  Each function
takes a GpuContext plus buffers and dimensions and returns a new arena
buffer, like its Rust counterpart."""
from . import activation, argmax, attention, norm, q4, rope  # noqa: F401
