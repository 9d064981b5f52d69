"""chat_wgpu_b200 -- B200-native (sm_100a) replacement for the GPU layer of
EggerMarc/chat-wgpu's batch-1 decode loop.

Layout:
  csrc/        CUDA kernels, the C-ABI (include/chatcuda.h), GGUF reader,
               model/session code -> libchatcuda.so (built in-tree)
  context.py   GpuContext (the surface of chat-wgpu src/context.rs)
  kernels/     per-op wrappers (the surface of chat-wgpu src/kernels/)
  model.py     Model / Session / generate (chat-wgpu src/model/)
  gguf.py      GGUF writer/reader and seeded random-init checkpoints
"""
from . import _lib  # noqa: F401
from ._lib import CwError  # noqa: F401

__all__ = ["CwError", "GpuContext", "Model", "Session", "generate", "build"]


def build(force: bool = False) -> str:
    """Compile libchatcuda.so for sm_100a with nvcc (no GPU needed)."""
    from .build import build_library
    return build_library(force=force)


def __getattr__(name):
    if name == "GpuContext":
        from .context import GpuContext
        return GpuContext
    if name in ("Model", "Session", "generate"):
        from . import model
        return getattr(model, name)
    raise AttributeError(name)
