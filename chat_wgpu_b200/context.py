"""GpuContext: the buffer / dispatch / readback surface of chat-wgpu's
src/context.rs, over libchatcuda.so.

Method names and meanings follow the reference: `storage`, `storage_u32`,
`empty` (a per-frame arena slot, context.rs:207-227), `empty_persistent`,
`copy` (offsets in f32 elements, context.rs:252-269), `read` (flush + wait +
copy back, context.rs:359-389), `flush`, `reset_frame`, `clear_cache`,
`begin_profile` / `report_profile` (context.rs:106-126).
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _lib


class Buffer:
    """A device buffer handle (the analogue of wgpu::Buffer)."""

    __slots__ = ("ctx", "handle")

    def __init__(self, ctx: "GpuContext", handle: int):
        self.ctx = ctx
        self.handle = int(handle)

    @property
    def nbytes(self) -> int:
        n = C.c_size_t()
        _lib.call("cw_buf_nbytes", self.ctx._h, self.handle, C.byref(n))
        return int(n.value)

    @property
    def device_ptr(self) -> int:
        p = C.c_void_p()
        _lib.call("cw_buf_device_ptr", self.ctx._h, self.handle, C.byref(p))
        return int(p.value or 0)

    def release(self) -> None:
        _lib.call("cw_buf_release", self.ctx._h, self.handle)

    def __repr__(self) -> str:
        return f"Buffer({self.handle})"


def _np(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=dtype))


class GpuContext:
    """GpuContext::new (context.rs:60-104) on CUDA device `device`."""

    def __init__(self, device: int = 0):
        _lib.load()
        h = C.c_void_p()
        _lib.call("cw_ctx_create", int(device), C.byref(h))
        self._h = h
        # models (and through them sessions) made on this context: released
        # before the context itself, whatever order Python drops them in
        self._dependents = weakref.WeakSet()
        buf = C.create_string_buffer(256)
        _lib.call("cw_ctx_backend", self._h, buf, 256)
        self.backend = buf.value.decode()
        self.device = int(device)

    # -- lifetime -------------------------------------------------------------
    def _adopt(self, obj) -> None:
        self._dependents.add(obj)

    def close(self) -> None:
        if getattr(self, "_h", None):
            for obj in list(getattr(self, "_dependents", ())):
                obj.close()
            _lib.load().cw_ctx_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    # -- buffers ----------------------------------------------------------------
    def _new(self, fn: str, *args) -> Buffer:
        b = C.c_uint64()
        _lib.call(fn, self._h, *args, C.byref(b))
        return Buffer(self, b.value)

    def storage(self, data) -> Buffer:
        """GpuContext::storage (context.rs:177-184)."""
        a = _np(data, np.float32).ravel()
        return self._new("cw_storage", a.ctypes.data, a.size)

    def storage_u32(self, data) -> Buffer:
        """GpuContext::storage_u32 (context.rs:187-194)."""
        a = _np(data, np.uint32).ravel()
        return self._new("cw_storage_u32", a.ctypes.data, a.size)

    def storage_bytes(self, data) -> Buffer:
        a = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) \
            else np.ascontiguousarray(data).view(np.uint8).ravel()
        return self._new("cw_storage_bytes", a.ctypes.data, a.size)

    def empty(self, length: int) -> Buffer:
        """GpuContext::empty (context.rs:207-227): arena slot, valid until reset_frame."""
        return self._new("cw_empty", int(length))

    def empty_persistent(self, length: int) -> Buffer:
        """GpuContext::empty_persistent (context.rs:229-232), zero-filled."""
        return self._new("cw_empty_persistent", int(length))

    def copy(self, src: Buffer, src_off: int, dst: Buffer, dst_off: int, length: int) -> None:
        """GpuContext::copy (context.rs:252-269); offsets/length in f32 elements."""
        _lib.call("cw_copy", self._h, src.handle, int(src_off), dst.handle, int(dst_off), int(length))

    def write(self, dst: Buffer, dst_off: int, data) -> None:
        a = _np(data, np.float32).ravel()
        _lib.call("cw_write", self._h, dst.handle, int(dst_off), a.ctypes.data, a.size)

    def read(self, src: Buffer, length: int) -> np.ndarray:
        """GpuContext::read (context.rs:359-389): flush, wait, copy `length` f32s back."""
        out = np.empty(int(length), dtype=np.float32)
        _lib.call("cw_read", self._h, src.handle, out.ctypes.data, out.size)
        return out

    def read_u32(self, src: Buffer, length: int) -> np.ndarray:
        """read() reinterpreted as u32 (the `.to_bits()` of src/model/mod.rs:103)."""
        out = np.empty(int(length), dtype=np.uint32)
        _lib.call("cw_read_u32", self._h, src.handle, out.ctypes.data, out.size)
        return out

    # -- frame / submission -----------------------------------------------------
    def flush(self) -> None:
        _lib.call("cw_flush", self._h)

    def sync(self) -> None:
        _lib.call("cw_sync", self._h)

    def reset_frame(self) -> None:
        _lib.call("cw_reset_frame", self._h)

    def clear_cache(self) -> None:
        _lib.call("cw_clear_cache", self._h)

    # -- profiler ---------------------------------------------------------------
    def begin_profile(self) -> None:
        _lib.call("cw_begin_profile", self._h)

    def report_profile(self) -> list[tuple[str, int, float]]:
        """(kernel, passes, total_ms) sorted by total descending (profile.rs:86-117)."""
        n = C.c_size_t()
        rows = (_lib.ProfileRow * 256)()
        _lib.call("cw_report_profile", self._h, rows, 256, C.byref(n))
        return [(rows[i].kernel.decode(), int(rows[i].passes), float(rows[i].total_ms))
                for i in range(min(n.value, 256))]


def print_report(rows) -> str:
    """Per-kernel breakdown table in the layout of src/profile.rs:121-134."""
    total = sum(r[2] for r in rows)
    lines = ["┌─ GPU per-kernel breakdown ──────────────────────────────────",
             f"│ {'kernel':<16} {'passes':>7} {'total ms':>10} {'µs/pass':>9} {'%':>6}",
             "├─────────────────────────────────────────────────────────────"]
    for name, count, ms in rows:
        per = ms * 1000.0 / count if count else 0.0
        pct = ms / total * 100.0 if total > 0 else 0.0
        lines.append(f"│ {name:<16} {count:>7} {ms:>10.3f} {per:>9.1f} {pct:>5.1f}%")
    lines.append("├─────────────────────────────────────────────────────────────")
    lines.append(f"│ {'TOTAL':<16} {'':>7} {total:>10.3f}")
    lines.append("└─────────────────────────────────────────────────────────────")
    return "\n".join(lines)
