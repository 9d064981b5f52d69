import ctypes as C

from .. import _lib
from ..context import Buffer


def op(ctx, fn: str, *args) -> Buffer:
    out = C.c_uint64()
    _lib.call(fn, ctx.handle, *args, C.byref(out))
    return Buffer(ctx, out.value)
