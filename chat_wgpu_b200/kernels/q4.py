"""q4 GEMV building blocks (chat-wgpu src/kernels/q4.rs) plus the GGUF-native
Q4_0 weight format that the B200 decode path keeps in HBM."""
from __future__ import annotations

import ctypes as C

import numpy as np

from .. import _lib
from ..context import Buffer
from ._util import op


def gemv(ctx, x: Buffer, scales: Buffer, quants: Buffer, in_f: int, out_f: int) -> Buffer:
    """q4::gemv (q4.rs:9-30): y[out_f] over the crate's re-quantised layout."""
    return op(ctx, "cw_q4_gemv", x.handle, scales.handle, quants.handle, int(in_f), int(out_f))


def quantize_q4_0(ctx, w: Buffer, out_f: int, in_f: int) -> tuple[Buffer, Buffer]:
    """q4::quantize_q4_0 (q4.rs:37-60) on the device -> (scales, quants)."""
    s, q = C.c_uint64(), C.c_uint64()
    _lib.call("cw_q4_quantize", ctx.handle, w.handle, int(out_f), int(in_f), C.byref(s), C.byref(q))
    return Buffer(ctx, s.value), Buffer(ctx, q.value)


def q4_0_upload(ctx, gguf_blocks, rows: int, in_f: int) -> Buffer:
    """Upload GGUF Q4_0 blocks of a [rows, in_f] tensor as a packed weight."""
    a = np.ascontiguousarray(gguf_blocks).view(np.uint8).ravel()
    if a.size != rows * (in_f // 32) * 18:
        raise ValueError(f"expected {rows * (in_f // 32) * 18} bytes of Q4_0 blocks, got {a.size}")
    return op(ctx, "cw_q4_0_upload", a.ctypes.data, int(rows), int(in_f))


def q4_0_pack(ctx, gguf_blocks: Buffer, rows: int, in_f: int) -> Buffer:
    return op(ctx, "cw_q4_0_pack", gguf_blocks.handle, int(rows), int(in_f))


def q4_0_gemv(ctx, x: Buffer, w: Buffer, in_f: int, out_f: int) -> Buffer:
    """y[out_f] = W x over a packed GGUF Q4_0 weight."""
    return op(ctx, "cw_q4_0_gemv", x.handle, w.handle, int(in_f), int(out_f))


def q4_0_gemm(ctx, x: Buffer, w: Buffer, rows: int, in_f: int, out_f: int) -> Buffer:
    """Y[rows, out_f] = X[rows, in_f] W^T over a packed Q4_0 weight on the
    tcgen05 tensor cores (the batched prefill form of q4_0_gemv)."""
    return op(ctx, "cw_q4_0_gemm", x.handle, w.handle, int(rows), int(in_f), int(out_f))


def q4_0_dequant(ctx, w: Buffer, rows: int, in_f: int) -> Buffer:
    """Exact f32 dequantisation of a packed weight (dequant.rs:62-78)."""
    return op(ctx, "cw_q4_0_dequant", w.handle, int(rows), int(in_f))


# ---- GGUF k-quants (raw blocks in HBM) -------------------------------------------
Q4_K, Q5_K, Q6_K = 12, 13, 14
KQ_BLOCK_BYTES = {Q4_K: 144, Q5_K: 176, Q6_K: 210}


def kquant_gemv(ctx, x: Buffer, w: Buffer, qtype: int, in_f: int, out_f: int) -> Buffer:
    """y[out_f] = W x over raw GGUF Q4_K / Q5_K / Q6_K blocks (cw_storage_bytes)."""
    return op(ctx, "cw_kquant_gemv", x.handle, w.handle, int(qtype), int(in_f), int(out_f))


def kquant_dequant(ctx, w: Buffer, qtype: int, rows: int, in_f: int) -> Buffer:
    """Exact f32 dequantisation of a raw k-quant weight [rows, in_f]."""
    return op(ctx, "cw_kquant_dequant", w.handle, int(qtype), int(rows), int(in_f))


def q6_k_split(ctx, w: Buffer, rows: int, in_f: int) -> Buffer:
    """Raw Q6_K blocks -> the streaming GEMV's aligned planes (a new buffer)."""
    return op(ctx, "cw_q6_k_split", w.handle, int(rows), int(in_f))


def q6_k_gemv(ctx, x: Buffer, w: Buffer, in_f: int, out_f: int) -> Buffer:
    """y[out_f] = W x over a q6_k_split weight (the streaming GEMV)."""
    return op(ctx, "cw_q6_k_gemv", x.handle, w.handle, int(in_f), int(out_f))


def q8_0_split(ctx, w: Buffer, rows: int, in_f: int) -> Buffer:
    """Raw Q8_0 blocks -> the streaming GEMV's code and scale planes (a new buffer)."""
    return op(ctx, "cw_q8_0_split", w.handle, int(rows), int(in_f))


def q8_0_gemv(ctx, x: Buffer, w: Buffer, in_f: int, out_f: int) -> Buffer:
    """y[out_f] = W x over a q8_0_split weight (the streaming GEMV)."""
    return op(ctx, "cw_q8_0_gemv", x.handle, w.handle, int(in_f), int(out_f))
