"""Malformed GGUF files give a status code, never a crash (CPU, no device).

The reference's loader panics on these (src/loader/gguf.rs:192,203,206: the
`expect`s on a missing or unreadable tensor); the C-ABI promises a status
instead.  cw_gguf_inspect runs the parser and the tensor-table checks that
cw_model_load_gguf runs before it touches the device, so every case here is
checked without a GPU: truncated headers, bad magic and version, a tensor
past the end of the file, a zero dimension (which would divide by zero when
the row count is formed), dimensions whose product overflows 64 bits, a
byte size that overflows, and an element count that wraps to a small
number."""
import ctypes as C
import struct

import numpy as np
import pytest

CW_OK, CW_ERR_NOT_FOUND, CW_ERR_FORMAT = 0, 4, 7
Q4_0, F32 = 2, 0


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def gguf_bytes(tensors, data_len=None, version=3, magic=b"GGUF", meta=None):
    """A GGUF v3 image.  tensors: (name, dims, type, offset).  The data
    section (zeros) is data_len bytes, by default exactly what the tensors
    claim."""
    meta = dict(meta or {})
    meta.setdefault("general.alignment", 32)
    head = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(meta)))
    for k, v in meta.items():
        head += _s(k) + struct.pack("<II", 4, v)  # u32 values
    for name, dims, typ, off in tensors:
        head += _s(name) + struct.pack("<I", len(dims))
        head += b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, off)
    head += b"\0" * ((-len(head)) % 32)
    if data_len is None:
        data_len = 0
        for _, dims, typ, off in tensors:
            n = int(np.prod(dims, dtype=object))
            data_len = max(data_len, off + (n * 4 if typ == F32 else n // 32 * 18))
    return bytes(head) + b"\0" * data_len


def inspect(tmp_path, blob: bytes, name="m.gguf"):
    from chat_wgpu_b200 import _lib
    lib = _lib.load()
    p = tmp_path / name
    p.write_bytes(blob)
    n = C.c_size_t(123)
    d = C.c_uint64(456)
    rc = lib.cw_gguf_inspect(str(p).encode(), C.byref(n), C.byref(d))
    return rc, n.value, d.value, (lib.cw_last_error() or b"").decode()


GOOD = [("blk.0.attn_q.weight", (64, 128), Q4_0, 0), ("output_norm.weight", (64,), F32, 4608)]


def test_well_formed_file(tmp_path):
    rc, n, d, _ = inspect(tmp_path, gguf_bytes(GOOD))
    assert rc == CW_OK and n == 2 and d == 4608 + 256


def test_synthetic_checkpoint_is_well_formed(tmp_path):
    from chat_wgpu_b200 import _lib, gguf
    p = gguf.synth_model(str(tmp_path / "tiny.gguf"), gguf.CONFIGS["tiny-qwen3"], seed=7)
    n = C.c_size_t()
    assert _lib.load().cw_gguf_inspect(p.encode(), C.byref(n), None) == CW_OK
    r = gguf.GgufReader(p)
    assert n.value == len(r.infos)
    r.close()


def test_missing_file(tmp_path):
    from chat_wgpu_b200 import _lib
    assert _lib.load().cw_gguf_inspect(str(tmp_path / "absent.gguf").encode(), None, None) == \
        CW_ERR_NOT_FOUND


@pytest.mark.parametrize("cut", [3, 4, 8, 20, 24, 40, 70, 100])
def test_truncated_header(tmp_path, cut):
    blob = gguf_bytes(GOOD)
    rc, *_ = inspect(tmp_path, blob[:cut])
    assert rc == CW_ERR_FORMAT


def test_bad_magic_and_version(tmp_path):
    assert inspect(tmp_path, gguf_bytes(GOOD, magic=b"GGUG"))[0] == CW_ERR_FORMAT
    assert inspect(tmp_path, gguf_bytes(GOOD, version=7))[0] == CW_ERR_FORMAT


def test_tensor_past_end_of_file(tmp_path):
    rc, _, _, msg = inspect(tmp_path, gguf_bytes(GOOD, data_len=4608 + 100))
    assert rc == CW_ERR_FORMAT and "past the end" in msg
    bad = [("w", (64, 128), Q4_0, 1 << 40)]
    assert inspect(tmp_path, gguf_bytes(bad, data_len=64))[0] == CW_ERR_FORMAT


def test_zero_dimension(tmp_path):
    bad = [("w", (0, 128), Q4_0, 0)]
    rc, _, _, msg = inspect(tmp_path, gguf_bytes(bad, data_len=64))
    assert rc == CW_ERR_FORMAT and "dimension" in msg
    bad = [("w", (64, 0), Q4_0, 0)]
    assert inspect(tmp_path, gguf_bytes(bad, data_len=64))[0] == CW_ERR_FORMAT


def test_overflowing_dimensions(tmp_path):
    # 2^33 x 2^33 elements: the element count overflows 64 bits
    bad = [("w", (1 << 33, 1 << 33), F32, 0)]
    assert inspect(tmp_path, gguf_bytes(bad, data_len=64))[0] == CW_ERR_FORMAT
    # 2^32 x 2^30 x 4: the count fits, wraps to 0 mod 2^64 only in bytes
    bad = [("w", (1 << 32, 1 << 30, 4), F32, 0)]
    assert inspect(tmp_path, gguf_bytes(bad, data_len=64))[0] == CW_ERR_FORMAT


def test_byte_size_overflow(tmp_path):
    # row bytes 2^62 (F32 rows of 2^60 elements) x 8 rows overflows size_t
    bad = [("w", (1 << 60, 8), F32, 0)]
    assert inspect(tmp_path, gguf_bytes(bad, data_len=64))[0] == CW_ERR_FORMAT


def test_too_many_dimensions(tmp_path):
    bad = [("w", (2, 2, 2, 2, 2), F32, 0)]
    assert inspect(tmp_path, gguf_bytes(bad, data_len=256))[0] == CW_ERR_FORMAT


def test_null_path():
    from chat_wgpu_b200 import _lib
    assert _lib.load().cw_gguf_inspect(None, None, None) == 1
