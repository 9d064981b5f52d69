"""GGUF v3 writing and seeded random-init checkpoints.

The writer produces the container that chat-wgpu's loader parses
(src/loader/gguf.rs:68-106): magic, version 3, tensor/metadata counts,
typed metadata, tensor infos, a data section aligned to `general.alignment`.

`synth_model` writes a random-init checkpoint of a model shape: every matrix
(projections and token_embd) as GGUF Q4_0 blocks with 4-bit codes uniform in
0..15 and per-block scales d ~ U(0.002, 0.02) rounded to f16; norm gains f32
~ N(1, 0.02) (UnitShift families: N(0, 0.02), so the applied gain 1 + w is
again near 1).  There are no real checkpoints on this machine; these files
stand in for them with the same tensor names, shapes and dtypes.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 0, 1, 2, 12, 13, 14
GGML_Q4_1, GGML_Q8_0, GGML_BF16 = 3, 8, 30

# metadata value type ids (gguf.rs:125-151)
_T_U8, _T_I8, _T_U16, _T_I16, _T_U32, _T_I32, _T_F32, _T_BOOL, _T_STR, _T_ARR, _T_U64, _T_I64, _T_F64 = range(13)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _meta_value(v) -> bytes:
    if isinstance(v, bool):
        return struct.pack("<IB", _T_BOOL, int(v))
    if isinstance(v, int):
        return struct.pack("<II", _T_U32, v) if 0 <= v < 2**32 else struct.pack("<Iq", _T_I64, v)
    if isinstance(v, float):
        return struct.pack("<If", _T_F32, v)
    if isinstance(v, str):
        return struct.pack("<I", _T_STR) + _str(v)
    if isinstance(v, (list, tuple)):
        body = b"".join(_str(x) if isinstance(x, str) else struct.pack("<I", x) for x in v)
        et = _T_STR if v and isinstance(v[0], str) else _T_U32
        return struct.pack("<IIQ", _T_ARR, et, len(v)) + body
    raise TypeError(f"unsupported metadata value {v!r}")


@dataclass
class Tensor:
    name: str
    ggml_type: int
    dims: tuple          # ne[0] = innermost (row length)
    data: object         # bytes-like, or a callable returning bytes (lazy)


@dataclass
class GgufWriter:
    meta: dict = field(default_factory=dict)
    tensors: list = field(default_factory=list)
    alignment: int = 32

    def add(self, name, ggml_type, dims, data):
        self.tensors.append(Tensor(name, ggml_type, tuple(int(d) for d in dims), data))

    @staticmethod
    def nbytes(t: Tensor) -> int:
        n = int(np.prod(t.dims))
        return {GGML_F32: 4 * n, GGML_F16: 2 * n, GGML_BF16: 2 * n, GGML_Q4_0: n // 32 * 18,
                GGML_Q4_1: n // 32 * 20, GGML_Q8_0: n // 32 * 34,
                GGML_Q4_K: n // 256 * 144, GGML_Q5_K: n // 256 * 176,
                GGML_Q6_K: n // 256 * 210}[t.ggml_type]

    def write(self, path: str) -> None:
        meta = dict(self.meta)
        meta.setdefault("general.alignment", self.alignment)
        head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(self.tensors), len(meta)))
        for k, v in meta.items():
            head += _str(k) + _meta_value(v)
        off = 0
        offsets = []
        for t in self.tensors:
            offsets.append(off)
            off += self.nbytes(t)
            off = (off + self.alignment - 1) // self.alignment * self.alignment
        for t, o in zip(self.tensors, offsets):
            head += _str(t.name) + struct.pack("<I", len(t.dims))
            head += b"".join(struct.pack("<Q", d) for d in t.dims)
            head += struct.pack("<IQ", t.ggml_type, o)
        pad = (-len(head)) % self.alignment
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            f.write(head + b"\0" * pad)
            pos = 0
            for t, o in zip(self.tensors, offsets):
                if o > pos:
                    f.write(b"\0" * (o - pos))
                    pos = o
                data = t.data() if callable(t.data) else t.data
                mv = memoryview(np.ascontiguousarray(data) if isinstance(data, np.ndarray) else data).cast("B")
                if len(mv) != self.nbytes(t):
                    raise ValueError(f"{t.name}: {len(mv)} bytes, expected {self.nbytes(t)}")
                f.write(mv)
                pos += len(mv)
        os.replace(tmp, path)


def random_q4_0_blocks(rng: np.random.Generator, rows: int, in_f: int) -> np.ndarray:
    """[rows * in_f/32, 18] uint8 GGUF Q4_0 blocks: f16 d ~ U(0.002, 0.02), codes uniform."""
    nb = rows * (in_f // 32)
    blocks = np.empty((nb, 18), dtype=np.uint8)
    d = rng.uniform(0.002, 0.02, size=nb).astype(np.float16)
    blocks[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    blocks[:, 2:] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    return blocks


def random_q8_0_blocks(rng: np.random.Generator, rows: int, in_f: int) -> np.ndarray:
    """[rows * in_f/32, 34] uint8 GGUF Q8_0 blocks (dequant.rs:46-58): f16 d ~
    U(0.0002, 0.002), int8 codes uniform in -127..127 (the spread of the Q4_0
    weights)."""
    nb = rows * (in_f // 32)
    out = np.empty((nb, 34), np.uint8)
    out[:, 0:2] = rng.uniform(0.0002, 0.002, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = rng.integers(-127, 128, (nb, 32)).astype(np.int8).view(np.uint8)
    return out


def random_q4_1_blocks(rng: np.random.Generator, rows: int, in_f: int) -> np.ndarray:
    """[rows * in_f/32, 20] uint8 GGUF Q4_1 blocks (dequant.rs:82-97): f16 d ~
    U(0.002, 0.02), f16 minimum m ~ U(-0.16, -0.016) (about -8 d, so the
    weights centre near zero), codes uniform in 0..15."""
    nb = rows * (in_f // 32)
    out = np.empty((nb, 20), np.uint8)
    d = rng.uniform(0.002, 0.02, nb)
    out[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:4] = (-8.0 * d * rng.uniform(0.9, 1.1, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 4:] = rng.integers(0, 256, (nb, 16), dtype=np.uint8)
    return out


def random_dense(rng: np.random.Generator, rows: int, in_f: int, kind: str) -> np.ndarray:
    """A [rows, in_f] F32 / F16 / BF16 weight ~ N(0, 0.05) (the spread of the
    Q4_0 weights), as the file's bytes."""
    w = rng.normal(0.0, 0.05, (rows, in_f)).astype(np.float32)
    if kind == "f16":
        return w.astype(np.float16)
    if kind == "bf16":  # round to nearest even on the top 16 bits
        u = w.view(np.uint32)
        u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return u
    return w


def random_q6_k_blocks(rng: np.random.Generator, rows: int, in_f: int) -> np.ndarray:
    """[rows * in_f/256, 210] uint8 GGUF Q6_K super-blocks (dequant.rs:102-131
    layout): random 6-bit codes, int8 sub-block scales in [-64, 64), f16 d ~
    U(2e-4, 1e-3) (so values span about the Q4_0 blocks' range)."""
    nb = rows * (in_f // 256)
    b = rng.integers(0, 256, size=(nb, 210), dtype=np.uint8)
    b[:, 192:208] = rng.integers(-64, 64, size=(nb, 16)).astype(np.int8).view(np.uint8)
    b[:, 208:210] = rng.uniform(2e-4, 1e-3, size=nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b


def random_q45_k_blocks(rng: np.random.Generator, rows: int, in_f: int, five: bool) -> np.ndarray:
    """[rows * in_f/256, 144 | 176] uint8 GGUF Q4_K / Q5_K super-blocks (ggml's
    block_q4_K / block_q5_K): random codes and 6-bit (scale, min) pairs, f16 d
    ~ U(1e-4, 3e-4) (Q5_K: half that) and dmin = d * (7.5 | 15.5) so the
    weights centre near zero and span about the Q4_0 blocks' range."""
    nb = rows * (in_f // 256)
    size = 176 if five else 144
    b = rng.integers(0, 256, size=(nb, size), dtype=np.uint8)
    d = rng.uniform(1e-4, 3e-4, size=nb) * (0.5 if five else 1.0)
    dmin = d * (15.5 if five else 7.5)
    b[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:4] = dmin.astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b


# Benchmark model shapes (random-init: Qwen3-0.6B/8B, Gemma-2-2B), plus the tiny
# shape of the reference's RandomWeights verify model (src/main.rs:166-174).
CONFIGS = {
    "qwen3-0.6b": dict(arch="qwen3", dim=1024, n_layers=28, n_heads=16, n_kv=8, head_dim=128,
                       hidden=3072, vocab=151936, eps=1e-6, theta=1e6, tied=True),
    "qwen3-8b": dict(arch="qwen3", dim=4096, n_layers=36, n_heads=32, n_kv=8, head_dim=128,
                     hidden=12288, vocab=151936, eps=1e-6, theta=1e6, tied=False),
    # Qwen3-8B layer and head shapes over two layers (profiling the step's stages)
    "qwen3-8b-2l": dict(arch="qwen3", dim=4096, n_layers=2, n_heads=32, n_kv=8, head_dim=128,
                        hidden=12288, vocab=151936, eps=1e-6, theta=1e6, tied=False),
    "gemma2-2b": dict(arch="gemma2", dim=2304, n_layers=26, n_heads=8, n_kv=4, head_dim=256,
                      hidden=9216, vocab=256000, eps=1e-6, theta=1e4, tied=True, window=4096,
                      attn_softcap=50.0, final_softcap=30.0),
    # Gemma-2 head and residual shapes (head_dim 256, dim 2304) over three layers,
    # a short window and tight soft-caps: the post-norm persistent step variant
    "mid-gemma2": dict(arch="gemma2", dim=2304, n_layers=3, n_heads=4, n_kv=2, head_dim=256,
                       hidden=1536, vocab=4096, eps=1e-6, theta=1e4, tied=True, window=80,
                       attn_softcap=5.0, final_softcap=8.0),
    "tiny-qwen3": dict(arch="qwen3", dim=64, n_layers=2, n_heads=4, n_kv=2, head_dim=16,
                       hidden=128, vocab=256, eps=1e-6, theta=1e6, tied=True),
    # small shapes that exercise the family switches in tests
    "small-qwen3": dict(arch="qwen3", dim=512, n_layers=4, n_heads=8, n_kv=4, head_dim=64,
                        hidden=1536, vocab=2048, eps=1e-6, theta=1e6, tied=True),
    # an odd layer count: the persistent step's per-layer accumulator parity
    # wraps differently from one step to the next
    "odd-qwen3": dict(arch="qwen3", dim=512, n_layers=3, n_heads=16, n_kv=4, head_dim=32,
                      hidden=1024, vocab=1024, eps=1e-6, theta=1e6, tied=True),
    "tiny-gemma2": dict(arch="gemma2", dim=256, n_layers=3, n_heads=4, n_kv=2, head_dim=64,
                        hidden=512, vocab=512, eps=1e-6, theta=1e4, tied=True, window=6,
                        attn_softcap=2.0, final_softcap=3.0),
    # eight kv heads and 64 FFN column blocks: splits 2, 4 and 8 ways (TP tests)
    "tp8-qwen3": dict(arch="qwen3", dim=512, n_layers=3, n_heads=16, n_kv=8, head_dim=64,
                      hidden=2048, vocab=2048, eps=1e-6, theta=1e6, tied=True),
    "tiny-qwen2": dict(arch="qwen2", dim=256, n_layers=2, n_heads=8, n_kv=2, head_dim=32,
                       hidden=768, vocab=300, eps=1e-6, theta=1e6, tied=False, bias=True),
    # more FFN column blocks (hidden / 32 = 192) than a B200 has SMs: CTAs of the
    # persistent step take several FFN units each
    "wide-ffn-qwen3": dict(arch="qwen3", dim=512, n_layers=2, n_heads=8, n_kv=4, head_dim=64,
                           hidden=6144, vocab=2048, eps=1e-6, theta=1e6, tied=True),
    # k-quant projections in the mixes of Q4_K_M-style files (q/k/v of different
    # types, Q6_K down projections, a Q4_K head; a Q5_K variant)
    "small-qwen3-q4km": dict(arch="qwen3", dim=512, n_layers=3, n_heads=8, n_kv=4, head_dim=64,
                             hidden=1536, vocab=2048, eps=1e-6, theta=1e6, tied=False,
                             embed_type="q4_k",
                             proj_types=dict(q="q4_k", k="q4_k", v="q6_k", o="q4_k",
                                             gate="q4_k", up="q4_k", down="q6_k", head="q4_k")),
    "tiny-qwen2-q5k": dict(arch="qwen2", dim=256, n_layers=2, n_heads=8, n_kv=2, head_dim=32,
                           hidden=768, vocab=300, eps=1e-6, theta=1e6, tied=True, bias=True,
                           proj_types=dict(q="q5_k", k="q5_k", v="q5_k", o="q5_k",
                                           gate="q5_k", up="q5_k", down="q5_k")),
    # Qwen3-0.6B shapes in a Q4_K_M-style mix (decode through the k-quant GEMVs)
    "qwen3-0.6b-q4km": dict(arch="qwen3", dim=1024, n_layers=28, n_heads=16, n_kv=8,
                            head_dim=128, hidden=3072, vocab=151936, eps=1e-6, theta=1e6,
                            tied=True, embed_type="q6_k",
                            proj_types=dict(q="q4_k", k="q4_k", v="q6_k", o="q4_k",
                                            gate="q4_k", up="q4_k", down="q6_k")),
    # Q4_0 projections under a Q5_K token embedding shared with the LM head
    "small-qwen3-q5k-embed": dict(arch="qwen3", dim=512, n_layers=2, n_heads=8, n_kv=4,
                                  head_dim=64, hidden=1536, vocab=2048, eps=1e-6, theta=1e6,
                                  tied=True, embed_type="q5_k"),
    # the other types the reference's loader takes (tensor_f32: F32, F16, Q4_1,
    # Q8_0) as projections, embeddings and heads, q/k/v of different types
    "small-qwen3-mixed": dict(arch="qwen3", dim=512, n_layers=3, n_heads=8, n_kv=4, head_dim=64,
                              hidden=1536, vocab=2048, eps=1e-6, theta=1e6, tied=False,
                              embed_type="q8_0",
                              proj_types=dict(q="f16", k="q8_0", v="q4_1", o="f32",
                                              gate="q8_0", up="q8_0", down="q4_1", head="f16")),
    # dense projections (the reference's Proj::Dense over an f32 file) with
    # q/k/v biases
    "tiny-qwen2-f32": dict(arch="qwen2", dim=256, n_layers=2, n_heads=8, n_kv=2, head_dim=32,
                           hidden=768, vocab=300, eps=1e-6, theta=1e6, tied=True, bias=True,
                           embed_type="f32",
                           proj_types=dict(q="f32", k="f32", v="f32", o="f32",
                                           gate="f32", up="f32", down="f32")),
    # BF16 projections under an F16 tied embedding (the reference decodes BF16,
    # dequant.rs:41-43, but its tensor_f32 does not dispatch it)
    "small-qwen3-bf16": dict(arch="qwen3", dim=512, n_layers=2, n_heads=8, n_kv=4, head_dim=64,
                             hidden=1536, vocab=2048, eps=1e-6, theta=1e6, tied=True,
                             embed_type="f16",
                             proj_types=dict(q="bf16", k="bf16", v="bf16", o="bf16",
                                             gate="bf16", up="bf16", down="bf16")),
    # Q6_K token embedding (tied head) / Q6_K output, the layout of real Q4_0 files
    "small-qwen3-q6k": dict(arch="qwen3", dim=512, n_layers=4, n_heads=8, n_kv=4, head_dim=64,
                            hidden=1536, vocab=2048, eps=1e-6, theta=1e6, tied=True,
                            embed_type="q6_k"),
    "tiny-gemma2-q6k": dict(arch="gemma2", dim=256, n_layers=3, n_heads=4, n_kv=2, head_dim=64,
                            hidden=512, vocab=512, eps=1e-6, theta=1e4, tied=False, window=6,
                            attn_softcap=2.0, final_softcap=3.0, embed_type="q6_k"),
}


def synth_model(path: str, cfg: dict, seed: int = 0) -> str:
    """Write a seeded random-init GGUF of shape `cfg` (see CONFIGS)."""
    arch = cfg["arch"]
    dim, L, nh, nkv, hd = cfg["dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv"], cfg["head_dim"]
    hid, vocab = cfg["hidden"], cfg["vocab"]
    qd, kvd = nh * hd, nkv * hd
    unit = arch == "gemma2"
    w = GgufWriter()
    w.meta["general.architecture"] = arch
    w.meta["general.name"] = f"synthetic-{arch}"
    p = arch + "."
    w.meta[p + "block_count"] = L
    w.meta[p + "context_length"] = 40960
    w.meta[p + "embedding_length"] = dim
    w.meta[p + "feed_forward_length"] = hid
    w.meta[p + "attention.head_count"] = nh
    w.meta[p + "attention.head_count_kv"] = nkv
    w.meta[p + "attention.key_length"] = hd
    w.meta[p + "attention.value_length"] = hd
    w.meta[p + "attention.layer_norm_rms_epsilon"] = float(cfg["eps"])
    w.meta[p + "rope.freq_base"] = float(cfg["theta"])
    w.meta[p + "vocab_size"] = vocab
    if arch == "gemma2":
        w.meta[p + "attention.sliding_window"] = int(cfg.get("window", 4096))
        w.meta[p + "attn_logit_softcapping"] = float(cfg.get("attn_softcap", 50.0))
        w.meta[p + "final_logit_softcapping"] = float(cfg.get("final_softcap", 30.0))
    idx = [0]

    def rng():  # one independent stream per tensor, in file order
        idx[0] += 1
        return np.random.default_rng(np.random.SeedSequence([seed, idx[0]]))

    def mat(name, rows, in_f, q6k=False, kind=None):
        r = rng()
        kind = kind or ("q6_k" if q6k else "q4_0")
        if kind == "q6_k":  # real Q4_0 checkpoints often keep token_embd / output in Q6_K
            w.add(name, GGML_Q6_K, (in_f, rows), lambda r=r: random_q6_k_blocks(r, rows, in_f))
        elif kind == "q8_0":
            w.add(name, GGML_Q8_0, (in_f, rows), lambda r=r: random_q8_0_blocks(r, rows, in_f))
        elif kind == "q4_1":
            w.add(name, GGML_Q4_1, (in_f, rows), lambda r=r: random_q4_1_blocks(r, rows, in_f))
        elif kind in ("f32", "f16", "bf16"):
            t = {"f32": GGML_F32, "f16": GGML_F16, "bf16": GGML_BF16}[kind]
            w.add(name, t, (in_f, rows), lambda r=r, k=kind: random_dense(r, rows, in_f, k))
        elif kind in ("q4_k", "q5_k"):
            five = kind == "q5_k"
            w.add(name, GGML_Q5_K if five else GGML_Q4_K, (in_f, rows),
                  lambda r=r: random_q45_k_blocks(r, rows, in_f, five))
        else:
            w.add(name, GGML_Q4_0, (in_f, rows), lambda r=r: random_q4_0_blocks(r, rows, in_f))

    # per-projection types ("q", "k", "v", "o", "gate", "up", "down", "head"):
    # the mixes of Q4_K_M-style files; Q4_0 where not named
    pt = cfg.get("proj_types", {})

    def vec(name, n, mean=None):
        r = rng()
        mean = (0.0 if unit else 1.0) if mean is None else mean
        w.add(name, GGML_F32, (n,), lambda r=r: r.normal(mean, 0.02, size=n).astype(np.float32))

    q6k = cfg.get("embed_type") == "q6_k"
    mat("token_embd.weight", vocab, dim, kind=cfg.get("embed_type"))
    for i in range(L):
        b = f"blk.{i}."
        vec(b + "attn_norm.weight", dim)
        mat(b + "attn_q.weight", qd, dim, kind=pt.get("q"))
        mat(b + "attn_k.weight", kvd, dim, kind=pt.get("k"))
        mat(b + "attn_v.weight", kvd, dim, kind=pt.get("v"))
        if cfg.get("bias"):
            vec(b + "attn_q.bias", qd, mean=0.0)
            vec(b + "attn_k.bias", kvd, mean=0.0)
            vec(b + "attn_v.bias", kvd, mean=0.0)
        mat(b + "attn_output.weight", dim, qd, kind=pt.get("o"))
        if arch == "qwen3":
            vec(b + "attn_q_norm.weight", hd)
            vec(b + "attn_k_norm.weight", hd)
        vec(b + "ffn_norm.weight", dim)
        mat(b + "ffn_gate.weight", hid, dim, kind=pt.get("gate"))
        mat(b + "ffn_up.weight", hid, dim, kind=pt.get("up"))
        mat(b + "ffn_down.weight", dim, hid, kind=pt.get("down"))
        if arch == "gemma2":
            vec(b + "post_attention_norm.weight", dim)
            vec(b + "post_ffw_norm.weight", dim)
    vec("output_norm.weight", dim)
    if not cfg.get("tied", True):
        mat("output.weight", vocab, dim, q6k, kind=pt.get("head"))
    w.write(path)
    return path


def cached_model(name: str, seed: int = 0, cfg: dict | None = None, directory: str | None = None) -> str:
    """Path of the synthetic GGUF for config `name`, written once per seed."""
    cfg = cfg or CONFIGS[name]
    directory = directory or os.environ.get("CW_MODEL_DIR", "/tmp/chat_wgpu_b200_models")
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{name}-seed{seed}.gguf")
    if not os.path.exists(path):
        synth_model(path, cfg, seed)
    return path


class GgufReader:
    """Minimal GGUF v3 reader (src/loader/gguf.rs:68-106) for host-side tools:
    metadata values and raw tensor bytes, memory-mapped."""

    _SIZES = {_T_U8: 1, _T_I8: 1, _T_U16: 2, _T_I16: 2, _T_U32: 4, _T_I32: 4, _T_F32: 4,
              _T_BOOL: 1, _T_U64: 8, _T_I64: 8, _T_F64: 8}
    _FMT = {_T_U8: "<B", _T_I8: "<b", _T_U16: "<H", _T_I16: "<h", _T_U32: "<I", _T_I32: "<i",
            _T_F32: "<f", _T_BOOL: "<B", _T_U64: "<Q", _T_I64: "<q", _T_F64: "<d"}

    def __init__(self, path: str):
        import mmap
        self._f = open(path, "rb")
        self.buf = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        buf = self.buf
        if buf[:4] != b"GGUF":
            raise ValueError("not a GGUF file")
        _ver, n_t, n_kv = struct.unpack_from("<IQQ", buf, 4)
        o = 24
        self.meta = {}
        for _ in range(n_kv):
            k, o = self._str(o)
            t = struct.unpack_from("<I", buf, o)[0]
            o += 4
            if t == _T_STR:
                v, o = self._str(o)
            elif t == _T_ARR:
                et, cnt = struct.unpack_from("<IQ", buf, o)
                o += 12
                v = []
                for _ in range(cnt):
                    if et == _T_STR:
                        x, o = self._str(o)
                    else:
                        x = struct.unpack_from(self._FMT[et], buf, o)[0]
                        o += self._SIZES[et]
                    v.append(x)
            else:
                v = struct.unpack_from(self._FMT[t], buf, o)[0]
                o += self._SIZES[t]
            self.meta[k] = v
        self.infos = {}
        for _ in range(n_t):
            nm, o = self._str(o)
            nd = struct.unpack_from("<I", buf, o)[0]
            o += 4
            dims = struct.unpack_from("<" + "Q" * nd, buf, o)
            o += 8 * nd
            tt, off = struct.unpack_from("<IQ", buf, o)
            o += 12
            self.infos[nm] = (tt, tuple(int(d) for d in dims), off)
        align = int(self.meta.get("general.alignment", 32)) or 32
        self.data_start = (o + align - 1) // align * align

    def _str(self, o):
        n = struct.unpack_from("<Q", self.buf, o)[0]
        return bytes(self.buf[o + 8:o + 8 + n]).decode(), o + 8 + n

    def has(self, name: str) -> bool:
        return name in self.infos

    def tensor(self, name: str):
        """(ggml_type, dims, bytes) of a tensor."""
        tt, dims, off = self.infos[name]
        n = int(np.prod(dims))
        nbytes = {GGML_F32: 4 * n, GGML_F16: 2 * n, GGML_Q4_0: n // 32 * 18,
                  GGML_Q4_K: n // 256 * 144, GGML_Q5_K: n // 256 * 176,
                  GGML_Q6_K: n // 256 * 210}[tt]
        s = self.data_start + off
        return tt, dims, self.buf[s:s + nbytes]

    def vector_f32(self, name: str) -> np.ndarray:
        tt, dims, raw = self.tensor(name)
        if tt == GGML_F32:
            return np.frombuffer(raw, dtype=np.float32).copy()
        if tt == GGML_F16:
            return np.frombuffer(raw, dtype=np.float16).astype(np.float32)
        raise ValueError(f"{name}: type {tt} is not a float vector")

    def close(self):
        self.buf.close()
        self._f.close()


def read_tensor_bytes(path: str, name: str) -> tuple[int, tuple, bytes]:
    """(ggml_type, dims, raw bytes) of one tensor of a GGUF file."""
    r = GgufReader(path)
    try:
        tt, dims, raw = r.tensor(name)
        return tt, dims, bytes(raw)
    finally:
        r.close()
