"""Model layer (chat-wgpu src/model/{mod,qwen3,layers,cache}.rs) over
libchatcuda.so.

`Model` / `Session` / `generate` drive the native decode path: weights stay
GGUF Q4_0 in HBM and each token is one CUDA-graph replay of fused kernels.

`OpByOpQwen3` + `generate_op_by_op` restate the reference's composition
(qwen3.rs:139-191, mod.rs:57-125) line by line through the per-op wrappers of
`chat_wgpu_b200.kernels`, i.e. a caller of the reference's op surface
running unchanged on the drop-in context.  It exists to show that surface
composes a model and to cross-check the fused path.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import _lib
from .context import GpuContext
from .gguf import GgufReader
from .kernels import activation, argmax, attention, norm, q4, rope


TP_ID_BYTES = 128
TP_HANDLE_BYTES = 128  # CW_TP_HANDLE_BYTES


def tp_unique_id() -> bytes:
    """A fresh NCCL communicator id for cw_model_load_gguf_tp (rank 0 makes it)."""
    buf = C.create_string_buffer(TP_ID_BYTES)
    _lib.call("cw_tp_unique_id", C.cast(buf, C.c_void_p), TP_ID_BYTES)
    return buf.raw


class Model:
    """Model::load (mod.rs:26) from a GGUF file; the native model handle."""

    def __init__(self, ctx: GpuContext, path: str, tp: "tuple[int, int, bytes] | None" = None):
        """`tp` = (rank, world, id): this process's shard of a tensor-parallel
        model (cw_model_load_gguf_tp); `id` from `tp_unique_id()` on rank 0."""
        self.ctx = ctx
        h = C.c_void_p()
        if tp is None:
            _lib.call("cw_model_load_gguf", ctx.handle, path.encode(), C.byref(h))
        else:
            rank, world, uid = tp
            ub = C.create_string_buffer(bytes(uid), TP_ID_BYTES)
            _lib.call("cw_model_load_gguf_tp", ctx.handle, path.encode(), int(rank), int(world),
                      C.cast(ub, C.c_void_p), C.byref(h))
        self._h = h
        self._sessions = weakref.WeakSet()  # released before the model
        ctx._adopt(self)
        info = _lib.ModelInfo()
        _lib.call("cw_model_get_info", self._h, C.byref(info))
        self.info = {k: (getattr(info, k).decode() if k == "arch" else getattr(info, k))
                     for k, _ in info._fields_}
        r, w, off, nv = C.c_int(), C.c_int(), C.c_uint32(), C.c_uint32()
        _lib.call("cw_model_tp_info", self._h, C.byref(r), C.byref(w), C.byref(off), C.byref(nv))
        self.tp_rank, self.tp_world = r.value, w.value
        self.vocab_offset, self.vocab_local = off.value, nv.value

    @property
    def handle(self):
        return self._h

    @property
    def vocab_size(self) -> int:
        return int(self.info["vocab"])

    def close(self):
        if getattr(self, "_h", None):
            for sess in list(getattr(self, "_sessions", ())):
                sess.close()
            _lib.load().cw_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_session(self, max_seq: int) -> "Session":
        """Model::new_cache (qwen3.rs:115) plus the per-token device state."""
        return Session(self, max_seq)


class Session:
    def __init__(self, model: Model, max_seq: int):
        self.model = model
        h = C.c_void_p()
        _lib.call("cw_session_create", model.handle, int(max_seq), C.byref(h))
        self._h = h
        self.max_seq = int(max_seq)
        model._sessions.add(self)

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().cw_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_graph(self, use_graph: bool) -> None:
        _lib.call("cw_session_set_graph", self._h, 1 if use_graph else 0)

    def set_persistent(self, on) -> None:
        """Select the step kernel: True/1 (or "split"/2, the same plan) one
        persistent cooperative launch per token (default where the family is
        covered), False/0 one kernel per stage."""
        mode = {"split": 2}.get(on, None) if isinstance(on, str) else (1 if on else 0)
        if mode is None:
            raise ValueError(f"unknown persistent mode {on!r}")
        _lib.call("cw_session_set_persistent", self._h, int(mode))

    def inject_stall(self, wait_us: int) -> None:
        """Fault injection for tests (cw_session_inject_stall): the next
        persistent step times out after wait_us microseconds."""
        _lib.call("cw_session_inject_stall", self._h, int(wait_us))

    @property
    def persistent(self) -> bool:
        v = C.c_int()
        _lib.call("cw_session_persistent", self._h, C.byref(v))
        return bool(v.value)

    def begin(self, prompt) -> None:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        _lib.call("cw_session_begin", self._h, p.ctypes.data, p.size)

    def run(self, n_steps: int) -> int:
        n = C.c_size_t()
        _lib.call("cw_session_run", self._h, int(n_steps), C.byref(n))
        return int(n.value)

    def set_sampling(self, temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0,
                     seed: int = 0) -> None:
        """Device-side sampling after the LM head (cw_session_set_sampling);
        temperature 0 = greedy."""
        _lib.call("cw_session_set_sampling", self._h, float(temperature), int(top_k),
                  float(top_p), int(seed) & (2**64 - 1))

    def set_eos(self, ids) -> None:
        """Stop tokens: the sequence ends, without emitting it, at the first one."""
        a = np.ascontiguousarray(list(ids), dtype=np.uint32)
        _lib.call("cw_session_set_eos", self._h, a.ctypes.data if a.size else None, a.size)

    @property
    def stopped(self) -> bool:
        v = C.c_int()
        _lib.call("cw_session_stopped", self._h, C.byref(v))
        return bool(v.value)

    # ---- hook taps (Hook::tap, src/model/mod.rs:155-165)
    TAPS = ("q", "post_attn", "layer_out")

    def add_tap(self, name: str, layer: int, cap: int) -> None:
        """Record `name` of `layer` at every position into a device ring of
        the last `cap` positions."""
        _lib.call("cw_session_add_tap", self._h, name.encode(), int(layer), int(cap))

    def clear_taps(self) -> None:
        _lib.call("cw_session_clear_taps", self._h)

    def read_tap(self, name: str, layer: int, pos: int) -> np.ndarray:
        I = self.model.info
        n = I["n_heads"] * I["head_dim"] if name == "q" else I["dim"]
        out = np.empty(n, np.float32)
        _lib.call("cw_session_read_tap", self._h, name.encode(), int(layer), int(pos),
                  out.ctypes.data, n)
        return out

    def prefill(self) -> int:
        """Run the remaining prompt positions but the last as one batch on the
        tensor cores (cw_session_prefill); returns the positions processed."""
        n = C.c_size_t()
        _lib.call("cw_session_prefill", self._h, C.byref(n))
        return n.value

    def set_prefill_chunk(self, rows: int) -> None:
        """Rows per prefill chunk (cw_session_set_prefill_chunk; 0 = default)."""
        _lib.call("cw_session_set_prefill_chunk", self._h, int(rows))

    def read_kv(self, layer: int, n_pos: int) -> tuple[np.ndarray, np.ndarray]:
        """K and V cache rows [0, n_pos) of `layer`, each [n_kv, n_pos, head_dim]."""
        I = self.model.info
        k = np.empty((I["n_kv"], n_pos, I["head_dim"]), np.float32)
        v = np.empty_like(k)
        _lib.call("cw_session_read_kv", self._h, int(layer), int(n_pos), k.ctypes.data,
                  v.ctypes.data)
        return k, v

    def tokens(self) -> np.ndarray:
        out = np.zeros(self.max_seq, dtype=np.uint32)
        n = C.c_size_t()
        _lib.call("cw_session_tokens", self._h, out.ctypes.data, out.size, C.byref(n))
        return out[: n.value].copy()

    def logits(self) -> np.ndarray:
        """The last decode step's logits (a tensor-parallel rank: its vocabulary
        rows [model.vocab_offset, + model.vocab_local))."""
        v = self.model.vocab_local
        out = np.zeros(v, dtype=np.float32)
        _lib.call("cw_session_logits", self._h, out.ctypes.data, v)
        return out

    def hidden(self) -> np.ndarray:
        d = int(self.model.info["dim"])
        out = np.zeros(d, dtype=np.float32)
        _lib.call("cw_session_hidden", self._h, out.ctypes.data, d)
        return out

    TOKEN_DEVICE = 0xFFFFFFFF

    def step(self, token_in: int = TOKEN_DEVICE) -> int:
        """One step with a host round trip (mod.rs:93-103); returns the produced
        token, or 0xFFFFFFFF for a prompt position."""
        out = C.c_uint32()
        _lib.call("cw_session_step", self._h, int(token_in), C.byref(out))
        return int(out.value)

    def run_timed(self, n_steps: int) -> float:
        """run(n_steps) timed with CUDA events on the context stream (ms)."""
        ms = C.c_double()
        _lib.call("cw_session_run_timed", self._h, int(n_steps), C.byref(ms))
        return float(ms.value)

    def launches(self) -> tuple[int, int]:
        """Kernel launches of one (prompt, decode) step."""
        a, b = C.c_size_t(), C.c_size_t()
        _lib.call("cw_session_launches", self._h, C.byref(a), C.byref(b))
        return int(a.value), int(b.value)

    def profile(self, n_steps: int) -> list[tuple[str, int, float]]:
        """Per-kernel device time of n_steps decode steps (kernel, launches, ms),
        sorted by total descending (cw_session_profile)."""
        cap = 128
        rows = (_lib.ProfileRow * cap)()
        n = C.c_size_t()
        _lib.call("cw_session_profile", self._h, int(n_steps), rows, cap, C.byref(n))
        return [(rows[i].kernel.decode(), int(rows[i].passes), float(rows[i].total_ms))
                for i in range(min(n.value, cap))]

    def tp_handle(self) -> bytes:
        """This rank's exchange-area handle for the peer all-reduces
        (cw_session_tp_handle); every rank's goes to every rank's tp_attach."""
        buf = C.create_string_buffer(TP_HANDLE_BYTES)
        _lib.call("cw_session_tp_handle", self._h, C.cast(buf, C.c_void_p), TP_HANDLE_BYTES)
        return buf.raw

    def tp_attach(self, handles: "list[bytes]") -> None:
        """Map every rank's exchange area (handles in rank order): the step's
        all-reduces then run over NVLink peer memory instead of NCCL
        (cw_session_tp_attach)."""
        blob = b"".join(handles)
        buf = C.create_string_buffer(blob, len(blob))
        _lib.call("cw_session_tp_attach", self._h, C.cast(buf, C.c_void_p), len(blob))

    def tp_attach_p2p(self, allgather) -> None:
        """tp_handle + tp_attach with a host exchange: allgather(bytes) returns
        every rank's bytes in rank order (e.g. torch.distributed
        all_gather_object); the ranks are synchronised by it."""
        self.tp_attach(list(allgather(self.tp_handle())))

    @property
    def pos(self) -> int:
        n = C.c_size_t()
        _lib.call("cw_session_pos", self._h, C.byref(n))
        return int(n.value)


class SessionGroup:
    """Co-batched decode of several sessions of one model (cw_group_*): each
    step runs every session's next position with one pass over the weights
    (streaming GEMVs over all rows for groups of up to 8 sessions of a
    pre-norm family, else tensor-core GEMMs)."""

    def __init__(self, sessions):
        self.sessions = list(sessions)
        arr = (C.c_void_p * len(self.sessions))(*[s._h for s in self.sessions])
        h = C.c_void_p()
        _lib.call("cw_group_create", arr, len(self.sessions), C.byref(h))
        self._h = h
        self.sessions[0].model._sessions.add(self)

    def close(self):
        if getattr(self, "_h", None):
            _lib.load().cw_group_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def path(self) -> int:
        """Projection path: 1 streaming GEMVs (integer-MMA products where K <=
        4096), 2 streaming GEMVs with dp4a products, 0 tensor-core GEMMs."""
        v = C.c_int()
        _lib.call("cw_group_set_streaming", self._h, -1, C.byref(v))
        return int(v.value)

    @property
    def streaming(self) -> bool:
        """Whether the projections run as streaming GEMVs (else tensor-core GEMMs)."""
        return self.path != 0

    def set_streaming(self, on) -> None:
        """Choose the projection path: True / 1 streaming (integer MMA where
        K <= 4096), 2 streaming with dp4a products, False / 0 tensor-core GEMMs.
        Streaming raises when the group does not qualify."""
        _lib.call("cw_group_set_streaming", self._h, int(on), None)

    def run(self, n_steps: int) -> None:
        _lib.call("cw_group_run", self._h, int(n_steps))

    def run_timed(self, n_steps: int) -> float:
        ms = C.c_double()
        _lib.call("cw_group_run_timed", self._h, int(n_steps), C.byref(ms))
        return ms.value


def generate(model: Model, prompt, max_new: int) -> np.ndarray:
    """model::generate (mod.rs:57-125) through cw_generate: greedy, one token
    read back per step; max_new == 0 still yields one token."""
    p = np.ascontiguousarray(prompt, dtype=np.uint32)
    out = np.zeros(max(int(max_new), 1), dtype=np.uint32)
    _lib.call("cw_generate", model.handle, p.ctypes.data, p.size, int(max_new), out.ctypes.data)
    return out


# ---------------------------------------------------------------------------
# reference-order composition over the per-op surface
# ---------------------------------------------------------------------------
class OpByOpQwen3:
    """Qwen3 (src/model/qwen3.rs) composed from the per-op wrappers: weights
    uploaded as packed Q4_0 (q4.q4_0_upload), norms as f32 storage, the
    embedding table dequantised once to dense f32 like qwen3.rs:92."""

    def __init__(self, ctx: GpuContext, path: str):
        self.ctx = ctx
        r = GgufReader(path)
        arch = r.meta.get("general.architecture", "qwen3")
        if arch != "qwen3":
            raise ValueError("OpByOpQwen3 composes the qwen3 architecture only")
        m = lambda k, d=None: r.meta.get(f"qwen3.{k}", d)  # noqa: E731
        self.n_layers = int(m("block_count"))
        self.dim = int(m("embedding_length"))
        self.n_heads = int(m("attention.head_count"))
        self.n_kv_heads = int(m("attention.head_count_kv"))
        self.head_dim = int(m("attention.key_length"))
        self.hidden = int(m("feed_forward_length"))
        self.eps = float(m("attention.layer_norm_rms_epsilon"))
        self.rope_theta = float(m("rope.freq_base"))
        self.vocab = int(m("vocab_size"))
        qd, kvd = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim

        def mat(name, rows, in_f):
            tt, dims, raw = r.tensor(name)
            assert tt == 2 and dims == (in_f, rows), (name, tt, dims)
            return (q4.q4_0_upload(ctx, np.frombuffer(raw, dtype=np.uint8), rows, in_f), in_f, rows)

        vec = lambda name: ctx.storage(r.vector_f32(name))  # noqa: E731
        self.layers = []
        for i in range(self.n_layers):
            b = f"blk.{i}."
            self.layers.append(dict(
                attn_norm=vec(b + "attn_norm.weight"),
                wq=mat(b + "attn_q.weight", qd, self.dim),
                wk=mat(b + "attn_k.weight", kvd, self.dim),
                wv=mat(b + "attn_v.weight", kvd, self.dim),
                wo=mat(b + "attn_output.weight", self.dim, qd),
                q_norm=vec(b + "attn_q_norm.weight"),
                k_norm=vec(b + "attn_k_norm.weight"),
                ffn_norm=vec(b + "ffn_norm.weight"),
                gate=mat(b + "ffn_gate.weight", self.hidden, self.dim),
                up=mat(b + "ffn_up.weight", self.hidden, self.dim),
                down=mat(b + "ffn_down.weight", self.dim, self.hidden),
            ))
        self.final_norm = vec("output_norm.weight")
        emb_w, _, _ = mat("token_embd.weight", self.vocab, self.dim)
        # qwen3.rs:92 keeps the embedding as dense f32 [vocab, dim]
        tbl = q4.q4_0_dequant(ctx, emb_w, self.vocab, self.dim)
        self.embed_tbl = ctx.empty_persistent(self.vocab * self.dim)
        ctx.copy(tbl, 0, self.embed_tbl, 0, self.vocab * self.dim)
        self.lm_head = mat("output.weight", self.vocab, self.dim) if r.has("output.weight") \
            else (emb_w, self.dim, self.vocab)
        self.zeros = ctx.empty_persistent(self.dim)
        r.close()

    def new_cache(self, max_seq: int):
        """KvCache::new (cache.rs:14-18): per-layer [max_seq, kv_dim] f32."""
        kvd = self.n_kv_heads * self.head_dim
        return [(self.ctx.empty_persistent(max_seq * kvd), self.ctx.empty_persistent(max_seq * kvd))
                for _ in range(self.n_layers)]

    def _proj(self, w, x):
        buf, in_f, out_f = w
        return q4.q4_0_gemv(self.ctx, x, buf, in_f, out_f)

    def embed(self, token: int):
        """qwen3.rs:128-133"""
        out = self.ctx.empty(self.dim)
        self.ctx.copy(self.embed_tbl, int(token) * self.dim, out, 0, self.dim)
        return out

    def logits(self, hidden):
        return self._proj(self.lm_head, hidden)

    def forward(self, x, pos: int, cache, hook=None):
        """qwen3.rs:139-191, one op per line as in the reference."""
        ctx, nh, nkv, hd = self.ctx, self.n_heads, self.n_kv_heads, self.head_dim
        kvd = nkv * hd
        hidden = attention.add(ctx, x, self.zeros, self.dim)  # clone_buf (qwen3.rs:194-197)
        for i, l in enumerate(self.layers):
            normed = norm.rmsnorm(ctx, hidden, l["attn_norm"], 1, self.dim, self.eps)
            q = self._proj(l["wq"], normed)
            k = self._proj(l["wk"], normed)
            v = self._proj(l["wv"], normed)
            q = norm.rmsnorm(ctx, q, l["q_norm"], nh, hd, self.eps)
            k = norm.rmsnorm(ctx, k, l["k_norm"], nkv, hd, self.eps)
            q = rope.rope(ctx, q, nh, hd, pos, self.rope_theta)
            k = rope.rope(ctx, k, nkv, hd, pos, self.rope_theta)
            if hook:
                hook("q", i, q, nh * hd)
            kc, vc = cache[i]
            ctx.copy(k, 0, kc, pos * kvd, kvd)  # cache.rs:21-24
            ctx.copy(v, 0, vc, pos * kvd, kvd)
            attn = attention.attention(ctx, q, kc, vc, nh, nkv, pos + 1, hd)
            attn_out = self._proj(l["wo"], attn)
            hidden = attention.add(ctx, hidden, attn_out, self.dim)
            if hook:
                hook("post_attn", i, hidden, self.dim)
            normed = norm.rmsnorm(ctx, hidden, l["ffn_norm"], 1, self.dim, self.eps)
            gate = self._proj(l["gate"], normed)
            up = self._proj(l["up"], normed)
            act = activation.swiglu(ctx, gate, up, self.hidden)
            ff = self._proj(l["down"], act)
            hidden = attention.add(ctx, hidden, ff, self.dim)
            if hook:
                hook("layer_out", i, hidden, self.dim)
        return norm.rmsnorm(ctx, hidden, self.final_norm, 1, self.dim, self.eps)


def generate_op_by_op(ctx: GpuContext, model: OpByOpQwen3, prompt, max_new: int,
                      want_logits: bool = False):
    """model::generate (mod.rs:57-125) over the per-op surface."""
    ctx.clear_cache()
    cache = model.new_cache(len(prompt) + max_new)
    total = len(prompt) + max_new
    produced, all_logits = [], []
    next_input = int(prompt[0])
    for pos in range(total):
        ctx.reset_frame()
        x = model.embed(next_input)
        hidden = model.forward(x, pos, cache)
        logits = model.logits(hidden)
        idx = argmax.argmax(ctx, logits, model.vocab)
        tok = int(ctx.read_u32(idx, 1)[0])
        if pos + 1 < len(prompt):
            next_input = int(prompt[pos + 1])
        else:
            if want_logits:
                all_logits.append(ctx.read(logits, model.vocab))
            produced.append(tok)
            next_input = tok
            if len(produced) >= max_new:
                break
    toks = np.array(produced, dtype=np.uint32)
    return (toks, np.stack(all_logits)) if want_logits else toks
