"""Host-side mirror of static-lm's operator and model API over libslm_b200.so.

The names follow the reference (Bluewraith04/static-lm):
  AlignedArena / ArenaSlice      -> Arena / Slice        (src/memory/arena.rs)
  gemv_q4_0_arena / gemm_q4_0_arena -> same names        (src/quant/kernels.rs:289, :398)
  JitEngine exec_* on FuseGraph ops -> exec_rmsnorm, ... (src/jit/engine.rs:153-206)
  TransformerModel::{forward_token, prefill_tokens, generate, embed_tokens}
                                 -> Model methods       (src/model/transformer.rs:747-948)
Every call goes through the C ABI of include/slm_b200.h; all compute runs
in the sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import JIT_KERNEL_FN, JIT_OPS, PHASES, Config, LayerWeights, ModelWeights, SlmError, Slice, lib

__all__ = ["Config", "Slice", "SlmError", "Arena", "QMatrix", "Model", "JitEngine", "lib",
           "gemv_q4_0_arena", "gemm_q4_0_arena", "rope_tables"]

Q4_BLOCK_BYTES = 18
Q8_BLOCK_BYTES = 34


def _np_ptr(a: np.ndarray) -> int:
    if not a.flags["C_CONTIGUOUS"]:
        raise ValueError("array must be C-contiguous")
    return a.ctypes.data


class Arena:
    """AlignedArena (arena.rs:40-122) living in device memory."""

    def __init__(self, capacity: int, device: int = 0):
        h = C.c_void_p()
        lib().slm_arena_create(device, capacity, C.byref(h))
        self.h = h
        self.device = device

    def close(self):
        if self.h:
            lib().slm_arena_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def alloc_slice(self, n: int) -> Slice:
        s = Slice()
        lib().slm_arena_alloc_slice(self.h, n, C.byref(s))
        return s

    def alloc_q8_scratch(self, num_blocks: int) -> Slice:
        s = Slice()
        lib().slm_arena_alloc_q8_scratch(self.h, num_blocks, C.byref(s))
        return s

    def reset(self):
        lib().slm_arena_reset(self.h)

    @property
    def capacity(self) -> int:
        return int(lib().slm_arena_capacity(self.h))

    @property
    def used(self) -> int:
        return int(lib().slm_arena_used(self.h))

    def device_ptr(self, s: Slice) -> int:
        p = lib().slm_arena_device_ptr(self.h, s)
        if not p:
            raise SlmError(2, lib().slm_last_error().decode())
        return p

    def write(self, s: Slice, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32)
        lib().slm_arena_write(self.h, s, _np_ptr(a), a.size)

    def read(self, s: Slice) -> np.ndarray:
        out = np.empty(s.len, dtype=np.float32)
        lib().slm_arena_read(self.h, s, _np_ptr(out), out.size)
        return out


class QMatrix:
    """A rows x cols BlockQ4_0 matrix uploaded to the device."""

    def __init__(self, blocks: np.ndarray, rows: int, cols: int, device: int = 0):
        b = np.ascontiguousarray(blocks)
        if b.nbytes != rows * cols // 32 * Q4_BLOCK_BYTES:
            raise SlmError(4, "weights block count mismatch")
        h = C.c_void_p()
        lib().slm_qmatrix_upload(device, _np_ptr(b), rows, cols, C.byref(h))
        self.h, self.rows, self.cols = h, rows, cols

    def download(self) -> np.ndarray:
        out = np.zeros(self.rows * self.cols // 32 * Q4_BLOCK_BYTES, dtype=np.uint8)
        lib().slm_qmatrix_download(self.h, _np_ptr(out))
        return out

    def close(self):
        if self.h:
            lib().slm_qmatrix_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemv_q4_0_arena(arena: Arena, w: QMatrix, inp: Slice, q8: Slice, out: Slice, rows: int,
                    cols: int, stream: int = 0) -> None:
    lib().slm_gemv_q4_0_arena(arena.h, w.h, inp, q8, out, rows, cols, stream)


def gemm_q4_0_arena(arena: Arena, w: QMatrix, inp: Slice, q8: Slice, out: Slice, batch: int,
                    rows: int, cols: int, stream: int = 0) -> None:
    lib().slm_gemm_q4_0_arena(arena.h, w.h, inp, q8, out, batch, rows, cols, stream)


def rope_tables(max_seq: int, head_dim: int):
    c = np.zeros(max_seq * (head_dim // 2), dtype=np.float32)
    s = np.zeros_like(c)
    lib().slm_rope_tables(max_seq, head_dim, _np_ptr(c), _np_ptr(s))
    return c, s


class JitEngine:
    """JitEngine (src/jit/engine.rs:28-206) on the device: compile() returns
    a function with the JitKernelFn calling convention (slm_jit_compile), and
    exec_unary / exec_binary / exec_with_weights call it on arena slices the
    way the reference's do (engine.rs:153-206)."""

    def __init__(self, stream: int = 0):
        self.stream = stream

    def compile(self, op: str, n: int = 0, eps: float = 0.0):
        fp = C.c_void_p()
        lib().slm_jit_compile(JIT_OPS[op], n, eps, self.stream or None, C.byref(fp))
        return JIT_KERNEL_FN(fp.value)

    @staticmethod
    def _call(kernel, ptrs, out_ptr, n):
        arr = (C.c_void_p * len(ptrs))(*ptrs)
        kernel(C.cast(arr, C.POINTER(C.c_void_p)), out_ptr, n)

    def exec_unary(self, kernel, arena: "Arena", src: Slice, dst: Slice):
        if src.len != dst.len:
            raise SlmError(4, "src and dst length mismatch")
        self._call(kernel, [arena.device_ptr(src)], arena.device_ptr(dst), dst.len)

    def exec_binary(self, kernel, arena: "Arena", a: Slice, b: Slice, dst: Slice):
        if a.len != dst.len or b.len != dst.len:
            raise SlmError(4, "src and dst length mismatch")
        self._call(kernel, [arena.device_ptr(a), arena.device_ptr(b)], arena.device_ptr(dst), dst.len)

    def exec_with_weights(self, kernel, arena: "Arena", src: Slice, weights_dev: int, dst: Slice):
        if src.len != dst.len:
            raise SlmError(4, "src and dst length mismatch")
        self._call(kernel, [arena.device_ptr(src), weights_dev], arena.device_ptr(dst), dst.len)


def _vp_array(ptrs):
    arr = (C.c_void_p * len(ptrs))(*ptrs)
    return C.cast(arr, C.POINTER(C.c_void_p)), arr


class Model:
    """TransformerModel (transformer.rs:698-949) for `max_sequences`
    independent sequences on one GPU."""

    def __init__(self, cfg: Config, weights, max_sequences: int = 1, max_rows: int | None = None,
                 device: int = 0):
        """`weights` has attributes token_embd, layers (list of dicts with the
        TransformerWeights field names), output_norm, lm_head (or None), vocab
        -- host numpy arrays in the reference's formats."""
        self.cfg = cfg
        self.vocab = weights.vocab
        self.num_layers = len(weights.layers)
        self._keep = []
        layers = (LayerWeights * self.num_layers)()
        keys = ["rms_att_weight", "wq", "wk", "wv", "wo", "rms_ffn_weight", "w_gate", "w_up",
                "w_down"]
        for l, lw in enumerate(weights.layers):
            arrs = [np.ascontiguousarray(lw[k]) for k in keys]
            self._keep += arrs
            layers[l] = LayerWeights(*[_np_ptr(a) for a in arrs])
        te = np.ascontiguousarray(weights.token_embd)
        on = np.ascontiguousarray(weights.output_norm, dtype=np.float32)
        lm = None if weights.lm_head is None else np.ascontiguousarray(weights.lm_head)
        self._keep += [te, on, lm]
        mw = ModelWeights(_np_ptr(te), layers, self.num_layers, _np_ptr(on),
                          _np_ptr(lm) if lm is not None else None, self.vocab)
        h = C.c_void_p()
        lib().slm_model_create(device, C.byref(cfg), C.byref(mw), max_sequences,
                               max_rows or max_sequences, C.byref(h))
        self.h = h
        self._keep = []  # weights were uploaded; host copies no longer needed
        self.max_sequences = max_sequences
        self.kv_dim = cfg.dim // cfg.num_heads * cfg.num_kv_heads

    def close(self):
        if getattr(self, "h", None):
            lib().slm_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return int(lib().slm_model_stream(self.h) or 0)

    @property
    def device_bytes(self) -> int:
        return int(lib().slm_model_device_bytes(self.h))

    def forward_token(self, token: int, pos: int, seq: int = 0) -> int:
        nxt = C.c_int32()
        lib().slm_model_forward_token(self.h, seq, token, pos, C.byref(nxt))
        return int(nxt.value)

    def prefill_tokens(self, tokens, start_pos: int = 0, seq: int = 0) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = C.c_int32()
        lib().slm_model_prefill_tokens(self.h, seq, t.ctypes.data_as(C.POINTER(C.c_int32)), t.size,
                                       start_pos, C.byref(nxt))
        return int(nxt.value)

    def prefill_batch(self, prompts, seqs=None):
        """Batched prefill of equal-length prompts (2-D array [nseq][n]); returns
        the greedy next token of each (slm_model_prefill_batch)."""
        t = np.ascontiguousarray(prompts, dtype=np.int32)
        nseq, n = t.shape
        s = np.ascontiguousarray(range(nseq) if seqs is None else seqs, dtype=np.uint32)
        nxt = np.zeros(nseq, dtype=np.int32)
        lib().slm_model_prefill_batch(self.h, nseq, s.ctypes.data_as(C.POINTER(C.c_uint32)),
                                      t.ctypes.data_as(C.POINTER(C.c_int32)), n,
                                      nxt.ctypes.data_as(C.POINTER(C.c_int32)))
        return nxt

    def attach_shard(self, nccl_id: bytes, nranks: int, rank: int):
        """Join the KV-head sharding group (collective over the ranks)."""
        buf = C.create_string_buffer(bytes(nccl_id), 128) if nranks > 1 else None
        lib().slm_model_attach_shard(self.h, buf, 128 if buf is not None else 0, nranks, rank)

    def set_comm_timeout(self, ms: int):
        """Bound (milliseconds) on the shard group's set-up and on each sharded
        prefill's wait for its collectives; past it the call raises TIMEOUT."""
        lib().slm_model_set_comm_timeout(self.h, ms)

    def set_prefill_mode(self, tensor_cores: bool):
        """Prefill attention on the tcgen05 tensor cores (3xTF32, ~1e-6
        relative to the exact path) or bit-exact on the CUDA cores (default)."""
        lib().slm_model_set_prefill_mode(self.h, 1 if tensor_cores else 0)

    def set_decode_mode(self, flash: bool):
        """Decode attention as split-K flash-decode (~1e-6 relative to the
        exact path) or bit-exact sequential chains (default)."""
        lib().slm_model_set_decode_mode(self.h, 1 if flash else 0)

    def generate(self, prompt, n_out: int, eos: int = -1, seq: int = 0):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_out, 1), dtype=np.int32)
        gen = C.c_uint32()
        lib().slm_model_generate(self.h, seq, p.ctypes.data_as(C.POINTER(C.c_int32)), p.size,
                                 out.ctypes.data_as(C.POINTER(C.c_int32)), n_out, eos,
                                 C.byref(gen))
        return out[:gen.value].tolist()

    def embed_tokens(self, tokens, seq: int = 0) -> np.ndarray:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(self.cfg.dim, dtype=np.float32)
        lib().slm_model_embed_tokens(self.h, seq, t.ctypes.data_as(C.POINTER(C.c_int32)), t.size,
                                     out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def decode_batch(self, seqs, tokens, pos) -> np.ndarray:
        s = np.ascontiguousarray(seqs, dtype=np.uint32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(pos, dtype=np.uint32)
        nxt = np.zeros(t.size, dtype=np.int32)
        lib().slm_model_decode_batch(self.h, t.size, s.ctypes.data_as(C.POINTER(C.c_uint32)),
                                     t.ctypes.data_as(C.POINTER(C.c_int32)),
                                     p.ctypes.data_as(C.POINTER(C.c_uint32)),
                                     nxt.ctypes.data_as(C.POINTER(C.c_int32)))
        return nxt

    def decode_steps_device(self, n: int, seqs_dev: int, tokens_dev: int, pos_dev: int,
                            steps: int, out_dev: int, max_pos_hint: int) -> None:
        lib().slm_model_decode_steps_device(self.h, n, seqs_dev, tokens_dev, pos_dev, steps,
                                            out_dev, max_pos_hint)

    def kv_write(self, seq: int, layer: int, which: int, row0: int, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32)
        nrows = a.size // self.kv_dim
        lib().slm_model_kv_write(self.h, seq, layer, which, row0, nrows, _np_ptr(a))

    def kv_write_device(self, seq: int, layer: int, which: int, row0: int, nrows: int,
                        src_dev: int) -> None:
        lib().slm_model_kv_write_device(self.h, seq, layer, which, row0, nrows, src_dev)

    def profile_decode(self, n: int, seqs_dev: int, tokens_dev: int, pos_dev: int, steps: int,
                       max_pos_hint: int) -> dict:
        ms = (C.c_float * len(PHASES))()
        lib().slm_model_profile_decode(self.h, n, seqs_dev, tokens_dev, pos_dev, steps,
                                       max_pos_hint, ms)
        return {name: float(ms[i]) for i, name in enumerate(PHASES)}

    def launches_per_decode_step(self, n: int) -> int:
        return int(lib().slm_model_launches_per_decode_step(self.h, n))

    def kv_read(self, seq: int, layer: int, which: int, row0: int, nrows: int) -> np.ndarray:
        out = np.zeros(nrows * self.kv_dim, dtype=np.float32)
        lib().slm_model_kv_read(self.h, seq, layer, which, row0, nrows, _np_ptr(out))
        return out

    def logits(self, row: int = 0) -> np.ndarray:
        out = np.zeros(self.vocab, dtype=np.float32)
        lib().slm_model_read_logits(self.h, row, _np_ptr(out))
        return out

    def hidden(self, row: int = 0) -> np.ndarray:
        out = np.zeros(self.cfg.dim, dtype=np.float32)
        lib().slm_model_read_hidden(self.h, row, _np_ptr(out))
        return out


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for Model.attach_shard."""
    buf = C.create_string_buffer(128)
    lib().slm_nccl_unique_id(buf, 128)
    return buf.raw


def shard_units(nseq: int, num_kv_heads: int, nranks: int, rank: int):
    """The (sequence*num_kv_heads + KV head) units `rank` computes in a sharded
    batched prefill, in all-gather order."""
    cap = max(1, nseq * num_kv_heads)
    out = np.zeros(cap, dtype=np.uint32)
    k = lib().slm_shard_units(nseq, num_kv_heads, nranks, rank,
                              out.ctypes.data_as(C.POINTER(C.c_uint32)), cap)
    return [int(u) for u in out[:k]]
