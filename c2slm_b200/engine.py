"""Python host side over the C ABI (include/c2slm_b200.h).

Mirrors the reference's Go surface for the token loop so callers and tests read
like the reference's own: ``Engine`` is c2slm.Engine minus the tokenizer
(c2slm.go:12-226) with engine.Forward / ComputeLogits and the KVCache
operations; the module-level functions are the tensor.* kernels.

There is no CPU fallback: if libc2slm_b200.so cannot be loaded, or no CUDA
device is present, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libc2slm_b200.so")

F32, Q5_0, Q8_0, Q4_K, Q6_K = 0, 6, 8, 12, 14
MAX_CONTEXT_LEN = 16384  # engine/kvcache.go:11

# exported symbols and their signatures (one line each, matching the header)
P, I, F = C.c_void_p, C.c_int, C.c_float
SIGNATURES = {
    "c2s_last_error": (C.c_char_p, []),
    "c2s_version": (C.c_char_p, []),
    "c2s_engine_open": (I, [C.c_char_p, I, I, C.POINTER(P)]),
    "c2s_engine_create": (I, [P, P, I, I, C.POINTER(P)]),
    "c2s_nccl_unique_id": (I, [P]),
    "c2s_tp_plan": (I, [P, I, I, P]),
    "c2s_engine_create_tp": (I, [P, P, I, I, I, I, P, C.POINTER(P)]),
    "c2s_engine_open_tp": (I, [C.c_char_p, I, I, I, I, P, C.POINTER(P)]),
    "c2s_engine_close": (None, [P]),
    "c2s_engine_desc": (I, [P, P]),
    "c2s_forward": (I, [P, C.c_int32, C.c_int32, P]),
    "c2s_compute_logits": (I, [P, P, P, I, P]),
    "c2s_kv_seq_len": (I, [P]),
    "c2s_kv_set_seq_len": (I, [P, I]),
    "c2s_kv_reset": (I, [P]),
    "c2s_kv_rewind": (I, [P, I]),
    "c2s_kv_store_token_id": (I, [P, I, C.c_int32]),
    "c2s_kv_token_ids": (I, [P, P, I]),
    "c2s_kv_get": (I, [P, I, I, I, I, P]),
    "c2s_prefill_debug": (I, [P, I, P, I]),
    "c2s_ingest_from": (I, [P, I, P, I, P]),
    "c2s_generate": (I, [P, I, F, I, I, P, C.POINTER(I)]),
    "c2s_decode_step": (I, [P, C.c_int32, F, I, C.POINTER(C.c_int32)]),
    "c2s_engine_sync": (I, [P]),
    "c2s_bench_decode": (I, [P, I, F, I]),
    "c2s_kernels_per_step": (I, [P]),
    "c2s_bench_decode_timed": (I, [P, I, F, I, I, C.POINTER(F)]),
    "c2s_profile_step": (I, [P, I, F, I, P, P]),
    "c2s_trace_decode": (I, [P, I, F, I, P, C.POINTER(I)]),
    "c2s_decode_launches": (I, [P, I]),
    "c2s_ring_groups": (I, [I, I]),
    "c2s_quantize_row_q8_k": (I, [P, P, I]),
    "c2s_gemv": (I, [I, P, P, P, I, I]),
    "c2s_gemv_noalloc": (I, [I, P, P, P, I, I]),
    "c2s_gemv_device": (I, [I, I, P, P, P, I, I]),
    "c2s_bench_gemv": (I, [I, I, P, C.c_size_t, I, P, P, I, I, I, C.POINTER(F)]),
    "c2s_kquant_partials": (I, [I, P, P, P, I, I]),
    "c2s_dot_rows_f32x": (I, [I, P, P, P, I, P, I, I]),
    "c2s_rmsnorm": (I, [P, P, P, I, F]),
    "c2s_swiglu": (I, [P, P, P, I]),
    "c2s_dequant_row": (I, [I, P, P, I]),
}


class C2SError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"c2slm_b200 error {code}: {msg}")
        self.code = code


_lib = None


def load_library(path: str = LIB_PATH) -> C.CDLL:
    """Loads the in-tree library (built by c2slm_b200.build / __graft_entry__.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with `python -m c2slm_b200.build`")
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _check(rc: int) -> int:
    if rc < 0:
        raise C2SError(rc, load_library().c2s_last_error().decode(errors="replace"))
    return rc


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    if isinstance(a, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(a), np.uint8)
    return np.ascontiguousarray(a, dtype=np.uint8)


class ModelDesc(C.Structure):
    _fields_ = [("embd", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("rope_base", C.c_float), ("eps", C.c_float),
                ("max_tokens", C.c_int32), ("im_end", C.c_int32), ("eos", C.c_int32)]


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_int32), ("n_dims", C.c_int32),
                ("dims", C.c_int64 * 4), ("data", C.c_void_p), ("nbytes", C.c_uint64)]


# ---------------------------------------------------------------------------
# tensor.* kernels
# ---------------------------------------------------------------------------
def quantize_row_q8_k(x) -> np.ndarray:
    """tensor.QuantizeRowQ8_K (tensor/ops.go:170)."""
    x = _f32(x)
    y = np.zeros((x.size // 256) * 292, np.uint8)
    _check(load_library().c2s_quantize_row_q8_k(_ptr(x), _ptr(y), x.size))
    return y


def gemv(kind: int, w, x, rows: int, cols: int) -> np.ndarray:
    """DispatchGEMV with a pool (engine/model.go:250, engine/pool.go:122-154)."""
    w, x = _u8(w), _f32(x)
    y = np.zeros(rows, np.float32)
    _check(load_library().c2s_gemv(kind, _ptr(w), _ptr(x), _ptr(y), rows, cols))
    return y


def gemv_noalloc(kind: int, w, x, rows: int, cols: int) -> np.ndarray:
    """c2s_gemv with the operands staged in the library's static device array
    (no device allocation or free); see c2s_gemv_noalloc in the header."""
    w, x = _u8(w), _f32(x)
    y = np.zeros(rows, np.float32)
    _check(load_library().c2s_gemv_noalloc(kind, _ptr(w), _ptr(x), _ptr(y), rows, cols))
    return y


def bench_gemv(device: int, kind: int, d_weight: int, copy_stride: int, n_copies: int, d_x: int, d_y: int,
               rows: int, cols: int, reps: int) -> float:
    """Device time (ms) of `reps` back-to-back matvecs on device pointers,
    launch i on weight copy i % n_copies (c2s_bench_gemv)."""
    ms = C.c_float(0.0)
    _check(load_library().c2s_bench_gemv(device, kind, C.c_void_p(d_weight), copy_stride, n_copies,
                                         C.c_void_p(d_x), C.c_void_p(d_y), rows, cols, reps, C.byref(ms)))
    return float(ms.value)


def kquant_partials(kind: int, w, x, rows: int, cols: int) -> np.ndarray:
    w, x = _u8(w), _f32(x)
    nsb = cols // 256
    out = np.zeros(rows * nsb * (8 if kind == Q4_K else 1), np.int32)
    _check(load_library().c2s_kquant_partials(kind, _ptr(w), _ptr(x), _ptr(out), rows, cols))
    return out.reshape(rows, nsb, 8) if kind == Q4_K else out.reshape(rows, nsb)


def dot_rows_f32x(kind: int, w, x, rows_idx, rows: int, cols: int) -> np.ndarray:
    w, x = _u8(w), _f32(x)
    idx = np.ascontiguousarray(rows_idx, np.int32)
    out = np.zeros(idx.size, np.float32)
    _check(load_library().c2s_dot_rows_f32x(kind, _ptr(w), _ptr(x), _ptr(idx), idx.size, _ptr(out), rows, cols))
    return out


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    out = np.zeros_like(x)
    _check(load_library().c2s_rmsnorm(_ptr(out), _ptr(x), _ptr(w), x.size, eps))
    return out


def swiglu(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    out = np.zeros_like(g)
    _check(load_library().c2s_swiglu(_ptr(out), _ptr(g), _ptr(u), g.size))
    return out


def dequant_row(kind: int, row, cols: int) -> np.ndarray:
    row = _u8(row)
    out = np.zeros(cols, np.float32)
    _check(load_library().c2s_dequant_row(kind, _ptr(row), _ptr(out), cols))
    return out


# ---------------------------------------------------------------------------
# Engine
# ---------------------------------------------------------------------------
NCCL_ID_BYTES = 128


def nccl_unique_id() -> bytes:
    """An NCCL unique id for a tensor-parallel group (rank 0 shares it)."""
    buf = (C.c_uint8 * NCCL_ID_BYTES)()
    _check(load_library().c2s_nccl_unique_id(buf))
    return bytes(buf)


def tp_plan(desc, rank: int, world: int) -> dict:
    """The shard of `rank` in a `world`-way tensor-parallel engine."""
    out = (C.c_int32 * 9)()
    _check(load_library().c2s_tp_plan(C.byref(desc), rank, world, out))
    return dict(zip(("h0", "h1", "g0", "g1", "f0", "f1", "v0", "v1", "vpad"), list(out)))


class Engine:
    """c2slm.Engine over one GPU (tokenizer stays with the caller)."""

    def __init__(self, path: str | None = None, device: int = 0, max_tokens: int = MAX_CONTEXT_LEN,
                 gguf_file=None, tp: tuple[int, int, bytes] | None = None):
        """tp = (rank, world, nccl_id): this process's shard of a tensor-parallel
        engine (every rank opens the same file with the same nccl_id, from
        nccl_unique_id() on rank 0, and then makes the same calls)."""
        lib = load_library()
        h = C.c_void_p()
        if tp is not None:
            rank, world, nid = tp
            if path is None or len(nid) != NCCL_ID_BYTES:
                raise ValueError("tensor parallel needs a GGUF path and a 128-byte NCCL id")
            idbuf = (C.c_uint8 * NCCL_ID_BYTES).from_buffer_copy(nid)
            _check(lib.c2s_engine_open_tp(path.encode(), device, max_tokens, rank, world, idbuf, C.byref(h)))
        elif gguf_file is not None:
            self._create_from_gguf(gguf_file, device, max_tokens, h)
        else:
            _check(lib.c2s_engine_open(path.encode(), device, max_tokens, C.byref(h)))
        self._h = h
        d = ModelDesc()
        _check(lib.c2s_engine_desc(self._h, C.byref(d)))
        self.desc = d
        self.device = device

    def _create_from_gguf(self, f, device, max_tokens, h):
        """The cgo path: tensors stay mapped by the caller's GGUF reader."""
        def u32(k2, k3, dflt):
            v, ok = f.get_uint32(k2)
            if not ok or v == 0:
                v, ok = f.get_uint32(k3)
            return v if v else dflt
        d = ModelDesc()
        d.embd = u32("qwen2.embedding_length", "qwen3.embedding_length", 896)
        d.n_layers = u32("qwen2.block_count", "qwen3.block_count", 24)
        d.n_heads = u32("qwen2.attention.head_count", "qwen3.attention.head_count", 14)
        d.n_kv_heads = u32("qwen2.attention.head_count_kv", "qwen3.attention.head_count_kv", 2)
        d.ffn = u32("qwen2.feed_forward_length", "qwen3.feed_forward_length", 4864)
        rb, _ = f.get_float32("qwen2.rope.freq_base")
        d.rope_base = rb or 1e6
        ep, _ = f.get_float32("qwen2.attention.layer_norm_rms_epsilon")
        d.eps = ep or 1e-6
        d.max_tokens = max_tokens
        toks, ok = f.get_string_slice("tokenizer.ggml.tokens")
        specials = {s: i for i, s in enumerate(toks or []) if s.startswith("<|") and s.endswith("|>")}
        d.im_end = specials.get("<|im_end|>", 0)
        d.eos = specials.get("<|endoftext|>", 0)
        descs = (TensorDesc * len(f.tensors))()
        self._keep = []
        for i, ti in enumerate(f.tensors):
            name = ti.name.encode()
            self._keep.append(name)
            arr = np.frombuffer(ti.data, np.uint8)
            self._keep.append(arr)
            descs[i].name = name
            descs[i].type = ti.type
            descs[i].n_dims = len(ti.dimensions)
            for k, v in enumerate(ti.dimensions[:4]):
                descs[i].dims[k] = v
            descs[i].data = arr.ctypes.data
            descs[i].nbytes = len(ti.data)
        del arr  # no view of the caller's mapping outlives this call, even when it raises
        try:
            _check(load_library().c2s_engine_create(C.byref(d), descs, len(f.tensors), device, C.byref(h)))
        finally:
            self._keep = None

    # lifecycle -------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            load_library().c2s_engine_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # engine.Forward / ComputeLogits ------------------------------------------
    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.desc.embd, np.float32)
        _check(load_library().c2s_forward(self._h, token, pos, _ptr(out)))
        return out

    def compute_logits(self, normx=None, targets=None, out=None) -> np.ndarray:
        lib = load_library()
        if out is None:
            out = np.zeros(self.desc.vocab, np.float32)
        nx = None if normx is None else _f32(normx)
        if targets is not None and len(targets) > 0:
            t = np.ascontiguousarray(targets, np.int32)
            _check(lib.c2s_compute_logits(self._h, None if nx is None else _ptr(nx), _ptr(t), t.size, _ptr(out)))
        else:
            _check(lib.c2s_compute_logits(self._h, None if nx is None else _ptr(nx), None, 0, _ptr(out)))
        return out

    # KVCache ----------------------------------------------------------------
    @property
    def seq_len(self) -> int:
        return _check(load_library().c2s_kv_seq_len(self._h))

    @seq_len.setter
    def seq_len(self, n: int) -> None:
        _check(load_library().c2s_kv_set_seq_len(self._h, n))

    @property
    def max_tokens(self) -> int:
        return self.desc.max_tokens

    def reset(self) -> None:
        _check(load_library().c2s_kv_reset(self._h))

    def rewind(self, n: int) -> None:
        _check(load_library().c2s_kv_rewind(self._h, n))

    def store_token_id(self, pos: int, token: int) -> None:
        _check(load_library().c2s_kv_store_token_id(self._h, pos, token))

    def token_ids(self, n: int | None = None) -> np.ndarray:
        n = self.seq_len if n is None else n
        out = np.zeros(max(n, 1), np.int32)
        _check(load_library().c2s_kv_token_ids(self._h, _ptr(out), n))
        return out[:n]

    def get_key(self, layer: int, kv_head: int, pos: int) -> np.ndarray:
        out = np.zeros(self.desc.head_dim, np.float32)
        _check(load_library().c2s_kv_get(self._h, 0, layer, kv_head, pos, _ptr(out)))
        return out

    def get_value(self, layer: int, kv_head: int, pos: int) -> np.ndarray:
        out = np.zeros(self.desc.head_dim, np.float32)
        _check(load_library().c2s_kv_get(self._h, 1, layer, kv_head, pos, _ptr(out)))
        return out

    def prefill_debug(self, which: str, n_tokens: int, n_heads: int) -> np.ndarray:
        """Test surface: the last layer's buffers of the last tensor-core
        prefill chunk, [n_tokens][n_heads * head_dim] -- which = "attention"
        (the causal attention output) or "queries" (the rotated queries)."""
        out = np.zeros((n_tokens, n_heads * self.desc.head_dim), np.float32)
        w = {"attention": 0, "queries": 1}[which]
        _check(load_library().c2s_prefill_debug(self._h, w, _ptr(out), out.size))
        return out

    # c2slm.Engine ------------------------------------------------------------
    def ingest_from(self, pos: int, tokens) -> np.ndarray | None:
        """c2slm.Engine.IngestFrom (c2slm.go:92-115)."""
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.desc.embd, np.float32)
        n = _check(load_library().c2s_ingest_from(self._h, pos, _ptr(t) if t.size else None, t.size, _ptr(out)))
        return out if n > 0 else None

    def generate(self, max_new: int, penalty: float = 1.15, window: int = 64,
                 stop_on_special: bool = True) -> np.ndarray:
        """The greedy loop of c2slm.Engine.generate (c2slm.go:144-223) on ids."""
        buf = np.zeros(max(max_new, 1), np.int32)
        n = C.c_int(0)
        _check(load_library().c2s_generate(self._h, max_new, penalty, window, 1 if stop_on_special else 0,
                                           _ptr(buf), C.byref(n)))
        return buf[:n.value].copy()

    def generate_stream(self, prompt_tokens, max_new: int, penalty: float = 1.15, window: int = 64,
                        stop_on_special: bool = True) -> np.ndarray:
        """GenerateStream on token ids (c2slm.go:64-82): reset, ingest, generate."""
        if len(prompt_tokens) == 0:
            raise ValueError("empty prompt tokens")
        if len(prompt_tokens) >= MAX_CONTEXT_LEN:
            raise ValueError(f"prompt ({len(prompt_tokens)}) exceeds max context ({MAX_CONTEXT_LEN})")
        self.reset()
        self.ingest_from(0, prompt_tokens)
        return self.generate(max_new, penalty, window, stop_on_special)

    def generate_stream_session(self, new_tokens, max_new: int, penalty: float = 1.15, window: int = 64,
                                stop_on_special: bool = True) -> np.ndarray:
        """GenerateStreamSession on token ids (c2slm.go:124-138)."""
        if len(new_tokens) == 0:
            raise ValueError("empty prompt tokens")
        if self.seq_len + len(new_tokens) >= MAX_CONTEXT_LEN:
            raise ValueError("session prompt exceeds max context")
        self.ingest_from(self.seq_len, new_tokens)
        return self.generate(max_new, penalty, window, stop_on_special)

    def decode_step(self, token: int, penalty: float = 1.15, window: int = 64) -> int:
        nxt = C.c_int32(0)
        _check(load_library().c2s_decode_step(self._h, token, penalty, window, C.byref(nxt)))
        return nxt.value

    def sync(self) -> None:
        _check(load_library().c2s_engine_sync(self._h))

    def bench_decode(self, n_steps: int, penalty: float = 1.15, window: int = 64) -> None:
        _check(load_library().c2s_bench_decode(self._h, n_steps, penalty, window))

    def bench_decode_timed(self, n_steps: int, penalty: float = 1.15, window: int = 64, period: int = 0) -> float:
        """Runs n_steps device-resident decode steps (rewinding to the current
        SeqLen every `period` steps); returns CUDA-event milliseconds."""
        ms = C.c_float(0)
        _check(load_library().c2s_bench_decode_timed(self._h, n_steps, penalty, window, period, C.byref(ms)))
        return ms.value

    STAGES = {1: "qkv", 2: "o_proj", 3: "gate_up", 4: "down", 5: "logits", 7: "attention"}

    def profile_step(self, n_steps: int, penalty: float = 1.15, window: int = 64) -> dict:
        """Per-stage CUDA-event timing table over n_steps decode steps."""
        ms = np.zeros(8, np.float32)
        cnt = np.zeros(8, np.int32)
        _check(load_library().c2s_profile_step(self._h, n_steps, penalty, window, _ptr(ms), _ptr(cnt)))
        return {name: {"ms": float(ms[k]), "launches": int(cnt[k])} for k, name in self.STAGES.items()}

    def trace_decode(self, n_steps: int, penalty: float = 1.15, window: int = 64, n_sms: int | None = None):
        """Per-phase stamps (ns) of the persistent decode kernel for every CTA:
        array [n_steps, nphase, n_sms, 8]: ns stamps (start, inputs ready,
        chunks done, end), then SM cycles (weight waits, grid barrier, chunk
        loop, cycle counter at start)."""
        import torch
        n_sms = n_sms or torch.cuda.get_device_properties(self.device).multi_processor_count
        nph = C.c_int(0)
        buf = np.zeros(n_steps * n_sms * 8 * (5 * self.desc.n_layers + 1), np.uint64)
        _check(load_library().c2s_trace_decode(self._h, n_steps, penalty, window, _ptr(buf), C.byref(nph)))
        return buf.reshape(n_steps, nph.value, n_sms, 8)

    @property
    def kernels_per_step(self) -> int:
        return load_library().c2s_kernels_per_step(self._h)

    def decode_launches(self, n_steps: int) -> int:
        """Kernel launches of one bench_decode(_timed) call of n_steps."""
        return load_library().c2s_decode_launches(self._h, n_steps)
