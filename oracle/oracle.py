"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py as the checker; the product (c2slm_b200) never imports
this module.  Each wrapper names the reference function it restates (see the
file:line comments in c2s_oracle.c).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, Q5_0, Q8_0, Q4_K, Q6_K = 0, 6, 8, 12, 14
BLOCK = {Q5_0: (32, 22), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), F32: (1, 4)}


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    src = os.path.join(HERE, "c2s_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I = C.c_int
F = C.c_float


def _declare(L: C.CDLL) -> None:
    sig = {
        "c2o_fp16_to_f32": (F, [C.c_uint16]),
        "c2o_quantize_row_q8_k": (None, [P, P, I]),
        "c2o_dot_q4_k_q8_k": (F, [P, P, I]),
        "c2o_gemv2_q4_k_q8_k": (None, [P, P, P, I, P, P]),
        "c2o_gemv2_q6_k_q8_k": (None, [P, P, P, I, P, P]),
        "c2o_dot_q5_0": (F, [P, P, I]),
        "c2o_dot_q8_0": (F, [P, P, I]),
        "c2o_dot_q4_k": (F, [P, P, I]),
        "c2o_dot_q6_k": (F, [P, P, I]),
        "c2o_q4k_q8k_partials": (None, [P, P, I, I, P, P]),
        "c2o_q6k_q8k_partials": (None, [P, P, I, I, P]),
        "c2o_gemv": (I, [I, P, P, P, I, I, P, I]),
        "c2o_gemv_f32x": (I, [I, P, P, P, I, I]),
        "c2o_dequant_row": (I, [I, P, P, I]),
        "c2o_rmsnorm": (None, [P, P, P, I, F]),
        "c2o_add_bias": (None, [P, P, I]),
        "c2o_rope_table": (None, [P, P, I, I, F]),
        "c2o_rope_apply": (None, [P, P, I, I, P, I, I, I]),
        "c2o_rope_neox": (None, [P, I, I, I, F]),
        "c2o_softmax": (None, [P, I]),
        "c2o_swiglu": (None, [P, P, P, I]),
        "c2o_attn_qk": (None, [P, P, I, I, F, P, I]),
        "c2o_attn_av": (None, [P, P, I, I, P, I]),
        "c2o_model_open": (P, [C.c_char_p, I, I, C.c_char_p, I]),
        "c2o_model_close": (None, [P]),
        "c2o_model_get_info": (None, [P, P]),
        "c2o_model_set_simd_order": (None, [P, I]),
        "c2o_attn_qk_simd": (None, [P, P, I, I, F, P, I]),
        "c2o_attn_av_simd": (None, [P, P, I, I, P, I]),
        "c2o_swiglu_simd": (None, [P, P, P, I]),
        "c2o_forward": (None, [P, C.c_int32, I, P]),
        "c2o_compute_logits": (None, [P, P, P, P, I]),
        "c2o_select": (C.c_int32, [P, P, I, F, I]),
        "c2o_kv_seq_len": (I, [P]),
        "c2o_kv_set_seq_len": (None, [P, I]),
        "c2o_kv_reset": (None, [P]),
        "c2o_kv_rewind": (None, [P, I]),
        "c2o_kv_store_token_id": (None, [P, I, C.c_int32]),
        "c2o_kv_token_id": (C.c_int32, [P, I]),
        "c2o_kv_get": (None, [P, I, I, I, I, P]),
        "c2o_ingest_from": (I, [P, I, P, I, P]),
        "c2o_generate": (I, [P, P, I, F, I, I, P, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(a), np.uint8) if isinstance(a, (bytes, bytearray)) else a, dtype=np.uint8)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- scalar kernels ---------------------------------------------------------
def fp16_to_f32(h: int) -> float:
    return lib().c2o_fp16_to_f32(h)


def quantize_row_q8_k(x) -> np.ndarray:
    x = _f32(x)
    y = np.zeros((x.size // 256) * 292, np.uint8)
    lib().c2o_quantize_row_q8_k(_p(x), _p(y), x.size)
    return y


def dot_q4_k_q8_k(w, q8k, cols: int) -> float:
    w, q8k = _u8(w), _u8(q8k)
    return lib().c2o_dot_q4_k_q8_k(_p(w), _p(q8k), cols)


def gemv2(kind: int, w0, w1, q8k, cols: int):
    w0, w1, q8k = _u8(w0), _u8(w1), _u8(q8k)
    o = np.zeros(2, np.float32)
    fn = lib().c2o_gemv2_q4_k_q8_k if kind == Q4_K else lib().c2o_gemv2_q6_k_q8_k
    fn(_p(w0), _p(w1), _p(q8k), cols, C.c_void_p(o.ctypes.data), C.c_void_p(o.ctypes.data + 4))
    return float(o[0]), float(o[1])


def dot_f32x(kind: int, w, x, cols: int) -> float:
    w, x = _u8(w), _f32(x)
    fn = {Q5_0: lib().c2o_dot_q5_0, Q8_0: lib().c2o_dot_q8_0,
          Q4_K: lib().c2o_dot_q4_k, Q6_K: lib().c2o_dot_q6_k}[kind]
    return fn(_p(w), _p(x), cols)


def q4k_q8k_partials(w, q8k, rows: int, cols: int):
    w, q8k = _u8(w), _u8(q8k)
    nsb = cols // 256
    dots = np.zeros(rows * nsb * 8, np.int32)
    pairs = np.zeros(nsb * 4, np.int32)
    lib().c2o_q4k_q8k_partials(_p(w), _p(q8k), rows, cols, _p(dots), _p(pairs))
    return dots.reshape(rows, nsb, 8), pairs.reshape(nsb, 4)


def q6k_q8k_partials(w, q8k, rows: int, cols: int):
    w, q8k = _u8(w), _u8(q8k)
    nsb = cols // 256
    isum = np.zeros(rows * nsb, np.int32)
    lib().c2o_q6k_q8k_partials(_p(w), _p(q8k), rows, cols, _p(isum))
    return isum.reshape(rows, nsb)


def gemv(kind: int, w, x, rows: int, cols: int, nthreads: int = 1) -> np.ndarray:
    """WorkerPool.ParallelGEMV semantics: K-quants go through Q8_K."""
    w, x = _u8(w), _f32(x)
    y = np.zeros(rows, np.float32)
    q8 = np.zeros((cols // 256 + 1) * 292, np.uint8)
    rc = lib().c2o_gemv(kind, _p(w), _p(x), _p(y), rows, cols, _p(q8), nthreads)
    assert rc == 0
    return y


def gemv_f32x(kind: int, w, x, rows: int, cols: int) -> np.ndarray:
    w, x = _u8(w), _f32(x)
    y = np.zeros(rows, np.float32)
    lib().c2o_gemv_f32x(kind, _p(w), _p(x), _p(y), rows, cols)
    return y


def dequant_row(kind: int, row, cols: int) -> np.ndarray:
    row = _u8(row)
    out = np.zeros(cols, np.float32)
    assert lib().c2o_dequant_row(kind, _p(row), _p(out), cols) == 0
    return out


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    out = np.zeros_like(x)
    lib().c2o_rmsnorm(_p(out), _p(x), _p(w), x.size, eps)
    return out


def rope_table(max_len: int, head_dim: int, theta: float):
    half = head_dim // 2
    c = np.zeros(max_len * half, np.float32)
    s = np.zeros(max_len * half, np.float32)
    lib().c2o_rope_table(_p(c), _p(s), max_len, head_dim, theta)
    return c, s


def rope_apply(table, max_len: int, head_dim: int, vec, num_heads: int, pos: int) -> np.ndarray:
    c, s = table
    v = _f32(vec).copy()
    lib().c2o_rope_apply(_p(c), _p(s), max_len, head_dim, _p(v), v.size, num_heads, pos)
    return v


def rope_neox(vec, num_heads: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    v = _f32(vec).copy()
    lib().c2o_rope_neox(_p(v), num_heads, head_dim, pos, theta)
    return v


def softmax(x) -> np.ndarray:
    v = _f32(x).copy()
    lib().c2o_softmax(_p(v), v.size)
    return v


def swiglu(g, u, simd: bool = False) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    out = np.zeros_like(g)
    (lib().c2o_swiglu_simd if simd else lib().c2o_swiglu)(_p(out), _p(g), _p(u), g.size)
    return out


def attn_qk(q, kbase, pos: int, stride: int, scale: float, hd: int, simd: bool = False) -> np.ndarray:
    q, kbase = _f32(q), _f32(kbase)
    s = np.zeros(pos + 1, np.float32)
    fn = lib().c2o_attn_qk_simd if simd else lib().c2o_attn_qk
    fn(_p(q), _p(kbase), pos, stride, scale, _p(s), hd)
    return s


def attn_av(scores, vbase, pos: int, stride: int, hd: int, simd: bool = False) -> np.ndarray:
    scores, vbase = _f32(scores), _f32(vbase)
    out = np.zeros(hd, np.float32)
    fn = lib().c2o_attn_av_simd if simd else lib().c2o_attn_av
    fn(_p(scores), _p(vbase), pos, stride, _p(out), hd)
    return out


# ---- model -----------------------------------------------------------------
class ModelInfo(C.Structure):
    _fields_ = [("embd", C.c_int32), ("n_layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32), ("ffn", C.c_int32),
                ("vocab", C.c_int32), ("rope_base", C.c_float), ("eps", C.c_float),
                ("max_tokens", C.c_int32), ("im_end", C.c_int32), ("eos", C.c_int32),
                ("tied_output", C.c_int32)]


class OracleModel:
    """engine.Model + KVCache + Arena on the CPU (engine/model.go:58, kvcache.go:49)."""

    def __init__(self, path: str, max_tokens: int = 16384, nthreads: int = 1, simd_order: bool = False):
        err = C.create_string_buffer(512)
        self._h = lib().c2o_model_open(path.encode(), max_tokens, nthreads, err, 512)
        if not self._h:
            raise RuntimeError(f"oracle load failed: {err.value.decode()}")
        info = ModelInfo()
        lib().c2o_model_get_info(self._h, C.byref(info))
        self.info = info
        if simd_order:  # evaluate like the reference's AVX2 build
            lib().c2o_model_set_simd_order(self._h, 1)

    def close(self):
        if self._h:
            lib().c2o_model_close(self._h)
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

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.info.embd, np.float32)
        lib().c2o_forward(self._h, token, pos, _p(out))
        return out

    def compute_logits(self, normx, targets=None) -> np.ndarray:
        normx = _f32(normx)
        out = np.zeros(self.info.vocab, np.float32)
        if targets is None or len(targets) == 0:
            lib().c2o_compute_logits(self._h, _p(normx), _p(out), None, 0)
        else:
            t = np.ascontiguousarray(targets, np.int32)
            lib().c2o_compute_logits(self._h, _p(normx), _p(out), _p(t), t.size)
        return out

    def select(self, logits, cur_pos: int, penalty: float = 1.15, window: int = 64):
        lg = _f32(logits).copy()
        best = lib().c2o_select(self._h, _p(lg), cur_pos, penalty, window)
        return int(best), lg

    @property
    def seq_len(self) -> int:
        return lib().c2o_kv_seq_len(self._h)

    @seq_len.setter
    def seq_len(self, n: int) -> None:
        lib().c2o_kv_set_seq_len(self._h, n)

    def reset(self):
        lib().c2o_kv_reset(self._h)

    def rewind(self, n: int):
        lib().c2o_kv_rewind(self._h, n)

    def store_token_id(self, pos: int, tok: int):
        lib().c2o_kv_store_token_id(self._h, pos, tok)

    def token_ids(self, n: int) -> np.ndarray:
        return np.array([lib().c2o_kv_token_id(self._h, i) for i in range(n)], np.int32)

    def kv_get(self, is_v: int, layer: int, kv_head: int, pos: int) -> np.ndarray:
        out = np.zeros(self.info.head_dim, np.float32)
        lib().c2o_kv_get(self._h, is_v, layer, kv_head, pos, _p(out))
        return out

    def ingest_from(self, pos: int, tokens) -> np.ndarray | None:
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.info.embd, np.float32)
        n = lib().c2o_ingest_from(self._h, pos, _p(t), t.size, _p(out))
        return out if n > 0 else None

    def generate(self, last_normx, max_new: int, penalty: float = 1.15, window: int = 64,
                 stop_on_special: bool = True):
        normx = _f32(last_normx)
        toks = np.zeros(max(max_new, 1), np.int32)
        margins = np.zeros(max(max_new, 1), np.float32)
        maxabs = np.zeros(max(max_new, 1), np.float32)
        n = lib().c2o_generate(self._h, _p(normx), max_new, penalty, window,
                               1 if stop_on_special else 0, _p(toks), _p(margins), _p(maxabs))
        return toks[:n].copy(), margins[:n].copy(), maxabs[:n].copy()
