"""Python handle on the oracle: the CPU restatement of SparseLattice's integer forward path.

TEST INFRASTRUCTURE ONLY. The tests, the smoke check and the bench's CPU-baseline / reference legs
use it as the checker; the product package never imports it. See slx_oracle.cpp for the
reference file:line each routine follows.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libslx_oracle.so")
_lock = threading.Lock()
_lib = None

I64P = ctypes.POINTER(ctypes.c_int64)
I32P = ctypes.POINTER(ctypes.c_int32)
U16P = ctypes.POINTER(ctypes.c_uint16)
U8P = ctypes.POINTER(ctypes.c_uint8)
F32P = ctypes.POINTER(ctypes.c_float)
U64P = ctypes.POINTER(ctypes.c_uint64)
VP = ctypes.c_void_p


def build() -> str:
    """Compile the oracle with its Makefile (g++ -fopenmp) if it is missing or stale."""
    src = os.path.join(_HERE, "slx_oracle.cpp")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def _sig(lib):
    def f(name, res, *args):
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = list(args)

    i, i64, f32 = ctypes.c_int, ctypes.c_int64, ctypes.c_float
    f("slxo_set_threads", i, i)
    f("slxo_half_to_float", f32, ctypes.c_uint16)
    f("slxo_float_to_half", ctypes.c_uint16, f32)
    f("slxo_half_to_float_n", None, U16P, i64, F32P)
    f("slxo_float_to_half_n", None, F32P, i64, U16P)
    f("slxo_dequantize", i, i, U8P, i64, F32P, i64)
    f("slxo_byte_count", i64, i, i64)
    f("slxo_quantize_from_float", None, F32P, i64, i, I64P)
    f("slxo_dot_int128", None, I64P, I64P, i, I64P)
    f("slxo_matmul_long", None, I64P, i, i, I64P, i, i, I64P)
    f("slxo_matmul_half", None, I64P, i, i, U16P, i, i, i, I64P)
    f("slxo_matmul_float", None, I64P, i, i, F32P, i, i, i, I64P)
    f("slxo_fixed_exp", i64, i64, i)
    f("slxo_fixed_sigmoid", i64, i64, i)
    f("slxo_fixed_silu", i64, i64, i)
    f("slxo_fixed_softmax", None, I64P, i, i)
    f("slxo_isqrt64", i64, i64)
    f("slxo_isqrt128", i64, i64, i64)
    f("slxo_layernorm", None, I64P, i, i, I64P, I64P)
    f("slxo_rmsnorm", None, I64P, i, i, I64P)
    f("slxo_rmsnorm_per_head", None, I64P, i, i, i, I64P)
    f("slxo_rope_cache", None, i, i, f32, i, I64P, I64P)
    f("slxo_apply_rope", i, I64P, i, i, i, i, i, f32, i)
    f("slxo_attention", None, I64P, I64P, I64P, i, i, i, i, i, i, i, i, i, I64P)
    f("slxo_silu_gate", None, I64P, I64P, i64, i)
    f("slxo_ffn_long", None, I64P, i, i, I64P, I64P, I64P, i, i, i, I64P)
    f("slxo_ffn_half", None, I64P, i, i, U16P, U16P, U16P, i, i, i, I64P)
    f("slxo_mean_pool", None, I64P, i, i, I64P)
    f("slxo_to_float_l2", None, I64P, i, i, F32P)
    f("slxo_argmax_half", i, F32P, U16P, i64, i, i)
    f("slxo_gguf_open", VP, ctypes.c_char_p, ctypes.POINTER(i))
    f("slxo_gguf_close", None, VP)
    f("slxo_gguf_info", i, VP, ctypes.POINTER(i))
    f("slxo_gguf_data_offset", i64, VP)
    f("slxo_gguf_arch", i, VP, ctypes.c_char_p, i)
    f("slxo_gguf_tensor_elements", i64, VP, ctypes.c_char_p)
    f("slxo_gguf_tensor_dtype", i, VP, ctypes.c_char_p)
    f("slxo_gguf_read_f32", i, VP, ctypes.c_char_p, F32P, i64)
    f("slxo_encoder_load", VP, ctypes.c_char_p, i, ctypes.POINTER(i))
    f("slxo_encoder_free", None, VP)
    f("slxo_encoder_info", i, VP, ctypes.POINTER(i))
    f("slxo_encoder_hidden", i, VP, I32P, i, i, I64P)
    f("slxo_encoder_forward", i, VP, I32P, i, i, I64P)
    f("slxo_causal_load", VP, ctypes.c_char_p, i, ctypes.POINTER(i))
    f("slxo_gemma_encoder_load", VP, ctypes.c_char_p, i, ctypes.POINTER(i))
    f("slxo_causal_free", None, VP)
    f("slxo_causal_info", i, VP, ctypes.POINTER(i))
    f("slxo_causal_hidden", i, VP, I32P, i, i, i, I64P)
    f("slxo_causal_forward_last", i, VP, I32P, i, I64P)
    f("slxo_causal_next_token", i, VP, I32P, i, I32P)
    f("slxo_causal_generate", i, VP, I32P, i, i, I32P, ctypes.POINTER(i))
    f("slxo_causal_next_token_lattice", i, VP, I32P, i, i, I32P)
    f("slxo_causal_generate_lattice", i, VP, I32P, i, i, i, I32P, ctypes.POINTER(i))
    f("slxo_gemma_encoder_forward", i, VP, I32P, i, i, I64P)
    f("slxo_quantize_dense", None, F32P, i64, f32, i64, I64P)
    f("slxo_distance_sq_l2_fast", ctypes.c_uint64, I64P, I64P, i)
    f("slxo_knn_l2", None, I64P, i64, i, I64P, i, i, i64, I64P, U64P)
    f("slxo_tree_build", VP, I64P, i64, i, i, ctypes.POINTER(i))
    f("slxo_tree_free", None, VP)
    f("slxo_tree_info", None, VP, I64P)
    f("slxo_tree_export", None, VP, I32P, I32P, I32P, I64P, I64P, I64P, I64P)
    f("slxo_slat_save", i64, VP, I64P, i, I32P, U8P, i64)
    f("slxo_slat_load", VP, U8P, i64, ctypes.POINTER(i), ctypes.POINTER(i64), ctypes.POINTER(i))
    f("slxo_slat_tree", VP, VP)
    f("slxo_slat_rows", None, VP, I64P, I32P)
    f("slxo_slat_free", None, VP)
    f("slxo_float_encoder_load", VP, ctypes.c_char_p, ctypes.POINTER(i))
    f("slxo_float_encoder_free", None, VP)
    f("slxo_float_encoder_forward", i, VP, I32P, i, F32P)


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            _lib = ctypes.CDLL(_SO)
            _sig(_lib)
    return _lib


class OracleError(RuntimeError):
    def __init__(self, status: int, what: str):
        super().__init__(f"{what}: oracle status {status}")
        self.status = status


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int64)


def set_threads(n: int) -> int:
    return lib().slxo_set_threads(int(n))


def half_to_float(h) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().slxo_half_to_float_n(_p(h, U16P), h.size, _p(out, F32P))
    return out


def float_to_half(f) -> np.ndarray:
    f = np.ascontiguousarray(f, dtype=np.float32)
    out = np.empty(f.shape, np.uint16)
    lib().slxo_float_to_half_n(_p(f, F32P), f.size, _p(out, U16P))
    return out


def dequantize(dtype: int, raw: bytes | np.ndarray, n: int) -> np.ndarray:
    buf = np.frombuffer(bytes(raw), dtype=np.uint8).copy() if not isinstance(raw, np.ndarray) else np.ascontiguousarray(raw, np.uint8)
    out = np.zeros(n, np.float32)
    st = lib().slxo_dequantize(int(dtype), _p(buf, U8P), buf.size, _p(out, F32P), int(n))
    if st:
        raise OracleError(st, "dequantize")
    return out


def quantize_from_float(x, bits: int = 30) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.int64)
    lib().slxo_quantize_from_float(_p(x, F32P), x.size, bits, _p(out, I64P))
    return out


def dot_int128(a, b) -> int:
    a, b = _i64(a), _i64(b)
    r = np.zeros(2, np.int64)
    lib().slxo_dot_int128(_p(a, I64P), _p(b, I64P), a.size, _p(r, I64P))
    return (int(r[1]) << 64) + (int(r[0]) & ((1 << 64) - 1))


def matmul_long(a, rows: int, cols: int, w, cols_b: int, shift: int = 0) -> np.ndarray:
    a, w = _i64(a), _i64(w)
    c = np.empty(rows * cols_b, np.int64)
    lib().slxo_matmul_long(_p(a, I64P), rows, cols, _p(w, I64P), cols_b, shift, _p(c, I64P))
    return c


def matmul_half(a, rows: int, cols: int, w_half, cols_b: int, scale_bits: int = 30, shift: int = 30) -> np.ndarray:
    a = _i64(a)
    w = np.ascontiguousarray(w_half, dtype=np.uint16)
    c = np.empty(rows * cols_b, np.int64)
    lib().slxo_matmul_half(_p(a, I64P), rows, cols, _p(w, U16P), cols_b, scale_bits, shift, _p(c, I64P))
    return c


def matmul_float(a, rows: int, cols: int, w, cols_b: int, scale_bits: int = 30, shift: int = 30) -> np.ndarray:
    a = _i64(a)
    w = np.ascontiguousarray(w, dtype=np.float32)
    c = np.empty(rows * cols_b, np.int64)
    lib().slxo_matmul_float(_p(a, I64P), rows, cols, _p(w, F32P), cols_b, scale_bits, shift, _p(c, I64P))
    return c


def fixed_exp(x: int, frac: int = 30) -> int:
    return lib().slxo_fixed_exp(int(x), frac)


def fixed_sigmoid(x: int, frac: int = 30) -> int:
    return lib().slxo_fixed_sigmoid(int(x), frac)


def fixed_silu(x: int, frac: int = 30) -> int:
    return lib().slxo_fixed_silu(int(x), frac)


def fixed_softmax(scores, frac: int = 30) -> np.ndarray:
    s = _i64(scores).copy()
    lib().slxo_fixed_softmax(_p(s, I64P), s.size, frac)
    return s


def isqrt64(v: int) -> int:
    return lib().slxo_isqrt64(int(v))


def isqrt128(v: int) -> int:
    lo = v & ((1 << 64) - 1)
    hi = (v >> 64) & ((1 << 64) - 1)
    to_s = lambda u: u - (1 << 64) if u >= (1 << 63) else u
    return lib().slxo_isqrt128(to_s(lo), to_s(hi))


def layernorm(x, seq: int, embd: int, w, b) -> np.ndarray:
    x = _i64(x).copy()
    w, b = _i64(w), _i64(b)
    lib().slxo_layernorm(_p(x, I64P), seq, embd, _p(w, I64P), _p(b, I64P))
    return x


def rmsnorm(x, seq: int, embd: int, w) -> np.ndarray:
    x = _i64(x).copy()
    w = _i64(w)
    lib().slxo_rmsnorm(_p(x, I64P), seq, embd, _p(w, I64P))
    return x


def rmsnorm_per_head(x, seq: int, nh: int, hd: int, w) -> np.ndarray:
    x = _i64(x).copy()
    w = _i64(w)
    lib().slxo_rmsnorm_per_head(_p(x, I64P), seq, nh, hd, _p(w, I64P))
    return x


def rope_cache(max_seq: int, head_dim: int, base: float, frac: int = 30):
    c = np.empty(max_seq * (head_dim // 2), np.int64)
    s = np.empty_like(c)
    lib().slxo_rope_cache(max_seq, head_dim, base, frac, _p(c, I64P), _p(s, I64P))
    return c, s


def apply_rope(x, seq: int, embd: int, nh: int, max_seq: int, head_dim: int, base: float, frac: int = 30) -> np.ndarray:
    x = _i64(x).copy()
    st = lib().slxo_apply_rope(_p(x, I64P), seq, embd, nh, max_seq, head_dim, base, frac)
    if st:
        raise OracleError(st, "apply_rope")
    return x


def attention(q, k, v, seq: int, q_embd: int, kv_dim: int, nh: int, nkv: int, scale_exp: int = -30,
              frac: int = 30, mode: int = 0, window: int = 0) -> np.ndarray:
    """mode 0: (Grouped)MultiHeadAttention, 1: causal (leaky -0.5 mask), 2: sliding window."""
    q, k, v = _i64(q), _i64(k), _i64(v)
    out = np.empty(seq * q_embd, np.int64)
    lib().slxo_attention(_p(q, I64P), _p(k, I64P), _p(v, I64P), seq, q_embd, kv_dim, nh, nkv, scale_exp, frac, mode,
                         window, _p(out, I64P))
    return out


def silu_gate(gate, up, frac: int = 30) -> np.ndarray:
    g = _i64(gate)
    u = _i64(up).copy()
    lib().slxo_silu_gate(_p(g, I64P), _p(u, I64P), g.size, frac)
    return u


def ffn_long(x, seq, embd, wg, wu, wd, nff, shift=30, frac=30) -> np.ndarray:
    x, wg, wu, wd = _i64(x), _i64(wg), _i64(wu), _i64(wd)
    out = np.empty(seq * embd, np.int64)
    lib().slxo_ffn_long(_p(x, I64P), seq, embd, _p(wg, I64P), _p(wu, I64P), _p(wd, I64P), nff, shift, frac, _p(out, I64P))
    return out


def mean_pool(x, T: int, d: int) -> np.ndarray:
    x = _i64(x)
    out = np.empty(d, np.int64)
    lib().slxo_mean_pool(_p(x, I64P), T, d, _p(out, I64P))
    return out


def to_float_l2(v, scale_bits: int = 30) -> np.ndarray:
    v = _i64(v)
    out = np.empty(v.size, np.float32)
    lib().slxo_to_float_l2(_p(v, I64P), v.size, scale_bits, _p(out, F32P))
    return out


def argmax_half(h, E_half, vocab: int, dims: int) -> int:
    h = np.ascontiguousarray(h, np.float32)
    E = np.ascontiguousarray(E_half, np.uint16)
    return lib().slxo_argmax_half(_p(h, F32P), _p(E, U16P), E.size, vocab, dims)


def quantize_dense(e, zero_threshold: float = 0.001, global_scale: int = 1_000_000_000) -> np.ndarray:
    """EmbeddingAdapter.QuantizeDense / Quantize (no sparsity budget) of float embeddings, any shape."""
    e = np.ascontiguousarray(e, dtype=np.float32)
    out = np.empty(e.shape, np.int64)
    lib().slxo_quantize_dense(_p(e, F32P), e.size, zero_threshold, int(global_scale), _p(out, I64P))
    return out


def distance_sq_l2_fast(a, b) -> int:
    a, b = _i64(a), _i64(b)
    return int(lib().slxo_distance_sq_l2_fast(_p(a, I64P), _p(b, I64P), a.size))


def knn_l2(db, queries, k: int, id_base: int = 0):
    """Exact k nearest rows of db ([n, dim] int64) for each query row, ascending (distance, id).
    Returns (ids [nq, k] int64, dist [nq, k] uint64); missing entries (k > n) are -1 / UINT64_MAX."""
    db, q = _i64(db), _i64(queries)
    n, dim = db.shape
    nq = q.shape[0]
    ids = np.empty((nq, k), np.int64)
    dist = np.empty((nq, k), np.uint64)
    lib().slxo_knn_l2(_p(db, I64P), n, dim, _p(q, I64P), nq, k, id_base, _p(ids, I64P), _p(dist, U64P))
    return ids, dist


def merge_topk(ids, dist):
    """Merge per-shard answers [parts][nq][k] (ascending, id -1 = empty) into [nq][k] by
    (distance, id); the k-way merge a sharded database needs after gathering its shards' answers."""
    ids = np.asarray(ids, np.int64)
    dist = np.asarray(dist, np.uint64)
    parts, nq, k = ids.shape
    out_i = np.full((nq, k), -1, np.int64)
    out_d = np.full((nq, k), np.iinfo(np.uint64).max, np.uint64)
    for q in range(nq):
        cand = sorted((int(dist[p, q, j]), int(ids[p, q, j])) for p in range(parts) for j in range(k) if ids[p, q, j] >= 0)
        for j, (d, i) in enumerate(cand[:k]):
            out_i[q, j], out_d[q, j] = i, d
    return out_i, out_d


class Gguf:
    """GgufReader restatement (GgufReader.cs:54-130) over a file."""

    def __init__(self, path: str):
        st = ctypes.c_int(0)
        self._h = lib().slxo_gguf_open(path.encode(), ctypes.byref(st))
        if not self._h:
            raise OracleError(st.value, f"open {path}")

    def close(self):
        if self._h:
            lib().slxo_gguf_close(self._h)
            self._h = None

    __del__ = close

    def info(self) -> dict:
        v = (ctypes.c_int * 11)()
        lib().slxo_gguf_info(self._h, v)
        keys = ["version", "embd", "ctx", "heads", "layers", "ff", "n_tokens", "bos", "eos", "unk", "n_tensors"]
        d = dict(zip(keys, list(v)))
        buf = ctypes.create_string_buffer(256)
        lib().slxo_gguf_arch(self._h, buf, 256)
        d["arch"] = buf.value.decode()
        d["data_offset"] = lib().slxo_gguf_data_offset(self._h)
        return d

    def elements(self, name: str) -> int:
        return lib().slxo_gguf_tensor_elements(self._h, name.encode())

    def read_f32(self, name: str) -> np.ndarray:
        n = self.elements(name)
        if n < 0:
            raise OracleError(3, f"tensor {name}")
        out = np.zeros(n, np.float32)
        st = lib().slxo_gguf_read_f32(self._h, name.encode(), _p(out, F32P), n)
        if st:
            raise OracleError(st, f"read {name}")
        return out


class Encoder:
    """IntegerTransformerSource (nomic-bert / bert) restatement."""

    def __init__(self, path: str, scale_bits: int = 30):
        st = ctypes.c_int(0)
        self._h = lib().slxo_encoder_load(path.encode(), scale_bits, ctypes.byref(st))
        if not self._h:
            raise OracleError(st.value, f"load {path}")
        v = (ctypes.c_int * 6)()
        lib().slxo_encoder_info(self._h, v)
        self.embd, self.heads, self.layers, self.ff, self.unk, self.vocab = list(v)

    def close(self):
        if getattr(self, "_h", None):
            lib().slxo_encoder_free(self._h)
            self._h = None

    __del__ = close

    def hidden(self, ids, n_layers: int = -1) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        x = np.empty(ids.size * self.embd, np.int64)
        st = lib().slxo_encoder_hidden(self._h, _p(ids, I32P), ids.size, n_layers, _p(x, I64P))
        if st:
            raise OracleError(st, "encoder hidden")
        return x.reshape(ids.size, self.embd)

    def forward(self, ids) -> np.ndarray:
        """ids [B, T] -> pooled Q30 [B, embd]."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.empty((B, self.embd), np.int64)
        st = lib().slxo_encoder_forward(self._h, _p(ids, I32P), B, T, _p(out, I64P))
        if st:
            raise OracleError(st, "encoder forward")
        return out


class Causal:
    """IntegerCausalSource (Gemma causal LM) restatement; gemma_encoder=True gives IntegerGemmaSource."""

    def __init__(self, path: str, scale_bits: int = 30, gemma_encoder: bool = False):
        st = ctypes.c_int(0)
        loader = lib().slxo_gemma_encoder_load if gemma_encoder else lib().slxo_causal_load
        self._h = loader(path.encode(), scale_bits, ctypes.byref(st))
        if not self._h:
            raise OracleError(st.value, f"load {path}")
        v = (ctypes.c_int * 12)()
        lib().slxo_causal_info(self._h, v)
        (self.embd, self.heads, self.kv_heads, self.head_dim, self.ff, self.layers, self.vocab, self.sliding,
         self.eos, self.unk, self.q_dim, self.kv_dim) = list(v)

    def close(self):
        if getattr(self, "_h", None):
            lib().slxo_causal_free(self._h)
            self._h = None

    __del__ = close

    def hidden(self, ids, n_layers: int = -1, final_norm: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        x = np.empty(ids.size * self.embd, np.int64)
        st = lib().slxo_causal_hidden(self._h, _p(ids, I32P), ids.size, n_layers, int(final_norm), _p(x, I64P))
        if st:
            raise OracleError(st, "causal hidden")
        return x.reshape(ids.size, self.embd)

    def forward_last(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(self.embd, np.int64)
        st = lib().slxo_causal_forward_last(self._h, _p(ids, I32P), ids.size, _p(out, I64P))
        if st:
            raise OracleError(st, "forward_last")
        return out

    def next_token(self, ids) -> int:
        ids = np.ascontiguousarray(ids, np.int32)
        nx = ctypes.c_int32(0)
        st = lib().slxo_causal_next_token(self._h, _p(ids, I32P), ids.size, ctypes.byref(nx))
        if st:
            raise OracleError(st, "next_token")
        return nx.value

    def generate(self, ids, max_new: int) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(max(max_new, 1), np.int32)
        n = ctypes.c_int(0)
        st = lib().slxo_causal_generate(self._h, _p(ids, I32P), ids.size, max_new, _p(out, I32P), ctypes.byref(n))
        if st:
            raise OracleError(st, "generate")
        return out[: n.value].copy()

    def next_token_lattice(self, ids, k: int = 64) -> int:
        """PredictNextToken with the VocabLattice (k nearest candidates, best sequential fp32 dot)."""
        ids = np.ascontiguousarray(ids, np.int32)
        nx = ctypes.c_int32(0)
        st = lib().slxo_causal_next_token_lattice(self._h, _p(ids, I32P), ids.size, k, ctypes.byref(nx))
        if st:
            raise OracleError(st, "next_token_lattice")
        return nx.value

    def generate_lattice(self, ids, max_new: int, k: int = 64) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.empty(max(max_new, 1), np.int32)
        n = ctypes.c_int(0)
        st = lib().slxo_causal_generate_lattice(self._h, _p(ids, I32P), ids.size, max_new, k, _p(out, I32P),
                                                 ctypes.byref(n))
        if st:
            raise OracleError(st, "generate_lattice")
        return out[: n.value].copy()

    def encode_pooled(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.empty((B, self.embd), np.int64)
        st = lib().slxo_gemma_encoder_forward(self._h, _p(ids, I32P), B, T, _p(out, I64P))
        if st:
            raise OracleError(st, "gemma encode")
        return out


# ---- KD-tree lattice and SLAT ---------------------------------------------------------------------

TREE_INFO_KEYS = ("nodes", "branches", "leaves", "occupants", "max_depth")


def _tree_dict(h, n_rows: int) -> dict:
    info = np.zeros(5, np.int64)
    lib().slxo_tree_info(h, _p(info, I64P))
    nn = int(info[0])
    kind, mask, dim = (np.zeros(max(nn, 1), np.int32) for _ in range(3))
    val, start, count = (np.zeros(max(nn, 1), np.int64) for _ in range(3))
    perm = np.zeros(max(n_rows, 1), np.int64)
    lib().slxo_tree_export(h, _p(kind, I32P), _p(mask, I32P), _p(dim, I32P), _p(val, I64P), _p(start, I64P),
                           _p(count, I64P), _p(perm, I64P))
    out = dict(zip(TREE_INFO_KEYS, (int(x) for x in info)))
    out.update(kind=kind[:nn], mask=mask[:nn], dim=dim[:nn], val=val[:nn], start=start[:nn], count=count[:nn],
               perm=perm[:n_rows])
    return out


def tree_build(rows, leaf_threshold: int = 16) -> dict:
    """EmbeddingLatticeBuilder.Build over dense quantized rows [n, dim] (row i is occupant i).
    Returns the tree flattened in pre-order (kind 0 leaf / 1 branch, child mask, split dimension and
    value, leaf start and count into `perm`, the row ids in leaf order) and its statistics."""
    rows = np.ascontiguousarray(np.atleast_2d(rows), np.int64)
    n, dim = rows.shape
    st = ctypes.c_int(0)
    h = lib().slxo_tree_build(_p(rows, I64P), n, dim, leaf_threshold, ctypes.byref(st))
    if not h:
        raise OracleError(st.value, "tree_build")
    try:
        return _tree_dict(h, n)
    finally:
        lib().slxo_tree_free(h)


def slat_save(rows, payload, leaf_threshold: int = 16) -> bytes:
    """SparseLatticeSerializer.Save (Int32PayloadSerializer) of the lattice built over `rows`."""
    rows = np.ascontiguousarray(np.atleast_2d(rows), np.int64)
    n, dim = rows.shape
    payload = np.ascontiguousarray(payload, np.int32)
    st = ctypes.c_int(0)
    h = lib().slxo_tree_build(_p(rows, I64P), n, dim, leaf_threshold, ctypes.byref(st))
    if not h:
        raise OracleError(st.value, "tree_build")
    try:
        size = lib().slxo_slat_save(h, _p(rows, I64P), dim, _p(payload, I32P), None, 0)
        buf = np.zeros(size, np.uint8)
        lib().slxo_slat_save(h, _p(rows, I64P), dim, _p(payload, I32P), _p(buf, U8P), size)
        return buf.tobytes()
    finally:
        lib().slxo_tree_free(h)


def slat_load(data: bytes) -> dict:
    """SparseLatticeSerializer.Load (Int32PayloadSerializer): dense rows [n, dim] in file order,
    payloads, and the tree as tree_build returns it (perm indexes the rows in file order)."""
    buf = np.frombuffer(bytes(data), np.uint8).copy()
    st, n, dim = ctypes.c_int(0), ctypes.c_int64(0), ctypes.c_int(0)
    h = lib().slxo_slat_load(_p(buf, U8P) if buf.size else None, buf.size, ctypes.byref(st), ctypes.byref(n),
                             ctypes.byref(dim))
    if not h:
        raise OracleError(st.value, "slat_load")
    try:
        rows = np.zeros((n.value, dim.value), np.int64)
        payload = np.zeros(n.value, np.int32)
        lib().slxo_slat_rows(h, _p(rows, I64P), _p(payload, I32P))
        out = _tree_dict(lib().slxo_slat_tree(h), n.value)
        out.update(rows=rows, payload=payload)
        return out
    finally:
        lib().slxo_slat_free(h)


class FloatEncoder:
    """TransformerEmbeddingSource (Gguf/TransformerEmbeddingSource.cs): the fp32 twin of the encoder."""

    def __init__(self, path: str):
        st = ctypes.c_int(0)
        self._h = lib().slxo_float_encoder_load(path.encode(), ctypes.byref(st))
        if not self._h:
            raise OracleError(st.value, f"float encoder load {path}")
        g = Gguf(path)
        try:
            self.embd = g.info()["embd"]
        finally:
            g.close()

    def close(self):
        if self._h:
            lib().slxo_float_encoder_free(self._h)
            self._h = None

    __del__ = close

    def forward(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        out = np.zeros(self.embd, np.float32)
        st = lib().slxo_float_encoder_forward(self._h, _p(ids, I32P), ids.size, _p(out, F32P))
        if st:
            raise OracleError(st, "float encoder forward")
        return out
