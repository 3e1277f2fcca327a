"""spatialdb_b200 -- SparseLattice's quantized integer transformer forward path on B200 (sm_100a).

Host-side mirror of the reference's model sources over the libslx C ABI (include/slx.h):

* IntegerTransformerSource  (SparseLattice/Gguf/IntegerTransformerSource*.cs) -- nomic-bert / bert
  encoder; forward(ids) -> pooled Q30 long, forward_float(ids) -> L2-normalised float.
* IntegerGemmaSource        (SparseLattice/Gguf/IntegerGemmaSource*.cs) -- Gemma encoder.
* IntegerCausalSource       (SparseLattice/Gguf/IntegerCausalSource*.cs) -- Gemma causal LM;
  forward_causal, next_token, generate (greedy, full re-forward per token).
* dequantize / read_tensor_f32  (SparseLattice/Gguf/GgufDequantizer.cs, GgufReader.cs).
* matmul_q30                (SparseLattice/Math/IntegerMatMul.cs) with GGUF-packed weights.

Tokenizers stay with the caller (the C# host keeps them); these entry points take token ids.
All work runs in the CUDA library; nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes
import weakref

import numpy as np

from . import _lib
from ._lib import I32P, I64P, F32P, U8P, U64P, VP

(SLX_OK, SLX_EINVAL, SLX_EFORMAT, SLX_ENOTFOUND, SLX_EUNSUPPORTED, SLX_EEOF, SLX_ERANGE, SLX_EOOM, SLX_ECUDA, SLX_ETIMEOUT,
 SLX_ESCRATCH) = range(11)
OPT_WAIT_LIMIT_CYCLES, OPT_TEST_STALL_MMA = 1, 2
MODEL_ENCODER, MODEL_CAUSAL, MODEL_GEMMA_ENCODER, MODEL_FLOAT_ENCODER = 0, 1, 2, 3


class SlxError(RuntimeError):
    """Raised for a non-zero slx_status; `status` holds the code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class InvalidDataError(SlxError):      # InvalidDataException
    pass


class NotSupportedError(SlxError):     # NotSupportedException
    pass


class NotFoundError(SlxError):         # FileNotFoundException / KeyNotFoundException
    pass


class EndOfStreamError(SlxError):      # EndOfStreamException
    pass


class IndexOutOfRangeError(SlxError):  # IndexOutOfRangeException
    pass


_EXC = {SLX_EFORMAT: InvalidDataError, SLX_EUNSUPPORTED: NotSupportedError, SLX_ENOTFOUND: NotFoundError,
        SLX_EEOF: EndOfStreamError, SLX_ERANGE: IndexOutOfRangeError}


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class Context:
    """One CUDA device and stream (slx_init)."""

    _default: "Context | None" = None

    def __init__(self, device: int = 0):
        self._lib = _lib.lib()
        h = VP()
        st = self._lib.slx_init(device, ctypes.byref(h))
        if st:
            raise SlxError(st, f"slx_init(device={device}) failed")
        self._h = h
        self.device = device
        self._children = weakref.WeakSet()

    @classmethod
    def default(cls) -> "Context":
        if cls._default is None:
            cls._default = Context(0)
        return cls._default

    def check(self, st: int):
        if st:
            msg = self._lib.slx_last_error(self._h).decode(errors="replace")
            raise _EXC.get(st, SlxError)(st, msg)

    def status(self, stream: int = 0):
        """slx_ctx_status: wait for `stream` (cudaStream_t as int, 0 = the context's stream), raise the
        device-side error recorded by work queued through the _device entry points, and clear it."""
        self.check(self._lib.slx_ctx_status(self._h, VP(stream or None)))

    def set_option(self, option: int, value: int):
        """slx_ctx_set_option (OPT_WAIT_LIMIT_CYCLES, OPT_TEST_STALL_MMA)."""
        self.check(self._lib.slx_ctx_set_option(self._h, option, int(value)))

    def _adopt(self, child):
        """Registers a handle created on this context (model, weight, lattice): closing the context
        closes them first, so a garbage collection that finalizes the context before them (objects in
        a reference cycle are finalized in no fixed order) never frees a handle after its context."""
        self._children.add(child)

    def close(self):
        if getattr(self, "_h", None):
            for c in list(getattr(self, "_children", ())):
                try:
                    c.close()
                except Exception:
                    pass
            self._lib.slx_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dequantize(dtype: int, raw, n: int, ctx: Context | None = None) -> np.ndarray:
    """GgufDequantizer for one raw tensor (n output floats)."""
    ctx = ctx or Context.default()
    buf = np.frombuffer(bytes(raw), np.uint8).copy() if not isinstance(raw, np.ndarray) else np.ascontiguousarray(raw, np.uint8)
    out = np.zeros(n, np.float32)
    ctx.check(ctx._lib.slx_dequantize(ctx._h, int(dtype), _p(buf, U8P), buf.size, _p(out, F32P), int(n)))
    return out


def read_tensor_f32(path: str, name: str, n: int, ctx: Context | None = None) -> np.ndarray:
    """GgufReader.ReadTensorF32 (n must be the tensor's element count)."""
    ctx = ctx or Context.default()
    out = np.zeros(n, np.float32)
    ctx.check(ctx._lib.slx_gguf_read_f32(ctx._h, path.encode(), name.encode(), _p(out, F32P), int(n)))
    return out


def matmul_q30(a: np.ndarray, dtype: int, w_raw, N: int, half_composite: bool = False, scale_bits: int = 30,
               shift: int = 30, ctx: Context | None = None) -> np.ndarray:
    """IntegerMatMul.MatMul of int64 a[M][K] with a GGUF weight of N rows of K (flat block order)."""
    ctx = ctx or Context.default()
    a = np.ascontiguousarray(np.atleast_2d(a), np.int64)
    M, K = a.shape
    w = np.frombuffer(bytes(w_raw), np.uint8).copy() if not isinstance(w_raw, np.ndarray) else np.ascontiguousarray(w_raw, np.uint8)
    c = np.empty((M, N), np.int64)
    ctx.check(ctx._lib.slx_matmul_q30(ctx._h, _p(a, I64P), M, K, int(dtype), _p(w, U8P), w.size, N, int(half_composite),
                                      scale_bits, shift, _p(c, I64P)))
    return c


class PreparedWeight:
    """A GGUF weight in device memory prepared once for repeated IntegerMatMul products
    (slx_weight_prepare): the tensor-core digit planes of its Q30 composites. `d_w` is a device
    pointer to the raw blocks, which must stay alive while this object does."""

    def __init__(self, d_w: int, w_bytes: int, dtype: int, N: int, K: int, half_composite: bool = False,
                 scale_bits: int = 30, ctx: Context | None = None):
        self.ctx = ctx or Context.default()
        h = VP()
        self.ctx.check(self.ctx._lib.slx_weight_prepare(self.ctx._h, VP(d_w), int(w_bytes), int(dtype), int(N), int(K),
                                                        int(half_composite), int(scale_bits), ctypes.byref(h)))
        self._h = h
        self.ctx._adopt(self)
        info = (ctypes.c_int32 * 4)()
        self.ctx._lib.slx_weight_info(h, info, 4)
        self.N, self.K, self.tensor_cores, self.digits = list(info)

    def matmul_device(self, d_a: int, M: int, d_c: int, shift: int = 30, stream: int = 0):
        """Queue c[M][N] = MatMul(a[M][K], w) >> shift on device buffers (raw pointers)."""
        self.ctx.check(self.ctx._lib.slx_matmul_q30_prepared(self._h, VP(d_a), int(M), int(shift), VP(d_c),
                                                             VP(stream or None)))

    def close(self):
        if getattr(self, "_h", None):
            self.ctx._lib.slx_weight_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def attention(q, k, v, seq: int, n_heads: int, n_kv_heads: int, scale_exp: int = -30, mode: int = 0,
              window: int = 0, ctx: Context | None = None) -> np.ndarray:
    """IntegerAttention on Q30 arrays of one sequence: mode 0 (grouped) multi-head, 1 causal, 2 sliding window."""
    ctx = ctx or Context.default()
    q = np.ascontiguousarray(q, np.int64).reshape(seq, -1)
    k = np.ascontiguousarray(k, np.int64).reshape(seq, -1)
    v = np.ascontiguousarray(v, np.int64).reshape(seq, -1)
    out = np.empty_like(q)
    ctx.check(ctx._lib.slx_attention(ctx._h, _p(q, I64P), _p(k, I64P), _p(v, I64P), seq, q.shape[1], k.shape[1], n_heads,
                                     n_kv_heads, scale_exp, mode, window, _p(out, I64P)))
    return out


class _Model:
    kind = -1

    def __init__(self, path: str, scale_bits: int = 30, ctx: Context | None = None):
        self.ctx = ctx or Context.default()
        h = VP()
        self.ctx.check(self.ctx._lib.slx_model_load_gguf(self.ctx._h, path.encode(), self.kind, scale_bits, ctypes.byref(h)))
        self._h = h
        self.ctx._adopt(self)
        info = np.zeros(12, np.int32)
        self.ctx._lib.slx_model_info(self._h, _p(info, I32P), 12)
        (_, self.embd, self.heads, self.kv_heads, self.head_dim, self.ff, self.layers, self.vocab, self.eos, self.unk,
         self.q_dim, self.kv_dim) = [int(v) for v in info]
        self.scale_bits = scale_bits
        self.path = path

    @classmethod
    def load(cls, path: str, scale_bits: int = 30, ctx: Context | None = None):
        return cls(path, scale_bits, ctx)

    @property
    def dimensions(self) -> int:
        return self.embd

    def close(self):
        if getattr(self, "_h", None):
            self.ctx._lib.slx_model_free(self._h)
            self._h = None

    def dispose(self):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def trace_hidden(self, ids, n_layers: int = -1, final_norm: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        x = np.empty((ids.size, self.embd), np.int64)
        self.ctx.check(self.ctx._lib.slx_trace_hidden(self._h, _p(ids, I32P), ids.size, n_layers, int(final_norm), _p(x, I64P)))
        return x


class _Encoder(_Model):
    def forward(self, ids) -> np.ndarray:
        """Forward on token ids [B, T] (or [T]) -> pooled Q30 long [B, embd]."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.empty((B, self.embd), np.int64)
        self.ctx.check(self.ctx._lib.slx_encode(self._h, _p(ids, I32P), B, T, _p(out, I64P), None))
        return out

    def forward_float(self, ids) -> np.ndarray:
        """ForwardFloat: pooled vectors dequantized and L2-normalised (float32)."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.empty((B, self.embd), np.int64)
        l2 = np.empty((B, self.embd), np.float32)
        self.ctx.check(self.ctx._lib.slx_encode(self._h, _p(ids, I32P), B, T, _p(out, I64P), _p(l2, F32P)))
        return l2

    def embed_batch(self, batch_ids) -> np.ndarray:
        """EmbedBatchAsync on equal-length id sequences, as one device batch."""
        return self.forward_float(batch_ids)

    def encode_device(self, d_ids_ptr: int, B: int, T: int, d_pooled_ptr: int, stream: int = 0):
        """Queue a forward on device buffers (raw device pointers, cudaStream_t as int)."""
        self.ctx.check(self.ctx._lib.slx_encode_device(self._h, VP(d_ids_ptr), B, T, VP(d_pooled_ptr), VP(stream or None)))


class IntegerTransformerSource(_Encoder):
    """nomic-bert / bert integer encoder (IntegerTransformerSource)."""
    kind = MODEL_ENCODER


class IntegerGemmaSource(_Encoder):
    """Gemma integer encoder, non-causal GQA, mean pooled (IntegerGemmaSource)."""
    kind = MODEL_GEMMA_ENCODER


class TransformerEmbeddingSource(_Model):
    """nomic-bert / bert encoder in fp32 (TransformerEmbeddingSource, Gguf/TransformerEmbeddingSource.cs):
    the float twin of IntegerTransformerSource. Agrees with the reference to fp32 rounding (its SIMD
    dot order is machine-dependent), not bit for bit."""
    kind = MODEL_FLOAT_ENCODER

    def forward(self, ids) -> np.ndarray:
        """Forward / EmbedBatchAsync on token ids [B, T] (or [T]): L2-normalised float embeddings [B, embd]."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.empty((B, self.embd), np.float32)
        self.ctx.check(self.ctx._lib.slx_encode(self._h, _p(ids, I32P), B, T, None, _p(out, F32P)))
        return out


class IntegerCausalSource(_Model):
    """Gemma causal LM in Q30 integer arithmetic (IntegerCausalSource)."""
    kind = MODEL_CAUSAL

    def forward_causal(self, ids) -> np.ndarray:
        """ForwardCausal: last position's hidden state after the output norm (Q30 long [embd])."""
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        out = np.empty(self.embd, np.int64)
        self.ctx.check(self.ctx._lib.slx_causal_forward_last(self._h, _p(ids, I32P), ids.size, _p(out, I64P)))
        return out

    def forward_causal_float(self, ids) -> np.ndarray:
        """ForwardCausalFloat: (float)(v * 2^-scale_bits) of forward_causal."""
        v = self.forward_causal(ids)
        return (v.astype(np.float64) * 2.0 ** -self.scale_bits).astype(np.float32)

    def next_token(self, ids, use_lattice: bool = False, lattice_k: int = 64) -> np.ndarray:
        """Greedy next id for each of B sequences [B, T]: PredictNextToken (IntegerCausalSource.cs:149-157)
        with the ArgmaxBruteForce head, or with the VocabLattice head and `lattice_k` candidates."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.empty(B, np.int32)
        lib = self.ctx._lib
        if use_lattice:
            self.ctx.check(lib.slx_causal_next_token_lattice(self._h, _p(ids, I32P), B, T, int(lattice_k), _p(out, I32P)))
        else:
            self.ctx.check(lib.slx_causal_next_token(self._h, _p(ids, I32P), B, T, _p(out, I32P)))
        return out

    def generate(self, ids, max_new_tokens: int = 64, use_lattice: bool = False, lattice_k: int = 64) -> list[np.ndarray]:
        """Generate on token ids [B, T] (IntegerCausalSource.cs:86-108): greedy, full re-forward per
        token, stop at EOS; `use_lattice` scores only the `lattice_k` VocabLattice candidates."""
        ids = np.ascontiguousarray(np.atleast_2d(ids), np.int32)
        B, T = ids.shape
        out = np.zeros((B, max(max_new_tokens, 1)), np.int32)
        n = np.zeros(B, np.int32)
        lib = self.ctx._lib
        if use_lattice:
            rc = lib.slx_causal_generate_lattice(self._h, _p(ids, I32P), B, T, max_new_tokens, int(lattice_k),
                                                 _p(out, I32P), _p(n, I32P))
        else:
            rc = lib.slx_causal_generate(self._h, _p(ids, I32P), B, T, max_new_tokens, _p(out, I32P), _p(n, I32P))
        self.ctx.check(rc)
        return [out[b, : n[b]].copy() for b in range(B)]

    def vocab_lattice_query(self, hidden, k: int = 64, return_distances: bool = False):
        """VocabLattice.QueryTopK (Lattice/VocabLattice.cs:43-58) for float hidden states [B, embd]:
        ids [B, k] ascending by (distance, row), -1 past the vocabulary; with return_distances also
        their DistanceSquaredL2Fast values (uint64 [B, k], UINT64_MAX past the vocabulary)."""
        h = np.ascontiguousarray(np.atleast_2d(hidden), np.float32)
        B = h.shape[0]
        if h.shape[1] != self.embd:
            raise ValueError(f"hidden width {h.shape[1]} != embd {self.embd}")
        k = max(int(k), 0)
        out = np.full((B, k), -1, np.int32)
        dist = np.full((B, k), np.iinfo(np.uint64).max, np.uint64)
        if k > 0 and B > 0:
            self.ctx.check(self.ctx._lib.slx_vocab_lattice_query(self._h, _p(h, F32P), B, k, _p(out, I32P),
                                                                 _p(dist, U64P) if return_distances else None))
        return (out, dist) if return_distances else out


# ---- lattice k-NN search --------------------------------------------------------------------------

KNN_EXACT = 1  # query flag: scan every row exactly instead of bounding with the tensor cores


class QuantizationOptions:
    """QuantizationOptions (Math/EmbeddingAdapter.cs:4-11). The class defaults are the reference's
    (ZeroThreshold 0.01, GlobalScale long.MaxValue); VocabLattice uses (0.001, 1e9), which is
    VOCAB_LATTICE_OPTIONS and the default of EmbeddingLattice here. No sparsity budget."""

    def __init__(self, zero_threshold: float = 0.01, global_scale: int = (1 << 63) - 1):
        self.zero_threshold = float(zero_threshold)
        self.global_scale = int(global_scale)


VOCAB_LATTICE_OPTIONS = QuantizationOptions(0.001, 1_000_000_000)


class EmbeddingLattice:
    """Exact k-nearest-neighbour search over float embeddings on the device: the rows are quantized
    with EmbeddingAdapter.Quantize (options as above) and query_k_nearest_l2 returns
    EmbeddingLattice.QueryKNearestL2's answer (Lattice/EmbeddingLattice.cs:70-77): the k smallest
    DistanceSquaredL2Fast distances, ascending, equal distances by id. ids are id_base + row."""

    def __init__(self, vectors, options: QuantizationOptions = VOCAB_LATTICE_OPTIONS, id_base: int = 0,
                 ctx: Context | None = None):
        self._ctx = ctx or Context.default()
        self.options = options
        v = np.ascontiguousarray(vectors, np.float32)
        if v.ndim != 2:
            raise ValueError("vectors must be [n, dim]")
        h = VP()
        self._ctx.check(self._ctx._lib.slx_lattice_build(self._ctx._h, _p(v, F32P), v.shape[0], v.shape[1],
                                                         options.zero_threshold, options.global_scale, int(id_base),
                                                         ctypes.byref(h)))
        self._h = h
        self._ctx._adopt(self)
        self.n, self.dim, self.id_base = v.shape[0], v.shape[1], int(id_base)
        self.last_exact = 0

    @classmethod
    def from_device(cls, d_vectors_ptr: int, n: int, dim: int, options: QuantizationOptions = VOCAB_LATTICE_OPTIONS,
                    id_base: int = 0, stream: int = 0, ctx: Context | None = None) -> "EmbeddingLattice":
        self = cls.__new__(cls)
        self._ctx = ctx or Context.default()
        self.options = options
        h = VP()
        self._ctx.check(self._ctx._lib.slx_lattice_build_device(self._ctx._h, VP(d_vectors_ptr), int(n), int(dim),
                                                                options.zero_threshold, options.global_scale,
                                                                int(id_base), VP(stream), ctypes.byref(h)))
        self._h = h
        self._ctx._adopt(self)
        self.n, self.dim, self.id_base = int(n), int(dim), int(id_base)
        self.last_exact = 0
        return self

    def query_k_nearest_l2(self, queries, k: int, exact: bool = False):
        """(ids [nq, k] int64, distances [nq, k] uint64); -1 / UINT64_MAX past the database."""
        q = np.ascontiguousarray(np.atleast_2d(queries), np.float32)
        nq = q.shape[0]
        ids = np.empty((nq, k), np.int64)
        dist = np.empty((nq, k), np.uint64)
        ne = ctypes.c_int(0)
        self._ctx.check(self._ctx._lib.slx_lattice_query_knn_l2(self._h, _p(q, F32P), nq, int(k),
                                                                KNN_EXACT if exact else 0, _p(ids, I64P),
                                                                _p(dist, U64P), ctypes.byref(ne)))
        self.last_exact = ne.value
        return ids, dist

    def query_device(self, d_queries_ptr: int, nq: int, k: int, d_ids_ptr: int, d_dist_ptr: int, exact: bool = False,
                     stream: int = 0) -> int:
        """Device buffers: queries [nq, dim] float32, ids [nq, k] int64, dist [nq, k] uint64. Returns the
        number of queries answered by an exact scan."""
        ne = ctypes.c_int(0)
        self._ctx.check(self._ctx._lib.slx_lattice_query_knn_l2_device(
            self._h, VP(d_queries_ptr), int(nq), int(k), KNN_EXACT if exact else 0, VP(d_ids_ptr), VP(d_dist_ptr),
            ctypes.byref(ne), VP(stream)))
        self.last_exact = ne.value
        return ne.value

    # ---- KD tree (EmbeddingLatticeBuilder) and SLAT (SparseLatticeSerializer) --------------------

    TREE_INFO_KEYS = ("nodes", "branches", "leaves", "occupants", "max_depth")

    def freeze(self, leaf_threshold: int = 16) -> "EmbeddingLattice":
        """Builds the KD tree over the rows (EmbeddingLatticeBuilder.Build with LatticeOptions.LeafThreshold)."""
        self._ctx.check(self._ctx._lib.slx_lattice_build_tree(self._h, int(leaf_threshold)))
        return self

    def collect_stats(self) -> dict:
        """SparseTreeStats: nodes, branches, leaves, occupants, max_depth."""
        info = np.zeros(5, np.int64)
        self._ctx.check(self._ctx._lib.slx_lattice_tree_info(self._h, _p(info, I64P), 5))
        return dict(zip(self.TREE_INFO_KEYS, (int(x) for x in info)))

    def tree(self) -> dict:
        """The tree in pre-order: kind, mask, dim, val, start, count per node and perm (row of each
        leaf-order position), plus the statistics."""
        st = self.collect_stats()
        nn = st["nodes"]
        kind, mask, dim = (np.zeros(max(nn, 1), np.int32) for _ in range(3))
        val, start, count = (np.zeros(max(nn, 1), np.int64) for _ in range(3))
        perm = np.zeros(max(st["occupants"], 1), np.int32)
        self._ctx.check(self._ctx._lib.slx_lattice_tree_export(self._h, _p(kind, I32P), _p(mask, I32P), _p(dim, I32P),
                                                               _p(val, I64P), _p(start, I64P), _p(count, I64P),
                                                               _p(perm, I32P)))
        st.update(kind=kind[:nn], mask=mask[:nn], dim=dim[:nn], val=val[:nn], start=start[:nn], count=count[:nn],
                  perm=perm[: st["occupants"]])
        return st

    def save(self, path: str | None = None) -> bytes | None:
        """SparseLatticeSerializer.Save (Int32 payloads): to `path`, or returns the bytes."""
        lib = self._ctx._lib
        if path is not None:
            self._ctx.check(lib.slx_lattice_save_slat(self._h, str(path).encode()))
            return None
        size = ctypes.c_int64(0)
        self._ctx.check(lib.slx_lattice_save_slat_mem(self._h, None, 0, ctypes.byref(size)))
        buf = bytearray(max(size.value, 1))
        ptr = (ctypes.c_uint8 * len(buf)).from_buffer(buf)
        self._ctx.check(lib.slx_lattice_save_slat_mem(self._h, ctypes.cast(ptr, U8P), len(buf), ctypes.byref(size)))
        del ptr
        return bytes(buf) if size.value == len(buf) else bytes(buf[: size.value])

    @classmethod
    def load(cls, source, options: QuantizationOptions = VOCAB_LATTICE_OPTIONS,
             ctx: Context | None = None) -> "EmbeddingLattice":
        """SparseLatticeSerializer.Load (Int32 payloads) from a path or bytes: the occupants become the
        rows (file order) with their tree; query ids are the payloads."""
        self = cls.__new__(cls)
        self._ctx = ctx or Context.default()
        self.options = options
        h = VP()
        lib = self._ctx._lib
        if isinstance(source, (bytes, bytearray, memoryview)):
            buf = np.frombuffer(bytes(source), np.uint8).copy()
            self._ctx.check(lib.slx_lattice_load_slat_mem(self._ctx._h, _p(buf, U8P) if buf.size else None, buf.size,
                                                          options.zero_threshold, options.global_scale,
                                                          ctypes.byref(h)))
        else:
            self._ctx.check(lib.slx_lattice_load_slat(self._ctx._h, str(source).encode(), options.zero_threshold,
                                                      options.global_scale, ctypes.byref(h)))
        self._h = h
        self._ctx._adopt(self)
        info = np.zeros(3, np.int64)
        lib.slx_lattice_info(h, _p(info, I64P), 3)
        self.n, self.dim, self.id_base = int(info[0]), int(info[1]), int(info[2])
        self.last_exact = 0
        return self

    def close(self):
        if getattr(self, "_h", None):
            self._ctx._lib.slx_lattice_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def knn_merge_device(d_ids_ptr: int, d_dist_ptr: int, parts: int, nq: int, k: int, d_out_ids_ptr: int,
                     d_out_dist_ptr: int, stream: int = 0, ctx: Context | None = None):
    """k-way merge of per-shard answers [parts][nq][k] into [nq][k] on the device."""
    ctx = ctx or Context.default()
    ctx.check(ctx._lib.slx_knn_merge_device(ctx._h, VP(d_ids_ptr), VP(d_dist_ptr), int(parts), int(nq), int(k),
                                            VP(d_out_ids_ptr), VP(d_out_dist_ptr), VP(stream)))
