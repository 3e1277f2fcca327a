"""Seeded synthetic GGUF models for the tests and the bench.

The file layout follows the reference test suite's in-memory writer
(SparseLattice.Test/Gguf/GgufReaderTests.cs:19-100 for metadata, :514-575 for raw quantized
tensors): magic, version 3, counts, metadata, tensor table, 32-byte padding, tensor data. Tensor
data offsets are kept 32-byte aligned inside the data section.

Quantized blocks use the reference's element order (GgufDequantizer.cs:31-76): Q8_0 is an f16
scale and 32 int8; Q4_0 is an f16 scale and 16 bytes where element 2j is the low nibble of byte j
and element 2j+1 its high nibble, both offset by 8.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

# GgufTypes.cs:4-38
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, T_UINT64, T_INT64, T_FLOAT64 = range(13)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, BF16, MXFP4 = 10, 11, 12, 13, 14, 15, 30, 39
DTYPE_NAMES = {"f32": F32, "f16": F16, "q4_0": Q4_0, "q8_0": Q8_0, "bf16": BF16}

GGUF_MAGIC = 0x46554747


def block_bytes(dtype: int, elements: int) -> int:
    """GgufTensorInfo.ComputeByteCount (GgufTensorInfo.cs:27-48)."""
    e = elements
    return {
        F32: e * 4, F16: e * 2, BF16: e * 2, Q8_0: (e // 32) * 34, Q4_0: (e // 32) * 18,
        Q4_1: (e // 32) * 20, Q5_0: (e // 32) * 22, Q5_1: (e // 32) * 24,
        Q2_K: (e // 256) * 84, Q3_K: (e // 256) * 110, Q4_K: (e // 256) * 144, Q5_K: (e // 256) * 176,
        Q6_K: (e // 256) * 210, Q8_K: (e // 256) * 292, MXFP4: (e // 32) * 17,
    }.get(dtype, e * 4)


# ----------------------------------------------------------------------------------------------
# block encoders
# ----------------------------------------------------------------------------------------------
def pack_q8_0(d16: np.ndarray, q: np.ndarray) -> np.ndarray:
    """d16: [nb] float16 scales, q: [nb, 32] int8 -> [nb, 34] bytes."""
    nb = d16.shape[0]
    out = np.empty((nb, 34), np.uint8)
    out[:, 0:2] = d16.astype(np.float16).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = q.astype(np.int8).view(np.uint8)
    return out


def pack_q4_0(d16: np.ndarray, nib: np.ndarray) -> np.ndarray:
    """d16: [nb] float16, nib: [nb, 32] values 0..15 -> [nb, 18] bytes (element 2j = low nibble)."""
    nb = d16.shape[0]
    out = np.empty((nb, 18), np.uint8)
    out[:, 0:2] = d16.astype(np.float16).view(np.uint8).reshape(nb, 2)
    nib = nib.astype(np.uint8)
    out[:, 2:] = nib[:, 0::2] | (nib[:, 1::2] << 4)
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Absmax Q8_0 of float32 values (length a multiple of 32) -> packed bytes."""
    b = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(b).max(axis=1)
    d = amax / 127.0
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.rint(b * inv[:, None]), -127, 127).astype(np.int8)
    return pack_q8_0(d.astype(np.float16), q).reshape(-1)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """Q4_0 of float32 values: scale from the signed element of largest magnitude / -8."""
    b = x.astype(np.float32).reshape(-1, 32)
    idx = np.abs(b).argmax(axis=1)
    mx = b[np.arange(b.shape[0]), idx]
    d = mx / -8.0
    inv = np.where(d != 0, 1.0 / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.floor(b * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    return pack_q4_0(d.astype(np.float16), q).reshape(-1)


def random_q8_0(rng: np.random.Generator, elements: int) -> np.ndarray:
    """Microbench blocks: q uniform in [-127, 127], scale f16(|N(0, 0.02)| / 127)."""
    nb = elements // 32
    q = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02 / 127)).astype(np.float16)
    return pack_q8_0(d, q).reshape(-1)


def random_q4_0(rng: np.random.Generator, elements: int) -> np.ndarray:
    """Microbench blocks: nibbles uniform in [0, 15] (value - 8), scale f16(|N(0, 0.02)| / 127)."""
    nb = elements // 32
    raw = rng.integers(0, 256, size=(nb, 16), dtype=np.uint16).astype(np.uint8)
    d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02 / 127)).astype(np.float16)
    out = np.empty((nb, 18), np.uint8)
    out[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = raw
    return out.reshape(-1)


def encode(dtype: int, x: np.ndarray) -> np.ndarray:
    if dtype == F32:
        return np.ascontiguousarray(x, np.float32).view(np.uint8).reshape(-1)
    if dtype == F16:
        return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint8).reshape(-1)
    if dtype == Q8_0:
        return quantize_q8_0(x)
    if dtype == Q4_0:
        return quantize_q4_0(x)
    raise ValueError(f"no encoder for dtype {dtype}")


# ----------------------------------------------------------------------------------------------
# writer
# ----------------------------------------------------------------------------------------------
def _s(b: bytearray, s: str):
    e = s.encode("utf-8")
    b += struct.pack("<Q", len(e))
    b += e


def _value(b: bytearray, t: int, v):
    if t == T_UINT8: b += struct.pack("<B", v)
    elif t == T_INT8: b += struct.pack("<b", v)
    elif t == T_UINT16: b += struct.pack("<H", v)
    elif t == T_INT16: b += struct.pack("<h", v)
    elif t == T_UINT32: b += struct.pack("<I", v)
    elif t == T_INT32: b += struct.pack("<i", v)
    elif t == T_FLOAT32: b += struct.pack("<f", v)
    elif t == T_BOOL: b += struct.pack("<B", 1 if v else 0)
    elif t == T_STRING: _s(b, v)
    elif t == T_UINT64: b += struct.pack("<Q", v)
    elif t == T_INT64: b += struct.pack("<q", v)
    elif t == T_FLOAT64: b += struct.pack("<d", v)
    elif t == T_ARRAY:
        et, items = v
        b += struct.pack("<IQ", et, len(items))
        if et == T_STRING:
            for it in items:
                _s(b, it)
        else:
            for it in items:
                _value(b, et, it)
    else:
        raise ValueError(t)


@dataclass
class _Tensor:
    name: str
    shape: tuple
    dtype: int
    data: np.ndarray  # raw bytes


class GgufWriter:
    """Collects metadata and tensors, then writes one GGUF v3 file."""

    def __init__(self, version: int = 3):
        self.version = version
        self.meta: list[tuple[str, int, object]] = []
        self.tensors: list[_Tensor] = []

    def kv(self, key: str, t: int, v):
        self.meta.append((key, t, v))

    def tensor_raw(self, name: str, shape: tuple, dtype: int, raw: np.ndarray):
        raw = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
        n = int(np.prod(shape))
        assert raw.size == block_bytes(dtype, n), (name, raw.size, block_bytes(dtype, n))
        self.tensors.append(_Tensor(name, tuple(int(s) for s in shape), dtype, raw))

    def tensor(self, name: str, shape: tuple, dtype: int, values: np.ndarray):
        self.tensor_raw(name, shape, dtype, encode(dtype, np.asarray(values).reshape(-1)))

    def write(self, path: str):
        h = bytearray()
        h += struct.pack("<IIQQ", GGUF_MAGIC, self.version, len(self.tensors), len(self.meta))
        for k, t, v in self.meta:
            _s(h, k)
            h += struct.pack("<I", t)
            _value(h, t, v)
        off = 0
        offsets = []
        for t in self.tensors:
            off = (off + 31) & ~31
            offsets.append(off)
            off += t.data.size
        for t, o in zip(self.tensors, offsets):
            _s(h, t.name)
            h += struct.pack("<I", len(t.shape))
            for s in t.shape:
                h += struct.pack("<Q", s)
            h += struct.pack("<IQ", t.dtype, o)
        pad = ((len(h) + 31) & ~31) - len(h)
        h += b"\0" * pad
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            f.write(h)
            pos = 0
            for t, o in zip(self.tensors, offsets):
                if o > pos:
                    f.write(b"\0" * (o - pos))
                    pos = o
                f.write(t.data.tobytes())
                pos += t.data.size
        os.replace(tmp, path)
        return path


# ----------------------------------------------------------------------------------------------
# model generators
# ----------------------------------------------------------------------------------------------
@dataclass
class EncoderShape:
    layers: int = 12
    embd: int = 768
    heads: int = 12
    ff: int = 3072
    vocab: int = 30522
    ctx: int = 512


def write_encoder(path: str, shape: EncoderShape, wtype: int = Q8_0, seed: int = 0, arch: str = "nomic-bert",
                  rope_base: float = 10000.0, unk: int | None = None, ffn_norm_scale: float = 1.0,
                  embd_norm_scale: float = 1.0) -> str:
    """nomic-bert style encoder with N(0, 0.02) weights quantized to `wtype` (norms and token types F32).

    Tensor names and shapes are those IntegerTransformerSource.LoadFromReader reads
    (Gguf/IntegerTransformerSource.Loading.cs:72-151); GGUF ne0 is the inner (K) dimension.
    ffn_norm_scale multiplies the weight of the norm in front of the FFN (attn_output_norm): large
    values make the FFN's activations exceed the tensor-core digit range. embd_norm_scale does the
    same for the embeddings' norm, so the first block's projections and attention inputs exceed it.
    """
    rng = np.random.default_rng(seed)
    d, F, V = shape.embd, shape.ff, shape.vocab
    w = GgufWriter()
    w.kv("general.architecture", T_STRING, arch)
    w.kv("general.name", T_STRING, f"synthetic-{arch}")
    w.kv(f"{arch}.embedding_length", T_UINT32, d)
    w.kv(f"{arch}.context_length", T_UINT32, shape.ctx)
    w.kv(f"{arch}.attention.head_count", T_UINT32, shape.heads)
    w.kv(f"{arch}.block_count", T_UINT32, shape.layers)
    w.kv(f"{arch}.feed_forward_length", T_UINT32, F)
    w.kv(f"{arch}.rope.freq_base", T_FLOAT32, rope_base)
    w.kv("tokenizer.ggml.tokens", T_ARRAY, (T_STRING, [f"t{i}" for i in range(V)]))
    w.kv("tokenizer.ggml.bos_token_id", T_UINT32, min(101, V - 1))
    w.kv("tokenizer.ggml.eos_token_id", T_UINT32, min(102, V - 1))
    w.kv("tokenizer.ggml.unknown_token_id", T_UINT32, min(100, V - 1) if unk is None else unk)

    def normal(n):
        return rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)

    w.tensor("token_embd.weight", (d, V), wtype, normal(d * V))
    w.tensor("token_types.weight", (d, 2), F32, normal(2 * d))
    w.tensor("token_embd_norm.weight", (d,), F32, (1 + normal(d)) * np.float32(embd_norm_scale))
    w.tensor("token_embd_norm.bias", (d,), F32, normal(d))
    for i in range(shape.layers):
        p = f"blk.{i}"
        w.tensor(f"{p}.attn_qkv.weight", (d, 3 * d), wtype, normal(3 * d * d))
        w.tensor(f"{p}.attn_output.weight", (d, d), wtype, normal(d * d))
        w.tensor(f"{p}.attn_output_norm.weight", (d,), F32, (1 + normal(d)) * np.float32(ffn_norm_scale))
        w.tensor(f"{p}.attn_output_norm.bias", (d,), F32, normal(d))
        w.tensor(f"{p}.ffn_up.weight", (d, F), wtype, normal(d * F))
        w.tensor(f"{p}.ffn_gate.weight", (d, F), wtype, normal(d * F))
        w.tensor(f"{p}.ffn_down.weight", (F, d), wtype, normal(F * d))
        w.tensor(f"{p}.layer_output_norm.weight", (d,), F32, 1 + normal(d))
        w.tensor(f"{p}.layer_output_norm.bias", (d,), F32, normal(d))
    return w.write(path)


@dataclass
class CausalShape:
    layers: int = 18
    embd: int = 2048
    heads: int = 8
    kv_heads: int = 1
    head_dim: int = 256
    ff: int = 16384
    vocab: int = 256000
    ctx: int = 8192
    sliding_window: int = 0


def write_causal(path: str, shape: CausalShape, wtype: int = Q4_0, norm_type: int = F16, seed: int = 0,
                 arch: str = "gemma", qk_norm: bool = True, eos: int | None = None,
                 token_rows: np.ndarray | None = None) -> str:
    """Gemma-shaped causal LM: projections and token_embd as random `wtype` blocks, norms 1+N(0,0.02).
    `token_rows` (float [vocab, embd]) replaces the random token table, stored as F16.

    Tensor names follow IntegerCausalSource.LoadFromReader (IntegerCausalSource.Loading.cs:74-195).
    """
    rng = np.random.default_rng(seed)
    d, F, V, hd = shape.embd, shape.ff, shape.vocab, shape.head_dim
    qd, kvd = shape.heads * hd, shape.kv_heads * hd
    w = GgufWriter()
    w.kv("general.architecture", T_STRING, arch)
    w.kv("general.name", T_STRING, f"synthetic-{arch}")
    w.kv(f"{arch}.embedding_length", T_UINT32, d)
    w.kv(f"{arch}.context_length", T_UINT32, shape.ctx)
    w.kv(f"{arch}.attention.head_count", T_UINT32, shape.heads)
    w.kv(f"{arch}.attention.head_count_kv", T_UINT32, shape.kv_heads)
    w.kv(f"{arch}.attention.key_length", T_UINT32, hd)
    w.kv(f"{arch}.block_count", T_UINT32, shape.layers)
    w.kv(f"{arch}.feed_forward_length", T_UINT32, F)
    w.kv(f"{arch}.rope.freq_base", T_FLOAT32, 10000.0)
    w.kv(f"{arch}.attention.layer_norm_rms_epsilon", T_FLOAT32, 1e-6)
    if shape.sliding_window > 0:
        w.kv(f"{arch}.attention.sliding_window", T_UINT32, shape.sliding_window)
    w.kv("tokenizer.ggml.tokens", T_ARRAY, (T_STRING, [f"t{i}" for i in range(V)]))
    w.kv("tokenizer.ggml.bos_token_id", T_UINT32, 2 % V)
    w.kv("tokenizer.ggml.eos_token_id", T_UINT32, (1 if eos is None else eos) % V)
    w.kv("tokenizer.ggml.unknown_token_id", T_UINT32, 3 % V)

    def blocks(n):
        if wtype == Q4_0:
            return random_q4_0(rng, n)
        if wtype == Q8_0:
            return random_q8_0(rng, n)
        return encode(wtype, rng.standard_normal(n, dtype=np.float32) * np.float32(0.02))

    def norm(n):
        return 1 + rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)

    if token_rows is None:
        w.tensor_raw("token_embd.weight", (d, V), wtype, blocks(d * V))
    else:
        w.tensor("token_embd.weight", (d, V), F16, np.asarray(token_rows, np.float32).reshape(V * d))
    w.tensor("output_norm.weight", (d,), norm_type, norm(d))
    for i in range(shape.layers):
        p = f"blk.{i}"
        w.tensor(f"{p}.attn_norm.weight", (d,), norm_type, norm(d))
        w.tensor_raw(f"{p}.attn_q.weight", (d, qd), wtype, blocks(d * qd))
        w.tensor_raw(f"{p}.attn_k.weight", (d, kvd), wtype, blocks(d * kvd))
        w.tensor_raw(f"{p}.attn_v.weight", (d, kvd), wtype, blocks(d * kvd))
        if qk_norm:
            w.tensor(f"{p}.attn_q_norm.weight", (hd,), norm_type, norm(hd))
            w.tensor(f"{p}.attn_k_norm.weight", (hd,), norm_type, norm(hd))
        w.tensor_raw(f"{p}.attn_output.weight", (qd, d), wtype, blocks(qd * d))
        w.tensor(f"{p}.post_attention_norm.weight", (d,), norm_type, norm(d))
        w.tensor(f"{p}.ffn_norm.weight", (d,), norm_type, norm(d))
        w.tensor_raw(f"{p}.ffn_gate.weight", (d, F), wtype, blocks(d * F))
        w.tensor_raw(f"{p}.ffn_up.weight", (d, F), wtype, blocks(d * F))
        w.tensor_raw(f"{p}.ffn_down.weight", (F, d), wtype, blocks(F * d))
        w.tensor(f"{p}.post_ffw_norm.weight", (d,), norm_type, norm(d))
    return w.write(path)


def model_dir() -> str:
    """Folder for generated models (kept out of git and out of the GPU snapshot)."""
    root = os.environ.get("SLX_MODEL_DIR") or os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_models")
    os.makedirs(root, exist_ok=True)
    return root


def cached(name: str, make) -> str:
    """Path of a generated model, written once by make(path). The file is written under a name of
    this process's own and renamed into place, so ranks that generate it at the same time never
    read a half-written file."""
    path = os.path.join(model_dir(), name)
    if not os.path.exists(path):
        tmp = f"{path}.tmp{os.getpid()}"
        make(tmp)
        os.replace(tmp, path)
    return path


# ----------------------------------------------------------------------------------------------
# the benchmark configurations' models (seeded; identical bytes on every machine)
# ----------------------------------------------------------------------------------------------
def encoder_q8_0_model() -> str:
    """CPU-runnable encoder configuration: nomic-bert 12L d768 H12 F3072 V30522, Q8_0 weights."""
    return cached("encoder_nomic_L12_d768_q8_0_seed1.gguf",
                  lambda p: write_encoder(p, EncoderShape(), Q8_0, seed=1))


def encoder_q4_0_model() -> str:
    """Batched-encoder configuration: the same architecture with Q4_0 weights."""
    return cached("encoder_nomic_L12_d768_q4_0_seed3.gguf",
                  lambda p: write_encoder(p, EncoderShape(), Q4_0, seed=3))


def gemma_model() -> str:
    """Gemma-2B-shaped causal LM: 18L d2048 8q/1kv hd256 F16384 V256000, Q4_0 projections and
    embeddings, F16 norms, EOS the last token (so greedy runs are not cut short by a random EOS)."""
    shape = CausalShape()
    return cached("gemma2b_shape_q4_0_f16norm_seed5.gguf",
                  lambda p: write_causal(p, shape, Q4_0, F16, seed=5, eos=shape.vocab - 1))


def gemma_prompts(batch: int, seq: int = 512, seed: int = 21) -> "np.ndarray":
    """Seeded prompt ids [batch, seq] drawn uniformly from [0, vocab - 1) (EOS excluded)."""
    return np.random.default_rng(seed).integers(0, CausalShape().vocab - 1, (batch, seq)).astype(np.int32)


def gaussian_mixture(rng: np.random.Generator, n: int, dim: int = 768, centres: int = 1024, sigma: float = 0.1,
                     centre_vectors: np.ndarray | None = None) -> np.ndarray:
    """Embed+search inputs: centres c ~ N(0, I) L2-normalized, points c + sigma N(0, I) L2-normalized
    (float32 [n, dim]). Pass centre_vectors to draw queries from the same mixture as a database."""
    c = centre_vectors
    if c is None:
        c = rng.standard_normal((centres, dim))
        c /= np.linalg.norm(c, axis=1, keepdims=True)
    x = c[rng.integers(0, c.shape[0], n)] + sigma * rng.standard_normal((n, dim))
    x /= np.linalg.norm(x, axis=1, keepdims=True)
    return x.astype(np.float32)


def mixture_centres(rng: np.random.Generator, dim: int = 768, centres: int = 1024) -> np.ndarray:
    c = rng.standard_normal((centres, dim))
    return c / np.linalg.norm(c, axis=1, keepdims=True)
