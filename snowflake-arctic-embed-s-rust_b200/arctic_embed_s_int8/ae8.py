"""The portable ``.ae8`` quantized model pack: reader and writer.

Layout (src/quantize.rs:20, :76-137, :168-209 of the reference crate): the 8-byte magic
``b"ARCTIC8\\x01"``, then length-prefixed little-endian vectors (u64 element count, then the
elements): word/pos/type embedding tables as int8 + per-row f32 scales, the embedding LayerNorm
weight and bias, then 12 layers of ``qkv`` (a linear), a ``has_split`` byte with optional
``q_only``/``kv_only`` linears, ``attn_out``, ``ln1`` weight/bias, ``ffn_inter``, ``ffn_out`` and
``ln2`` weight/bias. A linear is ``n_out`` (u64), ``k_in`` (u64), then int8 weights ``[n_out,k_in]``
row-major, ``w_scale[n_out]``, ``bias[n_out]`` and ``inv_smooth[k_in]``.
"""
from __future__ import annotations

import io
import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"ARCTIC8\x01"
HIDDEN_SIZE = 384
INTERMEDIATE_SIZE = 1536
NUM_HEADS = 12
HEAD_DIM = 32
NUM_LAYERS = 12
VOCAB_SIZE = 30522
MAX_POSITIONS = 512
TYPE_VOCAB_SIZE = 2
LAYER_NORM_EPS = 1e-12


class Ae8FormatError(ValueError):
    """Malformed pack (the reference returns ``io::ErrorKind::InvalidData`` / ``UnexpectedEof``)."""


@dataclass
class QuantizedLinear:
    """QuantizedLinearRaw, src/quantize.rs:22-30."""

    n_out: int
    k_in: int
    w_q: np.ndarray  # int8 [n_out, k_in]
    w_scale: np.ndarray  # f32 [n_out]
    bias: np.ndarray  # f32 [n_out]
    inv_smooth: np.ndarray  # f32 [k_in]


@dataclass
class QuantizedLayer:
    """QuantizedLayerRaw, src/quantize.rs:46-58."""

    qkv: QuantizedLinear
    q_only: QuantizedLinear | None
    kv_only: QuantizedLinear | None
    attn_out: QuantizedLinear
    ln1_weight: np.ndarray
    ln1_bias: np.ndarray
    ffn_inter: QuantizedLinear
    ffn_out: QuantizedLinear
    ln2_weight: np.ndarray
    ln2_bias: np.ndarray


@dataclass
class QuantizedModel:
    """QuantizedModelRaw, src/quantize.rs:60-72."""

    word_emb_q: np.ndarray
    word_emb_scale: np.ndarray
    pos_emb_q: np.ndarray
    pos_emb_scale: np.ndarray
    type_emb_q: np.ndarray
    type_emb_scale: np.ndarray
    emb_ln_weight: np.ndarray
    emb_ln_bias: np.ndarray
    layers: list[QuantizedLayer] = field(default_factory=list)


def _w_vec(f: io.BufferedIOBase, a: np.ndarray, dtype) -> None:
    a = np.ascontiguousarray(a, dtype=dtype).reshape(-1)
    f.write(struct.pack("<Q", a.size))
    f.write(a.astype(np.dtype(dtype).newbyteorder("<"), copy=False).tobytes())


def _w_linear(f, lin: QuantizedLinear) -> None:
    f.write(struct.pack("<QQ", lin.n_out, lin.k_in))
    _w_vec(f, lin.w_q, np.int8)
    _w_vec(f, lin.w_scale, np.float32)
    _w_vec(f, lin.bias, np.float32)
    _w_vec(f, lin.inv_smooth, np.float32)


def write_ae8(model: QuantizedModel, path_or_file) -> None:
    """Writes ``model`` in the layout QuantizedModelRaw::load_ae8 reads."""
    own = isinstance(path_or_file, (str, bytes)) or hasattr(path_or_file, "__fspath__")
    f = open(path_or_file, "wb") if own else path_or_file
    try:
        f.write(MAGIC)
        _w_vec(f, model.word_emb_q, np.int8)
        _w_vec(f, model.word_emb_scale, np.float32)
        _w_vec(f, model.pos_emb_q, np.int8)
        _w_vec(f, model.pos_emb_scale, np.float32)
        _w_vec(f, model.type_emb_q, np.int8)
        _w_vec(f, model.type_emb_scale, np.float32)
        _w_vec(f, model.emb_ln_weight, np.float32)
        _w_vec(f, model.emb_ln_bias, np.float32)
        for ly in model.layers:
            _w_linear(f, ly.qkv)
            split = ly.q_only is not None and ly.kv_only is not None
            f.write(bytes([1 if split else 0]))
            if split:
                _w_linear(f, ly.q_only)
                _w_linear(f, ly.kv_only)
            _w_linear(f, ly.attn_out)
            _w_vec(f, ly.ln1_weight, np.float32)
            _w_vec(f, ly.ln1_bias, np.float32)
            _w_linear(f, ly.ffn_inter)
            _w_linear(f, ly.ffn_out)
            _w_vec(f, ly.ln2_weight, np.float32)
            _w_vec(f, ly.ln2_bias, np.float32)
    finally:
        if own:
            f.close()


class _Cursor:
    def __init__(self, buf: bytes):
        self.buf = memoryview(buf)
        self.pos = 0

    def take(self, n: int) -> memoryview:
        if n < 0 or self.pos + n > len(self.buf):
            raise Ae8FormatError("unexpected end of .ae8 pack")
        out = self.buf[self.pos : self.pos + n]
        self.pos += n
        return out

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def vec(self, dtype) -> np.ndarray:
        n = self.u64()
        dt = np.dtype(dtype).newbyteorder("<")
        return np.frombuffer(self.take(n * dt.itemsize), dtype=dt).astype(dtype)

    def linear(self) -> QuantizedLinear:
        n_out, k_in = self.u64(), self.u64()
        w = self.vec(np.int8)
        ws = self.vec(np.float32)
        b = self.vec(np.float32)
        s = self.vec(np.float32)
        if w.size != n_out * k_in or ws.size != n_out or b.size != n_out or s.size != k_in:
            raise Ae8FormatError("linear layer has inconsistent vector lengths")
        return QuantizedLinear(n_out, k_in, w.reshape(n_out, k_in), ws, b, s)


def read_ae8(path_or_bytes) -> QuantizedModel:
    """QuantizedModelRaw::load_ae8 (src/quantize.rs:76-137), with the shape checks the reference
    performs later when packing (src/gemm.rs:206-212) done here."""
    if isinstance(path_or_bytes, (bytes, bytearray, memoryview)):
        buf = bytes(path_or_bytes)
    else:
        with open(path_or_bytes, "rb") as f:
            buf = f.read()
    c = _Cursor(buf)
    if bytes(c.take(8)) != MAGIC:
        raise Ae8FormatError("invalid .ae8 magic header")
    m = QuantizedModel(
        word_emb_q=c.vec(np.int8),
        word_emb_scale=c.vec(np.float32),
        pos_emb_q=c.vec(np.int8),
        pos_emb_scale=c.vec(np.float32),
        type_emb_q=c.vec(np.int8),
        type_emb_scale=c.vec(np.float32),
        emb_ln_weight=c.vec(np.float32),
        emb_ln_bias=c.vec(np.float32),
    )
    for _ in range(NUM_LAYERS):
        qkv = c.linear()
        split = bytes(c.take(1))[0] == 1
        q_only = kv_only = None
        if split:
            q_only, kv_only = c.linear(), c.linear()
        attn_out = c.linear()
        ln1w, ln1b = c.vec(np.float32), c.vec(np.float32)
        ffn_inter, ffn_out = c.linear(), c.linear()
        ln2w, ln2b = c.vec(np.float32), c.vec(np.float32)
        m.layers.append(QuantizedLayer(qkv, q_only, kv_only, attn_out, ln1w, ln1b, ffn_inter, ffn_out, ln2w, ln2b))
    return m
