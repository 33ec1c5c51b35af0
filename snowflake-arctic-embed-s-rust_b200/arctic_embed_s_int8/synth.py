"""Seeded synthetic arctic-embed-s model and token ids.

The real ``model.ae8`` is not available, so every test and benchmark runs on a synthetic pack with
the architecture of snowflake-arctic-embed-s (12 post-LN BERT layers, hidden 384, 12 heads x 32,
FFN 1536 with exact-erf GELU, LayerNorm eps 1e-12, vocab 30522, 512 positions, 2 token types):

* FP32 weights N(0, 0.02); LayerNorm gamma 1 + N(0, 0.05), beta N(0, 0.02); biases N(0, 0.02).
* SmoothQuant with alpha 0.5: for every linear, s_k = max|X_k|^0.5 / max|W[:,k]|^0.5 from an FP32
  calibration forward over 16 seeded 128-token sequences; W' = W diag(s), inv_smooth = 1 / s.
* Weights quantized symmetric per output channel (w_scale = max|row| / 127, round half even);
  embedding tables per row the same way.
* Layer 11 is written the way the reference's loader expects its pruned [CLS] layer: ``qkv`` with
  n_out = 0 keeping only ``inv_smooth`` (src/gemm.rs:195-205), ``has_split = 1``, and ``q_only`` /
  ``kv_only`` smoothed with the same s as the fused QKV (src/model.rs:226, :393 quantize the
  layer-11 input with ``layers[11].qkv.inv_smooth``).

Token ids follow ``[CLS]=101 + U{1000..30521}^(L-2) + [SEP]=102``.
"""
from __future__ import annotations

import hashlib
import os
import tempfile
from dataclasses import dataclass

import numpy as np

from .ae8 import (
    HIDDEN_SIZE as H,
    INTERMEDIATE_SIZE as INTER,
    NUM_HEADS,
    HEAD_DIM,
    NUM_LAYERS,
    VOCAB_SIZE,
    MAX_POSITIONS,
    TYPE_VOCAB_SIZE,
    LAYER_NORM_EPS,
    QuantizedLayer,
    QuantizedLinear,
    QuantizedModel,
    write_ae8,
)

CLS_ID = 101
SEP_ID = 102
SMOOTH_ALPHA = 0.5
CALIB_SEQS = 16
CALIB_LEN = 128


@dataclass
class Fp32Layer:
    wqkv: np.ndarray  # [1152, 384]
    bqkv: np.ndarray
    wo: np.ndarray  # [384, 384]
    bo: np.ndarray
    ln1w: np.ndarray
    ln1b: np.ndarray
    wi: np.ndarray  # [1536, 384]
    bi: np.ndarray
    wo2: np.ndarray  # [384, 1536]
    bo2: np.ndarray
    ln2w: np.ndarray
    ln2b: np.ndarray


@dataclass
class Fp32Model:
    word: np.ndarray
    pos: np.ndarray
    typ: np.ndarray
    emb_lnw: np.ndarray
    emb_lnb: np.ndarray
    layers: list


def token_ids(length: int, rng: np.random.Generator) -> np.ndarray:
    """``[101] + U{1000..30521}^(L-2) + [102]`` (length >= 2), uint16."""
    if length < 2:
        return np.full(max(length, 0), CLS_ID, dtype=np.uint16)
    mid = rng.integers(1000, VOCAB_SIZE, size=length - 2, endpoint=False)
    return np.concatenate([[CLS_ID], mid, [SEP_ID]]).astype(np.uint16)


def make_fp32_model(seed: int = 0) -> Fp32Model:
    rng = np.random.Generator(np.random.PCG64(seed))
    n = lambda *shape, s=0.02: (rng.standard_normal(shape, dtype=np.float64) * s).astype(np.float32)
    word, pos, typ = n(VOCAB_SIZE, H), n(MAX_POSITIONS, H), n(TYPE_VOCAB_SIZE, H)
    emb_lnw, emb_lnb = (1.0 + n(H, s=0.05)).astype(np.float32), n(H)
    layers = []
    for _ in range(NUM_LAYERS):
        layers.append(
            Fp32Layer(
                wqkv=n(3 * H, H), bqkv=n(3 * H), wo=n(H, H), bo=n(H),
                ln1w=(1.0 + n(H, s=0.05)).astype(np.float32), ln1b=n(H),
                wi=n(INTER, H), bi=n(INTER), wo2=n(H, INTER), bo2=n(H),
                ln2w=(1.0 + n(H, s=0.05)).astype(np.float32), ln2b=n(H),
            )
        )
    return Fp32Model(word, pos, typ, emb_lnw, emb_lnb, layers)


def _ln(x, w, b):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + LAYER_NORM_EPS) * w + b


def _gelu(x):
    from math import sqrt

    import scipy.special

    return 0.5 * x * (1.0 + scipy.special.erf(x / sqrt(2.0)))


def fp_forward(m: Fp32Model, ids: np.ndarray, dtype=np.float64, record: dict | None = None) -> np.ndarray:
    """Reference FP forward of the unquantized model (post-LN BERT, [CLS] pooling, L2 norm).

    ``record`` (optional) collects, per linear, the running max |x| of its input per channel, as
    needed for SmoothQuant calibration: keys ``(layer, name)``."""
    L = min(len(ids), MAX_POSITIONS)
    ids = np.asarray(ids[:L], dtype=np.int64)
    c = lambda a: a.astype(dtype)
    h = _ln(c(m.word[ids]) + c(m.pos[:L]) + c(m.typ[0]), c(m.emb_lnw), c(m.emb_lnb))

    def rec(key, x):
        if record is not None:
            mx = np.abs(x).max(0)
            record[key] = np.maximum(record.get(key, mx), mx)

    for li, ly in enumerate(m.layers):
        rec((li, "qkv"), h)
        qkv = h @ c(ly.wqkv).T + c(ly.bqkv)
        q, k, v = qkv[:, :H], qkv[:, H : 2 * H], qkv[:, 2 * H :]
        ctx = np.empty((L, H), dtype=dtype)
        for hh in range(NUM_HEADS):
            sl = slice(hh * HEAD_DIM, (hh + 1) * HEAD_DIM)
            s = (q[:, sl] / np.sqrt(HEAD_DIM)) @ k[:, sl].T
            s = np.exp(s - s.max(-1, keepdims=True))
            p = s / s.sum(-1, keepdims=True)
            ctx[:, sl] = p @ v[:, sl]
        rec((li, "attn_out"), ctx)
        h = _ln(ctx @ c(ly.wo).T + c(ly.bo) + h, c(ly.ln1w), c(ly.ln1b))
        rec((li, "ffn_inter"), h)
        g = _gelu(h @ c(ly.wi).T + c(ly.bi))
        rec((li, "ffn_out"), g)
        h = _ln(g @ c(ly.wo2).T + c(ly.bo2) + h, c(ly.ln2w), c(ly.ln2b))
    out = h[0]
    return (out / np.linalg.norm(out)).astype(np.float64)


def _quant_rows(w: np.ndarray):
    mx = np.abs(w).max(1)
    scale = np.where(mx > 0, mx / 127.0, 1.0).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def _smooth_linear(w: np.ndarray, b: np.ndarray, x_max: np.ndarray, alpha: float = SMOOTH_ALPHA):
    w64 = w.astype(np.float64)
    w_max = np.maximum(np.abs(w64).max(0), 1e-5)
    s = np.power(np.maximum(x_max, 1e-5), alpha) / np.power(w_max, 1.0 - alpha)
    s = np.clip(s, 1e-4, 1e4)
    wq, ws = _quant_rows((w64 * s[None, :]).astype(np.float32))
    inv = (1.0 / s).astype(np.float32)
    return QuantizedLinear(w.shape[0], w.shape[1], wq, ws, b.astype(np.float32), inv)


def quantize_model(m: Fp32Model, seed: int = 0) -> QuantizedModel:
    rng = np.random.Generator(np.random.PCG64(seed + 1))
    record: dict = {}
    for _ in range(CALIB_SEQS):
        fp_forward(m, token_ids(CALIB_LEN, rng), dtype=np.float32, record=record)
    wq, ws = _quant_rows(m.word)
    pq, ps = _quant_rows(m.pos)
    tq, ts = _quant_rows(m.typ)
    qm = QuantizedModel(wq, ws, pq, ps, tq, ts, m.emb_lnw.copy(), m.emb_lnb.copy())
    for li, ly in enumerate(m.layers):
        qkv = _smooth_linear(ly.wqkv, ly.bqkv, record[(li, "qkv")])
        q_only = kv_only = None
        if li == NUM_LAYERS - 1:
            q_only = QuantizedLinear(H, H, qkv.w_q[:H].copy(), qkv.w_scale[:H].copy(), qkv.bias[:H].copy(),
                                     qkv.inv_smooth.copy())
            kv_only = QuantizedLinear(2 * H, H, qkv.w_q[H:].copy(), qkv.w_scale[H:].copy(), qkv.bias[H:].copy(),
                                      qkv.inv_smooth.copy())
            qkv = QuantizedLinear(0, H, np.zeros((0, H), np.int8), np.zeros(0, np.float32), np.zeros(0, np.float32),
                                  qkv.inv_smooth)
        qm.layers.append(
            QuantizedLayer(
                qkv=qkv, q_only=q_only, kv_only=kv_only,
                attn_out=_smooth_linear(ly.wo, ly.bo, record[(li, "attn_out")]),
                ln1_weight=ly.ln1w.copy(), ln1_bias=ly.ln1b.copy(),
                ffn_inter=_smooth_linear(ly.wi, ly.bi, record[(li, "ffn_inter")]),
                ffn_out=_smooth_linear(ly.wo2, ly.bo2, record[(li, "ffn_out")]),
                ln2_weight=ly.ln2w.copy(), ln2_bias=ly.ln2b.copy(),
            )
        )
    return qm


def pack_path(seed: int = 0, cache_dir: str | None = None) -> str:
    """Path of the synthetic pack for ``seed``, generating and caching it on first use."""
    cache_dir = cache_dir or os.environ.get("ARCTIC_SYNTH_CACHE") or os.path.join(tempfile.gettempdir(), "arctic_synth")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"synthetic_seed{seed}.ae8")
    if not os.path.exists(path):
        qm = quantize_model(make_fp32_model(seed), seed)
        tmp = path + f".tmp{os.getpid()}"
        write_ae8(qm, tmp)
        os.replace(tmp, path)
    return path


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()
