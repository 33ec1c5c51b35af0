"""arctic_embed_s_int8 — host API of the B200 backend for the arctic-embed-s int8 W8A8 encoder.

Mirrors the public API of the reference crate (src/lib.rs of mdlockyer/snowflake-arctic-embed-s-rust):
``ArcticEmbedS.from_dir`` / ``embed_tokens`` / ``embed_batch`` / ``*_parallel``, ``Workspace``,
``ParallelContext`` and ``cosine_similarity``, over the C ABI of libarctic_cuda.so
(include/arctic_cuda.h). The forward pass runs only on the GPU: there is no CPU fallback, and
every entry point raises if the CUDA library or a B200 is unavailable.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import ae8
from ._lib import AeError, LayerDesc, LinearDesc, ModelDesc, check, lib

HIDDEN_SIZE = 384
MAX_POSITIONS = 512
MODEL_FILE = "model.ae8"
VOCAB_FILE = "vocab.txt"
MODEL_DIR_ENV_VAR = "ARCTIC_EMBED_MODEL_DIR"
# attention of layers 0-10 (ae_set_attention_mode): fp32 in the reference's x86 order, or its int8 scheme
ATTENTION_EXACT, ATTENTION_INT8 = 0, 1

__all__ = [
    "AeError", "Engine", "ArcticEmbedS", "Workspace", "ParallelContext", "cosine_similarity", "default_model_dir",
    "embed_batch_multi", "pack_sequences", "plan_shards", "HIDDEN_SIZE", "ATTENTION_EXACT", "ATTENTION_INT8",
]


def default_model_dir() -> str:
    """``$ARCTIC_EMBED_MODEL_DIR`` or ``./model`` (src/lib.rs:27-31)."""
    return os.environ.get(MODEL_DIR_ENV_VAR, "model")


def pack_sequences(seqs) -> tuple[np.ndarray, np.ndarray]:
    """Concatenates token-id sequences into (ids uint16 [T], cu_seqlens uint32 [n + 1])."""
    lens = np.array([len(s) for s in seqs], dtype=np.int64)
    cu = np.zeros(len(seqs) + 1, dtype=np.uint32)
    np.cumsum(lens, out=cu[1:])
    ids = np.concatenate([np.asarray(s, dtype=np.uint16) for s in seqs]) if len(seqs) else np.zeros(0, np.uint16)
    return np.ascontiguousarray(ids, dtype=np.uint16), cu


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
        return a.ctypes.data
    return a.data_ptr()  # torch tensor (device memory)


def _linear_desc(lin: ae8.QuantizedLinear | None, keep: list) -> LinearDesc:
    d = LinearDesc()
    if lin is None:
        return d
    arrs = [np.ascontiguousarray(lin.w_q, np.int8), np.ascontiguousarray(lin.w_scale, np.float32),
            np.ascontiguousarray(lin.bias, np.float32), np.ascontiguousarray(lin.inv_smooth, np.float32)]
    keep.extend(arrs)
    d.n_out, d.k_in = lin.n_out, lin.k_in
    d.w_q, d.w_scale, d.bias, d.inv_smooth = (a.ctypes.data if a.size else None for a in arrs)
    if lin.k_in and d.inv_smooth is None:
        d.inv_smooth = arrs[3].ctypes.data
    return d


def model_desc(m: ae8.QuantizedModel) -> tuple[ModelDesc, list]:
    """ae_model_desc over the arrays of a QuantizedModel (the arrays are kept alive in the list)."""
    keep: list = []

    def f(a, dt=np.float32):
        a = np.ascontiguousarray(a, dt)
        keep.append(a)
        return a.ctypes.data

    d = ModelDesc()
    d.word_emb_q, d.word_emb_scale = f(m.word_emb_q, np.int8), f(m.word_emb_scale)
    d.pos_emb_q, d.pos_emb_scale = f(m.pos_emb_q, np.int8), f(m.pos_emb_scale)
    d.type_emb_q, d.type_emb_scale = f(m.type_emb_q, np.int8), f(m.type_emb_scale)
    d.emb_ln_weight, d.emb_ln_bias = f(m.emb_ln_weight), f(m.emb_ln_bias)
    for i, ly in enumerate(m.layers):
        L = d.layers[i]
        L.qkv = _linear_desc(ly.qkv, keep)
        L.has_split = 1 if ly.q_only is not None else 0
        L.q_only = _linear_desc(ly.q_only, keep)
        L.kv_only = _linear_desc(ly.kv_only, keep)
        L.attn_out = _linear_desc(ly.attn_out, keep)
        L.ln1_weight, L.ln1_bias = f(ly.ln1_weight), f(ly.ln1_bias)
        L.ffn_inter = _linear_desc(ly.ffn_inter, keep)
        L.ffn_out = _linear_desc(ly.ffn_out, keep)
        L.ln2_weight, L.ln2_bias = f(ly.ln2_weight), f(ly.ln2_bias)
    return d, keep


class Engine:
    """One GPU context (ae_ctx): model on the device, workspace, stream, CUDA graphs."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        code = lib().ae_ctx_create(device, C.byref(h))
        if code != 0:
            raise AeError(code, lib().ae_last_error(None).decode())
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            try:
                lib().ae_ctx_destroy(self._h)
            except Exception:  # interpreter shutdown: modules may already be torn down
                pass
            self._h = None

    def __del__(self):
        self.close()

    def _check(self, code):
        check(self._h, code)

    def load_file(self, path: str) -> "Engine":
        self._check(lib().ae_model_load_file(self._h, os.fsencode(path)))
        return self

    def load(self, model: ae8.QuantizedModel) -> "Engine":
        d, keep = model_desc(model)
        self._check(lib().ae_model_load(self._h, C.byref(d)))
        del keep
        return self

    def reserve(self, max_tokens: int, max_seqs: int):
        self._check(lib().ae_reserve(self._h, max_tokens, max_seqs))

    def set_stream(self, stream) -> None:
        """Launch on a torch.cuda.Stream (or a raw cudaStream_t int); None = own stream."""
        s = None if stream is None else (stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))
        self._check(lib().ae_ctx_set_stream(self._h, s))

    def forward_cls(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint16)
        out = np.zeros(HIDDEN_SIZE, np.float32)
        self._check(lib().ae_forward_cls(self._h, _ptr(ids), len(ids), _ptr(out)))
        return out

    def forward_ragged(self, seqs) -> np.ndarray:
        ids, cu = pack_sequences(seqs)
        return self.forward_packed(ids, cu)

    def forward_packed(self, ids: np.ndarray, cu: np.ndarray) -> np.ndarray:
        n = len(cu) - 1
        out = np.zeros((n, HIDDEN_SIZE), np.float32)
        self._check(lib().ae_forward_ragged(self._h, _ptr(ids), _ptr(cu), n, _ptr(out)))
        return out

    def forward_device(self, d_ids, d_cu, n_seqs: int, total_tokens: int, max_len: int, d_out) -> None:
        """Asynchronous forward on device tensors (uint16 ids, int32/uint32 cu, float32 out [n, 384])."""
        self._check(lib().ae_forward_ragged_device(self._h, _ptr(d_ids), _ptr(d_cu), n_seqs, total_tokens, max_len,
                                                   _ptr(d_out)))

    TRACE_EMBED, TRACE_ATTN0 = 0, 1

    def trace(self, seqs, stage: int):
        """ae_trace_forward (a test hook): (f32 [T,384], q [T,384], scale [T]) of the forward pass of
        `seqs` stopped at TRACE_EMBED (embedding LayerNorm rows and their quantization) or
        TRACE_ATTN0 (layer 0's attention context and its quantization), rows in the caller's order."""
        ids, cu = pack_sequences(seqs)
        T = int(sum(min(len(s), MAX_POSITIONS) for s in seqs))
        f32 = np.zeros((T, HIDDEN_SIZE), np.float32)
        q = np.zeros((T, HIDDEN_SIZE), np.int8)
        sc = np.zeros(T, np.float32)
        self._check(lib().ae_trace_forward(self._h, _ptr(ids), _ptr(cu), len(seqs), stage, _ptr(f32), _ptr(q),
                                           _ptr(sc)))
        return f32, q, sc

    def gemm_i8(self, epi, a, a_scale, w, w_scale, bias, res=None, gamma=None, beta=None, inv_smooth=None, out=None,
                out_q=None, out_scale=None, acc=None) -> None:
        M, K = a.shape
        N = w.shape[0]
        self._check(lib().ae_gemm_i8(self._h, epi, M, N, K, _ptr(a), _ptr(a_scale), _ptr(w), _ptr(w_scale), _ptr(bias),
                                     _ptr(res), _ptr(gamma), _ptr(beta), _ptr(inv_smooth), _ptr(out), _ptr(out_q),
                                     _ptr(out_scale), _ptr(acc)))

    def attention_f32(self, qkv, cu, n_seqs: int, max_len: int, ctx) -> None:
        self._check(lib().ae_attention_f32(self._h, _ptr(qkv), _ptr(cu), n_seqs, max_len, _ptr(ctx)))

    def attention_i8(self, qkv, cu, n_seqs: int, max_len: int, ctx) -> None:
        """ae_attention_i8: the reference's int8 attention scheme on device buffers (every sequence)."""
        self._check(lib().ae_attention_i8(self._h, _ptr(qkv), _ptr(cu), n_seqs, max_len, _ptr(ctx)))

    def set_attention_mode(self, mode: int) -> "Engine":
        """ATTENTION_EXACT (fp32, default) or ATTENTION_INT8 (the reference's int8 scheme) for layers 0-10."""
        self._check(lib().ae_set_attention_mode(self._h, int(mode)))
        return self

    @property
    def attention_mode(self) -> int:
        return int(lib().ae_get_attention_mode(self._h))

    def measure_int8_peak(self, iters: int = 100000) -> tuple[float, float]:
        """ae_measure_int8_peak: (ms, int8 TOPS) of the resident-operand tcgen05 kind::i8 loop."""
        ms, tops = C.c_float(), C.c_double()
        self._check(lib().ae_measure_int8_peak(self._h, iters, C.byref(ms), C.byref(tops)))
        return float(ms.value), float(tops.value)

    def sync(self) -> None:
        self._check(lib().ae_sync(self._h))

    def selftest_wait_timeout(self, limit_us: int) -> None:
        """ae_selftest_wait_timeout: a bounded device wait that runs out; raises AeError(AE_ERR_DEVICE)."""
        self._check(lib().ae_selftest_wait_timeout(self._h, limit_us))

    def kernel_launches(self) -> int:
        return int(lib().ae_kernel_launches(self._h))

    KERNEL_KINDS = ("row_meta", "embed", "qkv", "attention", "ctx_quant", "attn_out", "ffn_up", "ffn_down", "cls_tail")

    def profile(self, enable: bool) -> None:
        """Start (clearing earlier records) or stop per-kernel CUDA-event timing of the forward pass."""
        self._check(lib().ae_profile(self._h, 1 if enable else 0))

    def profile_read(self) -> dict:
        """{kind: (total_ms, launches)} of everything recorded since profile(True); call after sync()."""
        ms = np.zeros(len(self.KERNEL_KINDS), np.float32)
        n = np.zeros(len(self.KERNEL_KINDS), np.uint32)
        self._check(lib().ae_profile_read(self._h, _ptr(ms), _ptr(n)))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(self.KERNEL_KINDS)}


def embed_batch_multi(engines, seqs=None, ids=None, cu=None, max_batch_tokens: int = 0) -> np.ndarray:
    """ae_embed_batch_multi: shards sequences across engines (GPUs); results in input order."""
    if seqs is not None:
        ids, cu = pack_sequences(seqs)
    n = len(cu) - 1
    out = np.zeros((n, HIDDEN_SIZE), np.float32)
    arr = (C.c_void_p * len(engines))(*[e.handle.value for e in engines])
    code = lib().ae_embed_batch_multi(arr, len(engines), _ptr(ids), _ptr(cu), n, max_batch_tokens, _ptr(out))
    check(engines[0].handle, code)
    return out


def plan_shards(cu: np.ndarray, n_shards: int) -> np.ndarray:
    """Shard index of every sequence (ae_plan_shards; host only)."""
    cu = np.ascontiguousarray(cu, np.uint32)
    out = np.zeros(len(cu) - 1, np.int32)
    code = lib().ae_plan_shards(_ptr(cu), len(cu) - 1, n_shards, _ptr(out))
    if code != 0:
        raise AeError(code, "ae_plan_shards: invalid arguments")
    return out


class Workspace:
    """Per-caller scratch of the reference (src/model.rs:123-173). On the GPU the workspace lives in
    the engine's context; this object only names the engine a caller drives, so code written
    against the reference's ``&mut Workspace`` keeps its shape."""

    def __init__(self, engine: Engine | None = None):
        self.engine = engine


class ParallelContext:
    """Latency mode (src/parallel.rs:137-254): one sequence on all SMs of one GPU. ``num_threads``
    is accepted for API parity and ignored — the GPU parallelises inside each kernel."""

    def __init__(self, num_threads: int = 0, engine: Engine | None = None):
        self.num_threads = num_threads
        self.engine = engine

    @classmethod
    def recommended(cls, engine: Engine | None = None) -> "ParallelContext":
        return cls(0, engine)

    def forward_cls(self, model: "ArcticEmbedS", input_ids) -> np.ndarray:
        return (self.engine or model.engine).forward_cls(input_ids)


class ArcticEmbedS:
    """src/lib.rs:34-260 on the GPU backend."""

    def __init__(self, engine: Engine, raw: ae8.QuantizedModel | None = None, tokenizer=None):
        self.engine = engine
        self.tokenizer = tokenizer
        self.raw_size_bytes = 0

    @classmethod
    def from_dir(cls, path: str | None = None, device: int = 0) -> "ArcticEmbedS":
        path = path or default_model_dir()
        eng = Engine(device).load_file(os.path.join(path, MODEL_FILE))
        tok = None
        vocab = os.path.join(path, VOCAB_FILE)
        if os.path.exists(vocab):
            from .tokenizer import BertTokenizer

            tok = BertTokenizer.from_vocab_file(vocab)
        return cls(eng, tokenizer=tok)

    @classmethod
    def from_pack(cls, pack_path: str, device: int = 0) -> "ArcticEmbedS":
        return cls(Engine(device).load_file(pack_path))

    def embed_tokens(self, input_ids, ws: Workspace | None = None) -> np.ndarray:
        return self.engine.forward_cls(input_ids)

    def embed_tokens_parallel(self, input_ids, par: ParallelContext) -> np.ndarray:
        return par.forward_cls(self, input_ids)

    def embed_document(self, text: str, ws: Workspace | None = None) -> np.ndarray:
        return self.embed_tokens(self._tok().encode(text), ws)

    def embed_query(self, query: str, ws: Workspace | None = None) -> np.ndarray:
        return self.embed_tokens(self._tok().encode_query(query), ws)

    def embed_document_parallel(self, text: str, par: ParallelContext) -> np.ndarray:
        return self.embed_tokens_parallel(self._tok().encode(text), par)

    def embed_query_parallel(self, query: str, par: ParallelContext) -> np.ndarray:
        return self.embed_tokens_parallel(self._tok().encode_query(query), par)

    def embed_batch_tokens(self, seqs, max_batch_tokens: int = 0) -> np.ndarray:
        return embed_batch_multi([self.engine], seqs=seqs, max_batch_tokens=max_batch_tokens)

    def embed_batch(self, texts, is_query: bool = False, num_threads: int = 0) -> np.ndarray:
        """src/lib.rs:138-260: texts tokenized on host threads (ae_tokenize_batch), then sharded and
        packed on the GPU(s). ``num_threads`` is accepted for API parity and ignored."""
        ids, cu = self._tok().encode_batch(list(texts), is_query)
        return embed_batch_multi([self.engine], ids=ids, cu=cu)

    def _tok(self):
        if self.tokenizer is None:
            raise RuntimeError("no vocab.txt was loaded; use embed_tokens / embed_batch_tokens with token ids")
        return self.tokenizer


def cosine_similarity(a, b) -> float:
    """src/lib.rs:263-271: dot product of two L2-normalised 384-d embeddings (sequential f32 sum)."""
    s = np.float32(0.0)
    for x, y in zip(np.asarray(a, np.float32), np.asarray(b, np.float32)):
        s = np.float32(s + np.float32(x * y))
    return float(s)
