"""ctypes binding of the CPU oracle (liboracle.so, built from oracle.cpp by the Makefile here).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg as the checker. The product library never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

BACKEND_AVX_VNNI = 5
BACKEND_AVX2 = 6
BACKEND_SCALAR = 7
H = 384
ATTENTION_EXACT, ATTENTION_INT8 = 0, 1  # or_model_set_attention_mode

_lib = None


def build() -> str:
    """Compiles liboracle.so in place (make)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = C.CDLL(_LIB_PATH)
    P = C.c_void_p
    u8p, i8p, u16p, u32p, f32p, i32p = (C.POINTER(t) for t in (C.c_uint8, C.c_int8, C.c_uint16, C.c_uint32, C.c_float, C.c_int32))
    L.or_detect_backend.restype = C.c_int
    L.or_has_avx2_fma.restype = C.c_int
    L.or_model_load.restype = P
    L.or_model_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_char_p)]
    L.or_model_load_mem.restype = P
    L.or_model_load_mem.argtypes = [u8p, C.c_uint64, C.c_int, C.POINTER(C.c_char_p)]
    L.or_model_free.argtypes = [P]
    L.or_model_backend.argtypes = [P]
    L.or_forward_cls.argtypes = [P, u16p, C.c_uint32, f32p]
    L.or_forward_ragged.argtypes = [P, u16p, u32p, C.c_uint32, f32p]
    L.or_embed_batch.argtypes = [P, u16p, u32p, C.c_uint32, C.c_uint32, f32p]
    L.or_forward_trace.argtypes = [P, u16p, C.c_uint32, i8p, f32p, f32p, f32p, f32p, i8p, f32p]
    L.or_embed_rows.argtypes = [P, u16p, C.c_uint32, f32p, i8p, f32p]
    L.or_gemm.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.c_uint32, i8p, f32p, i8p, f32p, f32p, f32p, f32p, i32p]
    L.or_layernorm_smooth_quantize_row.restype = C.c_float
    L.or_layernorm_smooth_quantize_row.argtypes = [f32p, f32p, f32p, f32p, i8p, C.c_uint32]
    L.or_smooth_quantize_row.restype = C.c_float
    L.or_smooth_quantize_row.argtypes = [f32p, f32p, i8p, C.c_uint32]
    L.or_gelu_smooth_quantize_row.restype = C.c_float
    L.or_gelu_smooth_quantize_row.argtypes = [f32p, f32p, i8p, C.c_uint32]
    L.or_layernorm_inplace_row.argtypes = [f32p, f32p, f32p, C.c_uint32]
    L.or_l2_normalize.argtypes = [f32p, C.c_uint32]
    L.or_attention_query.argtypes = [f32p, f32p, f32p, C.c_uint32, f32p]
    L.or_gelu_ref.argtypes = [f32p, f32p, C.c_uint32]
    L.or_model_set_attention_mode.argtypes = [P, C.c_int]
    L.or_attention_i8.argtypes = [f32p, C.c_uint32, f32p]
    _lib = L
    return L


def _p(a: np.ndarray | None, t):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.POINTER(t))


def detect_backend() -> int:
    return lib().or_detect_backend()


def pack_seqs(seqs) -> tuple[np.ndarray, np.ndarray]:
    """Concatenate sequences into (ids uint16, cu_seqlens uint32[n+1])."""
    lens = np.array([len(s) for s in seqs], dtype=np.uint32)
    cu = np.zeros(len(seqs) + 1, dtype=np.uint32)
    np.cumsum(lens, out=cu[1:])
    ids = np.concatenate([np.asarray(s, dtype=np.uint16) for s in seqs]) if seqs else np.zeros(0, np.uint16)
    return np.ascontiguousarray(ids, dtype=np.uint16), cu


class OracleModel:
    """The reference's PackedModel restated on the CPU."""

    def __init__(self, path: str, backend: int | None = None):
        self.backend = detect_backend() if backend is None else backend
        err = C.c_char_p()
        self._h = lib().or_model_load(path.encode(), self.backend, C.byref(err))
        if not self._h:
            raise ValueError(err.value.decode() if err.value else "oracle load failed")

    @classmethod
    def from_bytes(cls, buf: bytes, backend: int | None = None):
        self = cls.__new__(cls)
        self.backend = detect_backend() if backend is None else backend
        arr = np.frombuffer(buf, dtype=np.uint8)
        err = C.c_char_p()
        self._h = lib().or_model_load_mem(_p(np.ascontiguousarray(arr), C.c_uint8), len(buf), self.backend, C.byref(err))
        if not self._h:
            raise ValueError(err.value.decode() if err.value else "oracle load failed")
        return self

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_model_free(self._h)
            self._h = None

    def set_attention_mode(self, mode: int) -> "OracleModel":
        """ATTENTION_EXACT (fp32, the default) or ATTENTION_INT8 (the reference's int8 scheme)."""
        if lib().or_model_set_attention_mode(self._h, int(mode)) != 0:
            raise ValueError(f"unknown attention mode {mode}")
        return self

    def forward_cls(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint16)
        out = np.zeros(H, np.float32)
        lib().or_forward_cls(self._h, _p(ids, C.c_uint16), len(ids), _p(out, C.c_float))
        return out

    def forward_ragged(self, seqs) -> np.ndarray:
        ids, cu = pack_seqs(seqs)
        out = np.zeros((len(seqs), H), np.float32)
        lib().or_forward_ragged(self._h, _p(ids, C.c_uint16), _p(cu, C.c_uint32), len(seqs), _p(out, C.c_float))
        return out

    def embed_batch(self, seqs, threads: int = 1) -> np.ndarray:
        ids, cu = pack_seqs(seqs)
        return self.embed_batch_packed(ids, cu, threads)

    def embed_batch_packed(self, ids: np.ndarray, cu: np.ndarray, threads: int = 1) -> np.ndarray:
        n = len(cu) - 1
        out = np.zeros((n, H), np.float32)
        lib().or_embed_batch(self._h, _p(ids, C.c_uint16), _p(cu, C.c_uint32), n, threads, _p(out, C.c_float))
        return out

    def embed_rows(self, ids):
        """(hidden [L,384], q [L,384], scale [L]): the embedding LayerNorm rows of one sequence and their
        quantization for layer 0's QKV GEMM."""
        ids = np.ascontiguousarray(ids, dtype=np.uint16)
        L = min(len(ids), 512)
        hid = np.zeros((L, H), np.float32)
        q = np.zeros((L, H), np.int8)
        sc = np.zeros(L, np.float32)
        lib().or_embed_rows(self._h, _p(ids, C.c_uint16), len(ids), _p(hid, C.c_float), _p(q, C.c_int8), _p(sc, C.c_float))
        return hid, q, sc

    def trace(self, ids) -> dict:
        ids = np.ascontiguousarray(ids, dtype=np.uint16)
        L = min(len(ids), 512)
        t = {
            "gemm_in_q": np.zeros((12, L, H), np.int8),
            "gemm_in_s": np.zeros((12, L), np.float32),
            "qkv_out": np.zeros((11, L, 3 * H), np.float32),
            "ctx": np.zeros((11, L, H), np.float32),
            "hidden": np.zeros((11, L, H), np.float32),
            "down_in_q": np.zeros((11, L, 1536), np.int8),
            "down_in_s": np.zeros((11, L), np.float32),
        }
        lib().or_forward_trace(self._h, _p(ids, C.c_uint16), len(ids), _p(t["gemm_in_q"], C.c_int8),
                               _p(t["gemm_in_s"], C.c_float), _p(t["qkv_out"], C.c_float), _p(t["ctx"], C.c_float),
                               _p(t["hidden"], C.c_float), _p(t["down_in_q"], C.c_int8), _p(t["down_in_s"], C.c_float))
        return t


def gemm(backend, a_q, a_scale, w, w_scale, bias, res=None):
    """gemm_int8_fused on row-major W[N,K]: returns (out f32 [M,N], acc int32 [M,N])."""
    M, K = a_q.shape
    N = w.shape[0]
    out = np.zeros((M, N), np.float32)
    acc = np.zeros((M, N), np.int32)
    lib().or_gemm(backend, M, K, N, _p(np.ascontiguousarray(a_q, np.int8), C.c_int8),
                  _p(np.ascontiguousarray(a_scale, np.float32), C.c_float), _p(np.ascontiguousarray(w, np.int8), C.c_int8),
                  _p(np.ascontiguousarray(w_scale, np.float32), C.c_float), _p(np.ascontiguousarray(bias, np.float32), C.c_float),
                  _p(None if res is None else np.ascontiguousarray(res, np.float32), C.c_float), _p(out, C.c_float), _p(acc, C.c_int32))
    return out, acc


def ln_quant_rows(x, gamma, beta, inv_s):
    """layernorm_smooth_quantize_row over the rows of x: returns (y, q, scale)."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    q = np.zeros(y.shape, np.int8)
    sc = np.zeros(y.shape[0], np.float32)
    g, b, s = (np.ascontiguousarray(v, np.float32) for v in (gamma, beta, inv_s))
    for i in range(y.shape[0]):
        sc[i] = lib().or_layernorm_smooth_quantize_row(_p(y[i], C.c_float), _p(g, C.c_float), _p(b, C.c_float),
                                                       _p(s, C.c_float), _p(q[i], C.c_int8), y.shape[1])
    return y, q, sc


def smooth_quant_rows(x, inv_s):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(x.shape, np.int8)
    sc = np.zeros(x.shape[0], np.float32)
    s = np.ascontiguousarray(inv_s, np.float32)
    for i in range(x.shape[0]):
        sc[i] = lib().or_smooth_quantize_row(_p(x[i], C.c_float), _p(s, C.c_float), _p(q[i], C.c_int8), x.shape[1])
    return q, sc


def gelu_quant_rows(x, inv_s):
    g = np.array(x, dtype=np.float32, copy=True, order="C")
    q = np.zeros(g.shape, np.int8)
    sc = np.zeros(g.shape[0], np.float32)
    s = np.ascontiguousarray(inv_s, np.float32)
    for i in range(g.shape[0]):
        sc[i] = lib().or_gelu_smooth_quantize_row(_p(g[i], C.c_float), _p(s, C.c_float), _p(q[i], C.c_int8), g.shape[1])
    return g, q, sc


def attention_query(q32, k_head, v_head):
    q32, k, v = (np.ascontiguousarray(a, np.float32) for a in (q32, k_head, v_head))
    out = np.zeros(32, np.float32)
    lib().or_attention_query(_p(q32, C.c_float), _p(k, C.c_float), _p(v, C.c_float), k.shape[0], _p(out, C.c_float))
    return out


def attention_i8(qkv):
    """The reference's int8 attention scheme on one sequence: qkv [L, 1152] -> ctx [L, 384]."""
    qkv = np.ascontiguousarray(qkv, np.float32)
    out = np.zeros((qkv.shape[0], H), np.float32)
    lib().or_attention_i8(_p(qkv, C.c_float), qkv.shape[0], _p(out, C.c_float))
    return out


def gelu_ref(x):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    y = np.zeros_like(x)
    lib().or_gelu_ref(_p(x, C.c_float), _p(y, C.c_float), x.size)
    return y
