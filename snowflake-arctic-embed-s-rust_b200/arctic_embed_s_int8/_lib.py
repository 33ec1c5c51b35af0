"""ctypes binding of libarctic_cuda.so (the C ABI declared in include/arctic_cuda.h).

The library is loaded from the package's ``lib/`` folder. There is no CPU fallback: if the
library or a GPU is missing, loading fails with an error.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libarctic_cuda.so")
CSRC = os.path.join(_PKG_ROOT, "csrc")
HEADER = os.path.join(os.path.dirname(_PKG_ROOT), "include", "arctic_cuda.h")

AE_OK = 0
ERRORS = {
    -1: "AE_ERR_INVALID_ARG",
    -2: "AE_ERR_CUDA",
    -3: "AE_ERR_NO_MODEL",
    -4: "AE_ERR_BAD_PACK",
    -5: "AE_ERR_TOKEN_RANGE",
    -6: "AE_ERR_DEVICE",
    -7: "AE_ERR_CAPACITY",
}

# exported symbols (every function declared in include/arctic_cuda.h)
SYMBOLS = [
    "ae_ctx_create", "ae_ctx_destroy", "ae_last_error", "ae_ctx_set_stream", "ae_ctx_device",
    "ae_model_load", "ae_model_load_file", "ae_reserve", "ae_forward_cls", "ae_forward_ragged",
    "ae_forward_ragged_device", "ae_embed_batch_multi", "ae_gemm_i8", "ae_attention_f32", "ae_kernel_launches",
    "ae_plan_shards", "ae_forward_cls_noalloc", "ae_profile", "ae_profile_read", "ae_sync",
    "ae_tokenizer_create_from_file", "ae_tokenizer_create_from_vocab", "ae_tokenizer_destroy",
    "ae_tokenizer_vocab_size", "ae_tokenizer_last_error", "ae_tokenize", "ae_tokenize_batch",
    "ae_selftest_wait_timeout", "ae_set_attention_mode", "ae_get_attention_mode", "ae_attention_i8",
    "ae_trace_forward", "ae_measure_int8_peak",
]


class AeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class LinearDesc(C.Structure):
    _fields_ = [
        ("n_out", C.c_uint64), ("k_in", C.c_uint64), ("w_q", C.c_void_p), ("w_scale", C.c_void_p),
        ("bias", C.c_void_p), ("inv_smooth", C.c_void_p),
    ]


class LayerDesc(C.Structure):
    _fields_ = [
        ("qkv", LinearDesc), ("has_split", C.c_int32), ("q_only", LinearDesc), ("kv_only", LinearDesc),
        ("attn_out", LinearDesc), ("ln1_weight", C.c_void_p), ("ln1_bias", C.c_void_p),
        ("ffn_inter", LinearDesc), ("ffn_out", LinearDesc), ("ln2_weight", C.c_void_p), ("ln2_bias", C.c_void_p),
    ]


class ModelDesc(C.Structure):
    _fields_ = [
        ("word_emb_q", C.c_void_p), ("word_emb_scale", C.c_void_p), ("pos_emb_q", C.c_void_p),
        ("pos_emb_scale", C.c_void_p), ("type_emb_q", C.c_void_p), ("type_emb_scale", C.c_void_p),
        ("emb_ln_weight", C.c_void_p), ("emb_ln_bias", C.c_void_p), ("layers", LayerDesc * 12),
    ]


def build(force: bool = False) -> str:
    """Compiles the CUDA library for sm_100a (make in csrc/)."""
    if force or not os.path.exists(LIB_PATH):
        subprocess.run(["make", "-s", "-C", CSRC, "-j4"], check=True)
    else:
        subprocess.run(["make", "-s", "-C", CSRC, "-j4"], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {CSRC}` (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    P = C.c_void_p
    u32 = C.c_uint32
    L.ae_ctx_create.argtypes = [C.c_int, C.POINTER(P)]
    L.ae_ctx_destroy.argtypes = [P]
    L.ae_last_error.argtypes = [P]
    L.ae_last_error.restype = C.c_char_p
    L.ae_ctx_set_stream.argtypes = [P, P]
    L.ae_ctx_device.argtypes = [P]
    L.ae_model_load.argtypes = [P, C.POINTER(ModelDesc)]
    L.ae_model_load_file.argtypes = [P, C.c_char_p]
    L.ae_reserve.argtypes = [P, u32, u32]
    L.ae_forward_cls.argtypes = [P, P, u32, P]
    L.ae_forward_ragged.argtypes = [P, P, P, u32, P]
    L.ae_forward_ragged_device.argtypes = [P, P, P, u32, u32, u32, P]
    L.ae_embed_batch_multi.argtypes = [C.POINTER(P), C.c_int, P, P, u32, u32, P]
    L.ae_gemm_i8.argtypes = [P, C.c_int, u32, u32, u32] + [P] * 13
    L.ae_attention_f32.argtypes = [P, P, P, u32, u32, P]
    L.ae_attention_i8.argtypes = [P, P, P, u32, u32, P]
    L.ae_set_attention_mode.argtypes = [P, C.c_int]
    L.ae_get_attention_mode.argtypes = [P]
    L.ae_sync.argtypes = [P]
    L.ae_kernel_launches.argtypes = [P]
    L.ae_plan_shards.argtypes = [P, u32, C.c_int, P]
    L.ae_forward_cls_noalloc.argtypes = [P, P, u32, P]
    L.ae_profile.argtypes = [P, C.c_int]
    L.ae_profile_read.argtypes = [P, P, P]
    L.ae_selftest_wait_timeout.argtypes = [P, u32]
    L.ae_trace_forward.argtypes = [P, P, P, u32, C.c_int, P, P, P]
    L.ae_measure_int8_peak.argtypes = [P, u32, C.POINTER(C.c_float), C.POINTER(C.c_double)]
    L.ae_tokenizer_create_from_file.argtypes = [C.c_char_p, C.POINTER(P)]
    L.ae_tokenizer_create_from_vocab.argtypes = [C.c_char_p, C.c_size_t, C.POINTER(P)]
    L.ae_tokenizer_destroy.argtypes = [P]
    L.ae_tokenizer_vocab_size.argtypes = [P]
    L.ae_tokenizer_last_error.argtypes = []
    L.ae_tokenize.argtypes = [P, C.c_char_p, C.c_size_t, C.c_int, P, u32, C.POINTER(u32)]
    L.ae_tokenize_batch.argtypes = [P, C.POINTER(C.c_char_p), P, u32, C.c_int, P, C.c_size_t, P]
    for name in SYMBOLS:
        if name not in ("ae_last_error", "ae_kernel_launches", "ae_tokenizer_vocab_size", "ae_tokenizer_last_error"):
            getattr(L, name).restype = C.c_int
    L.ae_kernel_launches.restype = C.c_uint64
    L.ae_tokenizer_vocab_size.restype = C.c_uint32
    L.ae_tokenizer_last_error.restype = C.c_char_p
    _lib = L
    return L


def check(ctx, code: int) -> None:
    if code != AE_OK:
        msg = lib().ae_last_error(ctx)
        raise AeError(code, msg.decode() if msg else "")
