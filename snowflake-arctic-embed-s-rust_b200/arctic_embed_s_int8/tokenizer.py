"""BertTokenizer (src/tokenizer.rs:25-101) over the library's C++ WordPiece tokenizer
(ae_tokenizer_* in include/arctic_cuda.h). Host only: no GPU is needed."""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import AeError, lib

PAD_ID, UNK_ID, CLS_ID, SEP_ID, MASK_ID = 0, 100, 101, 102, 103
MAX_SEQ_LEN = 512
MAX_WORD_CHARS = 100
QUERY_PREFIX = "Represent this sentence for searching relevant passages: "


class BertTokenizer:
    def __init__(self, handle: C.c_void_p):
        self._h = handle

    @classmethod
    def from_vocab_file(cls, path: str) -> "BertTokenizer":
        h = C.c_void_p()
        code = lib().ae_tokenizer_create_from_file(path.encode(), C.byref(h))
        if code != 0:
            raise AeError(code, lib().ae_tokenizer_last_error().decode())
        return cls(h)

    @classmethod
    def from_vocab_str(cls, text: str) -> "BertTokenizer":
        b = text.encode("utf-8")
        h = C.c_void_p()
        code = lib().ae_tokenizer_create_from_vocab(b, len(b), C.byref(h))
        if code != 0:
            raise AeError(code, lib().ae_tokenizer_last_error().decode())
        return cls(h)

    def vocab_size(self) -> int:
        return int(lib().ae_tokenizer_vocab_size(self._h))

    def _encode(self, text: str, is_query: bool) -> np.ndarray:
        b = text.encode("utf-8")
        out = np.zeros(MAX_SEQ_LEN, np.uint16)
        n = C.c_uint32()
        code = lib().ae_tokenize(self._h, b, len(b), int(is_query), out.ctypes.data_as(C.c_void_p), MAX_SEQ_LEN,
                                 C.byref(n))
        if code != 0:
            raise AeError(code, "ae_tokenize failed")
        return out[: n.value].copy()

    def encode(self, text: str) -> np.ndarray:
        """[CLS] text [SEP], at most 512 ids (src/tokenizer.rs:74-79)."""
        return self._encode(text, False)

    def encode_query(self, query: str) -> np.ndarray:
        """[CLS] QUERY_PREFIX query [SEP], at most 512 ids (src/tokenizer.rs:80-87)."""
        return self._encode(query, True)

    def encode_batch(self, texts, is_query: bool = False):
        """Packed ids and cu_seqlens of many texts, tokenized on host threads (ae_tokenize_batch)."""
        bs = [t.encode("utf-8") for t in texts]
        n = len(bs)
        arr = (C.c_char_p * n)(*bs)
        lens = np.array([len(b) for b in bs], np.uint64)
        cap = n * MAX_SEQ_LEN
        ids = np.zeros(max(cap, 1), np.uint16)
        cu = np.zeros(n + 1, np.uint32)
        code = lib().ae_tokenize_batch(self._h, arr, lens.ctypes.data_as(C.c_void_p), n, int(is_query),
                                       ids.ctypes.data_as(C.c_void_p), cap, cu.ctypes.data_as(C.c_void_p))
        if code != 0:
            raise AeError(code, "ae_tokenize_batch failed")
        return ids[: int(cu[-1])].copy(), cu

    def close(self) -> None:
        if self._h:
            lib().ae_tokenizer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
