"""WordPiece tokenizer (C ABI ae_tokenize*, src/tokenizer.rs:25-327) on the CPU: the reference
crate's own known-answer vectors (12 short records, 7 long texts up to the 512-id limit), an
independent Python restatement on generated Unicode text, and the encode rules (query prefix,
truncation, vocabulary line handling, invalid UTF-8)."""
import ctypes as C
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from oracle.tokenizer_ref import QUERY_PREFIX, TokenizerRef  # noqa: E402
from arctic_embed_s_int8 import AeError  # noqa: E402
from arctic_embed_s_int8._lib import lib  # noqa: E402
from arctic_embed_s_int8.tokenizer import BertTokenizer  # noqa: E402

GOLDEN = os.path.join(ROOT, "tests", "golden", "tokenizer_vectors.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN, encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def vocab_text():
    from conftest import golden_vocab_text

    return golden_vocab_text()[0]


@pytest.fixture(scope="module")
def tok(vocab_text):
    return BertTokenizer.from_vocab_str(vocab_text)


def test_reference_vectors(tok, golden):
    """tests/accuracy_test.rs:90-94: the tokenizer reproduces the reference ids exactly."""
    for r in golden["records"]:
        ids = tok.encode_query(r["text"]) if r["kind"] == "query" else tok.encode(r["text"])
        assert list(map(int, ids)) == r["ids"], r["text"][:60]
    assert max(len(r["ids"]) for r in golden["records"]) == 512  # one long text hits the limit


def test_batch_equals_single(tok, golden):
    texts = [r["text"] for r in golden["records"]]
    ids, cu = tok.encode_batch(texts * 30)
    for i, t in enumerate(texts * 30):
        np.testing.assert_array_equal(ids[cu[i]:cu[i + 1]], tok.encode(t))
    qids, qcu = tok.encode_batch(texts, is_query=True)
    for i, t in enumerate(texts):
        np.testing.assert_array_equal(qids[qcu[i]:qcu[i + 1]], tok.encode_query(t))


def _random_text(r, words):
    pieces = []
    for _ in range(r.integers(0, 40)):
        k = r.integers(0, 12)
        if k < 5:
            w = words[r.integers(len(words))]
            if r.random() < 0.3:
                w = w.upper() if r.random() < 0.5 else w.capitalize()
            pieces.append(w)
        elif k == 5:
            pieces.append("".join(chr(int(c)) for c in r.integers(0x4E00, 0x9FFF, r.integers(1, 4))))
        elif k == 6:  # accented Latin, Greek, Cyrillic, Turkish dotted I, final sigma
            pieces.append("".join(r.choice(list("àÉîÕüÇñÿĀăĘğİıŁœŞžΣσςΑΩЖжÅØ"), r.integers(1, 6))))
        elif k == 7:  # combining marks and punctuation
            pieces.append("é" + r.choice(["!", "?", "...", "—", "«", "»", "¿", "‘", "’", "(", ")", "#", "##"]))
        elif k == 8:  # whitespace and control characters
            pieces.append(r.choice(["\t", "\n", "\r\n", " ", "　", " ", "\x0b", "\x00", "\x7f", "\u0085",
                                    "�", "​"]))
        elif k == 9:  # a long word
            pieces.append("x" * int(r.integers(90, 130)))
        elif k == 10:  # digits, symbols, emoji
            pieces.append(r.choice(["2023", "3.14", "$100", "a+b=c", "\U0001F600", "™", "½", "ﬁ", "ẞ"]))
        else:
            pieces.append(words[r.integers(len(words))] + words[r.integers(len(words))])
    seps = r.choice([" ", "", "  "], len(pieces))
    return "".join(p + s for p, s in zip(pieces, seps))


def test_matches_python_restatement(tok, vocab_text, golden):
    ref = TokenizerRef(vocab_text)
    words = [w for w in golden["vocab_subset"].values() if w.isalpha()]
    r = np.random.Generator(np.random.PCG64(17))
    texts = [_random_text(r, words) for _ in range(1500)]
    for t in texts:
        assert list(map(int, tok.encode(t))) == ref.encode(t), repr(t)
        assert list(map(int, tok.encode_query(t))) == ref.encode(t, True), repr(t)


def test_prefix_and_truncation(tok, vocab_text):
    ref = TokenizerRef(vocab_text)
    q = list(map(int, tok.encode_query("")))
    assert q[0] == 101 and q[-1] == 102 and q[1:-1] == ref.prefix and len(ref.prefix) == 8
    assert list(map(int, tok.encode(""))) == [101, 102]
    long = " ".join(["the"] * 2000)
    ids = tok.encode(long)
    assert len(ids) == 512 and ids[0] == 101 and ids[-1] == 102
    assert QUERY_PREFIX.startswith("Represent")


def test_vocabulary_lines():
    """str::lines: "\\r\\n" endings, no empty line after a final newline; a later duplicate wins;
    "##x" lines become continuation pieces."""
    vocab = ["[PAD]"] + [f"[unused{i}]" for i in range(99)] + ["[UNK]", "[CLS]", "[SEP]", "[MASK]"]
    vocab += ["play", "##ing", "##s", "foo", "play"]
    t = BertTokenizer.from_vocab_str("\r\n".join(vocab) + "\r\n")
    assert t.vocab_size() == len(vocab)
    assert list(map(int, t.encode("playing plays foo bar"))) == [101, len(vocab) - 1, 105, len(vocab) - 1, 106, 107,
                                                                  100, 102]


def test_invalid_utf8_and_errors(tok):
    out = np.zeros(512, np.uint16)
    n = C.c_uint32()
    bad = b"abc\xff\xfe"
    code = lib().ae_tokenize(tok._h, bad, len(bad), 0, out.ctypes.data_as(C.c_void_p), 512, C.byref(n))
    assert code == -1
    code = lib().ae_tokenize(tok._h, b"hello world", 11, 0, out.ctypes.data_as(C.c_void_p), 2, C.byref(n))
    assert code == -7 and n.value == 4  # AE_ERR_CAPACITY, the needed length reported
    with pytest.raises(AeError):
        BertTokenizer.from_vocab_file(os.path.join(ROOT, "no-such-vocab.txt"))
