"""Test infrastructure only: a pure-Python restatement of the reference's BertTokenizer
(src/tokenizer.rs:25-327), used by tests/test_tokenizer.py as an independent check of the C++
tokenizer on generated text. Lowercasing uses Python's Unicode database (`str.lower` of one code
point, as `char::to_lowercase`)."""

UNK_ID, CLS_ID, SEP_ID = 100, 101, 102
MAX_SEQ_LEN = 512
MAX_WORD_CHARS = 100
QUERY_PREFIX = "Represent this sentence for searching relevant passages: "

# src/tokenizer.rs:211-222 (char::is_whitespace = White_Space)
_WS = set([0x20, 0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000]) | set(range(0x09, 0x0E)) | set(
    range(0x2000, 0x200B))


def _ws(c):
    return ord(c) in _WS


def _control(c):  # src/tokenizer.rs:214-220 (general category Cc, minus \t \n \r)
    if c in "\t\n\r":
        return False
    o = ord(c)
    return o < 0x20 or 0x7F <= o <= 0x9F


_CJK = [(0x4E00, 0x9FFF), (0x3400, 0x4DBF), (0x20000, 0x2A6DF), (0x2A700, 0x2B73F), (0x2B740, 0x2B81F),
        (0x2B820, 0x2CEAF), (0xF900, 0xFAFF), (0x2F800, 0x2FA1F)]


def _chinese(c):  # src/tokenizer.rs:224-234
    o = ord(c)
    return any(a <= o <= b for a, b in _CJK)


_PUNCT_RANGES = [(33, 47), (58, 64), (91, 96), (123, 126), (0x2000, 0x206F), (0x3000, 0x303F), (0xFE30, 0xFE6F),
                 (0xFF01, 0xFF0F), (0xFF1A, 0xFF20), (0xFF3B, 0xFF40), (0xFF5B, 0xFF65)]
_PUNCT_EXTRA = {0xA1, 0xA7, 0xAB, 0xB6, 0xB7, 0xBB, 0xBF}


def _punct(c):  # src/tokenizer.rs:237-290
    o = ord(c)
    return any(a <= o <= b for a, b in _PUNCT_RANGES) or o in _PUNCT_EXTRA


_MARKS = [(0x0300, 0x036F), (0x1AB0, 0x1AFF), (0x1DC0, 0x1DFF), (0x20D0, 0x20FF), (0xFE20, 0xFE2F)]


def _mark(c):  # src/tokenizer.rs:293-300
    o = ord(c)
    return any(a <= o <= b for a, b in _MARKS)


_ACCENTS = [(0xC0, 0xC5, "a"), (0xE0, 0xE5, "a"), (0x100, 0x104, "a"), (0xC7, 0xC7, "c"), (0xE7, 0xE7, "c"),
            (0x106, 0x10C, "c"), (0x10E, 0x10F, "d"), (0xC8, 0xCB, "e"), (0xE8, 0xEB, "e"), (0x112, 0x11A, "e"),
            (0x11C, 0x122, "g"), (0x124, 0x125, "h"), (0xCC, 0xCF, "i"), (0xEC, 0xEF, "i"), (0x128, 0x12E, "i"),
            (0x134, 0x135, "j"), (0x136, 0x137, "k"), (0x139, 0x13E, "l"), (0xD1, 0xD1, "n"), (0xF1, 0xF1, "n"),
            (0x143, 0x147, "n"), (0xD2, 0xD6, "o"), (0xF2, 0xF6, "o"), (0x14C, 0x150, "o"), (0x154, 0x158, "r"),
            (0x15A, 0x161, "s"), (0x162, 0x164, "t"), (0xD9, 0xDC, "u"), (0xF9, 0xFC, "u"), (0x168, 0x172, "u"),
            (0x174, 0x175, "w"), (0xDD, 0xDD, "y"), (0xFD, 0xFD, "y"), (0xFF, 0xFF, "y"), (0x176, 0x178, "y"),
            (0x179, 0x17E, "z")]


def _strip_accent(c):  # src/tokenizer.rs:304-327
    o = ord(c)
    for a, b, base in _ACCENTS:
        if a <= o <= b:
            return base
    return c


class TokenizerRef:
    def __init__(self, vocab_text: str):
        lines = vocab_text.split("\n")
        if vocab_text.endswith("\n"):
            lines = lines[:-1]
        self.root, self.sub = {}, {}
        for i, ln in enumerate(lines):
            if ln.endswith("\r"):
                ln = ln[:-1]
            if ln.startswith("##") and len(ln) > 2:
                self.sub[ln[2:]] = i
            self.root[ln] = i
        self.prefix = []
        self._raw(QUERY_PREFIX, self.prefix)

    def _raw(self, text, out):  # encode_raw_into, src/tokenizer.rs:103-150
        norm = []
        for ch in text:
            if ch == "\0" or ch == "\ufffd" or _control(ch):
                continue
            if _ws(ch):
                norm.append(" ")
                continue
            if _chinese(ch):
                norm += [" ", ch, " "]
                continue
            if _mark(ch):
                continue
            for lc in _strip_accent(ch).lower():
                if not _mark(lc):
                    norm.append(lc)
        word = []
        for ch in norm:
            if ch == " ":
                self._wp("".join(word), out)
                word = []
            elif _punct(ch):
                self._wp("".join(word), out)
                word = []
                self._wp(ch, out)
            else:
                word.append(ch)
        self._wp("".join(word), out)

    def _wp(self, word, out):  # wordpiece_into, src/tokenizer.rs:152-201
        if not word:
            return
        if word in self.root:
            out.append(self.root[word])
            return
        if len(word) > MAX_WORD_CHARS:
            out.append(UNK_ID)
            return
        n0, start = len(out), 0
        while start < len(word):
            end, hit = len(word), None
            while end > start:
                piece = word[start:end]
                hit = (self.root if start == 0 else self.sub).get(piece)
                if hit is not None:
                    break
                end -= 1
            if hit is None:
                del out[n0:]
                out.append(UNK_ID)
                return
            out.append(hit)
            start = end

    def encode(self, text, is_query=False):  # encode_into, src/tokenizer.rs:90-101
        out = [CLS_ID] + (list(self.prefix) if is_query else [])
        self._raw(text, out)
        if len(out) >= MAX_SEQ_LEN:
            out = out[: MAX_SEQ_LEN - 1]
        out.append(SEP_ID)
        return out
