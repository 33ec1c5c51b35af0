// BERT WordPiece tokenizer of arctic-embed-s (host side of the embedding path): BertTokenizer,
// src/tokenizer.rs:25-327, behind the C ABI in include/arctic_cuda.h.
//
//   normalizer      src/tokenizer.rs:103-127  drop NUL / U+FFFD / control characters, whitespace
//                   -> ' ', CJK ideographs padded with spaces, combining marks dropped, Latin-1 /
//                   Latin Extended-A accents stripped, then lowercased (combining marks in the
//                   lowercase output dropped too)
//   pre-tokenizer   src/tokenizer.rs:129-149  split on ' ', every punctuation character is a word
//   WordPiece       src/tokenizer.rs:152-201  whole-word lookup, > 100 characters -> [UNK], then
//                   greedy longest match with "##" continuation pieces; no match -> one [UNK]
//   encode          src/tokenizer.rs:74-101   [CLS] (+ query prefix) ... [SEP], at most 512 ids
//
// The vocabulary lives in two open-addressing tables over one byte arena (whole tokens, and the
// "##" pieces without their prefix), so lookups of word slices allocate nothing.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "../../include/arctic_cuda.h"
#include "unicode_tables.h"

namespace {

constexpr uint16_t kUnkId = 100;
constexpr uint16_t kClsId = 101;
constexpr uint16_t kSepId = 102;
constexpr size_t kMaxSeqLen = 512;
constexpr size_t kMaxWordChars = 100;

thread_local std::string g_tok_err;

int tok_fail(int code, const char* msg) {
  g_tok_err = msg;
  return code;
}

// ---------------------------------------------------------------------------------------- vocab
class StrTable {
 public:
  void build(const std::vector<std::pair<std::string, uint16_t>>& entries) {
    size_t cap = 16;
    while (cap < entries.size() * 2) cap <<= 1;
    slots_.assign(cap, Slot{0, 0, 0, 0});
    mask_ = cap - 1;
    arena_.clear();
    for (const auto& e : entries) insert(e.first.data(), e.first.size(), e.second);
  }
  // id of the token with these bytes, or -1
  int find(const char* p, size_t n) const {
    if (slots_.empty()) return -1;
    for (size_t i = hash(p, n) & mask_;; i = (i + 1) & mask_) {
      const Slot& s = slots_[i];
      if (!s.used) return -1;
      if (s.len == n && std::memcmp(arena_.data() + s.off, p, n) == 0) return s.id;
    }
  }

 private:
  struct Slot {
    uint32_t off;
    uint32_t len;
    uint16_t id;
    uint16_t used;
  };
  static uint64_t hash(const char* p, size_t n) {  // FNV-1a
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; ++i) h = (h ^ uint8_t(p[i])) * 1099511628211ull;
    return h ^ (h >> 29);
  }
  void insert(const char* p, size_t n, uint16_t id) {  // a later duplicate replaces the id
    for (size_t i = hash(p, n) & mask_;; i = (i + 1) & mask_) {
      Slot& s = slots_[i];
      if (!s.used) {
        s = Slot{uint32_t(arena_.size()), uint32_t(n), id, 1};
        arena_.append(p, n);
        return;
      }
      if (s.len == n && std::memcmp(arena_.data() + s.off, p, n) == 0) {
        s.id = id;
        return;
      }
    }
  }
  std::vector<Slot> slots_;
  std::string arena_;
  size_t mask_ = 0;
};

// ------------------------------------------------------------------------------------- unicode
// UTF-8 -> code points; false on malformed input (overlong, surrogate, > U+10FFFF, truncated).
bool decode_utf8(const char* s, size_t n, std::u32string* out) {
  out->clear();
  out->reserve(n);
  const auto* u = reinterpret_cast<const uint8_t*>(s);
  for (size_t i = 0; i < n;) {
    const uint32_t b = u[i];
    uint32_t cp, len;
    if (b < 0x80) {
      cp = b, len = 1;
    } else if ((b & 0xE0) == 0xC0) {
      cp = b & 0x1F, len = 2;
    } else if ((b & 0xF0) == 0xE0) {
      cp = b & 0x0F, len = 3;
    } else if ((b & 0xF8) == 0xF0) {
      cp = b & 0x07, len = 4;
    } else {
      return false;
    }
    if (i + len > n) return false;
    for (uint32_t k = 1; k < len; ++k) {
      if ((u[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (u[i + k] & 0x3F);
    }
    static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
    if (cp < kMin[len] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    out->push_back(cp);
    i += len;
  }
  return true;
}

void append_utf8(std::string* s, uint32_t cp) {
  if (cp < 0x80) {
    s->push_back(char(cp));
  } else if (cp < 0x800) {
    s->push_back(char(0xC0 | (cp >> 6)));
    s->push_back(char(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    s->push_back(char(0xE0 | (cp >> 12)));
    s->push_back(char(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back(char(0x80 | (cp & 0x3F)));
  } else {
    s->push_back(char(0xF0 | (cp >> 18)));
    s->push_back(char(0x80 | ((cp >> 12) & 0x3F)));
    s->push_back(char(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back(char(0x80 | (cp & 0x3F)));
  }
}

// char::is_whitespace: the Unicode White_Space property.
bool is_whitespace(uint32_t c) {
  return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F ||
         c == 0x3000;
}

// is_bert_control: general category Cc, except tab, newline and carriage return.
bool is_control(uint32_t c) {
  if (c == '\t' || c == '\n' || c == '\r') return false;
  return c < 0x20 || (c >= 0x7F && c <= 0x9F);
}

bool is_chinese_char(uint32_t c) {
  return (c >= 0x4E00 && c <= 0x9FFF) || (c >= 0x3400 && c <= 0x4DBF) || (c >= 0x20000 && c <= 0x2A6DF) ||
         (c >= 0x2A700 && c <= 0x2B73F) || (c >= 0x2B740 && c <= 0x2B81F) || (c >= 0x2B820 && c <= 0x2CEAF) ||
         (c >= 0xF900 && c <= 0xFAFF) || (c >= 0x2F800 && c <= 0x2FA1F);
}

bool is_punctuation(uint32_t c) {
  if ((c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) || (c >= 123 && c <= 126)) return true;
  if ((c >= 0x2000 && c <= 0x206F) || (c >= 0x3000 && c <= 0x303F) || (c >= 0xFE30 && c <= 0xFE6F) ||
      (c >= 0xFF01 && c <= 0xFF0F) || (c >= 0xFF1A && c <= 0xFF20) || (c >= 0xFF3B && c <= 0xFF40) ||
      (c >= 0xFF5B && c <= 0xFF65))
    return true;
  // Latin-1 punctuation named by the reference (the U+20xx ones fall in the range above)
  return c == 0xA1 || c == 0xA7 || c == 0xAB || c == 0xB6 || c == 0xB7 || c == 0xBB || c == 0xBF;
}

bool is_combining_mark(uint32_t c) {
  return (c >= 0x0300 && c <= 0x036F) || (c >= 0x1AB0 && c <= 0x1AFF) || (c >= 0x1DC0 && c <= 0x1DFF) ||
         (c >= 0x20D0 && c <= 0x20FF) || (c >= 0xFE20 && c <= 0xFE2F);
}

// strip_latin_accent: precomposed Latin-1 / Latin Extended-A letters (U+00C0..U+017F) named by the
// reference -> their base letter; everything else unchanged.
uint32_t strip_latin_accent(uint32_t c) {
  if (c < 0xC0 || c > 0x17F) return c;
  struct R {
    uint16_t lo, hi;
    char base;
  };
  static const R kRanges[] = {
      {0xC0, 0xC5, 'a'},   {0xE0, 0xE5, 'a'},   {0x100, 0x104, 'a'}, {0xC7, 0xC7, 'c'},   {0xE7, 0xE7, 'c'},
      {0x106, 0x10C, 'c'}, {0x10E, 0x10F, 'd'}, {0xC8, 0xCB, 'e'},   {0xE8, 0xEB, 'e'},   {0x112, 0x11A, 'e'},
      {0x11C, 0x122, 'g'}, {0x124, 0x125, 'h'}, {0xCC, 0xCF, 'i'},   {0xEC, 0xEF, 'i'},   {0x128, 0x12E, 'i'},
      {0x134, 0x135, 'j'}, {0x136, 0x137, 'k'}, {0x139, 0x13E, 'l'}, {0xD1, 0xD1, 'n'},   {0xF1, 0xF1, 'n'},
      {0x143, 0x147, 'n'}, {0xD2, 0xD6, 'o'},   {0xF2, 0xF6, 'o'},   {0x14C, 0x150, 'o'}, {0x154, 0x158, 'r'},
      {0x15A, 0x161, 's'}, {0x162, 0x164, 't'}, {0xD9, 0xDC, 'u'},   {0xF9, 0xFC, 'u'},   {0x168, 0x172, 'u'},
      {0x174, 0x175, 'w'}, {0xDD, 0xDD, 'y'},   {0xFD, 0xFD, 'y'},   {0xFF, 0xFF, 'y'},   {0x176, 0x178, 'y'},
      {0x179, 0x17E, 'z'},
  };
  for (const R& r : kRanges)
    if (c >= r.lo && c <= r.hi) return uint32_t(r.base);
  return c;
}

// char::to_lowercase of one code point: one or two code points (second 0 if absent).
void to_lower(uint32_t c, uint32_t* a, uint32_t* b) {
  const ae::LowerMap* end = ae::kLowerMap + ae::kLowerMapSize;
  const ae::LowerMap* it =
      std::lower_bound(ae::kLowerMap, end, c, [](const ae::LowerMap& m, uint32_t v) { return m.cp < v; });
  if (it != end && it->cp == c) {
    *a = it->lo0;
    *b = it->lo1;
  } else {
    *a = c;
    *b = 0;
  }
}

}  // namespace

struct ae_tokenizer {
  StrTable root;      // every vocabulary line
  StrTable sub;       // "##x" lines, keyed by x
  uint32_t vocab_size = 0;
  std::vector<uint16_t> prefix_ids;

  // encode_raw_into (src/tokenizer.rs:103-150)
  bool encode_raw(const char* text, size_t len, std::vector<uint16_t>* out) const {
    std::u32string cps;
    if (!decode_utf8(text, len, &cps)) return false;
    std::u32string norm;
    norm.reserve(cps.size() + 16);
    for (uint32_t ch : cps) {
      if (ch == 0 || ch == 0xFFFD || is_control(ch)) continue;
      if (is_whitespace(ch)) {
        norm.push_back(' ');
        continue;
      }
      if (is_chinese_char(ch)) {
        norm.push_back(' ');
        norm.push_back(ch);
        norm.push_back(' ');
        continue;
      }
      if (is_combining_mark(ch)) continue;
      uint32_t a, b;
      to_lower(strip_latin_accent(ch), &a, &b);
      if (!is_combining_mark(a)) norm.push_back(a);
      if (b && !is_combining_mark(b)) norm.push_back(b);
    }
    std::string word;  // UTF-8 bytes of the current word
    auto flush = [&]() {
      if (!word.empty()) wordpiece(word, out);
      word.clear();
    };
    for (uint32_t ch : norm) {
      if (ch == ' ') {
        flush();
      } else if (is_punctuation(ch)) {
        flush();
        append_utf8(&word, ch);
        flush();
      } else {
        append_utf8(&word, ch);
      }
    }
    flush();
    return true;
  }

  // wordpiece_into (src/tokenizer.rs:152-201)
  void wordpiece(const std::string& w, std::vector<uint16_t>* out) const {
    const int whole = root.find(w.data(), w.size());
    if (whole >= 0) {
      out->push_back(uint16_t(whole));
      return;
    }
    size_t chars = 0;
    for (unsigned char c : w) chars += (c & 0xC0) != 0x80;
    if (chars > kMaxWordChars) {
      out->push_back(kUnkId);
      return;
    }
    const size_t start_len = out->size();
    size_t start = 0;
    while (start < w.size()) {
      size_t end = w.size();
      int id = -1;
      while (end > start) {
        id = start == 0 ? root.find(w.data(), end) : sub.find(w.data() + start, end - start);
        if (id >= 0) break;
        --end;  // back to the previous character boundary
        while (end > start && (uint8_t(w[end]) & 0xC0) == 0x80) --end;
      }
      if (id < 0) {
        out->resize(start_len);
        out->push_back(kUnkId);
        return;
      }
      out->push_back(uint16_t(id));
      start = end;
    }
  }

  // encode_into (src/tokenizer.rs:90-101)
  bool encode(const char* text, size_t len, bool is_query, std::vector<uint16_t>* out) const {
    out->clear();
    out->push_back(kClsId);
    if (is_query) out->insert(out->end(), prefix_ids.begin(), prefix_ids.end());
    if (!encode_raw(text, len, out)) return false;
    if (out->size() >= kMaxSeqLen) out->resize(kMaxSeqLen - 1);
    out->push_back(kSepId);
    return true;
  }
};

namespace {

// from_vocab_str (src/tokenizer.rs:40-68): str::lines semantics (split at '\n', one trailing '\r'
// removed, no empty line after a final '\n').
int build_tokenizer(const char* text, size_t len, ae_tokenizer** out) {
  std::vector<std::pair<std::string, uint16_t>> roots, subs;
  size_t pos = 0, id = 0;
  while (pos < len) {
    size_t e = pos;
    while (e < len && text[e] != '\n') ++e;
    size_t le = e;
    if (le > pos && text[le - 1] == '\r') --le;
    if (id > 65535) return tok_fail(AE_ERR_INVALID_ARG, "vocabulary has more than 65,536 lines");
    std::string tok(text + pos, le - pos);
    if (tok.size() > 2 && tok[0] == '#' && tok[1] == '#') subs.emplace_back(tok.substr(2), uint16_t(id));
    roots.emplace_back(std::move(tok), uint16_t(id));
    ++id;
    pos = e + 1;
  }
  if (id == 0) return tok_fail(AE_ERR_INVALID_ARG, "empty vocabulary");
  auto* t = new ae_tokenizer();
  t->root.build(roots);
  t->sub.build(subs);
  t->vocab_size = uint32_t(id);
  const char* prefix = AE_QUERY_PREFIX;
  t->encode_raw(prefix, std::strlen(prefix), &t->prefix_ids);
  *out = t;
  return AE_OK;
}

}  // namespace

extern "C" {

int ae_tokenizer_create_from_vocab(const char* vocab_text, size_t len, ae_tokenizer** out) {
  if (!vocab_text || !out) return tok_fail(AE_ERR_INVALID_ARG, "null pointer");
  *out = nullptr;
  return build_tokenizer(vocab_text, len, out);
}

int ae_tokenizer_create_from_file(const char* vocab_path, ae_tokenizer** out) {
  if (!vocab_path || !out) return tok_fail(AE_ERR_INVALID_ARG, "null pointer");
  *out = nullptr;
  FILE* f = std::fopen(vocab_path, "rb");
  if (!f) return tok_fail(AE_ERR_INVALID_ARG, "cannot open the vocabulary file");
  std::string text;
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
  std::fclose(f);
  return build_tokenizer(text.data(), text.size(), out);
}

int ae_tokenizer_destroy(ae_tokenizer* tok) {
  delete tok;
  return AE_OK;
}

uint32_t ae_tokenizer_vocab_size(const ae_tokenizer* tok) { return tok ? tok->vocab_size : 0; }

const char* ae_tokenizer_last_error(void) { return g_tok_err.c_str(); }

int ae_tokenize(const ae_tokenizer* tok, const char* text, size_t len, int is_query, uint16_t* ids, uint32_t cap,
                uint32_t* n_ids) {
  if (!tok || (!text && len) || !ids || !n_ids) return AE_ERR_INVALID_ARG;
  std::vector<uint16_t> v;
  if (!tok->encode(text ? text : "", len, is_query != 0, &v)) return AE_ERR_INVALID_ARG;
  *n_ids = uint32_t(v.size());
  if (v.size() > cap) return AE_ERR_CAPACITY;
  std::memcpy(ids, v.data(), v.size() * 2);
  return AE_OK;
}

int ae_tokenize_batch(const ae_tokenizer* tok, const char* const* texts, const size_t* lens, uint32_t n,
                      int is_query, uint16_t* ids, size_t ids_cap, uint32_t* cu_seqlens) {
  if (!tok || (n && (!texts || !lens || !ids)) || !cu_seqlens) return AE_ERR_INVALID_ARG;
  std::vector<std::vector<uint16_t>> enc(n);
  std::atomic<int> bad{0};
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  const unsigned workers = std::max(1u, std::min<unsigned>(hw, (n + 255) / 256));
  auto run = [&](unsigned w) {
    for (uint32_t i = w; i < n; i += workers)
      if (!tok->encode(texts[i] ? texts[i] : "", texts[i] ? lens[i] : 0, is_query != 0, &enc[i])) bad = 1;
  };
  std::vector<std::thread> th;
  for (unsigned w = 1; w < workers; ++w) th.emplace_back(run, w);
  run(0);
  for (auto& t : th) t.join();
  if (bad) return AE_ERR_INVALID_ARG;
  size_t total = 0;
  cu_seqlens[0] = 0;
  for (uint32_t i = 0; i < n; ++i) {
    total += enc[i].size();
    if (total > 0xFFFFFFFFull) return AE_ERR_CAPACITY;
    cu_seqlens[i + 1] = uint32_t(total);
  }
  if (total > ids_cap) return AE_ERR_CAPACITY;
  for (uint32_t i = 0; i < n; ++i) std::memcpy(ids + cu_seqlens[i], enc[i].data(), enc[i].size() * 2);
  return AE_OK;
}

}  // extern "C"
