// tokenizer.cpp - the reference's BPE tokenizer in C++ (src/snai_tokenizer.php).
//
// The PHP host encodes the prompt and decodes every generated id in PHP
// (src/snai_inference.php:107-115, :201-208); this is the same tokenizer as
// library calls, so a host loop needs no PHP string work per token.
//
// Kept from src/snai_tokenizer.php, step for step:
//   :23-38    vocab = model.vocab of the HF-style JSON, merge ranks "a b" ->
//             index in model.merges (a later duplicate overwrites), the
//             inverse map (a later token with the same id overwrites)
//   :56-116   bpe(): code points, repeatedly merge every occurrence (left to
//             right) of the lowest-ranked adjacent pair, memoised per chunk
//   :118-185  encode(): invalid UTF-8 -> '?'; a leading ' ' unless the text
//             starts with ' ', '[' or '<'; split on the special tokens the
//             vocab has (leftmost match, first in list order at a position);
//             ' ' -> U+2581; chunks (U+2581|\n)[^U+2581\n]* (text before a
//             part's first U+2581 or \n is dropped, as preg_match_all
//             drops it); pieces looked up, <unk> (else 0) when missing
//   :187-199  decode(): concatenate, U+2581 -> ' ', optional trim
// NFKC (:128-130) runs in PHP only when the intl extension is loaded; it is
// not applied here (the same as a PHP build without intl).
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/cortex.h"
#include "engine.h"

namespace snai {
namespace {

const char kMeta[] = "\xE2\x96\x81";  // U+2581
const char *const kSpecials[] = {"<unk>", "<pad>", "<s>", "</s>", "\n", "[USER]", "[SYMBIO]", "[SYSTEM]"};

// ---- a small JSON reader: just what the vocabulary file needs ----
struct JsonReader {
  const char *p, *end;
  std::string err;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const char *m) {
    if (err.empty()) err = m;
    return false;
  }
  bool expect(char c) {
    ws();
    if (p >= end || *p != c) return fail("unexpected character");
    ++p;
    return true;
  }
  static void put_utf8(std::string &s, unsigned cp) {
    if (cp < 0x80) {
      s.push_back((char)cp);
    } else if (cp < 0x800) {
      s.push_back((char)(0xC0 | (cp >> 6)));
      s.push_back((char)(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
      s.push_back((char)(0xE0 | (cp >> 12)));
      s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      s.push_back((char)(0x80 | (cp & 0x3F)));
    } else {
      s.push_back((char)(0xF0 | (cp >> 18)));
      s.push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
      s.push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
      s.push_back((char)(0x80 | (cp & 0x3F)));
    }
  }
  bool hex4(unsigned *v) {
    if (end - p < 4) return fail("short \\u escape");
    unsigned x = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = p[i];
      x <<= 4;
      if (c >= '0' && c <= '9') x |= (unsigned)(c - '0');
      else if (c >= 'a' && c <= 'f') x |= (unsigned)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') x |= (unsigned)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    p += 4;
    *v = x;
    return true;
  }
  bool string(std::string *out) {
    ws();
    if (p >= end || *p != '"') return fail("string expected");
    ++p;
    out->clear();
    while (p < end && *p != '"') {
      if (*p != '\\') {
        out->push_back(*p++);
        continue;
      }
      if (++p >= end) return fail("unterminated escape");
      const char c = *p++;
      switch (c) {
        case '"': out->push_back('"'); break;
        case '\\': out->push_back('\\'); break;
        case '/': out->push_back('/'); break;
        case 'b': out->push_back('\b'); break;
        case 'f': out->push_back('\f'); break;
        case 'n': out->push_back('\n'); break;
        case 'r': out->push_back('\r'); break;
        case 't': out->push_back('\t'); break;
        case 'u': {
          unsigned cp;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
            p += 2;
            unsigned lo;
            if (!hex4(&lo)) return false;
            if (lo >= 0xDC00 && lo < 0xE000) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(*out, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool number(long long *v) {
    ws();
    char *e = nullptr;
    const long long x = strtoll(p, &e, 10);
    if (e == p) return fail("number expected");
    p = e;
    while (p < end && (*p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-' || (*p >= '0' && *p <= '9'))) ++p;
    *v = x;
    return true;
  }
  // Skips any value.
  bool skip() {
    ws();
    if (p >= end) return fail("value expected");
    if (*p == '"') {
      std::string s;
      return string(&s);
    }
    if (*p == '{' || *p == '[') {
      const char close = *p == '{' ? '}' : ']';
      const bool obj = *p == '{';
      ++p;
      ws();
      if (p < end && *p == close) {
        ++p;
        return true;
      }
      for (;;) {
        if (obj) {
          std::string k;
          if (!string(&k) || !expect(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (p < end && *p == ',') {
          ++p;
          continue;
        }
        return expect(close);
      }
    }
    while (p < end && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n' && *p != '\r' && *p != '\t') ++p;
    return true;
  }
  // Calls f(key) for every member of an object; f consumes the value.
  template <class F>
  bool object(F &&f) {
    if (!expect('{')) return false;
    ws();
    if (p < end && *p == '}') {
      ++p;
      return true;
    }
    for (;;) {
      std::string k;
      if (!string(&k) || !expect(':') || !f(k)) return false;
      ws();
      if (p < end && *p == ',') {
        ++p;
        continue;
      }
      return expect('}');
    }
  }
  template <class F>
  bool array(F &&f) {
    if (!expect('[')) return false;
    ws();
    if (p < end && *p == ']') {
      ++p;
      return true;
    }
    for (;;) {
      if (!f()) return false;
      ws();
      if (p < end && *p == ',') {
        ++p;
        continue;
      }
      return expect(']');
    }
  }
};

// Memo of bpe() per chunk: open addressing over FNV-1a hashes, keys and ids
// in two arenas (a chunk is a few bytes; a node-based map spends more time
// chasing its nodes than hashing).
struct ChunkCache {
  struct Slot {
    uint64_t h = 0;
    uint32_t key = 0, klen = 0, ids = 0, n = 0;
    bool used = false;
  };
  std::vector<Slot> slots = std::vector<Slot>(1024);
  std::string keys;
  std::vector<int> ids;
  size_t count = 0;

  static uint64_t hash(const std::string &k) {
    uint64_t h = 1469598103934665603ull;
    for (unsigned char c : k) h = (h ^ c) * 1099511628211ull;
    return h;
  }
  // the ids of `k` (hash h) as (first, count) into `ids`, or false
  bool find(const std::string &k, uint64_t h, uint32_t *first, uint32_t *n) const {
    const size_t mask = slots.size() - 1;
    for (size_t i = h & mask;; i = (i + 1) & mask) {
      const Slot &s = slots[i];
      if (!s.used) return false;
      if (s.h == h && s.klen == k.size() && keys.compare(s.key, s.klen, k) == 0) {
        *first = s.ids;
        *n = s.n;
        return true;
      }
    }
  }
  void insert(const std::string &k, uint64_t h, const std::vector<int> &v, uint32_t *first) {
    if (2 * (count + 1) > slots.size()) {
      std::vector<Slot> old(2 * slots.size());
      old.swap(slots);
      const size_t mask = slots.size() - 1;
      for (const Slot &s : old)
        if (s.used) {
          size_t i = s.h & mask;
          while (slots[i].used) i = (i + 1) & mask;
          slots[i] = s;
        }
    }
    const size_t mask = slots.size() - 1;
    size_t i = h & mask;
    while (slots[i].used) i = (i + 1) & mask;
    Slot &s = slots[i];
    s.used = true;
    s.h = h;
    s.key = (uint32_t)keys.size();
    s.klen = (uint32_t)k.size();
    keys += k;
    s.ids = (uint32_t)ids.size();
    s.n = (uint32_t)v.size();
    ids.insert(ids.end(), v.begin(), v.end());
    ++count;
    *first = s.ids;
  }
};

struct Tokenizer {
  std::unordered_map<std::string, int> vocab;
  std::vector<std::pair<std::string, int>> vocab_order;  // key order of the file (first occurrence)
  std::unordered_map<int, std::string> inverse;
  std::vector<const std::string *> inverse_dense;  // inverse[] by id for ids in [0, 2^22), else via the map
  std::unordered_map<std::string, int> ranks;
  ChunkCache cache;  // chunk -> ids
  std::vector<std::string> specials;  // the special tokens the vocab has, in list order
  std::vector<int> special_ids;       // and their ids
  int unk = 0;
  std::mutex mu;
};

bool load_vocab(Tokenizer *t, const std::string &text, std::string *err) {
  JsonReader r{text.data(), text.data() + text.size(), {}};
  bool have_vocab = false;
  const bool ok = r.object([&](const std::string &k) {
    if (k != "model") return r.skip();
    return r.object([&](const std::string &mk) {
      if (mk == "vocab") {
        have_vocab = true;
        return r.object([&](const std::string &tok) {
          long long id;
          if (!r.number(&id)) return false;
          auto it = t->vocab.find(tok);
          if (it == t->vocab.end()) {
            t->vocab.emplace(tok, (int)id);
            t->vocab_order.push_back({tok, (int)id});
          } else {
            it->second = (int)id;  // a later duplicate key overwrites (json_decode)
            for (auto &kv : t->vocab_order)
              if (kv.first == tok) kv.second = (int)id;
          }
          return true;
        });
      }
      if (mk == "merges") {
        int i = 0;
        return r.array([&]() {
          r.ws();
          std::string key;
          if (r.p < r.end && *r.p == '[') {
            std::vector<std::string> parts;
            if (!r.array([&]() {
                  std::string s;
                  if (!r.string(&s)) return false;
                  parts.push_back(s);
                  return true;
                }))
              return false;
            for (size_t j = 0; j < parts.size(); ++j) key += (j ? " " : "") + parts[j];
          } else if (!r.string(&key)) {
            return false;
          }
          t->ranks[key] = i++;  // a later duplicate overwrites
          return true;
        });
      }
      return r.skip();
    });
  });
  if (!ok || !have_vocab) {
    *err = ok ? "no model.vocab in the file" : r.err;
    return false;
  }
  for (const auto &kv : t->vocab_order) t->inverse[kv.second] = kv.first;  // array_flip: later keys win
  int top = -1;
  for (const auto &kv : t->inverse)
    if (kv.first >= 0 && kv.first < (1 << 22)) top = std::max(top, kv.first);
  t->inverse_dense.assign((size_t)(top + 1), nullptr);
  for (const auto &kv : t->inverse)
    if (kv.first >= 0 && kv.first < (1 << 22)) t->inverse_dense[kv.first] = &kv.second;
  for (const char *s : kSpecials) {
    auto it = t->vocab.find(s);
    if (it != t->vocab.end()) {
      t->specials.push_back(s);
      t->special_ids.push_back(it->second);
    }
  }
  auto u = t->vocab.find("<unk>");
  t->unk = u == t->vocab.end() ? 0 : u->second;
  return true;
}

// mb_convert_encoding(text, 'UTF-8', 'UTF-8'): each invalid sequence
// (maximal subpart) becomes '?'.
std::string sanitize_utf8(const char *s, size_t n) {
  std::string out;
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    const unsigned char b = (unsigned char)s[i];
    if (b < 0x80) {
      // a run of ASCII bytes, eight at a time, copied at once
      size_t j = i + 1;
      while (j + 8 <= n) {
        uint64_t w;
        memcpy(&w, s + j, 8);
        if (w & 0x8080808080808080ull) break;
        j += 8;
      }
      while (j < n && (unsigned char)s[j] < 0x80) ++j;
      out.append(s + i, j - i);
      i = j;
      continue;
    }
    int need;
    unsigned char lo = 0x80, hi = 0xBF;
    if (b >= 0xC2 && b <= 0xDF) need = 1;
    else if (b == 0xE0) need = 2, lo = 0xA0;
    else if ((b >= 0xE1 && b <= 0xEC) || b == 0xEE || b == 0xEF) need = 2;
    else if (b == 0xED) need = 2, hi = 0x9F;
    else if (b == 0xF0) need = 3, lo = 0x90;
    else if (b >= 0xF1 && b <= 0xF3) need = 3;
    else if (b == 0xF4) need = 3, hi = 0x8F;
    else {
      out.push_back('?');
      ++i;
      continue;
    }
    size_t j = i + 1;
    bool ok = true;
    for (int k = 0; k < need; ++k) {
      if (j >= n) {
        ok = false;
        break;
      }
      const unsigned char c = (unsigned char)s[j];
      const unsigned char l = k == 0 ? lo : 0x80, h = k == 0 ? hi : 0xBF;
      if (c < l || c > h) {
        ok = false;
        break;
      }
      ++j;
    }
    if (ok) {
      out.append(s + i, j - i);
      i = j;
    } else {
      out.push_back('?');
      i = j > i + 1 ? j : i + 1;
    }
  }
  return out;
}

size_t utf8_len(unsigned char b) { return b < 0x80 ? 1 : b < 0xE0 ? 2 : b < 0xF0 ? 3 : 4; }

// :56-116 bpe() of one chunk, as vocabulary ids (memoised), appended to out.
void bpe_ids(Tokenizer &t, const std::string &chunk, std::vector<int> *out) {
  const uint64_t h = ChunkCache::hash(chunk);
  uint32_t first = 0, cnt = 0;
  if (t.cache.find(chunk, h, &first, &cnt)) {
    out->insert(out->end(), t.cache.ids.begin() + first, t.cache.ids.begin() + first + cnt);
    return;
  }
  std::vector<std::string> word;
  for (size_t i = 0; i < chunk.size();) {
    const size_t l = std::min(utf8_len((unsigned char)chunk[i]), chunk.size() - i);
    word.push_back(chunk.substr(i, l));
    i += l;
  }
  while (word.size() >= 2) {
    int best = -1;
    size_t bi = 0;
    for (size_t i = 0; i + 1 < word.size(); ++i) {
      auto it = t.ranks.find(word[i] + " " + word[i + 1]);
      if (it != t.ranks.end() && (best < 0 || it->second < best)) {
        best = it->second;
        bi = i;
      }
    }
    if (best < 0) break;
    const std::string first = word[bi], second = word[bi + 1];
    std::vector<std::string> nw;
    nw.reserve(word.size());
    for (size_t i = 0; i < word.size();) {
      if (i + 1 < word.size() && word[i] == first && word[i + 1] == second) {
        nw.push_back(first + second);
        i += 2;
      } else {
        nw.push_back(word[i]);
        i += 1;
      }
    }
    word.swap(nw);
  }
  std::vector<int> ids;
  for (const std::string &piece : word) {
    auto v = t.vocab.find(piece);
    ids.push_back(v == t.vocab.end() ? t.unk : v->second);
  }
  t.cache.insert(chunk, h, ids, &first);
  out->insert(out->end(), ids.begin(), ids.end());
}

void encode(Tokenizer &t, const char *text, size_t n, std::vector<int> *out) {
  std::string s = sanitize_utf8(text, n);
  if (!s.empty() && s[0] != ' ' && s[0] != '[' && s[0] != '<') s.insert(s.begin(), ' ');
  // the text between special tokens in chunks: a U+2581 (a space becomes
  // one) or \n, then everything up to the next one; the key is the chunk
  // with its space written as U+2581 (text before a part's first chunk
  // start is dropped)
  std::string key;
  auto chunks = [&](size_t a, size_t b) {
    auto is_start = [&](size_t k) {
      return s[k] == ' ' || s[k] == '\n' || (s[k] == kMeta[0] && k + 3 <= b && s.compare(k, 3, kMeta) == 0);
    };
    size_t i = a;
    while (i < b && !is_start(i)) ++i;
    while (i < b) {
      size_t j = i + (s[i] == kMeta[0] ? 3 : 1);
      while (j < b && !is_start(j)) ++j;
      key.clear();
      if (s[i] == ' ') {
        key.append(kMeta, 3);
        key.append(s, i + 1, j - i - 1);
      } else {
        key.append(s, i, j - i);
      }
      bpe_ids(t, key, out);
      i = j;
    }
  };
  // split on the special tokens (leftmost match; first in list order there);
  // only a position holding some special's first byte can start one
  bool lead[256] = {};
  for (const std::string &sp : t.specials) lead[(unsigned char)sp[0]] = true;
  size_t start = 0, pos = 0;
  while (pos < s.size()) {
    int hit = -1;
    if (lead[(unsigned char)s[pos]])
      for (size_t k = 0; k < t.specials.size(); ++k)
        if (s.compare(pos, t.specials[k].size(), t.specials[k]) == 0) {
          hit = (int)k;
          break;
        }
    if (hit < 0) {
      ++pos;
      continue;
    }
    if (pos > start) chunks(start, pos);
    out->push_back(t.special_ids[hit]);
    pos += t.specials[hit].size();
    start = pos;
  }
  if (start < s.size()) chunks(start, s.size());
}

}  // namespace
}  // namespace snai

using namespace snai;

extern "C" void *cortex_tokenizer_load(const char *vocab_json) {
  clear_error();
  FILE *f = vocab_json ? fopen(vocab_json, "rb") : nullptr;
  if (!f) {
    set_error("cannot open the vocabulary %s", vocab_json ? vocab_json : "(null)");
    return nullptr;
  }
  std::string text;
  char buf[1 << 16];
  size_t r;
  while ((r = fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, r);
  fclose(f);
  Tokenizer *t = new Tokenizer();
  std::string err;
  if (!load_vocab(t, text, &err)) {
    set_error("%s: %s", vocab_json, err.c_str());
    delete t;
    return nullptr;
  }
  return t;
}

extern "C" void cortex_tokenizer_free(void *tok) { delete static_cast<Tokenizer *>(tok); }

extern "C" int cortex_tokenizer_vocab_size(void *tok) {
  return tok ? (int)static_cast<Tokenizer *>(tok)->vocab.size() : 0;
}

extern "C" int cortex_tokenizer_encode(void *tok, const char *text, int text_len, int *ids, int max_ids) {
  clear_error();
  if (!tok || (!text && text_len != 0)) {
    set_error("tokenizer and text must not be NULL");
    return -1;
  }
  Tokenizer &t = *static_cast<Tokenizer *>(tok);
  std::vector<int> out;
  {
    std::lock_guard<std::mutex> g(t.mu);
    encode(t, text ? text : "", text_len < 0 ? strlen(text) : (size_t)text_len, &out);
  }
  const int n = (int)out.size();
  if (ids)
    for (int i = 0; i < n && i < max_ids; ++i) ids[i] = out[i];
  return n;
}

extern "C" int cortex_tokenizer_decode(void *tok, const int *ids, int n, int trim, char *out, int max_bytes) {
  clear_error();
  if (!tok || (!ids && n > 0)) {
    set_error("tokenizer and ids must not be NULL");
    return -1;
  }
  Tokenizer &t = *static_cast<Tokenizer *>(tok);
  std::string s;
  for (int i = 0; i < n; ++i) {
    const int id = ids[i];
    if (id >= 0 && (size_t)id < t.inverse_dense.size()) {
      if (const std::string *p = t.inverse_dense[id]) s += *p;
    } else if (id < 0 || id >= (1 << 22)) {
      auto it = t.inverse.find(id);
      if (it != t.inverse.end()) s += it->second;
    }
  }
  std::string o;
  o.reserve(s.size());
  for (size_t i = 0; i < s.size();) {
    if (s[i] == kMeta[0] && s.compare(i, 3, kMeta) == 0) {
      o.push_back(' ');
      i += 3;
    } else {
      o.push_back(s[i++]);
    }
  }
  if (trim) {  // PHP trim(): " \t\n\r\0\x0B" at both ends
    auto ws = [](char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\0' || c == '\x0B'; };
    size_t a = 0, b = o.size();
    while (a < b && ws(o[a])) ++a;
    while (b > a && ws(o[b - 1])) --b;
    o = o.substr(a, b - a);
  }
  if (out && max_bytes > 0) {
    const size_t c = std::min(o.size(), (size_t)max_bytes - 1);
    memcpy(out, o.data(), c);
    out[c] = '\0';
  }
  return (int)o.size();
}
