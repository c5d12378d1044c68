// Text -> token ids for the checkpoint's tokenizer.json, and the text-level Encoder.
//
// The reference tokenizes with the HF `tokenizers` crate 0.22.2 (Cargo.lock), calling
// `Tokenizer::encode_fast(text, false)` (src/encode.rs:114-129) on ModernBERT's byte-level
// BPE tokenizer. This file restates the published algorithm of that pipeline for the
// configurations that tokenizer.json family uses, and refuses anything else at load time:
//   * added tokens (tokenizer.json "added_tokens"): leftmost-longest matches, first of the
//     tokens with normalized=false on the raw text, then of the normalized=true tokens
//     (matched in normalized form) on each remaining piece after normalisation; lstrip /
//     rstrip widen a match over adjacent white space, single_word drops a match touching
//     a word character; matched pieces map straight to their ids;
//   * normalizer: none or NFC (Unicode canonical decomposition, canonical ordering,
//     canonical composition; tables in unicode_tables.h);
//   * pre_tokenizer ByteLevel: optional leading space per piece, the GPT-2 split
//     's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+, then
//     every byte mapped to its printable stand-in (the GPT-2 byte <-> unicode table);
//   * model BPE: merges applied lowest rank first (leftmost among equals), optional
//     ignore_merges, no unk token, no dropout, no sub-word prefix/suffix.
// On top of it, Encoder (src/encode.rs:25-137): tokenizer_config.json special tokens,
// LRU caches of token fragments and of whole request encodings, the text forms of a
// request, and Encoder::sequence (j1_encode_sequence).
#include <algorithm>
#include <atomic>
#include <charconv>
#include <cmath>
#include <cstring>
#include <fstream>
#include <list>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "json.h"
#include "model.h"
#include "unicode_tables.h"

using namespace j1rt;

namespace {

// ------------------------------------------------------------------ unicode
template <size_t N>
bool in_ranges(const uint32_t (&r)[N][2], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid][0])
      hi = mid;
    else if (cp > r[mid][1])
      lo = mid + 1;
    else
      return true;
  }
  return false;
}
bool is_letter(uint32_t c) {
  if (c < 0x80) return (c | 0x20) >= 'a' && (c | 0x20) <= 'z';
  return in_ranges(ucd::kLetter, c);
}
bool is_number(uint32_t c) {
  if (c < 0x80) return c >= '0' && c <= '9';
  return in_ranges(ucd::kNumber, c);
}
bool is_space(uint32_t c) {
  if (c < 0x80) return c == ' ' || (c >= 0x9 && c <= 0xD);
  return in_ranges(ucd::kWhiteSpace, c);
}

void utf8_decode(const char* text, size_t n, std::vector<uint32_t>& cps, std::vector<uint32_t>* offs = nullptr) {
  cps.clear();
  if (offs) offs->clear();
  const unsigned char* p = reinterpret_cast<const unsigned char*>(text);
  for (size_t i = 0; i < n;) {
    uint32_t c = p[i];
    size_t len = 1;
    if (c >= 0xF0 && i + 3 < n) {
      c = ((c & 0x07) << 18) | ((p[i + 1] & 0x3F) << 12) | ((p[i + 2] & 0x3F) << 6) | (p[i + 3] & 0x3F);
      len = 4;
    } else if (c >= 0xE0 && i + 2 < n) {
      c = ((c & 0x0F) << 12) | ((p[i + 1] & 0x3F) << 6) | (p[i + 2] & 0x3F);
      len = 3;
    } else if (c >= 0xC0 && i + 1 < n) {
      c = ((c & 0x1F) << 6) | (p[i + 1] & 0x3F);
      len = 2;
    }
    if (offs) offs->push_back(static_cast<uint32_t>(i));
    cps.push_back(c);
    i += len;
  }
  if (offs) offs->push_back(static_cast<uint32_t>(n));
}

void utf8_decode(const std::string& s, std::vector<uint32_t>& cps, std::vector<uint32_t>* offs = nullptr) {
  utf8_decode(s.data(), s.size(), cps, offs);
}

void utf8_append(std::string& s, uint32_t c) {
  if (c < 0x80) {
    s += static_cast<char>(c);
  } else if (c < 0x800) {
    s += static_cast<char>(0xC0 | (c >> 6));
    s += static_cast<char>(0x80 | (c & 0x3F));
  } else if (c < 0x10000) {
    s += static_cast<char>(0xE0 | (c >> 12));
    s += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
    s += static_cast<char>(0x80 | (c & 0x3F));
  } else {
    s += static_cast<char>(0xF0 | (c >> 18));
    s += static_cast<char>(0x80 | ((c >> 12) & 0x3F));
    s += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
    s += static_cast<char>(0x80 | (c & 0x3F));
  }
}

// Well-formed UTF-8 (RFC 3629): no overlong forms, no surrogates, nothing above U+10FFFF —
// what a Rust &str, the reference's input type, can hold.
bool valid_utf8(const std::string& s) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s.data());
  const size_t n = s.size();
  for (size_t i = 0; i < n;) {
    const unsigned c = p[i];
    size_t len = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 0;
    if (len == 0 || i + len > n) return false;
    uint32_t cp = len == 1 ? c : len == 2 ? (c & 0x1F) : len == 3 ? (c & 0x0F) : (c & 0x07);
    for (size_t k = 1; k < len; ++k) {
      if ((p[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    static const uint32_t kMin[5] = {0, 0, 0x80, 0x800, 0x10000};
    if (cp < kMin[len] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
  }
  return true;
}

// Unicode canonical normalisation form C (UAX #15), for the NFC normalizer.
struct Nfc {
  std::unordered_map<uint32_t, uint8_t> ccc;
  std::unordered_map<uint32_t, std::pair<uint32_t, uint32_t>> decomp;
  std::unordered_map<uint64_t, uint32_t> comp;
  std::unordered_set<uint32_t> seconds;  // code points some composition takes as its second part
  // per code point: 0 not yet known, 1 NFC_QC = Yes, 2 otherwise (filled on first use)
  std::unique_ptr<std::atomic<uint8_t>[]> qc;
  Nfc() : qc(new std::atomic<uint8_t>[0x110000]()) {
    for (const auto& e : ucd::kCombining) ccc[e[0]] = static_cast<uint8_t>(e[1]);
    for (const auto& e : ucd::kDecomposition) decomp[e[0]] = {e[1], e[2]};
    for (const auto& e : ucd::kComposition) {
      comp[(static_cast<uint64_t>(e[0]) << 32) | e[1]] = e[2];
      seconds.insert(e[1]);
    }
  }
  static constexpr uint32_t SBase = 0xAC00, LBase = 0x1100, VBase = 0x1161, TBase = 0x11A7;
  static constexpr uint32_t LCount = 19, VCount = 21, TCount = 28, NCount = VCount * TCount, SCount = LCount * NCount;
  int cc(uint32_t c) const {
    if (c < 0x300) return 0;
    auto it = ccc.find(c);
    return it == ccc.end() ? 0 : it->second;
  }
  void decompose(uint32_t c, std::vector<uint32_t>& out) const {
    if (c >= SBase && c < SBase + SCount) {
      const uint32_t s = c - SBase;
      out.push_back(LBase + s / NCount);
      out.push_back(VBase + (s % NCount) / TCount);
      if (s % TCount) out.push_back(TBase + s % TCount);
      return;
    }
    auto it = decomp.find(c);
    if (it == decomp.end()) {
      out.push_back(c);
      return;
    }
    decompose(it->second.first, out);
    if (it->second.second) decompose(it->second.second, out);
  }
  uint32_t compose(uint32_t a, uint32_t b) const {
    if (a >= LBase && a < LBase + LCount && b >= VBase && b < VBase + VCount)
      return SBase + ((a - LBase) * VCount + (b - VBase)) * TCount;
    if (a >= SBase && a < SBase + SCount && (a - SBase) % TCount == 0 && b > TBase && b < TBase + TCount)
      return a + (b - TBase);
    auto it = comp.find((static_cast<uint64_t>(a) << 32) | b);
    return it == comp.end() ? 0 : it->second;
  }
  // UAX #15 quick check of one code point, NFC_QC = Yes: a starter that no composition
  // takes as its second part (Hangul medial and final jamo included) and that NFC maps to
  // itself. Below U+0300 every character qualifies.
  bool qc_yes(uint32_t c) const {
    if (c < 0x300) return true;
    uint8_t v = qc[c].load(std::memory_order_relaxed);
    if (v == 0) {
      const bool hangul_vt = (c >= VBase && c < VBase + VCount) || (c > TBase && c < TBase + TCount);
      bool yes = cc(c) == 0 && !hangul_vt && !seconds.count(c);
      if (yes) {
        std::string one, t;
        utf8_append(one, c);
        t = one;
        normalize_full(t);
        yes = t == one;
      }
      v = yes ? 1 : 2;
      qc[c].store(v, std::memory_order_relaxed);
    }
    return v == 1;
  }
  // True when the (valid UTF-8) text is in NFC by the quick check: every code point is
  // NFC_QC = Yes, so no character can change or combine with a neighbour.
  bool quick_yes(const char* p, size_t n) const {
    const unsigned char* u = reinterpret_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n;) {
      const unsigned b = u[i];
      if (b < 0xCC) {  // ASCII, or a 2-byte lead below U+0300 (then its continuation byte)
        i += b < 0x80 ? 1 : 2;
        continue;
      }
      const size_t len = (b >> 5) == 6 ? 2 : (b >> 4) == 14 ? 3 : 4;
      if (i + len > n) return false;
      uint32_t c = len == 2 ? (b & 0x1F) : len == 3 ? (b & 0x0F) : (b & 0x07);
      for (size_t k = 1; k < len; ++k) c = (c << 6) | (u[i + k] & 0x3F);
      if (c > 0x10FFFF || !qc_yes(c)) return false;
      i += len;
    }
    return true;
  }
  void normalize(std::string& s) const {
    if (quick_yes(s.data(), s.size())) return;
    normalize_full(s);
  }
  void normalize_full(std::string& s) const {
    std::vector<uint32_t> cps, d;
    utf8_decode(s, cps);
    d.reserve(cps.size() + 8);
    for (uint32_t c : cps) decompose(c, d);
    // canonical ordering: stable sort of each run of non-starters by combining class
    for (size_t i = 0; i < d.size();) {
      if (cc(d[i]) == 0) {
        ++i;
        continue;
      }
      size_t j = i;
      while (j < d.size() && cc(d[j]) != 0) ++j;
      std::stable_sort(d.begin() + i, d.begin() + j, [&](uint32_t x, uint32_t y) { return cc(x) < cc(y); });
      i = j;
    }
    // canonical composition
    std::vector<uint32_t> out;
    out.reserve(d.size());
    long starter = -1;
    int last_cc = -1;  // class of the last character kept after the starter; -1: none
    for (uint32_t c : d) {
      const int k = cc(c);
      if (starter >= 0 && (last_cc == -1 || (last_cc != 0 && last_cc < k))) {
        const uint32_t m = compose(out[starter], c);
        if (m) {
          out[starter] = m;
          continue;
        }
      }
      if (k == 0) {
        starter = static_cast<long>(out.size());
        last_cc = -1;
      } else {
        last_cc = k;
      }
      out.push_back(c);
    }
    s.clear();
    for (uint32_t c : out) utf8_append(s, c);
  }
};

const Nfc& nfc_tables() {
  static const Nfc t;
  return t;
}

// ------------------------------------------------------------------ LRU cache (lru::LruCache semantics)
// Shared by the threads of a text encoder: get promotes the entry, put of a new key evicts
// the least recently used one when full. Values are shared (the reference keeps Arc values).
// Keys are hashed, and new entries built, outside the lock; inside it there is only a bucket
// lookup with one key comparison, a list splice and a shared_ptr copy, and evicted entries
// are freed after it, so threads encoding large requests rarely wait on one another.
template <typename V>
class Lru {
 public:
  using Ptr = std::shared_ptr<const V>;
  explicit Lru(size_t cap) : cap_(cap) {}
  Ptr get(const std::string& k) {
    if (cap_ == 0) return nullptr;
    const uint64_t h = hash(k);
    std::lock_guard<std::mutex> lk(mu_);
    const auto it = find(h, k);
    if (it == items_.end()) return nullptr;
    items_.splice(items_.begin(), items_, it);
    return it->value;
  }
  void put(const std::string& k, Ptr v) {
    if (cap_ == 0) return;
    const uint64_t h = hash(k);
    std::list<Node> node;  // the entry and its index slot are allocated before locking
    node.push_back(Node{h, k, std::move(v)});
    Index slot;
    slot.emplace(h, node.begin());
    auto handle = slot.extract(slot.begin());
    std::list<Node> evicted;  // declared before the lock: freed after it is released
    std::lock_guard<std::mutex> lk(mu_);
    const auto it = find(h, k);
    if (it != items_.end()) {
      std::swap(it->value, node.front().value);
      items_.splice(items_.begin(), items_, it);
      return;
    }
    if (items_.size() >= cap_) {
      const auto last = std::prev(items_.end());
      unindex(last);
      evicted.splice(evicted.begin(), items_, last);
    }
    items_.splice(items_.begin(), node, node.begin());
    handle.mapped() = items_.begin();
    index_.insert(std::move(handle));
  }
  void clear() {
    std::list<Node> items;
    Index index;
    std::lock_guard<std::mutex> lk(mu_);
    items.swap(items_);
    index.swap(index_);
  }

 private:
  struct Node {
    uint64_t hash;
    std::string key;
    Ptr value;
  };
  using It = typename std::list<Node>::iterator;
  using Index = std::unordered_multimap<uint64_t, It>;
  static uint64_t hash(const std::string& k) { return std::hash<std::string>()(k); }
  It find(uint64_t h, const std::string& k) {
    for (auto [b, e] = index_.equal_range(h); b != e; ++b)
      if (b->second->key == k) return b->second;
    return items_.end();
  }
  void unindex(It it) {
    for (auto [b, e] = index_.equal_range(it->hash); b != e; ++b)
      if (b->second == it) {
        index_.erase(b);
        return;
      }
  }
  size_t cap_;
  std::mutex mu_;
  std::list<Node> items_;
  Index index_;
};

}  // namespace

// ------------------------------------------------------------------ tokenizer
namespace {
std::atomic<uint64_t> g_tokenizer_generation{1};
}

struct j1_tokenizer {
  const uint64_t generation = g_tokenizer_generation++;  // keys the per-thread BPE caches
  struct Added {
    std::string content, pattern;  // pattern: content, normalised for normalized tokens
    uint32_t id;
    bool single_word, lstrip, rstrip, normalized;
  };
  std::unordered_map<std::string, uint32_t> vocab;
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;  // (a, b) -> (rank, merged id)
  std::vector<Added> added;
  std::vector<size_t> raw_by_byte[256], norm_by_byte[256];  // added tokens by first byte of their pattern
  bool nfc = false, prefix_space = false, use_regex = true, ignore_merges = false, has_pre = false;
  bool has_norm_tokens = false;  // added tokens matched in normalised form exist
  uint32_t byte_id[256];
  bool byte_ok[256];
  std::string byte_char[256];  // GPT-2 byte -> printable stand-in, UTF-8

  // ---- added tokens
  // One pass of leftmost-longest matching over `text` with the tokens of `by_byte`.
  // Returns pieces: (token index or -1, byte range).
  void split_added(const std::string& text, const std::vector<size_t> (&by_byte)[256],
                   std::vector<std::pair<long, std::pair<size_t, size_t>>>& out) const {
    out.clear();
    size_t start_offset = 0;
    const size_t n = text.size();
    for (size_t pos = 0; pos < n;) {
      const auto& cand = by_byte[static_cast<unsigned char>(text[pos])];
      long best = -1;
      size_t best_len = 0;
      for (size_t a : cand) {
        const std::string& pt = added[a].pattern;
        if (pt.size() > best_len && pt.size() <= n - pos && std::memcmp(text.data() + pos, pt.data(), pt.size()) == 0) {
          best = static_cast<long>(a);
          best_len = pt.size();
        }
      }
      if (best < 0) {
        ++pos;
        continue;
      }
      size_t start = pos, stop = pos + best_len;
      pos = stop;  // the matcher resumes after this match even when it is dropped below
      const Added& t = added[static_cast<size_t>(best)];
      if (t.single_word) {
        const bool start_space = start == 0 || !ends_with_word(text, start);
        const bool stop_space = stop == n || !starts_with_word(text, stop);
        if (!start_space || !stop_space) continue;
      }
      if (t.lstrip) start = std::max(space_leftmost_at_end(text, start), start_offset);
      if (t.rstrip) stop += space_rightmost_at_start(text, stop);
      if (start_offset < start) out.push_back({-1, {start_offset, start}});
      out.push_back({best, {start, stop}});
      start_offset = stop;
    }
    if (start_offset < n) out.push_back({-1, {start_offset, n}});
  }
  // regex \w (word characters for single_word tokens)
  static bool word_char(uint32_t c) {
    if (c < 0x80) return c == '_' || (c >= '0' && c <= '9') || ((c | 0x20) >= 'a' && (c | 0x20) <= 'z');
    return in_ranges(ucd::kWord, c);
  }
  static uint32_t last_cp(const std::string& s, size_t end) {
    size_t i = end;
    while (i > 0 && (static_cast<unsigned char>(s[i - 1]) & 0xC0) == 0x80) --i;
    if (i > 0) --i;
    std::vector<uint32_t> c;
    utf8_decode(s.substr(i, end - i), c);
    return c.empty() ? 0 : c.back();
  }
  static uint32_t first_cp(const std::string& s, size_t start, size_t* len) {
    const unsigned char c = static_cast<unsigned char>(s[start]);
    const size_t l = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : 4;
    std::vector<uint32_t> cp;
    utf8_decode(s.substr(start, std::min(l, s.size() - start)), cp);
    if (len) *len = l;
    return cp.empty() ? 0 : cp[0];
  }
  static bool ends_with_word(const std::string& s, size_t end) { return end > 0 && word_char(last_cp(s, end)); }
  static bool starts_with_word(const std::string& s, size_t start) {
    return start < s.size() && word_char(first_cp(s, start, nullptr));
  }
  // start of the white space that ends s[0, end)
  static size_t space_leftmost_at_end(const std::string& s, size_t end) {
    size_t i = end;
    while (i > 0) {
      size_t j = i;
      while (j > 0 && (static_cast<unsigned char>(s[j - 1]) & 0xC0) == 0x80) --j;
      --j;
      size_t l = 0;
      if (!is_space(first_cp(s, j, &l))) break;
      i = j;
    }
    return i;
  }
  // bytes of white space at the start of s[start, ...)
  static size_t space_rightmost_at_start(const std::string& s, size_t start) {
    size_t i = start;
    while (i < s.size()) {
      size_t l = 0;
      if (!is_space(first_cp(s, i, &l))) break;
      i += l;
    }
    return i - start;
  }

  // ---- ByteLevel pre-tokenizer: the GPT-2 split of one piece (code point ranges)
  static void gpt2_split(const std::vector<uint32_t>& c, std::vector<std::pair<size_t, size_t>>& out) {
    out.clear();
    const size_t n = c.size();
    size_t i = 0;
    auto run = [&](size_t j, auto pred) {
      while (j < n && pred(c[j])) ++j;
      return j;
    };
    auto other = [](uint32_t x) { return !is_space(x) && !is_letter(x) && !is_number(x); };
    while (i < n) {
      const uint32_t x = c[i];
      if (x == '\'' && i + 1 < n) {  // 's 't 're 've 'm 'll 'd
        const uint32_t a = c[i + 1], b = i + 2 < n ? c[i + 2] : 0;
        size_t len = 0;
        if (a == 's' || a == 't' || a == 'm' || a == 'd')
          len = 2;
        else if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l'))
          len = 3;
        if (len) {
          out.push_back({i, i + len});
          i += len;
          continue;
        }
      }
      const size_t k = (x == ' ' && i + 1 < n) ? i + 1 : i;  // optional leading space
      if (is_letter(c[k]) && (k == i || x == ' ')) {
        const size_t j = run(k, is_letter);
        out.push_back({i, j});
        i = j;
        continue;
      }
      if (is_number(c[k]) && (k == i || x == ' ')) {
        const size_t j = run(k, is_number);
        out.push_back({i, j});
        i = j;
        continue;
      }
      if (other(c[k]) && (k == i || x == ' ')) {
        const size_t j = run(k, other);
        out.push_back({i, j});
        i = j;
        continue;
      }
      // white space: \s+(?!\S) keeps the last space for the next token, else \s+
      const size_t j = run(i, is_space);
      if (j == n || j - i == 1) {
        out.push_back({i, j});
        i = j;
      } else {
        out.push_back({i, j - 1});
        i = j - 1;
      }
    }
  }

  // ---- BPE on one pre-token (its UTF-8 bytes)
  // Per-thread cache of whole pre-tokens (no locking): entries keyed by a 64-bit hash of
  // the bytes, which are kept and compared on a hit; a cache belongs to one tokenizer.
  struct WordCache {
    struct Entry {
      uint32_t boff, blen, ioff, ilen;
    };
    uint64_t owner = 0;
    std::unordered_map<uint64_t, Entry> map;
    std::string bytes;
    std::vector<uint32_t> ids;
    void reset(uint64_t o) {
      owner = o;
      map.clear();
      bytes.clear();
      ids.clear();
    }
  };
  static uint64_t hash_bytes(const char* p, size_t n) {
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; ++i) {
      h ^= static_cast<unsigned char>(p[i]);
      h *= 1099511628211ull;
    }
    return h ^ (n * 0x9E3779B97F4A7C15ull);
  }
  void bpe(const char* p, size_t n, std::vector<uint32_t>& ids) const {
    if (ignore_merges) {
      std::string mapped;
      for (size_t i = 0; i < n; ++i) mapped += byte_char[static_cast<unsigned char>(p[i])];
      auto it = vocab.find(mapped);
      if (it != vocab.end()) {
        ids.push_back(it->second);
        return;
      }
    }
    thread_local WordCache wc;
    if (wc.owner != generation) wc.reset(generation);
    const uint64_t h = hash_bytes(p, n);
    auto hit = wc.map.find(h);
    if (hit != wc.map.end()) {
      const WordCache::Entry& e = hit->second;
      if (e.blen == n && std::memcmp(wc.bytes.data() + e.boff, p, n) == 0) {
        ids.insert(ids.end(), wc.ids.begin() + e.ioff, wc.ids.begin() + e.ioff + e.ilen);
        return;
      }
    }
    thread_local std::vector<uint32_t> sym;
    sym.clear();
    for (size_t i = 0; i < n; ++i) {
      const unsigned char b = static_cast<unsigned char>(p[i]);
      if (byte_ok[b]) sym.push_back(byte_id[b]);  // a byte missing from the vocab is dropped (no unk token)
    }
    while (sym.size() > 1) {
      uint32_t best_rank = UINT32_MAX, best_id = 0;
      size_t best_pos = 0;
      for (size_t i = 0; i + 1 < sym.size(); ++i) {
        auto it = merges.find((static_cast<uint64_t>(sym[i]) << 32) | sym[i + 1]);
        if (it != merges.end() && it->second.first < best_rank) {
          best_rank = it->second.first;
          best_id = it->second.second;
          best_pos = i;
        }
      }
      if (best_rank == UINT32_MAX) break;
      sym[best_pos] = best_id;
      sym.erase(sym.begin() + static_cast<std::ptrdiff_t>(best_pos) + 1);
    }
    ids.insert(ids.end(), sym.begin(), sym.end());
    if (hit == wc.map.end()) {  // (a hash collision with another piece is left uncached)
      if (wc.map.size() > 200000 || wc.bytes.size() > (64u << 20)) wc.reset(generation);
      wc.map.emplace(h, WordCache::Entry{static_cast<uint32_t>(wc.bytes.size()), static_cast<uint32_t>(n),
                                         static_cast<uint32_t>(wc.ids.size()), static_cast<uint32_t>(sym.size())});
      wc.bytes.append(p, n);
      wc.ids.insert(wc.ids.end(), sym.begin(), sym.end());
    }
  }

  // pre-tokenize + BPE one normalised piece (no added tokens inside)
  void encode_piece(const char* p, size_t n, std::vector<uint32_t>& ids) const {
    if (n == 0) return;
    thread_local std::string spaced;
    if (prefix_space && p[0] != ' ') {
      spaced.assign(1, ' ');
      spaced.append(p, n);
      p = spaced.data();
      n = spaced.size();
    }
    if (!use_regex) {
      bpe(p, n, ids);
      return;
    }
    thread_local std::vector<uint32_t> cps, offs;
    thread_local std::vector<std::pair<size_t, size_t>> parts;
    utf8_decode(p, n, cps, &offs);
    gpt2_split(cps, parts);
    for (const auto& pr : parts) bpe(p + offs[pr.first], offs[pr.second] - offs[pr.first], ids);
  }

  // True when some byte of [p, p + n) begins the pattern of a normalised added token; only
  // then can matching on the normalised piece (equal to the piece when it is NFC-stable)
  // find one.
  bool may_start_norm_token(const char* p, size_t n) const {
    for (size_t i = 0; i < n; ++i)
      if (!norm_by_byte[static_cast<unsigned char>(p[i])].empty()) return true;
    return false;
  }

  // Tokenizer::encode_fast(text, add_special_tokens = false)
  void encode(const std::string& text, std::vector<uint32_t>& ids) const {
    ids.clear();
    std::vector<std::pair<long, std::pair<size_t, size_t>>> raw, nrm;
    split_added(text, raw_by_byte, raw);
    for (const auto& r : raw) {
      if (r.first >= 0) {
        ids.push_back(added[static_cast<size_t>(r.first)].id);
        continue;
      }
      const char* p = text.data() + r.second.first;
      const size_t n = r.second.second - r.second.first;
      // nothing to normalise, and no normalised added token can start in the piece: no copy
      if ((!nfc || nfc_tables().quick_yes(p, n)) && (!has_norm_tokens || !may_start_norm_token(p, n))) {
        encode_piece(p, n, ids);
        continue;
      }
      std::string piece(p, n);
      if (nfc) nfc_tables().normalize(piece);
      split_added(piece, norm_by_byte, nrm);
      for (const auto& q : nrm) {
        if (q.first >= 0)
          ids.push_back(added[static_cast<size_t>(q.first)].id);
        else
          encode_piece(piece.data() + q.second.first, q.second.second - q.second.first, ids);
      }
    }
  }

  bool token_to_id(const std::string& t, uint32_t& id) const {
    for (const auto& a : added)
      if (a.content == t) {
        id = a.id;
        return true;
      }
    auto it = vocab.find(t);
    if (it == vocab.end()) return false;
    id = it->second;
    return true;
  }
};

namespace {

j1_status load_tokenizer(const std::string& text, std::unique_ptr<j1_tokenizer>& out) {
  Json j;
  std::string err;
  if (!parse_json(text, j, err)) return set_error(J1_ERR_INVALID_ARG, "tokenizer.json: " + err);
  auto T = std::make_unique<j1_tokenizer>();
  const Json* model = j.get("model");
  if (!model || !model->get("type") || model->get("type")->str != "BPE")
    return set_error(J1_ERR_UNSUPPORTED, "tokenizer.json: only BPE models are supported");
  auto flag = [](const Json* o, const char* k) {
    const Json* v = o ? o->get(k) : nullptr;
    return v && v->kind == Json::Bool && v->b;
  };
  auto nonempty = [](const Json* o, const char* k) {
    const Json* v = o ? o->get(k) : nullptr;
    return v && v->kind == Json::String && !v->str.empty();
  };
  if (flag(model, "byte_fallback") || nonempty(model, "continuing_subword_prefix") ||
      nonempty(model, "end_of_word_suffix") || (model->get("dropout") && model->get("dropout")->kind != Json::Null) ||
      (model->get("unk_token") && model->get("unk_token")->kind != Json::Null))
    return set_error(J1_ERR_UNSUPPORTED,
                     "tokenizer.json: BPE with byte_fallback, unk_token, dropout or sub-word affixes is not supported");
  T->ignore_merges = flag(model, "ignore_merges");
  const Json* vocab = model->get("vocab");
  const Json* merges = model->get("merges");
  if (!vocab || vocab->kind != Json::Object || !merges || merges->kind != Json::Array)
    return set_error(J1_ERR_INVALID_ARG, "tokenizer.json: model.vocab / model.merges missing");
  T->vocab.reserve(vocab->obj.size() * 2);
  for (const auto& kv : vocab->obj) T->vocab[kv.first] = static_cast<uint32_t>(kv.second.num);
  uint32_t rank = 0;
  for (const Json& m : merges->arr) {
    std::string a, b;
    if (m.kind == Json::String) {
      const size_t sp = m.str.find(' ');
      if (sp == std::string::npos) return set_error(J1_ERR_INVALID_ARG, "tokenizer.json: bad merge " + m.str);
      a = m.str.substr(0, sp);
      b = m.str.substr(sp + 1);
    } else if (m.kind == Json::Array && m.arr.size() == 2) {
      a = m.arr[0].str;
      b = m.arr[1].str;
    } else {
      return set_error(J1_ERR_INVALID_ARG, "tokenizer.json: bad merge entry");
    }
    auto ia = T->vocab.find(a), ib = T->vocab.find(b), ic = T->vocab.find(a + b);
    if (ia == T->vocab.end() || ib == T->vocab.end() || ic == T->vocab.end())
      return set_error(J1_ERR_INVALID_ARG, "tokenizer.json: merge of tokens outside the vocabulary: " + a + " " + b);
    // a pair listed twice keeps its last rank (the reference collects the list into a map)
    T->merges[(static_cast<uint64_t>(ia->second) << 32) | ib->second] = {rank, ic->second};
    ++rank;
  }
  // normalizer
  const Json* norm = j.get("normalizer");
  if (norm && norm->kind != Json::Null) {
    const Json* t = norm->get("type");
    if (!t || t->str != "NFC") return set_error(J1_ERR_UNSUPPORTED, "tokenizer.json: only the NFC normalizer is supported");
    T->nfc = true;
  }
  // pre-tokenizer
  const Json* pre = j.get("pre_tokenizer");
  if (!pre || pre->kind == Json::Null || !pre->get("type") || pre->get("type")->str != "ByteLevel")
    return set_error(J1_ERR_UNSUPPORTED, "tokenizer.json: only the ByteLevel pre-tokenizer is supported");
  T->prefix_space = flag(pre, "add_prefix_space");
  T->use_regex = !pre->get("use_regex") || flag(pre, "use_regex");
  // GPT-2 byte <-> printable character table
  {
    std::vector<int> bs;
    for (int b = '!'; b <= '~'; ++b) bs.push_back(b);
    for (int b = 0xA1; b <= 0xAC; ++b) bs.push_back(b);
    for (int b = 0xAE; b <= 0xFF; ++b) bs.push_back(b);
    std::vector<uint32_t> cs(bs.begin(), bs.end());
    uint32_t extra = 0;
    for (int b = 0; b < 256; ++b)
      if (std::find(bs.begin(), bs.end(), b) == bs.end()) {
        bs.push_back(b);
        cs.push_back(256 + extra++);
      }
    for (size_t i = 0; i < bs.size(); ++i) {
      std::string ch;
      utf8_append(ch, cs[i]);
      T->byte_char[bs[i]] = ch;
    }
    for (int b = 0; b < 256; ++b) {
      auto it = T->vocab.find(T->byte_char[b]);
      T->byte_ok[b] = it != T->vocab.end();
      T->byte_id[b] = T->byte_ok[b] ? it->second : 0;
    }
  }
  // added tokens
  const Json* added = j.get("added_tokens");
  if (added && added->kind == Json::Array) {
    for (const Json& a : added->arr) {
      j1_tokenizer::Added t;
      const Json* c = a.get("content");
      const Json* id = a.get("id");
      if (!c || !id) return set_error(J1_ERR_INVALID_ARG, "tokenizer.json: added token without content/id");
      t.content = c->str;
      t.id = static_cast<uint32_t>(id->num);
      t.single_word = flag(&a, "single_word");
      t.lstrip = flag(&a, "lstrip");
      t.rstrip = flag(&a, "rstrip");
      t.normalized = flag(&a, "normalized");
      t.pattern = t.content;
      if (t.normalized && T->nfc) nfc_tables().normalize(t.pattern);
      if (t.pattern.empty()) continue;
      T->added.push_back(t);
    }
  }
  for (size_t i = 0; i < T->added.size(); ++i) {
    const unsigned char b0 = static_cast<unsigned char>(T->added[i].pattern[0]);
    (T->added[i].normalized ? T->norm_by_byte : T->raw_by_byte)[b0].push_back(i);
    T->has_norm_tokens = T->has_norm_tokens || T->added[i].normalized;
  }
  out = std::move(T);
  return J1_OK;
}

bool read_file(const std::string& path, std::string& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::ostringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

}  // namespace

// ------------------------------------------------------------------ text encoder
struct j1_text_encoder {
  std::unique_ptr<j1_tokenizer> tok;
  std::string mask_token;
  j1_encoder_options opts{};
  std::unique_ptr<Lru<std::vector<uint32_t>>> tokens;
  struct Enc {
    std::vector<uint32_t> ids, markers;
    int32_t truncated;
  };
  std::unique_ptr<Lru<Enc>> encodings;

  // Encoder::tokenize (src/encode.rs:114-129), with the token-fragment cache
  void tokenize(const std::string& text, std::vector<uint32_t>& ids) {
    if (const auto hit = tokens->get(text)) {
      ids = *hit;
      return;
    }
    tok->encode(text, ids);
    tokens->put(text, std::make_shared<const std::vector<uint32_t>>(ids));
  }
};

namespace {

std::string replace_all(const std::string& s, const std::string& from, const std::string& to) {
  if (from.empty()) return s;
  std::string out;
  size_t i = 0;
  for (;;) {
    const size_t j = s.find(from, i);
    if (j == std::string::npos) break;
    out.append(s, i, j - i);
    out += to;
    i = j + from.size();
  }
  out.append(s, i, std::string::npos);
  return out;
}

const char* qtype_name(uint8_t q) { return q == 0 ? "choice" : q == 1 ? "score" : "noul"; }

// ------------------------------------------------------------------ State::render for JSON states
// Python's json.dumps(value, ensure_ascii=False), byte for byte (src/pyjson.rs): ", " and
// ": " separators, key order kept, integers as written, other numbers as float.__repr__,
// the json module's escapes.

// float.__repr__: the shortest digits that round-trip, fixed notation for decimal
// exponents -4 < point <= 16, else d.ddde+XX.
std::string float_repr(double v) {
  if (std::isnan(v)) return "NaN";
  if (std::isinf(v)) return v > 0 ? "Infinity" : "-Infinity";
  if (v == 0.0) return std::signbit(v) ? "-0.0" : "0.0";
  char buf[64];
  const auto res = std::to_chars(buf, buf + sizeof(buf), std::fabs(v), std::chars_format::scientific);
  const std::string sci(buf, res.ptr);
  const size_t epos = sci.find('e');
  std::string digits;
  for (size_t i = 0; i < epos; ++i)
    if (sci[i] != '.') digits += sci[i];
  const int exponent = std::atoi(sci.c_str() + epos + 1);
  const int point = exponent + 1;  // v = 0.DIGITS x 10^point
  const int n = static_cast<int>(digits.size());
  std::string out = v < 0 ? "-" : "";
  if (-4 < point && point <= 16) {
    if (point <= 0) {
      out += "0.";
      out.append(static_cast<size_t>(-point), '0');
      out += digits;
    } else if (point >= n) {
      out += digits;
      out.append(static_cast<size_t>(point - n), '0');
      out += ".0";
    } else {
      out += digits.substr(0, static_cast<size_t>(point));
      out += '.';
      out += digits.substr(static_cast<size_t>(point));
    }
  } else {
    out += digits.substr(0, 1);
    if (n > 1) {
      out += '.';
      out += digits.substr(1);
    }
    const int e = point - 1;
    char eb[16];
    std::snprintf(eb, sizeof(eb), "e%c%02d", e < 0 ? '-' : '+', e < 0 ? -e : e);
    out += eb;
  }
  return out;
}

void py_dumps_string(std::string& out, const std::string& s) {
  out += '"';
  for (unsigned char c : s) {
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      case 0x08: out += "\\b"; break;
      case 0x0C: out += "\\f"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof(b), "\\u%04x", c);
          out += b;
        } else {
          out += static_cast<char>(c);
        }
    }
  }
  out += '"';
}

void py_dumps(std::string& out, const Json& v) {
  switch (v.kind) {
    case Json::Null: out += "null"; break;
    case Json::Bool: out += v.b ? "true" : "false"; break;
    case Json::Number:
      // the json module reads literals without '.', 'e' or 'E' as int, the rest as float
      if (v.str.find_first_of(".eE") != std::string::npos)
        out += float_repr(v.num);
      else if (v.str == "-0")
        out += '0';
      else
        out += v.str;
      break;
    case Json::String: py_dumps_string(out, v.str); break;
    case Json::Array:
      out += '[';
      for (size_t i = 0; i < v.arr.size(); ++i) {
        if (i) out += ", ";
        py_dumps(out, v.arr[i]);
      }
      out += ']';
      break;
    case Json::Object:
      out += '{';
      for (size_t i = 0; i < v.obj.size(); ++i) {
        if (i) out += ", ";
        py_dumps_string(out, v.obj[i].first);
        out += ": ";
        py_dumps(out, v.obj[i].second);
      }
      out += '}';
      break;
  }
}

// State::render of a JSON state (Request::validate: an object or an array).
j1_status render_json_state(const std::string& text, std::string& out) {
  Json j;
  std::string err;
  if (!parse_json(text, j, err)) return set_error(J1_ERR_INVALID_ARG, "state is not valid JSON: " + err);
  if (j.kind != Json::Object && j.kind != Json::Array)
    return set_error(J1_ERR_INVALID_ARG, "state must be text/JSON and question must be text");
  out.clear();
  py_dumps(out, j);
  return J1_OK;
}

// The text part of Encoder::sequence (src/encode.rs:138-150, 180): strict refusal of the mask
// token's text, the text replaced by a space otherwise, and the tokens of the head
// "<qtype> question: <question>", of each " <option>" and of the state.
j1_status request_tokens(j1_text_encoder* e, const std::string& st, const std::string& q,
                         const std::vector<std::string>& opts, uint8_t qtype, std::vector<uint32_t>& head,
                         std::vector<uint32_t>& opt_ids, std::vector<uint32_t>& opt_lens,
                         std::vector<uint32_t>& state_ids) {
  const std::string& mask = e->mask_token;
  if (e->opts.strict) {
    bool has = st.find(mask) != std::string::npos || q.find(mask) != std::string::npos;
    for (const auto& s : opts) has = has || s.find(mask) != std::string::npos;
    if (has) return set_error(J1_ERR_INVALID_ARG, "Reserved model marker in request");
  }
  auto clean = [&mask](const std::string& s) { return replace_all(s, mask, " "); };
  e->tokenize(std::string(qtype_name(qtype)) + " question: " + clean(q), head);
  opt_ids.clear();
  opt_lens.clear();
  for (const auto& s : opts) {
    std::vector<uint32_t> v;
    e->tokenize(" " + clean(s), v);
    opt_ids.insert(opt_ids.end(), v.begin(), v.end());
    opt_lens.push_back(static_cast<uint32_t>(v.size()));
  }
  e->tokenize(clean(st), state_ids);
  return J1_OK;
}

j1_status read_request(const char* state, const char* question, const char* const* options, size_t n_options,
                       uint8_t qtype, std::string& st, std::string& q, std::vector<std::string>& opts) {
  if (!state || !question || (n_options && !options)) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
  if (qtype > 2) return set_error(J1_ERR_INVALID_ARG, "qtype must be 0 (choice), 1 (score) or 2 (noul)");
  opts.assign(n_options, std::string());
  for (size_t k = 0; k < n_options; ++k) {
    if (!options[k]) return set_error(J1_ERR_INVALID_ARG, "NULL option");
    opts[k] = options[k];
  }
  st = state;
  q = question;
  for (const std::string* s : {&st, &q})
    if (!valid_utf8(*s)) return set_error(J1_ERR_INVALID_ARG, "text is not valid UTF-8");
  for (const auto& s : opts)
    if (!valid_utf8(s)) return set_error(J1_ERR_INVALID_ARG, "text is not valid UTF-8");
  return J1_OK;
}

}  // namespace

extern "C" {

j1_status j1_tokenizer_load(const char* path, j1_tokenizer** out) {
  return guard("j1_tokenizer_load", [&]() -> j1_status {
    if (!path || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    std::string text;
    if (!read_file(path, text)) return set_error(J1_ERR_IO, std::string("cannot read ") + path);
    std::unique_ptr<j1_tokenizer> t;
    if (j1_status s = load_tokenizer(text, t)) return s;
    *out = t.release();
    return J1_OK;
  });
}

j1_status j1_tokenizer_from_json(const char* json, size_t len, j1_tokenizer** out) {
  return guard("j1_tokenizer_from_json", [&]() -> j1_status {
    if (!json || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    std::unique_ptr<j1_tokenizer> t;
    if (j1_status s = load_tokenizer(std::string(json, len), t)) return s;
    *out = t.release();
    return J1_OK;
  });
}

void j1_tokenizer_destroy(j1_tokenizer* t) { delete t; }

int64_t j1_tokenizer_token_to_id(const j1_tokenizer* t, const char* token) {
  uint32_t id = 0;
  int64_t out = -1;
  guard("j1_tokenizer_token_to_id", [&]() -> j1_status {
    if (t && token && t->token_to_id(token, id)) out = id;
    return J1_OK;
  });
  return out;
}

j1_status j1_tokenizer_encode(const j1_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t cap,
                              size_t* n_ids) {
  return guard("j1_tokenizer_encode", [&]() -> j1_status {
    if (!t || (!text && len) || !n_ids) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    const std::string s(text ? text : "", len);
    if (!valid_utf8(s)) return set_error(J1_ERR_INVALID_ARG, "text is not valid UTF-8");
    std::vector<uint32_t> v;
    t->encode(s, v);
    *n_ids = v.size();
    if (v.size() > cap || (!ids && !v.empty()))
      return set_error(J1_ERR_INVALID_ARG, "ids buffer too small (" + std::to_string(v.size()) + " needed)");
    if (!v.empty()) std::memcpy(ids, v.data(), v.size() * 4);
    return J1_OK;
  });
}

j1_status j1_tokenizer_encode_batch(const j1_tokenizer* t, size_t n, const char* const* texts, const size_t* lens,
                                    int32_t threads, uint32_t* ids, size_t cap, size_t* offsets) {
  return guard("j1_tokenizer_encode_batch", [&]() -> j1_status {
    if (!t || !offsets || (n && (!texts || !lens))) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::vector<std::vector<uint32_t>> res(n);
    std::atomic<size_t> next{0};
    std::atomic<long> bad{-1};
    auto work = [&]() {
      for (size_t i = next++; i < n; i = next++) {
        const std::string s(texts[i] ? texts[i] : "", lens[i]);
        if (!valid_utf8(s)) {
          bad = static_cast<long>(i);
          continue;
        }
        t->encode(s, res[i]);
      }
    };
    const int nt = std::max(1, std::min<int>(threads > 0 ? threads : 1, static_cast<int>(std::max<size_t>(n, 1))));
    run_pool(nt, work);
    if (bad >= 0) return set_error(J1_ERR_INVALID_ARG, "text " + std::to_string(bad) + " is not valid UTF-8");
    offsets[0] = 0;
    for (size_t i = 0; i < n; ++i) offsets[i + 1] = offsets[i] + res[i].size();
    if (offsets[n] > cap || (!ids && offsets[n]))
      return set_error(J1_ERR_INVALID_ARG, "ids buffer too small (" + std::to_string(offsets[n]) + " needed)");
    for (size_t i = 0; i < n; ++i)
      if (!res[i].empty()) std::memcpy(ids + offsets[i], res[i].data(), res[i].size() * 4);
    return J1_OK;
  });
}

j1_status j1_text_encoder_load(const char* dir, int32_t max_length, int32_t head_length, int32_t strict,
                               int64_t token_cache, int64_t encoding_cache, j1_text_encoder** out) {
  return guard("j1_text_encoder_load", [&]() -> j1_status {
    if (!dir || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    const std::string root(dir);
    std::string tj, cj;
    if (!read_file(root + "/tokenizer.json", tj)) return set_error(J1_ERR_IO, "cannot read " + root + "/tokenizer.json");
    if (!read_file(root + "/tokenizer_config.json", cj))
      return set_error(J1_ERR_IO, "cannot read " + root + "/tokenizer_config.json");
    // Encoder::from_parts (src/encode.rs:55-101)
    if (static_cast<int64_t>(head_length) + 4 >= max_length)
      return set_error(J1_ERR_INVALID_ARG, "max_length must leave room beyond the question head");
    auto E = std::make_unique<j1_text_encoder>();
    if (j1_status s = load_tokenizer(tj, E->tok)) return s;
    Json cfg;
    std::string err;
    if (!parse_json(cj, cfg, err)) return set_error(J1_ERR_INVALID_ARG, "tokenizer_config.json: " + err);
    auto special = [&](const char* key, std::string& name, uint32_t& id) -> j1_status {
      const Json* v = cfg.get(key);
      if (!v || v->kind != Json::String) return set_error(J1_ERR_INVALID_ARG, std::string("tokenizer lacks ") + key);
      name = v->str;
      if (!E->tok->token_to_id(name, id))
        return set_error(J1_ERR_INVALID_ARG, std::string("unknown ") + key + " " + name);
      return J1_OK;
    };
    std::string unused;
    j1_encoder_options& o = E->opts;
    if (j1_status s = special("mask_token", E->mask_token, o.mask_id)) return s;
    if (j1_status s = special("cls_token", unused, o.cls_id)) return s;
    if (j1_status s = special("sep_token", unused, o.sep_id)) return s;
    uint32_t pad = 0;
    if (j1_status s = special("pad_token", unused, pad)) return s;
    o.max_length = max_length;
    o.head_length = head_length;
    o.strict = strict ? 1 : 0;
    E->tokens = std::make_unique<Lru<std::vector<uint32_t>>>(token_cache > 0 ? static_cast<size_t>(token_cache) : 0);
    E->encodings = std::make_unique<Lru<j1_text_encoder::Enc>>(encoding_cache > 0 ? static_cast<size_t>(encoding_cache)
                                                                                   : 0);
    *out = E.release();
    return J1_OK;
  });
}

void j1_text_encoder_destroy(j1_text_encoder* e) { delete e; }

void j1_text_encoder_clear_cache(j1_text_encoder* e) {
  if (!e) return;
  e->tokens->clear();
  e->encodings->clear();
}

j1_status j1_text_encoder_options(const j1_text_encoder* e, j1_encoder_options* out) {
  return guard("j1_text_encoder_options", [&]() -> j1_status {
    if (!e || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    *out = e->opts;
    return J1_OK;
  });
}

j1_status j1_text_encoder_tokenize(j1_text_encoder* e, const char* text, size_t len, uint32_t* ids, size_t cap,
                                   size_t* n_ids) {
  return guard("j1_text_encoder_tokenize", [&]() -> j1_status {
    if (!e || (!text && len) || !n_ids) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    const std::string s(text ? text : "", len);
    if (!valid_utf8(s)) return set_error(J1_ERR_INVALID_ARG, "text is not valid UTF-8");
    std::vector<uint32_t> v;
    e->tokenize(s, v);
    *n_ids = v.size();
    if (v.size() > cap || (!ids && !v.empty())) return set_error(J1_ERR_INVALID_ARG, "ids buffer too small");
    if (!v.empty()) std::memcpy(ids, v.data(), v.size() * 4);
    return J1_OK;
  });
}

j1_status j1_text_encoder_encode(j1_text_encoder* e, const char* state, int32_t state_is_json, const char* question,
                                 const char* const* options, size_t n_options, uint8_t qtype, uint32_t* ids,
                                 size_t cap, size_t* ids_len, uint32_t* markers, int32_t* truncated) {
  return guard("j1_text_encoder_encode", [&]() -> j1_status {
    if (!e || !ids_len) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::string st, q;
    std::vector<std::string> opts;
    if (j1_status s = read_request(state, question, options, n_options, qtype, st, q, opts)) return s;
    // Encoder::encode (src/encode.rs:131-154): whole-request cache keyed on its text
    std::string key;
    if (true) {
      key.reserve(st.size() + q.size() + 64);
      auto put = [&key](const std::string& s) {
        const uint64_t n = s.size();
        key.append(reinterpret_cast<const char*>(&n), 8);
        key += s;
      };
      put(st);
      put(q);
      for (const auto& s : opts) put(s);
      key += static_cast<char>(qtype);
      key += state_is_json ? 'j' : 't';
    }
    std::shared_ptr<const j1_text_encoder::Enc> hit = e->encodings->get(key);
    if (!hit) {
      j1_text_encoder::Enc enc;
      std::string rendered;
      if (state_is_json) {  // State::render (src/request.rs:49-54)
        if (j1_status s = render_json_state(st, rendered)) return s;
      }
      std::vector<uint32_t> head, opt_ids, opt_lens, state_ids;
      if (j1_status s = request_tokens(e, state_is_json ? rendered : st, q, opts, qtype, head, opt_ids, opt_lens,
                                       state_ids))
        return s;
      j1_tokenized_request r{head.data(), head.size(), opt_ids.data(), opt_lens.data(), n_options,
                             state_ids.data(), state_ids.size(), qtype};
      enc.ids.assign(static_cast<size_t>(e->opts.max_length), 0);
      enc.markers.assign(std::max<size_t>(n_options, 1), 0);
      size_t n = 0;
      if (j1_status s = j1_encode_sequence(&e->opts, &r, enc.ids.data(), enc.ids.size(), &n, enc.markers.data(),
                                           &enc.truncated))
        return s;
      enc.ids.resize(n);
      enc.markers.resize(n_options);
      hit = std::make_shared<const j1_text_encoder::Enc>(std::move(enc));
      e->encodings->put(key, hit);
    }
    const j1_text_encoder::Enc& enc = *hit;
    *ids_len = enc.ids.size();
    if (enc.ids.size() > cap || !ids || (!markers && n_options))
      return set_error(J1_ERR_INVALID_ARG, "output arrays too small (ids_cap >= max_length, markers >= n_options)");
    std::memcpy(ids, enc.ids.data(), enc.ids.size() * 4);
    if (n_options) std::memcpy(markers, enc.markers.data(), n_options * 4);
    if (truncated) *truncated = enc.truncated;
    return J1_OK;
  });
}

j1_status j1_json_dumps(const char* json, size_t len, char* out, size_t cap, size_t* out_len) {
  return guard("j1_json_dumps", [&]() -> j1_status {
    if ((!json && len) || !out_len) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    Json j;
    std::string err;
    if (!parse_json(std::string(json ? json : "", len), j, err)) return set_error(J1_ERR_INVALID_ARG, "invalid JSON: " + err);
    std::string s;
    py_dumps(s, j);
    *out_len = s.size();
    if (s.size() > cap || (!out && !s.empty()))
      return set_error(J1_ERR_INVALID_ARG, "output buffer too small (" + std::to_string(s.size()) + " bytes needed)");
    if (!s.empty()) std::memcpy(out, s.data(), s.size());
    return J1_OK;
  });
}

namespace {

// Engine::encode's parallel Encoder::encode over rows[0, n); a failing row is reported as
// "JSONL line <line0 + its index + 1>" (the first failing one, as an in-order encode would).
j1_status encode_rows(j1_text_encoder* e, size_t n, const j1_text_request* rows, int32_t threads, size_t line0,
                      uint32_t* ids, size_t cap, size_t* offsets, uint32_t* markers, size_t mcap, size_t* moffsets,
                      int32_t* truncated) {
  if (!e || !offsets || !moffsets || (n && !rows)) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
  struct Out {
    std::vector<uint32_t> ids, markers;
    int32_t truncated = 0;
    j1_status status = J1_OK;
    std::string err;
  };
  std::vector<Out> res(n);
  const size_t row_cap = static_cast<size_t>(std::max(e->opts.max_length, 1));
  std::atomic<size_t> next{0};
  auto work = [&]() {
    for (size_t i = next++; i < n; i = next++) {
      const j1_text_request& r = rows[i];
      Out& o = res[i];
      o.ids.resize(row_cap);
      o.markers.resize(std::max<size_t>(r.n_options, 1));
      size_t len = 0;
      o.status = j1_text_encoder_encode(e, r.state, r.state_is_json, r.question, r.options, r.n_options, r.qtype,
                                        o.ids.data(), o.ids.size(), &len, o.markers.data(), &o.truncated);
      if (o.status) {
        char buf[512];
        j1_last_error(buf, sizeof(buf));  // the message is thread-local: keep it with the row
        o.err = buf;
        continue;
      }
      o.ids.resize(len);
      o.markers.resize(r.n_options);
    }
  };
  const int nt = std::max(1, std::min<int>(threads > 0 ? threads : 1, static_cast<int>(std::max<size_t>(n, 1))));
  run_pool(nt, work);
  for (size_t i = 0; i < n; ++i)  // the first failing row, as an in-order encode would report it
    if (res[i].status) return set_error(res[i].status, "JSONL line " + std::to_string(line0 + i + 1) + ": " + res[i].err);
  offsets[0] = moffsets[0] = 0;
  for (size_t i = 0; i < n; ++i) {
    offsets[i + 1] = offsets[i] + res[i].ids.size();
    moffsets[i + 1] = moffsets[i] + res[i].markers.size();
  }
  if (offsets[n] > cap || moffsets[n] > mcap || (offsets[n] && !ids) || (moffsets[n] && !markers))
    return set_error(J1_ERR_INVALID_ARG, "output arrays too small (" + std::to_string(offsets[n]) + " ids, " +
                                             std::to_string(moffsets[n]) + " markers needed)");
  for (size_t i = 0; i < n; ++i) {
    if (!res[i].ids.empty()) std::memcpy(ids + offsets[i], res[i].ids.data(), res[i].ids.size() * 4);
    if (!res[i].markers.empty()) std::memcpy(markers + moffsets[i], res[i].markers.data(), res[i].markers.size() * 4);
    if (truncated) truncated[i] = res[i].truncated;
  }
  return J1_OK;
}

}  // namespace

j1_status j1_text_encoder_encode_batch(j1_text_encoder* e, size_t n, const j1_text_request* rows, int32_t threads,
                                      uint32_t* ids, size_t cap, size_t* offsets, uint32_t* markers, size_t mcap,
                                      size_t* moffsets, int32_t* truncated) {
  return guard("j1_text_encoder_encode_batch", [&]() -> j1_status {
    return encode_rows(e, n, rows, threads, 0, ids, cap, offsets, markers, mcap, moffsets, truncated);
  });
}

namespace {

// The calling thread's last error message, for handing it to another thread.
std::string last_error_text() {
  const size_t n = j1_last_error(nullptr, 0);
  std::string m(n + 1, '\0');
  j1_last_error(&m[0], m.size());
  m.resize(n);
  return m;
}

// One chunk of rows [r0, r1) of a j1_engine_logits_text call, encoded for the engine.
struct TextChunk {
  size_t r0 = 0, r1 = 0;
  std::vector<uint32_t> ids, markers, lens, nmark;
  std::vector<uint8_t> qt;
  std::vector<size_t> offs, moffs;
  j1_status st = J1_OK;
  std::string err;
};

void encode_chunk(j1_text_encoder* e, const j1_text_request* rows, const std::vector<size_t>& mstart,
                  int32_t threads, TextChunk& c) noexcept {
  try {
    const size_t m = c.r1 - c.r0;
    const size_t L = static_cast<size_t>(std::max(e->opts.max_length, 1));
    c.ids.resize(m * L);
    c.markers.resize(std::max<size_t>(mstart[c.r1] - mstart[c.r0], 1));
    c.offs.resize(m + 1);
    c.moffs.resize(m + 1);
    c.st = encode_rows(e, m, rows + c.r0, threads, c.r0, c.ids.data(), c.ids.size(), c.offs.data(),
                       c.markers.data(), c.markers.size(), c.moffs.data(), nullptr);
    if (c.st) {
      c.err = last_error_text();
      return;
    }
    c.lens.resize(m);
    c.nmark.resize(m);
    c.qt.resize(m);
    for (size_t i = 0; i < m; ++i) {
      c.lens[i] = static_cast<uint32_t>(c.offs[i + 1] - c.offs[i]);
      c.nmark[i] = static_cast<uint32_t>(c.moffs[i + 1] - c.moffs[i]);
      c.qt[i] = rows[c.r0 + i].qtype;
    }
  } catch (const std::bad_alloc&) {
    c.st = J1_ERR_OOM;  // the caller words the message
  } catch (...) {
    c.st = J1_ERR_INTERNAL;
  }
}

}  // namespace

j1_status j1_engine_logits_text(j1_engine* engine, j1_text_encoder* e, size_t n, const j1_text_request* rows,
                                int32_t threads, float* logits_out) {
  return guard("j1_engine_logits_text", [&]() -> j1_status {
    if (!engine || !e) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (n == 0) return J1_OK;
    if (!rows || !logits_out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    // Request::validate for every row before any encoding (src/engine.rs:183-188)
    for (size_t i = 0; i < n; ++i) {
      const j1_text_request& r = rows[i];
      bool empty = r.n_options && !r.options;
      for (size_t k = 0; k < r.n_options && !empty; ++k) empty = !r.options[k] || !r.options[k][0];
      if (r.n_options < 2 || r.n_options > 20 || empty)
        return set_error(J1_ERR_INVALID_ARG, "JSONL line " + std::to_string(i + 1) +
                                                 ": options must contain 2–20 nonempty rendered descriptions");
      if (r.qtype == 2 && r.n_options != 2)
        return set_error(J1_ERR_INVALID_ARG,
                         "JSONL line " + std::to_string(i + 1) + ": noul options must be ordered [false, true]");
    }
    if (e->opts.max_length > j1_engine_max_length(engine))
      return set_error(J1_ERR_INVALID_ARG, "encoder max_length exceeds the engine's max_length");
    // Engine::logits (src/engine.rs:236-243) encodes every row, then scores them all. Here the
    // rows go in chunks of a few engine micro-batches and a helper thread encodes chunk k + 1
    // while this thread scores chunk k. A row's logits do not depend on the rows batched
    // with it, so the results are the same bits; an encoding error (the first failing row)
    // still takes precedence over a forward error, as in encode-then-score order.
    std::vector<size_t> mstart(n + 1, 0);
    for (size_t i = 0; i < n; ++i) mstart[i + 1] = mstart[i] + rows[i].n_options;
    const size_t R = std::max<size_t>(1, engine_pipeline_rows(engine));
    auto failed = [](const TextChunk& c) {
      return set_error(c.st, !c.err.empty() ? c.err
                             : c.st == J1_ERR_OOM ? "j1_engine_logits_text: host memory exhausted"
                                                  : "j1_engine_logits_text: encoding failed");
    };
    TextChunk cur, next;
    cur.r1 = std::min(n, std::max<size_t>(R / 4, 1));  // a short first chunk: less encoding left unhidden
    encode_chunk(e, rows, mstart, threads, cur);
    j1_status fwd = J1_OK;
    std::string fwd_msg;
    while (true) {
      if (cur.st) return failed(cur);
      const bool more = cur.r1 < n;
      std::thread helper;
      if (more) {
        next = TextChunk();
        next.r0 = cur.r1;
        next.r1 = std::min(n, next.r0 + R);
        try {
          helper = std::thread([&] { encode_chunk(e, rows, mstart, threads, next); });
        } catch (...) {  // no helper thread: encode the next chunk after this one's forward
        }
      }
      // Nothing between the helper's start and its join may throw (a joinable std::thread
      // must not be destroyed): the forward entry point returns a status, never throws.
      const bool async = helper.joinable();
      j1_status fs = J1_OK;
      if (!fwd)
        fs = j1_engine_logits_encoded(engine, cur.r1 - cur.r0, cur.ids.data(), cur.lens.data(), cur.markers.data(),
                                      cur.nmark.data(), cur.qt.data(), logits_out + mstart[cur.r0]);
      if (async) helper.join();
      if (fs) {  // this thread's message, taken before any encoding on this thread replaces it
        fwd = fs;
        fwd_msg = last_error_text();
      }
      if (!async && more) encode_chunk(e, rows, mstart, threads, next);
      if (!more) break;
      cur = std::move(next);
    }
    if (fwd) return set_error(fwd, fwd_msg);
    return J1_OK;
  });
}

j1_status j1_text_encoder_request_tokens(j1_text_encoder* e, const char* state, const char* question,
                                         const char* const* options, size_t n_options, uint8_t qtype, uint32_t* ids,
                                         size_t cap, size_t* total, uint32_t* piece_lens) {
  return guard("j1_text_encoder_request_tokens", [&]() -> j1_status {
    if (!e || !total) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::string st, q;
    std::vector<std::string> opts;
    if (j1_status s = read_request(state, question, options, n_options, qtype, st, q, opts)) return s;
    std::vector<uint32_t> head, opt_ids, opt_lens, state_ids;
    if (j1_status s = request_tokens(e, st, q, opts, qtype, head, opt_ids, opt_lens, state_ids)) return s;
    *total = head.size() + opt_ids.size() + state_ids.size();
    if (!ids || !piece_lens) return J1_OK;  // size query
    if (*total > cap) return set_error(J1_ERR_INVALID_ARG, "ids buffer too small");
    std::memcpy(ids, head.data(), head.size() * 4);
    std::memcpy(ids + head.size(), opt_ids.data(), opt_ids.size() * 4);
    std::memcpy(ids + head.size() + opt_ids.size(), state_ids.data(), state_ids.size() * 4);
    piece_lens[0] = static_cast<uint32_t>(head.size());
    for (size_t k = 0; k < n_options; ++k) piece_lens[1 + k] = opt_lens[k];
    piece_lens[1 + n_options] = static_cast<uint32_t>(state_ids.size());
    return J1_OK;
  });
}

}  // extern "C"
