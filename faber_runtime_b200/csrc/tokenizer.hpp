// tokenizer.hpp — GPT-2 byte-level BPE with the `smollm` pre-tokenizer
// (src/tokenizer/mod.rs, pretoken.rs, bpe.rs), host code. text -> ids:
//  1. special-token partition: with parse_special, every control, unknown
//     and user-defined token text found in the input becomes its id
//     (longest texts first); without it, only user-defined ones do;
//  2. pre-tokenizer: each number codepoint becomes its own piece, then the
//     GPT-2 splitter 's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+|
//     ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+ runs over each piece;
//  3. every byte of a piece maps to its GPT-2 display character;
//  4. BPE: adjacent symbols merge lowest merge rank first (ties: leftmost);
//     a final symbol that is not a token falls back to one token per raw
//     byte that has a single-byte ASCII token.
// Construction is fail-closed like the reference (mod.rs:329-530): model
// "gpt2", pre "smollm", exact vocabulary and merge counts, no scores,
// well-formed merges, non-empty token texts without a literal space, ids in
// range, add_bos_token and add_space_prefix false. The caller states the
// expected counts (the pinned row's are 49 152 tokens and 48 900 merges).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace faber {
namespace tok {

#include "unicode_classes.inc"

constexpr uint64_t kPinnedVocab = 49152;           // mod.rs:94
constexpr uint64_t kPinnedMerges = 48900;          // mod.rs:96
constexpr uint64_t kMaxTokenBytes = 4096;          // mod.rs:113
constexpr uint64_t kMaxMergeBytes = 2 * kMaxTokenBytes + 1;
constexpr uint64_t kMaxSpecials = 1024;            // mod.rs:117
constexpr uint64_t kMaxInputBytes = 1ull << 20;    // mod.rs:119
constexpr uint64_t kMaxOutputTokens = 1ull << 20;  // mod.rs:121

// llama token types (tokenizer.ggml.token_type)
constexpr int32_t kTypeNormal = 1, kTypeUnknown = 2, kTypeControl = 3, kTypeUserDefined = 4;

constexpr uint32_t kClassNumber = 2, kClassLetter = 4, kClassSpace = 0x100;

[[noreturn]] inline void tok_fail(const std::string& kind, const std::string& detail, int code = 1) {
  throw Error(code, kind + ": " + detail);
}

// Unicode White_Space property (PropList.txt).
inline bool is_white_space(uint32_t cp) {
  return (cp >= 0x09 && cp <= 0x0D) || cp == 0x20 || cp == 0x85 || cp == 0xA0 || cp == 0x1680 ||
         (cp >= 0x2000 && cp <= 0x200A) || cp == 0x2028 || cp == 0x2029 || cp == 0x202F || cp == 0x205F ||
         cp == 0x3000;
}

inline uint32_t cp_class(uint32_t cp) {
  constexpr size_t n = sizeof(kUnicodeClassRanges) / sizeof(kUnicodeClassRanges[0]);
  size_t lo = 0, hi = n;  // last range whose start <= cp
  while (hi - lo > 1) {
    const size_t mid = (lo + hi) / 2;
    if (kUnicodeClassRanges[mid][0] <= cp) lo = mid; else hi = mid;
  }
  return kUnicodeClassRanges[lo][1] | (is_white_space(cp) ? kClassSpace : 0u);
}

// GPT-2's bytes-to-unicode map: printable bytes ('!'-'~', 0xA1-0xAC,
// 0xAE-0xFF) stand for themselves, the other 68 take codepoints 256.. in
// byte order.
struct ByteMap {
  uint32_t to_cp[256];
  std::unordered_map<uint32_t, uint8_t> from_cp;
  ByteMap() {
    uint32_t extra = 0;
    for (uint32_t b = 0; b < 256; ++b) {
      const bool keep = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE);
      to_cp[b] = keep ? b : 256 + extra++;
      from_cp[to_cp[b]] = (uint8_t)b;
    }
  }
};

inline const ByteMap& byte_map() {
  static const ByteMap m;
  return m;
}

inline void put_utf8(std::string& s, uint32_t cp) {
  if (cp < 0x80) {
    s += (char)cp;
  } else if (cp < 0x800) {
    s += (char)(0xC0 | cp >> 6);
    s += (char)(0x80 | (cp & 0x3F));
  } else if (cp < 0x10000) {
    s += (char)(0xE0 | cp >> 12);
    s += (char)(0x80 | (cp >> 6 & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  } else {
    s += (char)(0xF0 | cp >> 18);
    s += (char)(0x80 | (cp >> 12 & 0x3F));
    s += (char)(0x80 | (cp >> 6 & 0x3F));
    s += (char)(0x80 | (cp & 0x3F));
  }
}

// Codepoints of valid UTF-8 with each one's byte offset (offsets has one
// more entry: the end). Invalid input is refused.
inline void decode_utf8(const std::string& s, std::vector<uint32_t>& cps, std::vector<size_t>& offsets) {
  cps.clear();
  offsets.clear();
  size_t i = 0;
  const auto* p = reinterpret_cast<const uint8_t*>(s.data());
  while (i < s.size()) {
    const uint8_t c = p[i];
    uint32_t cp = 0, len = 0, min = 0;
    if (c < 0x80) { cp = c; len = 1; }
    else if ((c & 0xE0) == 0xC0) { cp = c & 0x1F; len = 2; min = 0x80; }
    else if ((c & 0xF0) == 0xE0) { cp = c & 0x0F; len = 3; min = 0x800; }
    else if ((c & 0xF8) == 0xF0) { cp = c & 0x07; len = 4; min = 0x10000; }
    else tok_fail("InvalidUtf8", "byte " + std::to_string(i));
    if (i + len > s.size()) tok_fail("InvalidUtf8", "truncated sequence at byte " + std::to_string(i));
    for (uint32_t k = 1; k < len; ++k) {
      if ((p[i + k] & 0xC0) != 0x80) tok_fail("InvalidUtf8", "byte " + std::to_string(i + k));
      cp = cp << 6 | (p[i + k] & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))
      tok_fail("InvalidUtf8", "codepoint at byte " + std::to_string(i));
    cps.push_back(cp);
    offsets.push_back(i);
    i += len;
  }
  offsets.push_back(s.size());
}

struct Facts {
  std::string model, pre;
  std::vector<std::string> tokens;
  std::vector<int32_t> token_types;
  std::vector<std::string> merges;
  bool scores_present = false;
  uint32_t bos = 1, eos = 2, pad = 2, unk = 0;
  bool add_bos = false, add_space_prefix = false;
  uint64_t expected_vocab = kPinnedVocab, expected_merges = kPinnedMerges;
};

struct PairHash {
  size_t operator()(const std::pair<std::string, std::string>& p) const {
    return std::hash<std::string>()(p.first) * 1000003u ^ std::hash<std::string>()(p.second);
  }
};

class Tokenizer {
 public:
  // Gpt2BpeTokenizer::new: every fact checked in the reference's order.
  explicit Tokenizer(const Facts& f) {
    if (f.model != "gpt2") tok_fail("UnsupportedModel", "tokenizer model \"" + f.model + "\" is not \"gpt2\"");
    if (f.pre != "smollm") tok_fail("UnsupportedPreTokenizer", "tokenizer pre \"" + f.pre + "\" is not \"smollm\"");
    if (f.tokens.size() != f.expected_vocab)
      tok_fail("VocabSizeMismatch", "vocab count " + std::to_string(f.tokens.size()) + " != expected " +
                                        std::to_string(f.expected_vocab));
    if (f.token_types.size() != f.tokens.size())
      tok_fail("TokenTypeCountMismatch", "token_type count " + std::to_string(f.token_types.size()) +
                                             " != vocab count " + std::to_string(f.tokens.size()));
    if (f.merges.size() != f.expected_merges)
      tok_fail("MergesCountMismatch", "merges count " + std::to_string(f.merges.size()) + " != expected " +
                                          std::to_string(f.expected_merges));
    if (f.scores_present) tok_fail("ScoresPresent", "tokenizer.ggml.scores is present");
    if (f.add_bos) tok_fail("AddBosTokenNotSupported", "add_bos_token = true");
    if (f.add_space_prefix) tok_fail("AddSpacePrefixNotSupported", "add_space_prefix = true");
    vocab_ = f.tokens.size();
    std::fill(std::begin(byte_fallback_), std::end(byte_fallback_), UINT32_MAX);
    text_.reserve(vocab_);
    for (size_t id = 0; id < vocab_; ++id) {
      const std::string& t = f.tokens[id];
      if (t.empty() || t.size() > kMaxTokenBytes || t.find(' ') != std::string::npos)
        tok_fail("ByteBoundaryViolation", "token " + std::to_string(id) + " is empty, overlong or has a space");
      id_.emplace(t, (uint32_t)id);  // the first id of a text wins
      text_.push_back(t);
      if (t.size() == 1 && (uint8_t)t[0] < 0x80) byte_fallback_[(uint8_t)t[0]] = (uint32_t)id;
    }
    for (size_t i = 0; i < f.merges.size(); ++i) {
      const std::string& m = f.merges[i];
      // the first space splits the pair; one at position 0 is malformed
      const size_t sep = m.size() > kMaxMergeBytes ? std::string::npos : m.find(' ');
      if (sep == std::string::npos || sep == 0 || sep + 1 >= m.size())
        tok_fail("MalformedMergeString", "merge " + std::to_string(i) + ": \"" + m + "\"");
      rank_.emplace(std::make_pair(m.substr(0, sep), m.substr(sep + 1)), (uint32_t)i);  // first wins
    }
    for (uint32_t id : {f.bos, f.eos, f.pad, f.unk})
      if (id >= vocab_)
        tok_fail("TokenIdOutOfRange", "token id " + std::to_string(id) + " out of [0, " + std::to_string(vocab_) + ")");
    for (size_t id = 0; id < vocab_; ++id) {
      const int32_t t = f.token_types[id];
      if (t == kTypeControl || t == kTypeUnknown || t == kTypeUserDefined)
        specials_.push_back({f.tokens[id], (uint32_t)id, t});
    }
    if (specials_.size() > kMaxSpecials) tok_fail("ArithmeticOverflow", "special token cache ceiling");
    std::stable_sort(specials_.begin(), specials_.end(), [](const Special& a, const Special& b) {
      return a.text.size() != b.text.size() ? a.text.size() > b.text.size() : a.id < b.id;
    });
    // end-of-generation ids: tokens with these texts, then eos
    static const char* kEog[] = {"<|eot_id|>", "<|im_end|>", "<|end|>", "<|return|>", "<|call|>",
                                 "<|flush|>", "<|calls|>", "<end_of_turn>", "<|endoftext|>", "</s>",
                                 "<|eom_id|>", "<EOT>", "_<EOT>", "[EOT]", "[EOS]", "<|end_of_text|>",
                                 "<end_of_utterance>", "<eos>", "<turn|>", "<|tool_response>",
                                 "<\xEF\xBD\x9C" "end\xE2\x96\x81" "of\xE2\x96\x81" "sentence\xEF\xBD\x9C>",
                                 "[e~["};
    for (size_t id = 0; id < vocab_; ++id)
      for (const char* e : kEog)
        if (f.tokens[id] == e) {
          eog_.push_back((uint32_t)id);
          break;
        }
    if (std::find(eog_.begin(), eog_.end(), f.eos) == eog_.end()) eog_.push_back(f.eos);
    bos_ = f.bos;
    eos_ = f.eos;
    pad_ = f.pad;
    unk_ = f.unk;
  }

  size_t vocab_size() const { return vocab_; }
  const std::vector<uint32_t>& eog() const { return eog_; }
  uint32_t bos() const { return bos_; }
  uint32_t eos() const { return eos_; }
  uint32_t pad() const { return pad_; }
  uint32_t unk() const { return unk_; }

  // encode (mod.rs:690-770).
  std::vector<uint32_t> encode(const std::string& text, bool parse_special) const {
    std::vector<uint32_t> out;
    if (text.empty()) return out;
    if (text.size() > kMaxInputBytes)
      tok_fail("InputTooLarge", "encode input " + std::to_string(text.size()) + " bytes exceeds " +
                                    std::to_string(kMaxInputBytes));
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    decode_utf8(text, cps, offs);
    // 1. special partition: fragments are (start, len, id), id UINT32_MAX for text
    struct Frag { size_t start, len; uint32_t id; };
    std::vector<Frag> frags{{0, text.size(), UINT32_MAX}};
    for (const Special& sp : specials_) {
      if (!parse_special && sp.type != kTypeUserDefined) continue;
      std::vector<Frag> next;
      for (const Frag& fr : frags) {
        if (fr.id != UINT32_MAX) {
          next.push_back(fr);
          continue;
        }
        size_t base = fr.start;
        const size_t end = fr.start + fr.len;
        while (base < end) {
          const size_t m = text.find(sp.text, base);
          if (m == std::string::npos || m + sp.text.size() > end) break;
          if (m > base) next.push_back({base, m - base, UINT32_MAX});
          next.push_back({m, sp.text.size(), sp.id});
          base = m + sp.text.size();
        }
        if (base < end) next.push_back({base, end - base, UINT32_MAX});
      }
      frags.swap(next);
    }
    for (const Frag& fr : frags) {
      if (fr.id != UINT32_MAX) {
        push(out, fr.id);
        continue;
      }
      // the fragment's codepoint range (special texts are whole UTF-8)
      const size_t c0 = std::lower_bound(offs.begin(), offs.end(), fr.start) - offs.begin();
      const size_t c1 = std::lower_bound(offs.begin(), offs.end(), fr.start + fr.len) - offs.begin();
      std::vector<std::pair<size_t, size_t>> words;
      pre_tokenize(cps, c0, c1, words);
      for (const auto& w : words) bpe_word(text.substr(offs[w.first], offs[w.second] - offs[w.first]), out);
    }
    return out;
  }

  // Token texts through the inverse display map (text outside the map, such
  // as special tokens, is kept as it is).
  std::string decode(const std::vector<uint32_t>& ids) const {
    std::string out;
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    for (uint32_t id : ids) {
      if (id >= vocab_) tok_fail("TokenIdOutOfRange", "token id " + std::to_string(id));
      decode_utf8(text_[id], cps, offs);
      for (size_t k = 0; k < cps.size(); ++k) {
        auto it = byte_map().from_cp.find(cps[k]);
        if (it != byte_map().from_cp.end()) out += (char)it->second;
        else out.append(text_[id], offs[k], offs[k + 1] - offs[k]);
      }
    }
    return out;
  }

 private:
  struct Special {
    std::string text;
    uint32_t id;
    int32_t type;
  };
  size_t vocab_ = 0;
  std::unordered_map<std::string, uint32_t> id_;
  std::unordered_map<std::pair<std::string, std::string>, uint32_t, PairHash> rank_;
  std::vector<std::string> text_;
  std::vector<Special> specials_;
  uint32_t byte_fallback_[256];
  std::vector<uint32_t> eog_;
  uint32_t bos_ = 0, eos_ = 0, pad_ = 0, unk_ = 0;

  static void push(std::vector<uint32_t>& out, uint32_t id) {
    if (out.size() >= kMaxOutputTokens)
      tok_fail("OutputTooLarge", "encode output exceeds " + std::to_string(kMaxOutputTokens) + " tokens");
    out.push_back(id);
  }

  // smollm pre-tokenizer (pretoken.rs:21-180): number codepoints alone, then
  // the GPT-2 splitter over each piece. Appends codepoint ranges.
  static void pre_tokenize(const std::vector<uint32_t>& cps, size_t c0, size_t c1,
                           std::vector<std::pair<size_t, size_t>>& words) {
    size_t cur = c0;
    for (size_t i = c0; i < c1; ++i)
      if (cp_class(cps[i]) & kClassNumber) {
        if (i > cur) split_gpt2(cps, cur, i, words);
        split_gpt2(cps, i, i + 1, words);
        cur = i + 1;
      }
    if (cur < c1) split_gpt2(cps, cur, c1, words);
  }

  static void split_gpt2(const std::vector<uint32_t>& cps, size_t ini, size_t end,
                         std::vector<std::pair<size_t, size_t>>& words) {
    auto cp = [&](size_t p) -> int64_t { return p >= ini && p < end ? (int64_t)cps[p] : -1; };
    auto cls = [&](size_t p) -> uint32_t { return p >= ini && p < end ? cp_class(cps[p]) : 0u; };
    size_t prev = ini, pos = ini;
    auto emit = [&](size_t p) {
      if (p > prev) {
        words.push_back({prev, p});
        prev = p;
      }
    };
    while (pos < end) {
      const int64_t c = cp(pos);
      // contractions, lowercase only
      if (c == '\'' && pos + 1 < end) {
        const int64_t n1 = cp(pos + 1);
        if (n1 == 's' || n1 == 't' || n1 == 'm' || n1 == 'd') {
          pos += 2;
          emit(pos);
          continue;
        }
        const int64_t n2 = cp(pos + 2);
        if (pos + 2 < end && ((n1 == 'r' && n2 == 'e') || (n1 == 'v' && n2 == 'e') || (n1 == 'l' && n2 == 'l'))) {
          pos += 3;
          emit(pos);
          continue;
        }
      }
      const uint32_t f = c == ' ' ? cls(pos + 1) : cls(pos);  // an optional leading space
      const size_t lead = c == ' ' ? 1 : 0;
      if (f & kClassLetter) {
        pos += lead;
        while (cls(pos) & kClassLetter) ++pos;
        emit(pos);
        continue;
      }
      if (f & kClassNumber) {
        pos += lead;
        while (cls(pos) & kClassNumber) ++pos;
        emit(pos);
        continue;
      }
      const uint32_t other = kClassSpace | kClassLetter | kClassNumber;
      if (f != 0 && !(f & other)) {
        pos += lead;
        while (cls(pos) != 0 && !(cls(pos) & other)) ++pos;
        emit(pos);
        continue;
      }
      size_t ws = 0;
      while (cls(pos + ws) & kClassSpace) ++ws;
      if (ws > 1 && cp(pos + ws) >= 0) {  // \s+(?!\S): the last space joins the next word
        pos += ws - 1;
        emit(pos);
        continue;
      }
      pos += ws > 0 ? ws : 1;
      emit(pos);
    }
  }

  // bpe.rs:49-213 over one word's display form.
  void bpe_word(const std::string& word, std::vector<uint32_t>& out) const {
    std::string display;
    for (unsigned char b : word) put_utf8(display, byte_map().to_cp[b]);
    std::vector<uint32_t> cps;
    std::vector<size_t> offs;
    decode_utf8(display, cps, offs);
    const size_t n = cps.size();
    if (n == 0) return;
    struct Sym { long prev, next; size_t start, len; };
    std::vector<Sym> sym(n);
    for (size_t i = 0; i < n; ++i) sym[i] = {(long)i - 1, i + 1 == n ? -1 : (long)i + 1, offs[i], offs[i + 1] - offs[i]};
    struct Cand {
      uint32_t rank;
      size_t left, right, len;
      bool operator<(const Cand& o) const {  // the queue pops the lowest rank, then the leftmost
        return rank != o.rank ? rank > o.rank : left > o.left;
      }
    };
    std::priority_queue<Cand> q;
    auto piece = [&](size_t i) { return display.substr(sym[i].start, sym[i].len); };
    auto add = [&](long l, long r) {
      if (l < 0 || r < 0) return;
      auto it = rank_.find({piece((size_t)l), piece((size_t)r)});
      if (it != rank_.end()) q.push({it->second, (size_t)l, (size_t)r, sym[l].len + sym[r].len});
    };
    for (size_t i = 1; i < n; ++i) add((long)i - 1, (long)i);
    while (!q.empty()) {
      const Cand c = q.top();
      q.pop();
      Sym& L = sym[c.left];
      Sym& R = sym[c.right];
      // stale: a side merged since (its length changed or it is gone)
      if (L.len == 0 || R.len == 0 || L.next != (long)c.right || L.len + R.len != c.len) continue;
      L.len += R.len;
      L.next = R.next;
      R.len = 0;
      if (L.next >= 0) sym[L.next].prev = (long)c.left;
      add(L.prev, (long)c.left);
      add((long)c.left, L.next);
    }
    for (long i = 0; i >= 0; i = sym[i].next) {
      if (sym[i].len == 0) continue;
      const std::string t = piece((size_t)i);
      auto it = id_.find(t);
      if (it != id_.end()) {
        push(out, it->second);
      } else {
        for (unsigned char b : t)
          if (byte_fallback_[b] != UINT32_MAX) push(out, byte_fallback_[b]);
      }
    }
  }
};

}  // namespace tok
}  // namespace faber
