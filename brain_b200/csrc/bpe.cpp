// Native BPE encoder: splits text on whitespace, maps each word's code points to symbol ids (the last one
// carrying the end-of-word suffix), and merges the adjacent pair of lowest rank until none is left,
// then emits the vocabulary ids. This is the hot loop of the Python BpeTokenizer (brain_b200/text.py)
// for large corpora; both follow the byte-pair-encoding merge rule of Sennrich et al. (2016) as the
// reference tokenizer does (crates/brain-text/src/tokenizer/bpe.rs:76-135).
//
// Symbols are integers: the caller registers every vocabulary string (id = registration order) and
// every merge as (left id, right id, merged id) in rank order. Words are cached.
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#define BRAIN_API extern "C" __attribute__((visibility("default")))

namespace {

struct PairHash {
  size_t operator()(uint64_t k) const { return std::hash<uint64_t>()(k * 0x9E3779B97F4A7C15ull); }
};

struct Bpe {
  std::unordered_map<std::string, int32_t> vocab;
  std::unordered_map<uint64_t, std::pair<int32_t, int32_t>, PairHash> merges;  // (a, b) -> (rank, merged)
  std::string suffix;
  int32_t unk = -1;
  std::unordered_map<std::string, std::vector<int32_t>> cache;
};

inline uint64_t key(int32_t a, int32_t b) { return (uint64_t)(uint32_t)a << 32 | (uint32_t)b; }

// Length in bytes of the UTF-8 sequence starting with byte c (1 for invalid lead bytes).
inline int utf8_len(unsigned char c) {
  if (c < 0x80) return 1;
  if ((c >> 5) == 6) return 2;
  if ((c >> 4) == 14) return 3;
  if ((c >> 3) == 30) return 4;
  return 1;
}

void encode_word(Bpe& b, const std::string& w, std::vector<int32_t>& out) {
  auto hit = b.cache.find(w);
  if (hit != b.cache.end()) {
    out.insert(out.end(), hit->second.begin(), hit->second.end());
    return;
  }
  std::vector<std::string> chars;
  for (size_t i = 0; i < w.size();) {
    const int n = utf8_len((unsigned char)w[i]);
    chars.emplace_back(w.substr(i, (size_t)n));
    i += (size_t)n;
  }
  if (!chars.empty()) chars.back() += b.suffix;
  std::vector<int32_t> sym;
  sym.reserve(chars.size());
  for (auto& c : chars) {
    auto it = b.vocab.find(c);
    sym.push_back(it == b.vocab.end() ? b.unk : it->second);
  }
  while (sym.size() > 1) {
    int32_t best = INT32_MAX, idx = -1, merged = -1;
    for (size_t i = 0; i + 1 < sym.size(); ++i) {
      if (sym[i] < 0 || sym[i + 1] < 0) continue;
      auto it = b.merges.find(key(sym[i], sym[i + 1]));
      if (it != b.merges.end() && it->second.first < best) {
        best = it->second.first;
        idx = (int32_t)i;
        merged = it->second.second;
      }
    }
    if (idx < 0) break;
    sym[(size_t)idx] = merged;
    sym.erase(sym.begin() + idx + 1);
  }
  b.cache.emplace(w, sym);
  out.insert(out.end(), sym.begin(), sym.end());
}

}  // namespace

BRAIN_API void* brain_bpe_create(const char* suffix) {
  auto* b = new Bpe();
  b->suffix = suffix ? suffix : "";
  return b;
}

// Registers vocabulary string number `id` (UTF-8, len bytes); `is_unk` marks the unknown token.
BRAIN_API int brain_bpe_add_token(void* h, const char* s, int64_t len, int id, int is_unk) {
  auto* b = static_cast<Bpe*>(h);
  if (!b || !s || len < 0) return -10;
  b->vocab[std::string(s, (size_t)len)] = id;
  if (is_unk) b->unk = id;
  return 0;
}

// Registers merges (left, right) -> merged for ranks 0..n-1; triples is [n, 3] int32.
BRAIN_API int brain_bpe_add_merges(void* h, const int32_t* triples, int64_t n) {
  auto* b = static_cast<Bpe*>(h);
  if (!b || (!triples && n)) return -10;
  for (int64_t r = 0; r < n; ++r)
    b->merges[key(triples[3 * r], triples[3 * r + 1])] = {(int32_t)r, triples[3 * r + 2]};
  return 0;
}

// Encodes UTF-8 text (len bytes) into ids; returns the number of ids (which may exceed cap: the caller
// then retries with a larger buffer) or a negative error.
BRAIN_API int64_t brain_bpe_encode(void* h, const char* text, int64_t len, int32_t* out, int64_t cap) {
  auto* b = static_cast<Bpe*>(h);
  if (!b || (!text && len)) return -10;
  std::vector<int32_t> ids;
  int64_t i = 0;
  while (i < len) {
    while (i < len && (text[i] == ' ' || text[i] == '\t' || text[i] == '\n' || text[i] == '\r' || text[i] == '\f' ||
                       text[i] == '\v'))
      ++i;
    int64_t j = i;
    while (j < len && !(text[j] == ' ' || text[j] == '\t' || text[j] == '\n' || text[j] == '\r' || text[j] == '\f' ||
                        text[j] == '\v'))
      ++j;
    if (j > i) encode_word(*b, std::string(text + i, (size_t)(j - i)), ids);
    i = j;
  }
  const int64_t n = (int64_t)ids.size();
  if (out && n <= cap) std::memcpy(out, ids.data(), (size_t)n * sizeof(int32_t));
  return n;
}

BRAIN_API int brain_bpe_destroy(void* h) {
  delete static_cast<Bpe*>(h);
  return 0;
}
