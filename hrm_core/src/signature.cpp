// Text -> 2048-bin quantised signature.
// Features: word 3-grams (word = maximal run of ASCII alphanumerics or '\'', lower-cased, the three words joined by
// 0x1F) followed by character 5-grams of the whitespace-collapsed, lower-cased, trimmed text; at most 20000
// features in total.  Each feature is hashed with 64-bit FNV-1a and counted in bin (hash & 2047); the count is
// quantised as min(15, count * 2048 / total).  (The hash seed differs from textbook FNV-1a, see kFnvBasis.)  Character classes are those of the "C" locale.
#include "hrm/hrm.h"

#include <stdexcept>

namespace hrm {
namespace {

// Offset value used by the reference's fnv1a_64 (signature.cpp:11 there).  It is NOT the published FNV-1a 64-bit
// offset basis (14695981039346656037, one digit longer); it is kept so signatures, indexes and scores stay
// bit-identical with indexes built by the reference.
constexpr uint64_t kFnvBasis = 1469598103934665603ULL;
constexpr uint64_t kFnvPrime = 1099511628211ULL;          // FNV-1a 64-bit prime
constexpr uint32_t kMaxFeatures = 20000;

inline bool is_word(unsigned char c) {
  return (c >= '0' && c <= '9') || (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || c == '\'';
}
inline bool is_space(unsigned char c) { return c == ' ' || (c >= '\t' && c <= '\r'); }
inline unsigned char lower(unsigned char c) { return (c >= 'A' && c <= 'Z') ? (unsigned char)(c + 32) : c; }

inline uint64_t fnv_feed(uint64_t h, const unsigned char* p, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= kFnvPrime;
  }
  return h;
}

}  // namespace

Sig signature(const std::string& text) {
  // words as [begin, end) ranges into a lower-cased copy
  std::string low(text.size(), '\0');
  for (size_t i = 0; i < text.size(); ++i) low[i] = (char)lower((unsigned char)text[i]);
  std::vector<std::pair<size_t, size_t>> words;
  words.reserve(text.size() / 4 + 1);
  size_t i = 0;
  const size_t n = low.size();
  while (i < n) {
    while (i < n && !is_word((unsigned char)low[i])) ++i;
    const size_t b = i;
    while (i < n && is_word((unsigned char)low[i])) ++i;
    if (i > b) words.emplace_back(b, i);
  }

  uint32_t counts[kBins] = {0};
  uint32_t total = 0;
  const unsigned char sep = 0x1F;
  const auto* lp = reinterpret_cast<const unsigned char*>(low.data());
  for (size_t w = 0; w + 3 <= words.size(); ++w) {
    if (total >= kMaxFeatures) break;
    uint64_t h = kFnvBasis;
    for (int j = 0; j < 3; ++j) {
      if (j) h = fnv_feed(h, &sep, 1);
      h = fnv_feed(h, lp + words[w + j].first, words[w + j].second - words[w + j].first);
    }
    ++counts[h & (kBins - 1)];
    ++total;
  }

  // whitespace-collapsed, lower-cased, trimmed text
  std::string norm;
  norm.reserve(n);
  bool in_ws = false;
  for (size_t k = 0; k < n; ++k) {
    const unsigned char c = (unsigned char)text[k];
    if (is_space(c)) {
      if (!in_ws) norm.push_back(' ');
      in_ws = true;
    } else {
      norm.push_back((char)lower(c));
      in_ws = false;
    }
  }
  size_t a = 0, e = norm.size();
  while (a < e && norm[a] == ' ') ++a;
  while (e > a && norm[e - 1] == ' ') --e;
  const auto* np = reinterpret_cast<const unsigned char*>(norm.data()) + a;
  const size_t nn = e - a;
  for (size_t k = 0; k + 5 <= nn; ++k) {
    if (total >= kMaxFeatures) break;
    ++counts[fnv_feed(kFnvBasis, np + k, 5) & (kBins - 1)];
    ++total;
  }

  if (total == 0) {
    counts[0] = 1;
    total = 1;
  }
  Sig q(kBins);
  for (int b = 0; b < kBins; ++b) {
    const uint32_t v = counts[b] * (uint32_t)kBins / total;
    q[b] = (uint8_t)(v > (uint32_t)(kLevels - 1) ? kLevels - 1 : v);
  }
  return q;
}

std::vector<uint8_t> pack_nibbles(const Sig& q) {
  if (q.size() != (size_t)kBins) throw std::runtime_error("signature must have 2048 bins");
  std::vector<uint8_t> out(kBlobBytes);
  for (int j = 0; j < kBlobBytes; ++j) out[j] = (uint8_t)(((q[2 * j] & 15) << 4) | (q[2 * j + 1] & 15));
  return out;
}

Sig unpack_nibbles(const std::vector<uint8_t>& blob) {
  if (blob.size() != (size_t)kBlobBytes) throw std::runtime_error("signature blob must have 1024 bytes");
  Sig q(kBins);
  for (int j = 0; j < kBlobBytes; ++j) {
    q[2 * j] = (uint8_t)(blob[j] >> 4);
    q[2 * j + 1] = (uint8_t)(blob[j] & 15);
  }
  return q;
}

int overlap_sig_sig(const uint8_t* a, const uint8_t* b) {
  int s = 0;
  for (int i = 0; i < kBins; ++i) s += a[i] < b[i] ? a[i] : b[i];
  return s;
}

std::string cid_str(uint32_t cid) {
  char buf[16];
  std::snprintf(buf, sizeof(buf), "%04u", cid);
  return buf;
}

std::string sid_str(uint32_t cid, uint32_t sidx) {
  char buf[32];
  std::snprintf(buf, sizeof(buf), "%04u#s%04u", cid, sidx);
  return buf;
}

uint32_t parse_cid(const std::string& s) { return (uint32_t)std::stoul(s); }

}  // namespace hrm
