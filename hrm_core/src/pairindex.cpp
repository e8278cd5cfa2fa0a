// PairIndex tokenizer (see include/hrm/pairindex.h).
// Reference behaviour: experiments/run_llm_orig.sh:61-307 (index_build_v7) and llm_engine.cu:141-336.
#include "hrm/pairindex.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <stdexcept>

namespace hrm {
namespace pairidx {
namespace {

inline uint16_t pack(uint8_t a, uint8_t b) { return (uint16_t)(a | (uint16_t)(b << 8)); }
inline uint32_t key2(uint16_t a, uint16_t b) { return ((uint32_t)a << 16) | b; }
inline uint32_t slot_of(uint32_t k, uint32_t mask) { return (k * 2654435761u) & mask; }

std::vector<uint8_t> read_file(const std::string& p) {
  std::ifstream f(p, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + p);
  return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

// ranking: count descending, key ascending
template <typename K>
void rank(std::vector<std::pair<uint64_t, K>>& items) {
  std::sort(items.begin(), items.end(), [](const auto& x, const auto& y) {
    return x.first != y.first ? x.first > y.first : x.second < y.second;
  });
}

void stage1_from_counts(PairIndex& pi, const std::vector<uint64_t>& cnt, int k1) {
  std::vector<std::pair<uint64_t, uint16_t>> items;
  for (uint32_t p = 0; p < 65536; ++p)
    if (cnt[p]) items.push_back({cnt[p], (uint16_t)p});
  rank(items);
  pi.k1 = k1;
  pi.id2pair.clear();
  for (size_t i = 0; i < items.size() && (int)pi.id2pair.size() < k1; ++i) pi.id2pair.push_back(items[i].second);
  // fewer distinct pairs than k1: pad with unused pairs in key order (keeps the layout fixed-size)
  for (uint32_t p = 0; p < 65536 && (int)pi.id2pair.size() < k1; ++p)
    if (!cnt[p]) pi.id2pair.push_back((uint16_t)p);
  pi.pair2id.assign(65536, -1);
  for (int i = 0; i < k1; ++i) pi.pair2id[pi.id2pair[i]] = kBaseV + i;
}

// greedy stage-1 scan: calls emit(id) per token
template <typename F>
void scan1(const PairIndex& pi, const uint8_t* b, size_t n, F&& emit) {
  size_t i = 0;
  while (i < n) {
    if (i + 1 < n) {
      const int32_t id = pi.pair2id[pack(b[i], b[i + 1])];
      if (id >= 0) {
        emit((uint16_t)id);
        i += 2;
        continue;
      }
    }
    emit((uint16_t)b[i]);
    i += 1;
  }
}

void stage2_from_keys(PairIndex& pi, std::vector<uint32_t>& keys, int k2) {
  pi.k2 = k2;
  pi.id2pair2.clear();
  if (k2 > 0) {
    std::sort(keys.begin(), keys.end());
    std::vector<std::pair<uint64_t, uint32_t>> items;
    for (size_t i = 0; i < keys.size();) {
      size_t j = i;
      while (j < keys.size() && keys[j] == keys[i]) ++j;
      items.push_back({(uint64_t)(j - i), keys[i]});
      i = j;
    }
    rank(items);
    for (size_t i = 0; i < items.size() && (int)pi.id2pair2.size() < k2; ++i) pi.id2pair2.push_back(items[i].second);
    // small corpus: unreachable keys (first half 0xFFFF is never a stage-1 id)
    for (size_t j = pi.id2pair2.size(); (int)j < k2; ++j) pi.id2pair2.push_back((0xFFFFu << 16) | (uint32_t)(j & 0xFFFFu));
  }
  uint32_t need = 2;
  while (need < (uint32_t)(2 * k2)) need <<= 1;
  pi.hkeys.assign(need, kEmptyKey);
  pi.hvals.assign(need, kEmptyVal);
  pi.hmask = need - 1;
  for (int i = 0; i < k2; ++i) {
    const uint32_t k = pi.id2pair2[i];
    uint32_t h = slot_of(k, pi.hmask);
    while (pi.hkeys[h] != kEmptyKey) h = (h + 1) & pi.hmask;
    pi.hkeys[h] = k;
    pi.hvals[h] = (uint16_t)(kBaseV + pi.k1 + i);
  }
}

void check_sizes(int k1, int k2) {
  if (k1 < 0 || k2 < 0 || kBaseV + k1 + k2 >= 65536) throw std::runtime_error("vocabulary exceeds uint16 ids");
}

}  // namespace

uint32_t PairIndex::pow2() const {
  uint32_t p = 0;
  while ((1u << p) < hkeys.size()) ++p;
  return p;
}

uint16_t PairIndex::lookup2(uint16_t a, uint16_t b) const {
  if (k2 <= 0) return kEmptyVal;
  const uint32_t k = key2(a, b);
  for (uint32_t h = slot_of(k, hmask);; h = (h + 1) & hmask) {
    if (hkeys[h] == kEmptyKey) return kEmptyVal;
    if (hkeys[h] == k) return hvals[h];
  }
}

PairIndex build_from_files(std::vector<std::string> paths, int k1, int k2) {
  check_sizes(k1, k2);
  std::sort(paths.begin(), paths.end());
  std::vector<uint64_t> cnt(65536, 0);
  for (const auto& p : paths) {
    const auto b = read_file(p);
    for (size_t i = 0; i + 1 < b.size(); ++i) cnt[pack(b[i], b[i + 1])]++;
  }
  PairIndex pi;
  stage1_from_counts(pi, cnt, k1);
  std::vector<uint32_t> keys;
  for (const auto& p : paths) {
    const auto b = read_file(p);
    bool have = false;
    uint16_t prev = 0;
    scan1(pi, b.data(), b.size(), [&](uint16_t id) {
      if (have) keys.push_back(key2(prev, id));
      prev = id;
      have = true;
    });
  }
  stage2_from_keys(pi, keys, k2);
  return pi;
}

PairIndex build_from_bytes(const uint8_t* data, size_t n, int k1, int k2) {
  check_sizes(k1, k2);
  std::vector<uint64_t> cnt(65536, 0);
  for (size_t i = 0; i + 1 < n; ++i) cnt[pack(data[i], data[i + 1])]++;
  PairIndex pi;
  stage1_from_counts(pi, cnt, k1);
  std::vector<uint32_t> keys;
  bool have = false;
  uint16_t prev = 0;
  scan1(pi, data, n, [&](uint16_t id) {
    if (have) keys.push_back(key2(prev, id));
    prev = id;
    have = true;
  });
  stage2_from_keys(pi, keys, k2);
  return pi;
}

PairIndex from_tables(int k1, int k2, const uint16_t* id2pair, const uint32_t* id2pair2, uint32_t hsize,
                      const uint32_t* hkeys, const uint16_t* hvals) {
  check_sizes(k1, k2);
  if (hsize < 2 || (hsize & (hsize - 1))) throw std::runtime_error("hash table size must be a power of two >= 2");
  PairIndex pi;
  pi.k1 = k1;
  pi.k2 = k2;
  pi.id2pair.assign(id2pair, id2pair + k1);
  pi.pair2id.assign(65536, -1);
  for (int i = 0; i < k1; ++i) pi.pair2id[pi.id2pair[i]] = kBaseV + i;
  pi.id2pair2.assign(id2pair2, id2pair2 + k2);
  pi.hkeys.assign(hkeys, hkeys + hsize);
  pi.hvals.assign(hvals, hvals + hsize);
  pi.hmask = hsize - 1;
  return pi;
}

void save_idx7(const PairIndex& pi, const std::string& path) {
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  auto u32 = [&](uint32_t v) { f.write(reinterpret_cast<const char*>(&v), 4); };
  f.write("IDX7", 4);
  u32(1u);
  u32((uint32_t)pi.k1);
  u32((uint32_t)pi.k2);
  u32(pi.pow2());
  u32(0u);
  f.write(reinterpret_cast<const char*>(pi.id2pair.data()), (std::streamsize)(pi.id2pair.size() * 2));
  f.write(reinterpret_cast<const char*>(pi.id2pair2.data()), (std::streamsize)(pi.id2pair2.size() * 4));
  f.write(reinterpret_cast<const char*>(pi.hkeys.data()), (std::streamsize)(pi.hkeys.size() * 4));
  f.write(reinterpret_cast<const char*>(pi.hvals.data()), (std::streamsize)(pi.hvals.size() * 2));
  if (!f) throw std::runtime_error("write failed: " + path);
}

PairIndex load_idx7(const std::string& path) {
  const auto b = read_file(path);
  if (b.size() < 24 || std::memcmp(b.data(), "IDX7", 4) != 0) throw std::runtime_error("bad index magic: " + path);
  uint32_t h[5];
  std::memcpy(h, b.data() + 4, 20);
  if (h[0] != 1u) throw std::runtime_error("unsupported index version");
  const int k1 = (int)h[1], k2 = (int)h[2];
  if (h[3] > 30) throw std::runtime_error("bad index table size");
  const uint32_t hs = 1u << h[3];
  const size_t need = 24 + (size_t)k1 * 2 + (size_t)k2 * 4 + (size_t)hs * 6;
  if (b.size() < need) throw std::runtime_error("index file truncated: " + path);
  const uint8_t* p = b.data() + 24;
  std::vector<uint16_t> i1(k1);
  std::vector<uint32_t> i2(k2), hk(hs);
  std::vector<uint16_t> hv(hs);
  std::memcpy(i1.data(), p, (size_t)k1 * 2);
  p += (size_t)k1 * 2;
  std::memcpy(i2.data(), p, (size_t)k2 * 4);
  p += (size_t)k2 * 4;
  std::memcpy(hk.data(), p, (size_t)hs * 4);
  p += (size_t)hs * 4;
  std::memcpy(hv.data(), p, (size_t)hs * 2);
  return from_tables(k1, k2, i1.data(), i2.data(), hs, hk.data(), hv.data());
}

std::vector<uint16_t> encode(const PairIndex& pi, const uint8_t* data, size_t n) {
  std::vector<uint16_t> s1;
  s1.reserve(n);
  scan1(pi, data, n, [&](uint16_t id) { s1.push_back(id); });
  std::vector<uint16_t> out;
  out.reserve(s1.size());
  // merge adjacent stage-1 pairs that are macros, left to right; an unmerged right token is retried as the left
  // token of the next pair
  size_t i = 0;
  while (i < s1.size()) {
    if (i + 1 < s1.size()) {
      const uint16_t m = pi.lookup2(s1[i], s1[i + 1]);
      if (m != kEmptyVal) {
        out.push_back(m);
        i += 2;
        continue;
      }
    }
    out.push_back(s1[i]);
    i += 1;
  }
  return out;
}

namespace {
void decode_one(const PairIndex& pi, uint16_t id, std::string& out, int depth) {
  if (depth > 8) return;
  if (id < kBaseV) {
    out.push_back((char)id);
  } else if (id < kBaseV + pi.k1) {
    const uint16_t p = pi.id2pair[id - kBaseV];
    out.push_back((char)(p & 0xFF));
    out.push_back((char)(p >> 8));
  } else if (id < kBaseV + pi.k1 + pi.k2) {
    const uint32_t k = pi.id2pair2[id - kBaseV - pi.k1];
    decode_one(pi, (uint16_t)(k >> 16), out, depth + 1);
    decode_one(pi, (uint16_t)(k & 0xFFFFu), out, depth + 1);
  }
}
}  // namespace

std::string decode(const PairIndex& pi, const uint16_t* ids, size_t n) {
  std::string out;
  for (size_t i = 0; i < n; ++i) decode_one(pi, ids[i], out, 0);
  return out;
}

}  // namespace pairidx
}  // namespace hrm

// ------------------------------------------------------------------------------------------------------- C ABI
namespace {
thread_local std::string g_pi_err;
using hrm::pairidx::PairIndex;

template <typename F>
auto guarded(F&& f) -> decltype(f()) {
  g_pi_err.clear();
  try {
    return f();
  } catch (const std::exception& e) {
    g_pi_err = e.what();
  } catch (...) {
    g_pi_err = "unknown error";
  }
  return decltype(f())();
}
PairIndex* as_pi(void* h) {
  if (!h) throw std::runtime_error("null handle");
  return static_cast<PairIndex*>(h);
}
}  // namespace

extern "C" {
void* hrm_pi_build_files(const char* const* paths, int n_paths, int k1, int k2) {
  return guarded([&]() -> void* {
    std::vector<std::string> v;
    for (int i = 0; i < n_paths; ++i) v.emplace_back(paths[i]);
    if (v.empty()) throw std::runtime_error("no input files");
    return new PairIndex(hrm::pairidx::build_from_files(v, k1, k2));
  });
}
void* hrm_pi_build_bytes(const uint8_t* data, size_t n, int k1, int k2) {
  return guarded([&]() -> void* { return new PairIndex(hrm::pairidx::build_from_bytes(data, n, k1, k2)); });
}
void* hrm_pi_load(const char* path) {
  return guarded([&]() -> void* { return new PairIndex(hrm::pairidx::load_idx7(path)); });
}
void* hrm_pi_from_tables(int k1, int k2, const uint16_t* id2pair, const uint32_t* id2pair2, uint32_t hsize,
                         const uint32_t* hkeys, const uint16_t* hvals) {
  return guarded([&]() -> void* {
    return new PairIndex(hrm::pairidx::from_tables(k1, k2, id2pair, id2pair2, hsize, hkeys, hvals));
  });
}
int hrm_pi_save(void* h, const char* path) {
  return guarded([&]() -> int {
    hrm::pairidx::save_idx7(*as_pi(h), path);
    return 1;
  });
}
int hrm_pi_info(void* h, int* k1, int* k2, uint32_t* hsize) {
  return guarded([&]() -> int {
    const PairIndex* p = as_pi(h);
    if (k1) *k1 = p->k1;
    if (k2) *k2 = p->k2;
    if (hsize) *hsize = (uint32_t)p->hkeys.size();
    return 1;
  });
}
int hrm_pi_tables(void* h, uint16_t* id2pair, uint32_t* id2pair2, uint32_t* hkeys, uint16_t* hvals) {
  return guarded([&]() -> int {
    const PairIndex* p = as_pi(h);
    if (id2pair) std::copy(p->id2pair.begin(), p->id2pair.end(), id2pair);
    if (id2pair2) std::copy(p->id2pair2.begin(), p->id2pair2.end(), id2pair2);
    if (hkeys) std::copy(p->hkeys.begin(), p->hkeys.end(), hkeys);
    if (hvals) std::copy(p->hvals.begin(), p->hvals.end(), hvals);
    return 1;
  });
}
size_t hrm_pi_encode(void* h, const uint8_t* data, size_t n, uint16_t* out, size_t cap) {
  return guarded([&]() -> size_t {
    const auto ids = hrm::pairidx::encode(*as_pi(h), data, n);
    if (out) std::copy(ids.begin(), ids.begin() + (ptrdiff_t)std::min(cap, ids.size()), out);
    return ids.size();
  });
}
size_t hrm_pi_decode(void* h, const uint16_t* ids, size_t n, uint8_t* out, size_t cap) {
  return guarded([&]() -> size_t {
    const auto s = hrm::pairidx::decode(*as_pi(h), ids, n);
    if (out) std::memcpy(out, s.data(), std::min(cap, s.size()));
    return s.size();
  });
}
void hrm_pi_free(void* h) { delete static_cast<PairIndex*>(h); }
const char* hrm_pi_last_error(void) { return g_pi_err.c_str(); }
}
