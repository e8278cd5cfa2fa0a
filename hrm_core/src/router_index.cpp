// Flat inverted router index: for every (level, bin) slot the sorted, de-duplicated list of cluster ids whose
// signature reaches that level in that bin.  File layout ("HRMIDX2" truncated to its 6-byte magic, as written by
// the reference's save_router_index): magic, u32 bins, u32 levels, u32 max_cid, u64 n_offsets, u64 n_cids,
// u64 offsets[], u32 cids[] (host little-endian).
#include "hrm/hrm.h"

#include <algorithm>
#include <cstring>
#include <fstream>
#include <stdexcept>

namespace hrm {
namespace {
constexpr char kMagic[6] = {'H', 'R', 'M', 'I', 'D', 'X'};
}

RouterIndex build_router(const std::vector<std::pair<uint32_t, Sig>>& cluster_sigs) {
  RouterIndex idx;
  // count pass then fill pass (no per-slot vectors)
  std::vector<uint64_t> cnt(idx.slots() + 1, 0);
  for (const auto& cs : cluster_sigs) {
    idx.max_cid = std::max(idx.max_cid, cs.first);
    for (uint32_t b = 0; b < idx.bins; ++b)
      for (uint32_t lvl = 1; lvl <= cs.second[b]; ++lvl) ++cnt[(size_t)lvl * idx.bins + b];
  }
  idx.offsets.assign(idx.slots() + 1, 0);
  for (size_t s = 0; s < idx.slots(); ++s) idx.offsets[s + 1] = idx.offsets[s] + cnt[s];
  std::vector<uint32_t> raw(idx.offsets.back());
  std::vector<uint64_t> pos(idx.offsets.begin(), idx.offsets.end() - 1);
  for (const auto& cs : cluster_sigs)
    for (uint32_t b = 0; b < idx.bins; ++b)
      for (uint32_t lvl = 1; lvl <= cs.second[b]; ++lvl) raw[pos[(size_t)lvl * idx.bins + b]++] = cs.first;
  // sort + unique per slot, compacting
  idx.cids.reserve(raw.size());
  std::vector<uint64_t> out_off(idx.slots() + 1, 0);
  for (size_t s = 0; s < idx.slots(); ++s) {
    auto a = raw.begin() + idx.offsets[s], e = raw.begin() + idx.offsets[s + 1];
    std::sort(a, e);
    e = std::unique(a, e);
    out_off[s] = idx.cids.size();
    idx.cids.insert(idx.cids.end(), a, e);
  }
  out_off[idx.slots()] = idx.cids.size();
  idx.offsets.swap(out_off);
  return idx;
}

void save_router(const RouterIndex& idx, const std::string& path) {
  if (idx.offsets.size() != idx.slots() + 1 || idx.offsets.back() != idx.cids.size())
    throw std::runtime_error("router index is inconsistent");
  std::ofstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot write " + path);
  const uint64_t off_n = idx.offsets.size(), cid_n = idx.cids.size();
  f.write(kMagic, sizeof(kMagic));
  f.write(reinterpret_cast<const char*>(&idx.bins), 4);
  f.write(reinterpret_cast<const char*>(&idx.levels), 4);
  f.write(reinterpret_cast<const char*>(&idx.max_cid), 4);
  f.write(reinterpret_cast<const char*>(&off_n), 8);
  f.write(reinterpret_cast<const char*>(&cid_n), 8);
  f.write(reinterpret_cast<const char*>(idx.offsets.data()), (std::streamsize)(off_n * 8));
  f.write(reinterpret_cast<const char*>(idx.cids.data()), (std::streamsize)(cid_n * 4));
  if (!f) throw std::runtime_error("write failed: " + path);
}

RouterIndex load_router(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot read router_index");
  char magic[6];
  f.read(magic, 6);
  if (!f || std::memcmp(magic, kMagic, 6) != 0) throw std::runtime_error("bad router index magic");
  RouterIndex idx;
  uint64_t off_n = 0, cid_n = 0;
  f.read(reinterpret_cast<char*>(&idx.bins), 4);
  f.read(reinterpret_cast<char*>(&idx.levels), 4);
  f.read(reinterpret_cast<char*>(&idx.max_cid), 4);
  f.read(reinterpret_cast<char*>(&off_n), 8);
  f.read(reinterpret_cast<char*>(&cid_n), 8);
  if (!f || idx.bins == 0 || idx.levels == 0 || off_n != idx.slots() + 1) throw std::runtime_error("offset size mismatch");
  idx.offsets.resize(off_n);
  idx.cids.resize(cid_n);
  f.read(reinterpret_cast<char*>(idx.offsets.data()), (std::streamsize)(off_n * 8));
  f.read(reinterpret_cast<char*>(idx.cids.data()), (std::streamsize)(cid_n * 4));
  if (!f) throw std::runtime_error("truncated router_index");
  if (idx.offsets.back() != idx.cids.size()) throw std::runtime_error("offsets/cids mismatch");
  return idx;
}

}  // namespace hrm
