// Query engine.
//   1. route: score[cid] += level for every level 1..q[bin] of the prompt signature and every cid posted there;
//   2. top_k cids by (score desc, cid asc), positive scores only;
//   3. candidates = every snippet of those cids (cid order, then sidx), rel = sum_i min(q_prompt_i, q_snip_i),
//      sorted by (rel desc, sid asc), truncated to top_m;
//   4. MMR: k rounds picking max rel*lam_den - lam_num*max_overlap(candidate, chosen); ties -> smaller sid.
// Same ranking and tie rules as the reference Engine::query / mmr_select (engine.cpp:22-73, rank.cpp:35-61).
#include "hrm/hrm.h"

#include <algorithm>
#include <stdexcept>

namespace hrm {

void Engine::open(const std::string& model_dir) {
  close();
  router_ = load_router(model_dir + "/router_index.bin");
  Store st;
  st.open(model_dir + "/index.sqlite", false);
  for (auto& s : st.all()) {
    Row r{std::move(s.sid), std::move(s.txt), s.cid, unpack_nibbles(s.blob)};
    rows_[s.cid].push_back(std::move(r));
  }
  open_ = true;
}

void Engine::close() {
  rows_.clear();
  router_ = RouterIndex();
  open_ = false;
}

QueryResult Engine::query(const std::string& prompt, const QueryParams& qp) const {
  if (!open_) throw std::runtime_error("engine not open");
  QueryResult out;
  const Sig q = signature(prompt);

  std::vector<int32_t> score((size_t)router_.max_cid + 1, 0);
  for (uint32_t b = 0; b < router_.bins && b < (uint32_t)kBins; ++b) {
    for (uint32_t lvl = 1; lvl <= q[b] && lvl < router_.levels; ++lvl) {
      const size_t slot = (size_t)lvl * router_.bins + b;
      for (uint64_t i = router_.offsets[slot]; i < router_.offsets[slot + 1]; ++i) {
        const uint32_t cid = router_.cids[i];
        if (cid <= router_.max_cid) score[cid] += (int32_t)lvl;
      }
    }
  }
  std::vector<std::pair<int32_t, uint32_t>> ranked;
  for (uint32_t cid = 0; cid < score.size(); ++cid)
    if (score[cid] > 0) ranked.emplace_back(score[cid], cid);
  std::sort(ranked.begin(), ranked.end(), [](const auto& a, const auto& b) {
    return a.first != b.first ? a.first > b.first : a.second < b.second;
  });
  for (size_t i = 0; i < ranked.size() && (int)i < qp.top_k; ++i) out.cids.push_back(ranked[i].second);

  struct Cand {
    const Row* row;
    int rel;
  };
  std::vector<Cand> cand;
  for (uint32_t cid : out.cids) {
    auto it = rows_.find(cid);
    if (it == rows_.end()) continue;
    for (const Row& r : it->second) cand.push_back({&r, overlap_sig_sig(q.data(), r.sig.data())});
  }
  std::sort(cand.begin(), cand.end(), [](const Cand& a, const Cand& b) {
    return a.rel != b.rel ? a.rel > b.rel : a.row->sid < b.row->sid;
  });
  if ((int)cand.size() > qp.top_m) cand.resize(qp.top_m < 0 ? 0 : qp.top_m);

  // MMR with a running max-overlap per candidate
  const size_t n = cand.size();
  std::vector<int> red(n, 0);
  std::vector<char> used(n, 0);
  for (int it = 0; it < qp.k && it < (int)n; ++it) {
    long long best_score = 0;
    int best = -1;
    for (size_t i = 0; i < n; ++i) {
      if (used[i]) continue;
      const long long s = (long long)cand[i].rel * qp.lam_den - (long long)qp.lam_num * red[i];
      if (best < 0 || s > best_score || (s == best_score && cand[i].row->sid < cand[best].row->sid)) {
        best = (int)i;
        best_score = s;
      }
    }
    if (best < 0) break;
    used[best] = 1;
    const Row& c = *cand[best].row;
    out.chosen.push_back(Hit{c.sid, c.cid, c.txt, cand[best].rel});
    for (size_t i = 0; i < n; ++i) {
      if (used[i]) continue;
      const int ov = overlap_sig_sig(cand[i].row->sig.data(), c.sig.data());
      if (ov > red[i]) red[i] = ov;
    }
  }
  return out;
}

}  // namespace hrm
