// `hrm build`: payloads.jsonl -> model directory (index.sqlite, router_index.bin, meta.json).
// Snippet signatures and per-cluster signatures (snippets joined with '\n' after each) are computed on all host
// cores; rows are written in (cid, sidx) order with a commit every 20000 rows, as the reference CLI does
// (src/cli/main.cpp:130-180 there).
#include "hrm/hrm.h"

#include <algorithm>
#include <atomic>
#include <filesystem>
#include <fstream>
#include <thread>

namespace hrm {

template <class F>
static void parallel_for(size_t n, F&& f) {
  const size_t nt = std::max<size_t>(1, std::min<size_t>(n, std::thread::hardware_concurrency()));
  std::atomic<size_t> next{0};
  std::vector<std::thread> ts;
  for (size_t t = 0; t < nt; ++t)
    ts.emplace_back([&] {
      for (size_t i; (i = next.fetch_add(1)) < n;) f(i);
    });
  for (auto& t : ts) t.join();
}

uint64_t build_model(const std::string& payloads_path, const std::string& outdir) {
  std::filesystem::create_directories(outdir);
  const auto payloads = read_payloads(payloads_path);

  std::vector<std::pair<size_t, size_t>> items;   // (payload, snippet)
  for (size_t p = 0; p < payloads.size(); ++p)
    for (size_t s = 0; s < payloads[p].snippets.size(); ++s) items.emplace_back(p, s);
  std::vector<std::vector<uint8_t>> blobs(items.size());
  parallel_for(items.size(), [&](size_t i) {
    blobs[i] = pack_nibbles(signature(payloads[items[i].first].snippets[items[i].second]));
  });
  std::vector<std::pair<uint32_t, Sig>> csig(payloads.size());
  parallel_for(payloads.size(), [&](size_t p) {
    std::string joined;
    for (const auto& s : payloads[p].snippets) {
      joined += s;
      joined.push_back('\n');
    }
    csig[p] = {payloads[p].cid, signature(joined)};
  });

  Store st;
  st.open(outdir + "/index.sqlite", true);
  st.create_schema();
  st.begin();
  uint64_t n = 0;
  for (size_t i = 0; i < items.size(); ++i) {
    const Payload& p = payloads[items[i].first];
    const uint32_t sidx = (uint32_t)items[i].second;
    st.put(Snip{sid_str(p.cid, sidx), p.cid, sidx, p.snippets[sidx], blobs[i]});
    if (++n % 20000 == 0) {
      st.commit();
      st.begin();
    }
  }
  st.commit();
  st.close();

  const RouterIndex idx = build_router(csig);
  save_router(idx, outdir + "/router_index.bin");
  std::ofstream m(outdir + "/meta.json");
  m << "{\"bins\":" << kBins << ",\"levels\":" << kLevels << ",\"max_cid\":" << idx.max_cid << ",\"snips\":" << n
    << "}\n";
  return n;
}

}  // namespace hrm
