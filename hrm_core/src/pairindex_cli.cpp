// `pairindex` CLI: build / encode / decode / info for the PairIndex tokenizer (IDX7 files).
// Reference: the index_build_v7 tool of experiments/run_llm_orig.sh:308-340 (--k1 --k2 --out --inputs a:b:c).
#include "hrm/pairindex.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>
#include <vector>

using namespace hrm::pairidx;

static int usage() {
  std::fprintf(stderr,
               "pairindex build  --inputs a.txt[:b.txt...] [--k1 8192] [--k2 8192] --out index_v7.bin\n"
               "pairindex encode --index index_v7.bin --in text.txt --out ids.u16\n"
               "pairindex decode --index index_v7.bin --in ids.u16 --out text.txt\n"
               "pairindex info   --index index_v7.bin\n");
  return 2;
}

static std::vector<uint8_t> slurp(const std::string& p) {
  std::ifstream f(p, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + p);
  return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
}

int main(int argc, char** argv) {
  if (argc < 2) return usage();
  const std::string cmd = argv[1];
  std::string inputs, out, index, in;
  int k1 = 8192, k2 = 8192;
  for (int i = 2; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) throw std::runtime_error("missing value for " + a);
      return argv[++i];
    };
    try {
      if (a == "--inputs") inputs = next();
      else if (a == "--out") out = next();
      else if (a == "--index") index = next();
      else if (a == "--in") in = next();
      else if (a == "--k1") k1 = std::atoi(next().c_str());
      else if (a == "--k2") k2 = std::atoi(next().c_str());
      else { std::fprintf(stderr, "unknown arg: %s\n", a.c_str()); return 2; }
    } catch (const std::exception& e) {
      std::fprintf(stderr, "%s\n", e.what());
      return 2;
    }
  }
  try {
    if (cmd == "build") {
      if (inputs.empty() || out.empty()) return usage();
      std::vector<std::string> paths;
      size_t s = 0;
      while (s <= inputs.size()) {
        size_t e = inputs.find(':', s);
        if (e == std::string::npos) e = inputs.size();
        if (e > s) paths.push_back(inputs.substr(s, e - s));
        s = e + 1;
      }
      const PairIndex pi = build_from_files(paths, k1, k2);
      save_idx7(pi, out);
      std::fprintf(stderr, "[pairindex] inputs=%zu K1=%d K2=%d table=%zu -> %s\n", paths.size(), pi.k1, pi.k2,
                   pi.hkeys.size(), out.c_str());
    } else if (cmd == "encode" || cmd == "decode") {
      if (index.empty() || in.empty() || out.empty()) return usage();
      const PairIndex pi = load_idx7(index);
      const auto b = slurp(in);
      std::ofstream f(out, std::ios::binary);
      if (cmd == "encode") {
        const auto ids = encode(pi, b.data(), b.size());
        f.write(reinterpret_cast<const char*>(ids.data()), (std::streamsize)(ids.size() * 2));
        std::fprintf(stderr, "[pairindex] %zu bytes -> %zu ids\n", b.size(), ids.size());
      } else {
        const std::string s = decode(pi, reinterpret_cast<const uint16_t*>(b.data()), b.size() / 2);
        f.write(s.data(), (std::streamsize)s.size());
      }
    } else if (cmd == "info") {
      if (index.empty()) return usage();
      const PairIndex pi = load_idx7(index);
      std::printf("{\"k1\": %d, \"k2\": %d, \"vocab\": %d, \"table\": %zu}\n", pi.k1, pi.k2, pi.vocab(), pi.hkeys.size());
    } else {
      return usage();
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "FATAL: %s\n", e.what());
    return 1;
  }
  return 0;
}
