// Unit tests of the HRM core (run by `make -C hrm_core test`): signature locality, nibble packing, payload
// parsing with escapes, router-index round trip, compress_line rules, MMR tie-breaking.
#include "hrm/hrm.h"

#include <cstdio>
#include <filesystem>
#include <fstream>
#include <stdexcept>

namespace {
int failures = 0;
void check(bool ok, const char* what) {
  if (!ok) {
    std::fprintf(stderr, "FAIL: %s\n", what);
    ++failures;
  }
}
int ov(const hrm::Sig& a, const hrm::Sig& b) { return hrm::overlap_sig_sig(a.data(), b.data()); }

void signature_locality() {
  auto a = hrm::signature("Romeo Romeo wherefore art thou Romeo");
  auto typo = hrm::signature("romoe romeo wherefore art thou romeo");
  auto other = hrm::signature("completely unrelated query about physics");
  check(a.size() == (size_t)hrm::kBins, "2048 bins");
  check(ov(a, a) > 0, "non-empty signature");
  check(ov(a, a) >= ov(a, typo) && ov(a, typo) >= ov(a, other), "self >= typo >= unrelated");
  auto empty = hrm::signature("");
  check(empty[0] == 15 && ov(empty, empty) == 15, "empty text -> bin 0 saturated");
  check(hrm::unpack_nibbles(hrm::pack_nibbles(a)) == a, "nibble round trip");
}

void payload_and_prep() {
  auto dir = std::filesystem::temp_directory_path() / "hrm_core_test";
  std::filesystem::create_directories(dir);
  {
    std::ofstream f(dir / "p.jsonl");
    f << "{\"cid\":\"0007\",\"title\":\"cluster\",\"snippets\":[\"a \\\"q\\\" b\",\"tab\\there\",\"back\\\\slash\"]}\n";
    f << "{\"cid\":\"0002\",\"snippets\":[\"x\"]}\n";
    f << "not json\n";
  }
  auto ps = hrm::read_payloads((dir / "p.jsonl").string());
  check(ps.size() == 2 && ps[0].cid == 2 && ps[1].cid == 7, "cid parse + sort");
  check(ps[1].snippets.size() == 3 && ps[1].snippets[0] == "a \"q\" b" && ps[1].snippets[1] == "tab\there" &&
            ps[1].snippets[2] == "back\\slash",
        "snippet escapes");
  {
    std::ofstream f(dir / "in.txt");
    f << "line one\r\n\n   \t\nline \"two\"\nline three\n";
  }
  hrm::write_payloads_from_text((dir / "in.txt").string(), (dir / "out.jsonl").string(), 2);
  auto back = hrm::read_payloads((dir / "out.jsonl").string());
  check(back.size() == 2 && back[0].snippets.size() == 2 && back[0].snippets[1] == "line \"two\"" &&
            back[1].snippets[0] == "line three",
        "prep clusters non-blank lines");
}

void router_roundtrip() {
  std::vector<std::pair<uint32_t, hrm::Sig>> cs = {{0, hrm::signature("alpha beta gamma delta")},
                                                   {3, hrm::signature("epsilon zeta eta theta")}};
  auto idx = hrm::build_router(cs);
  auto path = (std::filesystem::temp_directory_path() / "hrm_router_test.bin").string();
  hrm::save_router(idx, path);
  auto r = hrm::load_router(path);
  check(r.max_cid == 3 && r.offsets == idx.offsets && r.cids == idx.cids, "router index round trip");
  bool sorted = true;
  for (size_t s = 0; s < r.slots(); ++s)
    for (uint64_t i = r.offsets[s] + 1; i < r.offsets[s + 1]; ++i) sorted &= r.cids[i - 1] < r.cids[i];
  check(sorted, "postings sorted and unique");
}

void compose_rules() {
  check(hrm::compress_line("ROMEO: But soft (aside) what [light] breaks") == "But soft what breaks", "speaker+groups");
  check(hrm::compress_line("romeo: lower case speaker stays") == "romeo: lower case speaker stays", "speaker case");
  std::string long_line(100, 'a');
  long_line += ". ";
  long_line += std::string(200, 'b');
  check(hrm::compress_line(long_line) == std::string(100, 'a') + "...", "cut at last period");
  check(hrm::compress_line(std::string(300, 'c')) == std::string(240, 'c') + "...", "hard cut");
}

}  // namespace

int main() {
  try {
    signature_locality();
    payload_and_prep();
    router_roundtrip();
    compose_rules();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "exception: %s\n", e.what());
    return 1;
  }
  if (failures) return 1;
  std::puts("hrm_tests: all passed");
  return 0;
}
