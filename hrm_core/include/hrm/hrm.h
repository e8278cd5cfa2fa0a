// HRM retrieval core: hashed n-gram signatures, flat inverted router index, SQLite snippet store, MMR selection.
//
// Behaviour (scores, tie-breaks, file formats, JSON) is identical to the reference core
// (hrm_core/src/hrm/{signature,router_index,sqlite_store,rank,engine,compose,payload_jsonl}.cpp); the
// implementation is this project's own: signatures are computed in one pass with a fixed-size count table, the
// snippet rows are loaded once per open into memory (queries never touch SQLite), unpacked 2048-byte signatures
// keep the overlap loops vectorisable, and MMR keeps each candidate's running max-overlap instead of rescanning
// the chosen set every iteration.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

struct sqlite3;
struct sqlite3_stmt;

namespace hrm {

constexpr int kBins = 2048;     // signature bins
constexpr int kLevels = 16;     // quantisation levels 0..15
constexpr int kBlobBytes = kBins / 2;

// ---------------------------------------------------------------- ids
std::string cid_str(uint32_t cid);                   // "%04u"
std::string sid_str(uint32_t cid, uint32_t sidx);    // "%04u#s%04u"
uint32_t parse_cid(const std::string& s);           // decimal, leading zeros allowed

// ---------------------------------------------------------------- signature
using Sig = std::vector<uint8_t>;                    // kBins values in 0..15
Sig signature(const std::string& text);
std::vector<uint8_t> pack_nibbles(const Sig& q);    // byte j = q[2j] << 4 | q[2j+1]
Sig unpack_nibbles(const std::vector<uint8_t>& blob);

int overlap_sig_sig(const uint8_t* a, const uint8_t* b);   // sum_i min(a_i, b_i) over kBins

// ---------------------------------------------------------------- router index (HRMIDX2 file)
struct RouterIndex {
  uint32_t bins = kBins, levels = kLevels, max_cid = 0;
  std::vector<uint64_t> offsets;   // levels*bins + 1, slot = level*bins + bin (level 0 unused)
  std::vector<uint32_t> cids;
  size_t slots() const { return (size_t)levels * bins; }
};
RouterIndex build_router(const std::vector<std::pair<uint32_t, Sig>>& cluster_sigs);
void save_router(const RouterIndex& idx, const std::string& path);
RouterIndex load_router(const std::string& path);

// ---------------------------------------------------------------- payloads (JSONL) and prep
struct Payload {
  uint32_t cid = 0;
  std::vector<std::string> snippets;
};
std::vector<Payload> read_payloads(const std::string& path);
void write_payloads_from_text(const std::string& input_txt, const std::string& out_jsonl, size_t cluster_size);

// ---------------------------------------------------------------- snippet store (SQLite)
struct Snip {
  std::string sid;
  uint32_t cid = 0, sidx = 0;
  std::string txt;
  std::vector<uint8_t> blob;   // kBlobBytes
};
class Store {
 public:
  Store() = default;
  Store(const Store&) = delete;
  Store& operator=(const Store&) = delete;
  ~Store();
  void open(const std::string& path, bool writable);
  void close();
  void create_schema();
  void begin();
  void commit();
  void put(const Snip& s);
  std::vector<Snip> by_cid(uint32_t cid) const;
  std::vector<Snip> all() const;   // ordered by cid, sidx
 private:
  ::sqlite3* db_ = nullptr;
  ::sqlite3_stmt* ins_ = nullptr;
};

// ---------------------------------------------------------------- engine
struct QueryParams {
  int top_k = 5, top_m = 400, k = 8, lam_num = 7, lam_den = 10;
};
struct Hit {
  std::string sid;
  uint32_t cid = 0;
  std::string txt;
  int rel = 0;
};
struct QueryResult {
  std::vector<uint32_t> cids;
  std::vector<Hit> chosen;
};

class Engine {
 public:
  void open(const std::string& model_dir);
  void close();
  bool is_open() const { return open_; }
  QueryResult query(const std::string& prompt, const QueryParams& qp) const;
 private:
  struct Row {
    std::string sid, txt;
    uint32_t cid;
    Sig sig;   // unpacked
  };
  RouterIndex router_;
  std::unordered_map<uint32_t, std::vector<Row>> rows_;   // cid -> rows in sidx order
  bool open_ = false;
};

// ---------------------------------------------------------------- compose / output
std::string compress_line(const std::string& txt, size_t max_len = 240);
std::string render_answer(const std::string& prompt, const std::vector<Hit>& chosen);
std::string json_escape(const std::string& s);
std::string result_json(const std::string& prompt, const QueryResult& r);

// ---------------------------------------------------------------- build (prep -> payloads -> model dir)
uint64_t build_model(const std::string& payloads_path, const std::string& outdir);

}  // namespace hrm
