// PairIndex: deterministic two-stage byte-pair tokenizer of the experiments plane.
//
// Stage 1 maps the K1 most frequent byte pairs to ids 256 .. 256+K1-1 (bytes keep ids 0..255); text is encoded
// greedily left to right (a pair if the table has it, else one byte).  Stage 2 maps the K2 most frequent adjacent
// stage-1 id pairs to "macro" ids 256+K1 .. 256+K1+K2-1, looked up in an open-addressing table.  Ties in every
// frequency ranking go to the smaller key, so the index is a pure function of the corpus bytes (files are read in
// sorted path order).  The on-disk "IDX7" layout and the table construction (multiplicative hash 2654435761,
// linear probing, power-of-two size >= 2*K2) are kept identical to the reference tokenizer so index files and
// checkpoints interoperate.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace hrm {
namespace pairidx {

constexpr int kBaseV = 256;
constexpr uint32_t kEmptyKey = 0xFFFFFFFFu;
constexpr uint16_t kEmptyVal = 0xFFFFu;

struct PairIndex {
  int k1 = 0, k2 = 0;
  std::vector<uint16_t> id2pair;    // [k1] packed byte pair: first byte in the low 8 bits
  std::vector<int32_t> pair2id;     // [65536] packed pair -> stage-1 id, or -1
  std::vector<uint32_t> id2pair2;   // [k2] (a << 16) | b over stage-1 ids
  std::vector<uint32_t> hkeys;      // [2^pow2] kEmptyKey = free
  std::vector<uint16_t> hvals;      // [2^pow2] macro id
  uint32_t hmask = 0;

  int vocab() const { return kBaseV + k1 + k2; }
  uint32_t pow2() const;
  uint16_t lookup2(uint16_t a, uint16_t b) const;   // macro id or kEmptyVal
};

// Build from corpus files (v7 semantics: counts summed over files, stage-2 pairs never cross a file boundary,
// stage 1 padded with unused pairs when the corpus has fewer than k1 distinct pairs, stage 2 with unreachable keys).
PairIndex build_from_files(std::vector<std::string> paths, int k1, int k2);
PairIndex build_from_bytes(const uint8_t* data, size_t n, int k1, int k2);
// Tables -> index (used when loading a checkpoint that embeds them).
PairIndex from_tables(int k1, int k2, const uint16_t* id2pair, const uint32_t* id2pair2, uint32_t hsize,
                      const uint32_t* hkeys, const uint16_t* hvals);

void save_idx7(const PairIndex& pi, const std::string& path);
PairIndex load_idx7(const std::string& path);

std::vector<uint16_t> encode(const PairIndex& pi, const uint8_t* data, size_t n);
std::string decode(const PairIndex& pi, const uint16_t* ids, size_t n);

}  // namespace pairidx
}  // namespace hrm

extern "C" {
// C ABI (libhrm_pairindex.so).  Handles are opaque; every call returns 0 / nullptr on failure and records a
// message readable with hrm_pi_last_error() (per thread).
void* hrm_pi_build_files(const char* const* paths, int n_paths, int k1, int k2);
void* hrm_pi_build_bytes(const uint8_t* data, size_t n, int k1, int k2);
void* hrm_pi_load(const char* path);
void* hrm_pi_from_tables(int k1, int k2, const uint16_t* id2pair, const uint32_t* id2pair2, uint32_t hsize,
                         const uint32_t* hkeys, const uint16_t* hvals);
int hrm_pi_save(void* h, const char* path);
int hrm_pi_info(void* h, int* k1, int* k2, uint32_t* hsize);
// copies the tables into caller buffers sized from hrm_pi_info
int hrm_pi_tables(void* h, uint16_t* id2pair, uint32_t* id2pair2, uint32_t* hkeys, uint16_t* hvals);
// returns the number of ids; writes at most cap of them (call with cap = 0 to size the output)
size_t hrm_pi_encode(void* h, const uint8_t* data, size_t n, uint16_t* out, size_t cap);
size_t hrm_pi_decode(void* h, const uint16_t* ids, size_t n, uint8_t* out, size_t cap);
void hrm_pi_free(void* h);
const char* hrm_pi_last_error(void);
}
