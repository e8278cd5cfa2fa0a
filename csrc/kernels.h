// Host-visible launchers of the non-GEMM kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace hrm {

// Programmatic dependent launch of the decode-path kernels (GEMM, tensor-core decode attention, split combine):
// on unless HRM_PDL=0 is set in the environment; set_pdl_enabled switches it at run time.
bool pdl_enabled();
void set_pdl_enabled(bool on);


void rmsnorm_launch(float* x, const float* delta, const float* w, __half* out, int M, int H, float eps,
                    cudaStream_t s);
void norm_prep_launch(float* x, const float* delta, const float* gamma, __half* xg, float* ssq, int M, int H,
                      cudaStream_t s);
// PHO index prototype: scores[i] = #(record id == query id pairs) - 0.05 * |len_i - q_len|; rec_ids [n][8] u32.
void pho_score_launch(const uint32_t* rec_ids, const uint32_t* rec_len, const uint32_t* q, int q_len, float* scores,
                      long long n, int sm_count, cudaStream_t s);
// Trainer optimizer step over one flat fp32 buffer: device-side global-norm clip factor, then AdamW.
void grad_clip_factor_launch(const float* g, long long n, float clip, float* partial, float* scalars, cudaStream_t s);
void adamw_flat_launch(float* w, float* m, float* v, const float* g, long long n, float lr, float wd, float b1,
                       float b2, float eps, int* step, const float* scalars, int sm_count, cudaStream_t s);
// Trainer causal attention (head dim 16 or 32, fp32, [B, T, H, D] rows, lse [B, H, T] in base-2 units): forward,
// then backward as a dQ pass and a dK/dV pass (deterministic, no atomics).  rpt: rows per thread (2: the D = 16
// kernels that share each shared-memory read between two rows; 1: one row per thread).
void flash_train_fwd_launch(const float* q, const float* k, const float* v, float* o, float* lse, int B, int T, int H,
                            int D, int rpt, cudaStream_t s);
void flash_train_bwd_launch(const float* q, const float* k, const float* v, const float* o, const float* lse,
                            const float* dout, float* dq, float* dk, float* dv, int B, int T, int H, int D, int rpt,
                            cudaStream_t s);
void embed_q8_launch(const int64_t* ids, const int8_t* q, const float* scale, float* out, int M, int H,
                     int vocab_start, int vocab_local, cudaStream_t s);

// Paged decode attention (one query token per sequence), split-K over the context + combine.
struct DecodeAttnArgs {
  const __nv_bfloat16* q;      // [B, Hq, D]
  const __nv_bfloat16* k_cache;  // [num_blocks, Hk, bs, D]
  const __nv_bfloat16* v_cache;
  const int* block_tables;     // [B, max_blocks]
  const int* context_lens;     // [B]
  __half* out;                 // [B, Hq, D]
  float* ws;                   // split partials: [B, Hq, splits, D + 2]
  int B, Hq, Hk, D, block_size, max_blocks, splits, keys_per_split;
  float scale;
  // 1: the kernel launched right before this one writes no block table / context length and no KV entry except the
  // last key of each sequence (one decode step), so the tensor-core kernel may stream older KV tiles before it ends
  int kv_prefetch;
  // optional [B * Hk] int32 tickets, zero at rest: the tensor-core kernel then merges the splits itself (the CTA
  // that finishes last among the splits of a (sequence, kv head) combines them and re-arms its ticket)
  int* tickets;
};
void decode_attn_launch(const DecodeAttnArgs& a, cudaStream_t s);
void decode_combine_launch(const DecodeAttnArgs& a, cudaStream_t s);
// tcgen05 variant (head_dim 128, block size 16, group <= 16, keys_per_split a multiple of 128)
bool decode_attn_tc_supported(const DecodeAttnArgs& a);
int decode_attn_tc_merge_max();   // largest (heads per kv head) x splits the in-kernel split merge handles
void decode_attn_tc_launch(const DecodeAttnArgs& a, int num_blocks, int* status, cudaStream_t s);
size_t decode_attn_ws_floats(int B, int Hq, int D, int splits);

// Paged prefill attention over varlen query chunks (causal with absolute positions).
struct PrefillAttnArgs {
  const __nv_bfloat16* q;      // [Tq, Hq, D] (all sequences' chunk tokens, concatenated)
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  const int* block_tables;     // [S, max_blocks]
  const int* cu_q;             // [S + 1] query offsets
  const int* q_start;          // [S] absolute position of each sequence's first chunk token
  const int* context_lens;     // [S] keys visible to the chunk's last token (q_start + chunk len)
  __half* out;                 // [Tq, Hq, D]
  int S, Hq, Hk, D, block_size, max_blocks, max_q;
  float scale;
};
void prefill_attn_launch(const PrefillAttnArgs& a, cudaStream_t s);
// tcgen05 variant (head_dim 128, block size 16); total_q = rows of q
bool prefill_attn_tc_supported(const PrefillAttnArgs& a);
void prefill_attn_tc_launch(const PrefillAttnArgs& a, int num_blocks, int total_q, int* status, cudaStream_t s);

// Row argmax of fp32 logits [M, V] -> packed (order(value) << 32 | ~global_idx) keys, and token ids.
// Split argmax: `scratch` = 2 * kArgmaxMaxRows zero-initialised u64 (row accumulators, then tickets; the kernel
// re-arms them), or nullptr for one CTA per row.  Rows beyond kArgmaxMaxRows also take one CTA per row.
constexpr int kArgmaxMaxRows = 4096;
void argmax_launch(const float* logits, int M, int V, int ld, int vocab_start, unsigned long long* keys,
                   int64_t* tokens, unsigned long long* scratch, int sms, cudaStream_t s);

// Tensor-parallel greedy pick without a collective library call: every rank holds the logits of its vocab slice.
// The CTA that finishes a row's local argmax stores the row's packed key into slot [epoch parity][rank][row] of
// EVERY rank's symmetric buffer (NVLink stores), fences once and stores the epoch into flag [rank][row] of every
// rank; it waits (bounded) until all ranks' flags of that row reached the epoch in its own buffer and takes the
// maximum of the keys.  The packed key orders by value, then by the lower global token id, so every rank picks the
// same token as one argmax over the whole vocabulary (the reference's distributed greedy rule,
// engine/llama_tp.py:317-335, without its three collectives and per-row broadcasts).  Key slots are
// double-buffered by epoch parity: a rank cannot start exchange e + 2 before every rank has finished reading
// exchange e, because exchange e + 1 needs every rank's flags.
struct ArgmaxXchg {
  const long long* peers;   // device table: base address of every rank's symmetric buffer (local one included)
  int rank, world, max_rows;
  long long off_keys;       // byte offset of int64 [2][world][max_rows] key slots in every buffer
  long long off_flags;      // byte offset of the epoch flags [world][max_rows], one 128-byte line each
  int* epoch;               // this rank's exchange counter (local memory); the launch's last row advances it
  int* row_ticket;          // rows finished in the current launch (local memory; zero between launches)
  int* status;              // bounded-wait error word
};
void argmax_xchg_launch(const float* logits, int M, int V, int ld, int vocab_start, unsigned long long* keys,
                        int64_t* tokens, unsigned long long* scratch, int sms, const ArgmaxXchg& x, cudaStream_t s);

// Sampled pick (temperature / top-k, Gumbel-max) on the argmax path; per-row arrays on the device.
struct SampleArgs {
  const float* inv_temp;              // [M] 1 / temperature; 0 keeps the row greedy
  const float* thresh;                // [M] keep logits >= thresh (-inf: every token); nullptr: every token
  const unsigned long long* seed;     // [M] per-request seed
  const int* pos;                     // [M] position of the row's input token (the noise counter)
};
void argmax_sample_launch(const float* logits, int M, int V, int ld, int vocab_start, unsigned long long* keys,
                          int64_t* tokens, unsigned long long* scratch, int sms, const SampleArgs& sp,
                          const ArgmaxXchg* x, cudaStream_t s);
// Top-k thresholds: out[r] = k[r]-th largest of x[r, 0:n] (-inf when k[r] <= 0 or >= n); candidates: the values
// above thresh[r] then thresh[r] up to k[r] slots, then -inf, in [rows, kmax] (k[r] <= kmax) (sampling.cu).
// kth_largest needs kth_largest_state_words(rows) u32 of scratch (initialised by the launch itself).
int kth_largest_state_words(int rows);
void kth_largest_launch(const float* x, int rows, int n, int ld, const int* k, float* out, uint32_t* state, int sms,
                        cudaStream_t s);
void topk_candidates_launch(const float* x, int rows, int n, int ld, const float* thresh, const int* k, int kmax,
                            float* cand, cudaStream_t s);

// Dense NT GEMM for the experiments plane: C [M, N] fp32 = A [M, K] . B [N, K]^T, A and B row-major bf16 (or f16),
// leading dimensions in elements (multiples of 8), N and ldc multiples of 4 (gemm_nt.cu).
void gemm_nt_launch(const void* A, int lda, const void* B, int ldb, float* C, int ldc, int M, int N, int K,
                    bool bf16, int* status, cudaStream_t stream);

void decode_prepare_launch(const int* positions, const int* tables, int maxb, int bs, const int* active, int* slots,
                           int* context_lens, int B, cudaStream_t s);
void decode_advance_launch(const int64_t* tokens, int64_t* ids, int* positions, const int* active, int B,
                           cudaStream_t s);

}  // namespace hrm
