// Host-visible declarations of the W8A16 tcgen05 GEMM (see gemm_w8a16.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

namespace hrm {

enum GemmEpilogue : int {
  EPI_F16 = 0,     // out f16 [M, ldo]            = acc * scale (+ bias)
  EPI_F32 = 1,     // out f32 [M, ldo]            = acc * scale (+ bias)
  EPI_RESID = 2,   // resid f32 [M, ldr]         += acc * scale (+ bias)
  EPI_SWIGLU = 3,  // out f16 [M, N/2]            = silu(gate) * up, rows interleaved 64 gate / 64 up per tile
  EPI_QKV = 4,     // q_out bf16 [M, q_rows]; K/V rows -> paged cache (bias + rotate-half RoPE on q and k)
  EPI_RESID_AR = 5,  // tensor-parallel residual GEMM: partial tiles all-reduced over peer memory, then as EPI_RESID
};

#if defined(__CUDACC__)
#define HRM_TILE_HD __host__ __device__ __forceinline__
#else
#define HRM_TILE_HD inline
#endif

// Output-tile numbering of the stream-K GEMM and the walk over consecutive pipeline units
// (unit = tile * k_tiles + kt).  n-fastest: tile = m_tile * n_tiles + n_tile, so CTAs running side by side hold
// different weight tiles of one token block (one pass over the weights per token block; the decode default, where
// there is one token block).  m-fastest: tile = n_tile * m_tiles + m_tile, so a CTA keeps one weight tile for every
// token block in turn and the weights leave DRAM once (multi-token-block, i.e. prefill, GEMMs).  Shared by the
// kernel's producer and epilogue and by the host-side test of the walk.
struct TileWalk {
  int n_tiles, m_tiles, k_tiles, m_fastest;
  int n_tile, m_tile, kt;
  HRM_TILE_HD static void coords(int tile, int n_tiles, int m_tiles, int m_fastest, int& n_tile, int& m_tile) {
    if (m_fastest) { n_tile = tile / m_tiles; m_tile = tile - n_tile * m_tiles; }
    else { m_tile = tile / n_tiles; n_tile = tile - m_tile * n_tiles; }
  }
  HRM_TILE_HD void start(long long unit) {
    const int tile = (int)(unit / k_tiles);
    kt = (int)(unit - (long long)tile * k_tiles);
    coords(tile, n_tiles, m_tiles, m_fastest, n_tile, m_tile);
  }
  HRM_TILE_HD void next() {
    if (++kt < k_tiles) return;
    kt = 0;
    if (m_fastest) {
      if (++m_tile == m_tiles) { m_tile = 0; ++n_tile; }
    } else if (++n_tile == n_tiles) {
      n_tile = 0;
      ++m_tile;
    }
  }
};

// k-segments of the stream-K tile whose units are [f, f + k_tiles) when U units are split evenly over G CTAs (CTA c
// holds [c*U/G, (c+1)*U/G)): the number of CTAs holding part of the tile, and the index of the segment that starts
// at unit u.  With at least as many units as CTAs every CTA holds a unit, so a tile's owners are consecutive CTAs.
// With fewer units than CTAs (a multi-phase chain runs every phase on all SMs) each CTA holds at most one unit and
// the owners are spread out with empty CTAs between them: a tile then has one segment per unit.  Shared by the
// kernels and the host-side test of the partition.
HRM_TILE_HD void tile_segments(long long f, int k_tiles, long long u, long long U, long long G, int& nseg,
                               int& segidx) {
  auto owner = [U, G](long long x) { return (int)(((x + 1) * G - 1) / U); };
  if (U >= G) {
    const int first = owner(f);
    nseg = owner(f + k_tiles - 1) - first + 1;
    segidx = owner(u) - first;
  } else {
    nseg = k_tiles;
    segidx = (int)(u - f);
  }
}

struct GemmArgs {
  int M, N, K;
  int k_tiles, n_tiles, tiles, max_seg;     // filled by the launcher from the plan (k_tiles = units per tile)
  int ku;                                   // 64-wide k-tiles per pipeline unit (1, 2 or 4)
  const float* scale;                       // [N]
  // Pre-tiled weights (preferred): [ceil(N/128)][K/64][8192] int8, each 8 KB block the 64-byte-swizzled image of
  // one 128-row x 64-k tile, fetched with one contiguous bulk copy.  nullptr: plain row-major [N, K] via 2-D TMA.
  const int8_t* w_tiles;
  const float* bias;                        // [N] or nullptr
  void* out;                                // EPI_F16 / EPI_F32 / EPI_SWIGLU
  int ldo;
  float* resid;                             // EPI_RESID
  int ldr;
  // EPI_RESID optional outputs feeding the next RMSNorm without a norm kernel:
  //   xg_out[m, n] = f16(x_new[m, n] * gamma_next[n]);  ssq_out[n_tile * M + m] = sum over the tile's rows of x_new^2
  __half* xg_out;
  int ldxg;
  const float* gamma_next;
  float* ssq_out;
  // consumer side: every output of token m is multiplied by rsqrt(sum_t in_ssq[t * M + m] * in_inv_h + in_eps)
  // (the RMSNorm of the un-normalised GEMM input, whose gamma is already folded into X)
  const float* in_ssq;
  int in_ssq_tiles;
  float in_inv_h, in_eps;
  // EPI_RESID_AR: symmetric buffers of all ranks (peers[r] = base address of rank r's buffer, mapped locally)
  const long long* peers;
  int tp_rank, tp_world;
  long long off_partials, off_final, off_flags;   // byte offsets inside every rank's buffer
  long long off_tile_flags;                       // int32 [world][ar_max_tiles]: epoch of each (source rank, tile)
  long long off_ll;                               // u64 [2][world][ar_max_tiles][ar_tile_floats]: epoch-tagged words
  int ar_ll;                                      // 1: epoch-tagged words (no fence, no flag); 0: partials + flags
  int ar_tile_floats;                             // floats per tile slot (max_bn * 128)
  int ar_max_tiles;
  int* epoch;                                     // this rank's launch epoch counter (in its symmetric buffer)
  int* launch_ticket;                             // [2] CTA tickets: phase-1 barrier, kernel end (zero between launches)
  int ep_offset;                                  // this all-reduce's epoch = *epoch + 1 + ep_offset (0 unless chained)
  int m_fastest;                                  // tile numbering: 0 n-fastest, 1 m-fastest (see TileWalk)
  float* ws;                                // stream-K partials: plan.ws_floats floats
  int* counters;                            // stream-K tickets: plan.counters ints, zero before first use
  // EPI_QKV
  int q_rows, kv_rows, head_dim, kv_heads, block_size;
  const int* positions;                     // [M] absolute positions
  const int* slots;                         // [M] block * block_size + offset, or -1 to skip the KV write
  const float* cos_t;                       // [max_pos, head_dim / 2]
  const float* sin_t;
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_cache;                   // [num_blocks, kv_heads, block_size, head_dim]
  __nv_bfloat16* v_cache;
  int* status;                              // bounded-wait error word (may be nullptr)
  long long* trace;                         // optional stamps: [16][kGemmTraceLen] (see trace_mark / trace_cta)
};

constexpr int kGemmTraceLen = 1024;

// Persistent stream-K plan: `ctas` CTAs share tiles*k_tiles (tile, k) units evenly; a tile is cut into at most
// `max_seg` k-segments (== `splits`), whose partials need `ws_floats` floats of workspace and `counters` tickets.
struct GemmPlan {
  int bn, n_tiles, m_tiles, k_tiles, tiles, ctas, max_seg, splits;   // k_tiles: pipeline units per output tile
  int ku;                                                            // 64-wide k-tiles per unit
  size_t ws_floats;
  int counters;
};

GemmPlan gemm_plan(int M, int N, int K, int force_ctas = 0);

// ---------------------------------------------------------------------------------------------- multi-phase chain
// Up to kMaxChainPhases decode GEMMs in one persistent cooperative launch, phase p + 1 reading phase p's outputs
// (grid barrier in between; the next phase's weights stream before it).  Supported epilogue sequences:
// {RESID, SWIGLU, RESID, QKV}, {RESID, SWIGLU, RESID}, the tensor-parallel {RESID_AR, SWIGLU, RESID_AR, QKV} /
// {RESID_AR, SWIGLU, RESID_AR} and {F16, F16}; pre-tiled weights; M <= 32.
constexpr int kMaxChainPhases = 4;
struct ChainArgs {
  int nph;
  GemmArgs ph[kMaxChainPhases];
  int* bar;       // [kMaxChainPhases + 1] zero-initialised: phase arrival counters, then the kernel-end ticket
  int* status;
};
struct ChainPhaseDesc {
  const void* x;  // f16 activations [M, ldx] of this phase (may be an earlier phase's output)
  int ldx;
  int epi;        // GemmEpilogue
  GemmArgs a;     // M, N, K, scale, w_tiles and the epilogue's fields; ws / counters shared by all phases
};
// Plan of one chain phase on exactly `ctas` CTAs (no clamp to the unit count).
GemmPlan gemm_chain_phase_plan(int M, int N, int K, int ctas);
void gemm_chain_launch(const ChainPhaseDesc* ph, int nph, int* bar, cudaStream_t stream);
void gemm_w8a16_launch(const void* x, int ldx, const int8_t* w, int epi, GemmArgs a, const GemmPlan& p,
                       cudaStream_t stream);
void make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz);
int gemm_sm_count();
// m-fastest tile numbering for GEMMs with more than one token block (default off; env HRM_GEMM_MFAST=1).
bool gemm_m_fastest();
void set_gemm_m_fastest(bool on);
void set_status_word(int device, int* p);
// Per-stage timestamps of CTA 0 for every following launch (nullptr switches tracing off).
void set_gemm_trace(long long* p);
int* status_word();

}  // namespace hrm
