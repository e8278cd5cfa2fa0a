// Shared device code of the W8A16 tcgen05 GEMM kernels (single launch in gemm_w8a16.cu, multi-phase chain in
// gemm_chain.cu): constants, per-width pipeline shapes, the epilogue variants, the peer-memory all-reduce epilogue and
// the host helpers both launchers use.  The design is described at the top of gemm_w8a16.cu.
#pragma once
#include "common.cuh"
#include "gemm_w8a16.h"

#include <cstdint>

namespace hrm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kDqWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kFirstDqWarp = 2;
constexpr int kFirstEpiWarp = kFirstDqWarp + kDqWarps;
constexpr int kMma2Warp = kFirstEpiWarp + kEpiWarps;         // second MMA issuer (warp 14)
constexpr int kThreads = (kMma2Warp + 1) * 32;               // 480
constexpr int kDqThreads = kDqWarps * 32;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kWrawBytes = kBM * kBK;          // int8 tile, 8 KB
constexpr int kW16Bytes = kBM * kBK * 2;       // f16 tile, 16 KB
constexpr int kChunk = 16;                     // epilogue columns per TMEM load

// Pipeline shape per token-tile width BN.
//  TS (BN <= 128, decode): dequantised A tiles go to tensor memory and the MMA reads A from TMEM; one dequant group
//    of 8 warps converts each unit (thread = weight row = TMEM lane; the two warps of a lane quarter take alternate
//    k-tiles of the unit).  Shared memory then carries 2 bytes per weight byte (bulk-copy
//    write + one conflict-free read) instead of 6.
//  SS (BN = 256, prefill): A tiles in shared memory (F stages of 16 KB, 128-byte swizzle); 4 dequant groups of
//    2 warps.  Here the MMA time per tile hides the extra shared-memory traffic.
// KU: 64-wide k-tiles per pipeline unit.  At decode widths every per-unit step (barrier waits, commits, TMA issue)
// costs hundreds of cycles, so units of KU k-tiles (KU x 8 KB of weights, KU x 4 MMAs) amortise them; the launcher
// picks ku = KU, or 2 / 1 when K/64 is not a multiple of KU.
// RW: raw weight ring (units), released by its dequant group once the unit is in registers.  RX: activation ring
// (units), released by the MMA.  F: A stages (units).  RW and F are multiples of the group count, so every slot of
// those rings is always consumed by the same group, in order: no waiter can ever mistake a phase two generations
// old for the one it waits for.
// NACC: MMA-issuing warps.  A single thread issuing one unit's small-N MMAs and then its commits and barrier waits
// leaves the tensor core idle during the bookkeeping; with two issuers (warps 1 and 14) taking alternate units, one
// issues while the other does its bookkeeping.  Each issuer accumulates into its own partial accumulator; the
// epilogue sums the partials that the segment wrote.
template <int BN> struct GemmCfg;
template <> struct GemmCfg<16>  { static constexpr bool TS = true;  static constexpr int KU = 4, RW = 4, RX = 8, F = 3, NACC = 2; };
template <> struct GemmCfg<32>  { static constexpr bool TS = true;  static constexpr int KU = 4, RW = 4, RX = 4, F = 3, NACC = 2; };
template <> struct GemmCfg<64>  { static constexpr bool TS = true;  static constexpr int KU = 4, RW = 4, RX = 2, F = 2, NACC = 2; };
template <> struct GemmCfg<128> { static constexpr bool TS = true;  static constexpr int KU = 4, RW = 2, RX = 2, F = 2, NACC = 1; };
template <> struct GemmCfg<256> { static constexpr bool TS = false; static constexpr int KU = 1, RW = 4, RX = 3, F = 4, NACC = 1; };

template <int BN>
struct GemmSmem {
  static constexpr bool TS = GemmCfg<BN>::TS;
  static constexpr int KU = GemmCfg<BN>::KU;
  static constexpr int RW = GemmCfg<BN>::RW, RX = GemmCfg<BN>::RX, F = GemmCfg<BN>::F;
  static constexpr int NACC = GemmCfg<BN>::NACC;
  static constexpr int kAccCols = NACC * BN;                            // one accumulator buffer (NACC partials)
  static constexpr int NG = TS ? 1 : 4;                                // dequant groups
  static constexpr int kGroupThreads = kDqThreads / NG;
  static constexpr int kXSub = BN * kBK * 2;                           // one k-tile of activations
  static constexpr int kXSlot = KU * kXSub;
  static constexpr int kWSlot = KU * kWrawBytes;
  static constexpr int kW16Off = 0;                                    // SS only: F x 16 KB
  static constexpr int kXOff = kW16Off + (TS ? 0 : F * kW16Bytes);
  static constexpr int kWrawOff = kXOff + RX * kXSlot;
  static constexpr int kStageOff = kWrawOff + RW * kWSlot;             // [16 cols][128 rows] fp32 = 8 KB
  static constexpr int kInvOff = kStageOff + kChunk * kBM * 4;         // [BN] per-token input row scale
  static constexpr int kSsqOff = kInvOff + BN * 4;                     // [4 warps][16] partial sums of squares
  static constexpr int kBarOff = kSsqOff + kEpiWarps * kChunk * 4;
  static constexpr int kNumBars = 2 * RW + 2 * RX + 2 * F + 5;
  static constexpr int kBytes = kBarOff + kNumBars * 8 + 32;
  static constexpr int kAlloc = kBytes + 1024;
  static constexpr int kAcol = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;  // first TMEM column of the A stages (TS)
  static constexpr int kAStageCols = KU * 32;
  static constexpr int kTmemCols = 512;
  static_assert(kAlloc <= 227 * 1024, "shared memory budget exceeded");
  static_assert(RW % NG == 0 && F % NG == 0, "ring depths must be multiples of the dequant group count");
  static_assert(!TS || kAcol + F * kAStageCols <= kTmemCols, "TMEM budget exceeded");
  static_assert(TS || (2 * kAccCols <= kTmemCols && KU == 1), "SS path: TMEM budget / unit size");
  static_assert(NACC == 1 || NACC == 2, "one or two MMA issuers");
};

// Pipeline trace for performance analysis: clock64 of CTA 0 at each stage of unit i (points listed at the call
// sites: 0 load issued, 1 raw tile landed, 2 A stage free, 3 dequant done, 4 MMA operands ready, 5/6 epilogue
// start/end of segment i, 7 kernel start/end).  Off (a.trace == nullptr) in normal launches.
HRM_DEVINL void trace_mark(const GemmArgs& a, int point, int64_t i) {
  if (a.trace != nullptr && blockIdx.x == 0 && i < kGemmTraceLen) a.trace[point * kGemmTraceLen + i] = clock64();
}
// Per-CTA %globaltimer stamps (rows 8..11: CTA start, first weight unit landed, mainloop done, CTA end; fused
// all-reduce rows 12..15: tile pushed, peers' flags seen / (chain) fence + grid ticket done, reduction written).
HRM_DEVINL void trace_cta(const GemmArgs& a, int row) {
  if (a.trace != nullptr && blockIdx.x < kGemmTraceLen) a.trace[row * kGemmTraceLen + blockIdx.x] = (long long)global_ns();
}

// 16 accumulator columns summed over the partial accumulators whose bit is set in `valid` (all are loaded, so the
// warp-collective loads stay uniform; one wait).
template <int BN, int NACC>
HRM_DEVINL void tmem_ld_acc(uint32_t taddr, float (&v)[16], uint32_t valid) {
  if constexpr (NACC == 1) {
    tmem_ld16(taddr, v);
  } else {
    uint32_t r[NACC][16];
#pragma unroll
    for (int j = 0; j < NACC; ++j)
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(r[j][0]), "=r"(r[j][1]), "=r"(r[j][2]), "=r"(r[j][3]), "=r"(r[j][4]), "=r"(r[j][5]),
            "=r"(r[j][6]), "=r"(r[j][7]), "=r"(r[j][8]), "=r"(r[j][9]), "=r"(r[j][10]), "=r"(r[j][11]),
            "=r"(r[j][12]), "=r"(r[j][13]), "=r"(r[j][14]), "=r"(r[j][15])
          : "r"(taddr + (uint32_t)(j * BN)));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < NACC; ++j)
        if (valid & (1u << j)) acc += __uint_as_float(r[j][i]);
      v[i] = acc;
    }
  }
}

// Sum of a tile's k-segment partials for one thread's row and 16 columns [c0, c0 + 16), in k order (segment 0
// first), so the result does not depend on which CTA finished last.  Partials are [segment][BN / 4][128 rows] float4
// in L2 (column-group-major: a warp reads 512 contiguous bytes per token group);
// the loads of four segments are issued before their adds, so a tile cut into many segments (narrow projections
// at high tensor-parallel degree) costs a few L2 round trips instead of one per segment.
template <int BN>
HRM_DEVINL void sum_segments(const float* ws_tile, int nseg, int row, int c0, float (&v)[16]) {
  const size_t seg4 = (size_t)BN * 128 / 4;   // float4s per segment partial
  const float4* p0 = reinterpret_cast<const float4*>(ws_tile) + (c0 / 4) * 128 + row;
  float4 acc[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) acc[q] = __ldcg(p0 + q * 128);
  int sg = 1;
  for (; sg + 4 <= nseg; sg += 4) {
    float4 t[4][4];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int q = 0; q < 4; ++q) t[s][q] = __ldcg(p0 + (size_t)(sg + s) * seg4 + q * 128);
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[q].x += t[s][q].x; acc[q].y += t[s][q].y; acc[q].z += t[s][q].z; acc[q].w += t[s][q].w;
      }
  }
  for (; sg < nseg; ++sg) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = __ldcg(p0 + (size_t)sg * seg4 + q * 128);
      acc[q].x += t.x; acc[q].y += t.y; acc[q].z += t.z; acc[q].w += t.w;
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[4 * q] = acc[q].x; v[4 * q + 1] = acc[q].y; v[4 * q + 2] = acc[q].z; v[4 * q + 3] = acc[q].w;
  }
}

// ------------------------------------------------------------------ stream-K partition helpers (device + host)
HRM_DEVINL int64_t unit_start(int64_t c, int64_t U, int64_t G) { return (c * U) / G; }
HRM_DEVINL int owner_of(int64_t x, int64_t U, int64_t G) { return (int)(((x + 1) * G - 1) / U); }

// Per-token input row scale (RMSNorm folded into the consumer GEMM): inv[j] for the tile's BN tokens.
template <int BN>
HRM_DEVINL void compute_row_scale(const GemmArgs& a, int m_tile, float* inv, int et) {
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");   // previous tile's readers are done with inv
  for (int j = et; j < BN; j += kEpiThreads) {
    const int m = m_tile * BN + j;
    float s = 0.f;
    if (m < a.M)
      for (int t = 0; t < a.in_ssq_tiles; ++t) s += a.in_ssq[(size_t)t * a.M + m];
    inv[j] = rsqrtf(s * a.in_inv_h + a.in_eps);
  }
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
}

// x_new of 16 tokens for this thread's row -> residual, xg = x * gamma_next, per-tile sums of squares.
template <int BN>
HRM_DEVINL void store_residual_outputs(const GemmArgs& a, int n_tile, int m_tile, int row, int c0,
                                       const float (&xn)[kChunk], int et, float* ssq_red) {
  const int n = n_tile * kBM + row;
  const float gn = (a.gamma_next != nullptr && n < a.N) ? a.gamma_next[n] : 0.f;
  float sq[kChunk];
#pragma unroll
  for (int j = 0; j < kChunk; ++j) {
    const int m = m_tile * BN + c0 + j;
    const bool ok = m < a.M && n < a.N;
    if (ok) {
      a.resid[(size_t)m * a.ldr + n] = xn[j];
      if (a.xg_out != nullptr) a.xg_out[(size_t)m * a.ldxg + n] = __float2half_rn(xn[j] * gn);
    }
    sq[j] = ok ? xn[j] * xn[j] : 0.f;
  }
  if (a.ssq_out != nullptr) {
    const int w = et >> 5, lane = et & 31;
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const float s = warp_sum(sq[j]);
      if (lane == 0) ssq_red[w * kChunk + j] = s;
    }
    asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
    if (et < kChunk) {
      const int m = m_tile * BN + c0 + et;
      const float s = ssq_red[et] + ssq_red[kChunk + et] + ssq_red[2 * kChunk + et] + ssq_red[3 * kChunk + et];
      if (m < a.M) a.ssq_out[(size_t)n_tile * a.M + m] = s;
    }
    asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
  }
}

// Tensor-parallel residual epilogue: one-shot all-reduce by peer-memory PUSH over NVLink (decode, one m tile).
// Receive area of every rank: [launch parity][source rank][tile][max_bn / 4 token groups][128 rows] float4
// (double-buffered by launch parity: a slow peer may still be reading the previous launch's data).
// Phase 1 (per finished tile, in the overlapped epilogue): the tile's partial is stored into the source-rank slot of
// EVERY rank's receive area (posted NVLink writes: no round trip on the critical path).
// Phase 2 (once per CTA, after the mainloop): the CTAs of this rank meet at a grid-wide ticket; the last one fences
// and writes this rank's epoch into every rank's flag array.  Each CTA waits on its LOCAL flags, then reduces its
// share of the tiles from local memory: x = resid + sum over source ranks in rank order, so every rank computes
// bit-identical x / xg / ssq.  One flag hop per launch; every load is local.
// A tile slot is laid out column-group-major: float4 element (row r, tokens 4g..4g+3) at index g * 128 + r, so the
// 32 rows of a warp store / load 512 contiguous bytes per instruction (one NVLink write burst, not 32 short ones).
HRM_DEVINL float4* ar_slot(const GemmArgs& a, int dst, int src, int par, int tile) {
  float* base = reinterpret_cast<float*>(reinterpret_cast<char*>(a.peers[dst]) + a.off_partials);
  return reinterpret_cast<float4*>(base + (((size_t)par * a.tp_world + src) * a.ar_max_tiles + tile) *
                                              a.ar_tile_floats);
}
// Epoch-tagged receive slot of the flag-free variant: word (token m, row r) at m * 128 + r holds the fp32 partial in
// its low half and the launch epoch in its high half.
HRM_DEVINL unsigned long long* ar_ll_slot(const GemmArgs& a, int dst, int src, int par, int tile) {
  unsigned long long* base = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(a.peers[dst]) + a.off_ll);
  return base + (((size_t)par * a.tp_world + src) * a.ar_max_tiles + tile) * a.ar_tile_floats;
}
// Flags of the per-tile protocol: one 128-byte line per (source rank, tile), so pollers of different tiles and the
// peers' flag stores never share a line.
constexpr int kFlagStrideInts = 32;
HRM_DEVINL int* ar_tile_flag(const GemmArgs& a, int dst, int src, int tile) {
  int* f = reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[dst]) + a.off_tile_flags);
  return f + ((size_t)src * a.ar_max_tiles + tile) * kFlagStrideInts;
}

// Reduction of tile t from the receive area (every rank's partial has arrived): x = resid + sum over source ranks
// in rank order, then residual / xg / ssq outputs.  Every rank computes bit-identical results.
template <int BN>
HRM_DEVINL void ar_reduce_tile(const GemmArgs& a, int t, int par, int row, int et, float* ssq_red) {
  const int n = t * kBM + row;
  for (int c0 = 0; c0 < BN && c0 < a.M; c0 += kChunk) {
    float xr[kChunk];   // residual rows, loaded before the partials so both latencies overlap
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int m = c0 + j;
      xr[j] = (m < a.M && n < a.N) ? a.resid[(size_t)m * a.ldr + n] : 0.f;
    }
    float sum[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) sum[j] = 0.f;
    // source ranks two at a time: their loads are in flight together, the adds stay in rank order
    for (int s0 = 0; s0 < a.tp_world; s0 += 2) {
      float4 v[2][kChunk / 4];
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        if (s0 + s < a.tp_world) {
          const float4* p = ar_slot(a, a.tp_rank, s0 + s, par, t) + (c0 / 4) * kBM + row;
#pragma unroll
          for (int q = 0; q < kChunk / 4; ++q) v[s][q] = __ldcg(p + q * kBM);
        }
      }
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        if (s0 + s < a.tp_world) {
#pragma unroll
          for (int q = 0; q < kChunk / 4; ++q) {
            sum[4 * q] += v[s][q].x; sum[4 * q + 1] += v[s][q].y;
            sum[4 * q + 2] += v[s][q].z; sum[4 * q + 3] += v[s][q].w;
          }
        }
      }
    }
    float xn[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int m = c0 + j;
      xn[j] = (m < a.M && n < a.N) ? xr[j] + sum[j] : 0.f;
    }
    store_residual_outputs<BN>(a, t, 0, row, c0, xn, et, ssq_red);
  }
}

// Per-tile all-reduce of the single-launch fused row-parallel GEMM.  The CTA that completed output tile t (its
// last k-segment) has just stored the tile's fp32 partial into slot [epoch parity][this rank][t] of EVERY rank's
// receive area (epilogue_store, EPI_RESID_AR).  Then:
//  1. the epilogue threads meet at their named barrier (every push issued); one thread fences once at system scope
//     (cumulative over the CTA's pushes, ordered before it by the barrier) and stores the epoch, relaxed, into flag
//     [this rank][t] of every rank: a release pattern;
//  2. thread r < world polls this rank's flag [r][t] (relaxed, bounded) and fences once it reached the epoch;
//  3. after the barrier the tile is reduced from local memory (ar_reduce_tile).
// There is no grid-wide ticket and no whole-launch flag: tile t waits only for tile t of the other ranks, which the
// same CTA index completes at about the same time on every rank (identical plans).  Key slots are double-buffered by
// epoch parity: a rank cannot push launch e + 2 before every rank finished launch e, because finishing launch e + 1
// needs every rank's launch-(e + 1) pushes, which come after that rank's launch e (stream order).
template <int BN>
HRM_DEVINL void ar_tile_finish(const GemmArgs& a, int t, int row, int et, int ep, float* ssq_red) {
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
  if (et == 0) {
    trace_cta(a, 12);
    fence_acq_rel_sys();
    for (int d = 0; d < a.tp_world; ++d) st_relaxed_sys(ar_tile_flag(a, d, a.tp_rank, t), ep);
  }
  if (et < a.tp_world) wait_flag_acquire(ar_tile_flag(a, a.tp_rank, et, t), ep, a.status);
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
  if (et == 0) trace_cta(a, 14);   // every rank's partial of this tile has arrived
  ar_reduce_tile<BN>(a, t, ep & 1, row, et, ssq_red);
  if (et == 0) trace_cta(a, 15);
}

// Flag-free variant of ar_tile_finish (GemmArgs::ar_ll): every pushed element is one 64-bit word {epoch, fp32}
// stored with a single relaxed system-scope store, so a word is either wholly this launch's or not yet arrived.  The
// tile's owner polls the words themselves (a source rank's 16 words in flight at a time), so there is no fence, no
// flag store and no flag round trip; the NVLink bytes double (8 per element).  Sums stay in rank order.
template <int BN>
HRM_DEVINL void ar_tile_finish_ll(const GemmArgs& a, int t, int row, int et, int ep, float* ssq_red) {
  if (et == 0) trace_cta(a, 12);
  const unsigned want = (unsigned)ep;
  const int n = t * kBM + row;
  const uint64_t t0 = global_ns();
  bool gave_up = false;
  for (int c0 = 0; c0 < BN && c0 < a.M; c0 += kChunk) {
    float xr[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int m = c0 + j;
      xr[j] = (m < a.M && n < a.N) ? a.resid[(size_t)m * a.ldr + n] : 0.f;
    }
    float sum[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) sum[j] = 0.f;
    for (int src = 0; src < a.tp_world; ++src) {
      const unsigned long long* p = ar_ll_slot(a, a.tp_rank, src, ep & 1, t) + (size_t)c0 * kBM + row;
      unsigned long long w[kChunk];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) w[j] = ld_relaxed_sys_u64(p + (size_t)j * kBM);
#pragma unroll 1
      for (int j = 0; j < kChunk; ++j) {
        unsigned long long x = w[j];
        for (uint32_t i = 0; (unsigned)(x >> 32) != want && !gave_up; ++i) {   // not arrived yet: poll the word
          __nanosleep(32);
          x = ld_relaxed_sys_u64(p + (size_t)j * kBM);
          if ((i & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) {
            record_error(a.status, kErrTimeoutPeer);
            gave_up = true;
          }
        }
        w[j] = x;
      }
#pragma unroll
      for (int j = 0; j < kChunk; ++j) sum[j] += __uint_as_float((unsigned)w[j]);
    }
    if (et == 0) trace_cta(a, 14);
    float xn[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int m = c0 + j;
      xn[j] = (m < a.M && n < a.N) ? xr[j] + sum[j] : 0.f;
    }
    store_residual_outputs<BN>(a, t, 0, row, c0, xn, et, ssq_red);
  }
  if (et == 0) trace_cta(a, 15);
}

// Whole-launch variant (multi-phase chain): all CTAs meet at a grid ticket, the last one publishes one flag per
// rank, every CTA then reduces a share of the tiles.
template <int BN>
HRM_DEVINL void ar_oneshot(const GemmArgs& a, int row, int et, int ep, float* ssq_red) {
  int* my_flags = reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[a.tp_rank]) + a.off_flags);
  __threadfence_system();   // this thread's pushed partials are visible system-wide before the ticket
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
  if (et == 0) {
    if (atomicAdd(&a.launch_ticket[0], 1) == (int)gridDim.x - 1) {
      a.launch_ticket[0] = 0;   // re-arm for the next launch (every CTA has arrived)
      __threadfence_system();
      for (int r = 0; r < a.tp_world; ++r)
        st_release_sys(reinterpret_cast<int*>(reinterpret_cast<char*>(a.peers[r]) + a.off_flags) + a.tp_rank, ep);
    }
  }
  if (et < a.tp_world) wait_peer_flag(my_flags + et, ep, a.status);
  asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
  const int par = ep & 1;
  for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
    const int n = t * kBM + row;
    for (int c0 = 0; c0 < BN && c0 < a.M; c0 += kChunk) {
      float sum[kChunk];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) sum[j] = 0.f;
      for (int src = 0; src < a.tp_world; ++src) {
        const float4* p = ar_slot(a, a.tp_rank, src, par, t) + (c0 / 4) * kBM + row;
#pragma unroll
        for (int q = 0; q < kChunk / 4; ++q) {
          const float4 v = __ldcg(p + q * kBM);
          sum[4 * q] += v.x; sum[4 * q + 1] += v.y; sum[4 * q + 2] += v.z; sum[4 * q + 3] += v.w;
        }
      }
      float xn[kChunk];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        const int m = c0 + j;
        xn[j] = (m < a.M && n < a.N) ? a.resid[(size_t)m * a.ldr + n] + sum[j] : 0.f;
      }
      store_residual_outputs<BN>(a, t, 0, row, c0, xn, et, ssq_red);
    }
  }
}

template <int BN, int EPI>
HRM_DEVINL void epilogue_store(const GemmArgs& a, int n_tile, int m_tile, int row, int c0, const float (&v0)[kChunk],
                               float* stage, int et, const float* inv, float* ssq_red) {
  const int n = n_tile * kBM + row;
  const float sc = (n < a.N) ? a.scale[n] : 0.f;
  const float bi = (a.bias != nullptr && n < a.N) ? a.bias[n] : 0.f;
  float v[kChunk];
#pragma unroll
  for (int j = 0; j < kChunk; ++j) v[j] = a.in_ssq != nullptr ? v0[j] * inv[c0 + j] : v0[j];
  if constexpr (EPI == EPI_SWIGLU || EPI == EPI_QKV) {
#pragma unroll
    for (int j = 0; j < kChunk; ++j) stage[j * kBM + row] = v[j] * sc + bi;
    asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
    if constexpr (EPI == EPI_SWIGLU) {
      // rows [0,64) are gate rows, [64,128) the matching up rows; output column n_tile*64 + i
      for (int idx = et; idx < kChunk * 64; idx += kEpiThreads) {
        const int j = idx >> 6, i = idx & 63;
        const int m = m_tile * BN + c0 + j;
        const int oc = n_tile * 64 + i;
        if (m < a.M && oc * 2 < a.N) {
          const float g = stage[j * kBM + i];
          const float u = stage[j * kBM + 64 + i];
          reinterpret_cast<__half*>(a.out)[(size_t)m * a.ldo + oc] = __float2half_rn(silu(g) * u);
        }
      }
    } else {
      const int D = a.head_dim, halfD = D >> 1;
      for (int idx = et; idx < kChunk * kBM; idx += kEpiThreads) {
        const int j = idx >> 7, rr = idx & (kBM - 1);
        const int m = m_tile * BN + c0 + j;
        const int gn = n_tile * kBM + rr;
        if (m >= a.M || gn >= a.N) continue;
        const int d = gn % D;
        const float* srow = stage + j * kBM;
        float y;
        if (gn < a.q_rows + a.kv_rows) {
          const int pos = a.positions[m];
          const int dd = d < halfD ? d : d - halfD;
          const float c = a.cos_t[(size_t)pos * halfD + dd];
          const float s = a.sin_t[(size_t)pos * halfD + dd];
          y = d < halfD ? srow[rr] * c - srow[rr + halfD] * s : srow[rr - halfD] * s + srow[rr] * c;
        } else {
          y = srow[rr];
        }
        if (gn < a.q_rows) {
          a.q_out[(size_t)m * a.q_rows + gn] = __float2bfloat16_rn(y);
        } else {
          const int slot = a.slots[m];
          if (slot < 0) continue;
          const bool is_k = gn < a.q_rows + a.kv_rows;
          const int kvh = (gn - a.q_rows - (is_k ? 0 : a.kv_rows)) / D;
          const int blk = slot / a.block_size, off = slot - blk * a.block_size;
          __nv_bfloat16* cache = is_k ? a.k_cache : a.v_cache;
          cache[(((size_t)blk * a.kv_heads + kvh) * a.block_size + off) * D + d] = __float2bfloat16_rn(y);
        }
      }
    }
    asm volatile("bar.sync 2, %0;" ::"n"(kEpiThreads) : "memory");
  } else if constexpr (EPI == EPI_RESID) {
    float xn[kChunk];
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int m = m_tile * BN + c0 + j;
      xn[j] = (m < a.M && n < a.N) ? a.resid[(size_t)m * a.ldr + n] + (v[j] * sc + bi) : 0.f;
    }
    store_residual_outputs<BN>(a, n_tile, m_tile, row, c0, xn, et, ssq_red);
  } else if constexpr (EPI == EPI_RESID_AR) {
    // this rank's partial tile -> its symmetric buffer ([token][128 rows], one slot per n tile)
    // push this rank's partial (16 tokens of this thread's row) into every rank's receive slot for this rank
    const int ep = *reinterpret_cast<const volatile int*>(a.epoch) + 1 + a.ep_offset;
    if (a.ar_ll) {   // epoch-tagged words: token-major per slot, a warp stores 32 consecutive words per token
      const unsigned long long tag = (unsigned long long)(unsigned)ep << 32;
      for (int dst = 0; dst < a.tp_world; ++dst) {
        unsigned long long* w = ar_ll_slot(a, dst, a.tp_rank, ep & 1, n_tile) + (size_t)c0 * kBM + row;
#pragma unroll
        for (int j = 0; j < kChunk; ++j) st_relaxed_sys_u64(w + (size_t)j * kBM, tag | __float_as_uint(v[j] * sc));
      }
      return;
    }
    float4 q[kChunk / 4];
#pragma unroll
    for (int i = 0; i < kChunk / 4; ++i) q[i] = make_float4(v[4 * i] * sc, v[4 * i + 1] * sc, v[4 * i + 2] * sc, v[4 * i + 3] * sc);
    for (int dst = 0; dst < a.tp_world; ++dst) {
      float4* p = ar_slot(a, dst, a.tp_rank, ep & 1, n_tile) + (c0 / 4) * kBM + row;
#pragma unroll
      for (int i = 0; i < kChunk / 4; ++i) p[i * kBM] = q[i];
    }
  } else {
#pragma unroll
    for (int j = 0; j < kChunk; ++j) {
      const int m = m_tile * BN + c0 + j;
      if (m < a.M && n < a.N) {
        const float y = v[j] * sc + bi;
        if constexpr (EPI == EPI_F16) {
          reinterpret_cast<__half*>(a.out)[(size_t)m * a.ldo + n] = __float2half_rn(y);
        } else {
          reinterpret_cast<float*>(a.out)[(size_t)m * a.ldo + n] = y;
        }
      }
    }
  }
}


// ------------------------------------------------------------------ host helpers shared by the launchers
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tmap_encode_fn();
int gemm_pick_bn(int M);
inline int owner_host(int64_t x, int64_t U, int64_t G) { return (int)(((x + 1) * G - 1) / U); }

}  // namespace hrm
