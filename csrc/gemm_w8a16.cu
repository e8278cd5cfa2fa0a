// W8A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM, TMA-fed), persistent stream-K, fused epilogues.
//
//   Y[m, n] = sum_k X[m, k] * (Wq[n, k] * scale[n])        X: f16 [M, K], Wq: int8 [N, K] (DSI8 row layout)
//
// Replaces the reference's DP4A GEMVs (`gemv_w8_prequant` / `gemv_w8`, scripts/deepseek_native_engine.sh:446-529)
// and the fp16 library matmuls of the torch TP path (tp/parallel_linear.py:31-35,59-66).
//
// Design ("swap-AB": weight rows on the MMA M side, tokens on N):
//  * persistent grid, one CTA per SM.  The work is the list of (tile, k-tile) units, tile = 128 weight rows x BN
//    tokens (BN in {16..256}); CTA c takes the contiguous unit range [c*U/G, (c+1)*U/G) ("stream-K"), so every SM
//    streams the same number of weight bytes whatever the tile count.  A tile cut between CTAs is a set of k-segments
//    whose fp32 partials go to a caller-provided workspace; the last segment to finish (atomic ticket) sums them in
//    k order, so results are bitwise deterministic whatever the scheduling.
//  * warp 0: TMA producer.  Raw int8 weight tiles [128 x 64] (64-byte swizzle) stream through a deep ring that the
//    dequant warps release as soon as a tile is in registers; the f16 activation tile [BN x 64] (128-byte swizzle,
//    canonical K-major UMMA layout) has its own ring released by the MMA.  Both rings run across segment and tile
//    boundaries, so HBM sees a continuous stream.
//  * warps 2-9: dequant int8 -> f16 exactly (prmt + f16x2 subtract); the per-row scale is applied once in the
//    epilogue.  Decode widths (BN <= 128) write the f16 A tile straight into tensor memory (tcgen05.st, thread =
//    row = TMEM lane) and the MMA reads A from TMEM: shared memory then carries 2 bytes per weight byte instead of 6,
//    which is what bounds a weight-streaming GEMM.  The prefill width (BN = 256) keeps A in 128-byte-swizzled
//    shared memory.
//  * warp 1: one thread issues tcgen05.mma (kind::f16, fp32 accumulate) into one of two TMEM accumulators and
//    tcgen05.commit releases ring slots / publishes a finished accumulator.
//  * warps 10-13: epilogue (thread = TMEM lane = weight row), overlapped with the next segment's mainloop: plain
//    f16/f32 stores, residual add, SwiGLU over gate/up rows interleaved per tile, or QKV bias + rotate-half RoPE +
//    paged-KV append (cross-row pairs exchanged through a 16-column smem chunk).
//  * every wait is bounded; a timeout sets the CTA abort flag, records an error code, drains in-flight TMA/MMA and
//    exits without hanging.
#include "common.cuh"
#include "gemm_w8a16.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

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
// Per-CTA %globaltimer stamps (rows 8..11: CTA start, first weight unit landed, mainloop done, CTA end).
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

// ------------------------------------------------------------------ peer-memory (NVLink) flags for EPI_RESID_AR
HRM_DEVINL void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HRM_DEVINL int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait for a peer flag to reach `want` (epochs only grow).  Records kErrTimeoutPeer on timeout.
HRM_DEVINL bool wait_peer_flag(const int* p, int want, int* status) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_sys(p) - want >= 0) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      record_error(status, kErrTimeoutPeer);
      return false;
    }
  }
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
// Receive area of every rank: [launch parity][source rank][tile][128 rows][max_bn tokens] fp32 (double-buffered by
// launch parity: a slow peer may still be reading the previous launch's data).
// Phase 1 (per finished tile, in the overlapped epilogue): the tile's partial is stored into the source-rank slot of
// EVERY rank's receive area (posted NVLink writes: no round trip on the critical path).
// Phase 2 (once per CTA, after the mainloop): the CTAs of this rank meet at a grid-wide ticket; the last one fences
// and writes this rank's epoch into every rank's flag array.  Each CTA waits on its LOCAL flags, then reduces its
// share of the tiles from local memory: x = resid + sum over source ranks in rank order, so every rank computes
// bit-identical x / xg / ssq.  One flag hop per launch; every load is local.
HRM_DEVINL float* ar_slot(const GemmArgs& a, int dst, int src, int par, int tile) {
  float* base = reinterpret_cast<float*>(reinterpret_cast<char*>(a.peers[dst]) + a.off_partials);
  return base + (((size_t)par * a.tp_world + src) * a.ar_max_tiles + tile) * a.ar_tile_floats;
}

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
  const int stride = a.ar_tile_floats / kBM;   // tokens per row slot (max_bn)
  for (int t = blockIdx.x; t < a.n_tiles; t += gridDim.x) {
    const int n = t * kBM + row;
    for (int c0 = 0; c0 < BN && c0 < a.M; c0 += kChunk) {
      float sum[kChunk];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) sum[j] = 0.f;
      for (int src = 0; src < a.tp_world; ++src) {
        const float4* p = reinterpret_cast<const float4*>(ar_slot(a, a.tp_rank, src, par, t) + (size_t)row * stride + c0);
#pragma unroll
        for (int q = 0; q < kChunk / 4; ++q) {
          const float4 v = __ldcg(p + q);
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
    const int stride = a.ar_tile_floats / kBM;
    float4 q[kChunk / 4];
#pragma unroll
    for (int i = 0; i < kChunk / 4; ++i) q[i] = make_float4(v[4 * i] * sc, v[4 * i + 1] * sc, v[4 * i + 2] * sc, v[4 * i + 3] * sc);
    for (int dst = 0; dst < a.tp_world; ++dst) {
      float4* p = reinterpret_cast<float4*>(ar_slot(a, dst, a.tp_rank, ep & 1, n_tile) + (size_t)row * stride + c0);
#pragma unroll
      for (int i = 0; i < kChunk / 4; ++i) p[i] = q[i];
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

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
w8a16_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const GemmArgs a) {
  using S = GemmSmem<BN>;
  constexpr int RW = S::RW, RX = S::RX, F = S::F, NG = S::NG;
  constexpr bool TS = S::TS;
  // TS with a single dequant group and an activation ring deeper than the A-stage ring: the dequant warps wait for
  // the unit's activation tile (they run ahead of the MMA anyway), so the MMA thread waits on one barrier per unit.
  constexpr bool kFoldX = TS && NG == 1 && RX > F;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w16 = base + S::kW16Off;
  uint8_t* xs = base + S::kXOff;
  uint8_t* wraw = base + S::kWrawOff;
  float* stage = reinterpret_cast<float*>(base + S::kStageOff);
  float* inv = reinterpret_cast<float*>(base + S::kInvOff);
  float* ssq_red = reinterpret_cast<float*>(base + S::kSsqOff);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(base + S::kBarOff);   // [RW] raw weight tile landed (TMA)
  uint64_t* wempty = wfull + RW;                                      // [RW] raw tile read by its dequant group
  uint64_t* xfull = wempty + RW;                                      // [RX] activation tile landed (TMA)
  uint64_t* xempty = xfull + RX;                                      // [RX] activation tile consumed (MMA)
  uint64_t* ffull = xempty + RX;                                      // [F] A stage written (dequant)
  uint64_t* fempty = ffull + F;                                       // [F] A stage consumed (MMA)
  uint64_t* afull = fempty + F;      // [2] accumulator ready (MMA -> epilogue)
  uint64_t* aempty = afull + 2;      // [2] accumulator drained (epilogue -> MMA)
  uint64_t* mdone = aempty + 2;      // all MMAs of this CTA complete (drain before TMEM is freed)
  int* misc = reinterpret_cast<int*>(mdone + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  int* last_flag = misc + 1;
  volatile int* abort_flag = misc + 2;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int64_t U = (int64_t)a.tiles * a.k_tiles;
  const int64_t u0 = unit_start(blockIdx.x, U, G), u1 = unit_start(blockIdx.x + 1, U, G);
  if (threadIdx.x == 0) {
    trace_mark(a, 7, 0);
    trace_cta(a, 8);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < RW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], S::kGroupThreads);
    }
    for (int s = 0; s < RX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < F; ++s) {
      mbar_init(&ffull[s], S::kGroupThreads);
      mbar_init(&fempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&afull[s], S::NACC);
      mbar_init(&aempty[s], kEpiThreads);
    }
    mbar_init(mdone, S::NACC);   // every MMA issuer commits once at the end
    *last_flag = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ku = a.ku;                       // k-tiles per unit (<= KU)
  const int kt_total = a.k_tiles * ku;       // 64-wide k-tiles per output tile
  // Only the producer thread runs ahead of the previous grid (int8 weights are never written by a kernel of the
  // inference step); every other thread starts on dependent data (activations, residual, workspace, tickets).
  const bool producer = warp == 0 && lane == 0;
  if (!producer) {
    pdl_wait();
    pdl_trigger();
  }

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      if (a.w_tiles == nullptr) tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      // the first RW units' weight tiles go out before waiting for the previous grid (ring slots start free)
      const int64_t pre = (u1 - u0) < RW ? (u1 - u0) : RW;
      {
        const int tile0 = (int)(u0 / a.k_tiles);
        int kt = (int)(u0 % a.k_tiles), n_tile = tile0 % a.n_tiles;
        for (int64_t i = 0; i < pre; ++i) {
          uint8_t* dst = wraw + i * S::kWSlot;
          mbar_arrive_expect_tx(&wfull[i], (uint32_t)(ku * kWrawBytes));
          if (a.w_tiles != nullptr) {
            bulk_load(dst, a.w_tiles + ((size_t)n_tile * kt_total + (size_t)kt * ku) * kWrawBytes,
                      (uint32_t)(ku * kWrawBytes), &wfull[i]);
          } else {
            for (int j = 0; j < ku; ++j)
              tma_load_2d(dst + j * kWrawBytes, &tmW, &wfull[i], (kt * ku + j) * kBK, n_tile * kBM);
          }
          if (++kt == a.k_tiles) {
            kt = 0;
            if (++n_tile == a.n_tiles) n_tile = 0;
          }
        }
      }
      pdl_wait();
      pdl_trigger();
      int64_t nw = pre, nx = 0;   // units issued into each ring
      // (n-tile, m-tile, unit-within-tile) of the current unit, advanced incrementally (no divisions in the loop)
      const int tile0 = (int)(u0 / a.k_tiles);
      int kt = (int)(u0 % a.k_tiles);
      int n_tile = tile0 % a.n_tiles, m_tile = tile0 / a.n_tiles;
      int sw = 0, sx = 0;
      uint32_t pw = 1u, px = 1u;   // producer-side parities of the empty barriers (first pass: free)
      for (int64_t u = u0; u < u1; ++u) {
        const int64_t i = u - u0;
        trace_mark(a, 0, i);
        if (i >= pre) {
          if (!mbar_wait_ab(&wempty[sw], pw, a.status, kErrTimeoutEmpty, abort_flag)) break;
          mbar_arrive_expect_tx(&wfull[sw], (uint32_t)(ku * kWrawBytes));
          uint8_t* dst = wraw + sw * S::kWSlot;
          if (a.w_tiles != nullptr) {
            bulk_load(dst, a.w_tiles + ((size_t)n_tile * kt_total + (size_t)kt * ku) * kWrawBytes,
                      (uint32_t)(ku * kWrawBytes), &wfull[sw]);
          } else {
            for (int j = 0; j < ku; ++j)
              tma_load_2d(dst + j * kWrawBytes, &tmW, &wfull[sw], (kt * ku + j) * kBK, n_tile * kBM);
          }
          nw = i + 1;
        }
        if (!mbar_wait_ab(&xempty[sx], px, a.status, kErrTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&xfull[sx], (uint32_t)(ku * S::kXSub));
        tma_load_3d(xs + sx * S::kXSlot, &tmX, &xfull[sx], 0, m_tile * BN, kt * ku);
        nx = i + 1;
        if (++sw == RW) { sw = 0; pw ^= 1u; }
        if (++sx == RX) { sx = 0; px ^= 1u; }
        if (++kt == a.k_tiles) {
          kt = 0;
          if (++n_tile == a.n_tiles) { n_tile = 0; ++m_tile; }
        }
      }
      // drain: every issued load must have landed before exit (earlier ones were consumed, hence landed)
      for (int64_t j = (nw > RW ? nw - RW : 0); j < nw; ++j)
        mbar_wait(&wfull[j % RW], (uint32_t)(j / RW) & 1u, a.status, kErrTimeoutFull);
      for (int64_t j = (nx > RX ? nx - RX : 0); j < nx; ++j)
        mbar_wait(&xfull[j % RX], (uint32_t)(j / RX) & 1u, a.status, kErrTimeoutFull);
    }
  } else if (warp == 1 || warp == kMma2Warp) {
    // ------------------------------------------------------------------ MMA issuers (NACC of them)
    const int mw = warp == 1 ? 0 : 1;   // issuer index = its partial accumulator
    if (lane == 0 && mw < S::NACC) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
      const uint64_t xdesc0 = sdesc_sw128(smem_u32(xs));
      const uint64_t wdesc0 = sdesc_sw128(smem_u32(w16));
      int seg = 0;
      bool ok = true;
      int sx = 0, f = 0;                  // ring slots of the current unit
      uint32_t phx = 0u, phf = 0u;        // their full-barrier parities
      // issuer mw takes the units whose CTA-local index is congruent to mw (mod NACC); the slot counters still step
      // over every unit so they stay in lock-step with the rings
      for (int64_t u = u0; ok && u < u1; ++seg) {
        const int tile = (int)(u / a.k_tiles);
        const int64_t tile_end = (int64_t)(tile + 1) * a.k_tiles;
        const int64_t ue = tile_end < u1 ? tile_end : u1;
        const int acc = seg & 1;
        const uint32_t acc_addr = tmem + (uint32_t)(acc * S::kAccCols + mw * BN);
        ok = mbar_wait_ab(&aempty[acc], ((uint32_t)(seg >> 1) & 1u) ^ 1u, a.status, kErrTimeoutAccum, abort_flag);
        tc_fence_after();
        bool first = true;                  // this issuer's first unit of the segment overwrites its partial
        for (int64_t k = u; ok && k < ue; ++k) {
          if (((k - u0) % S::NACC) != mw) {
            if (++sx == RX) { sx = 0; phx ^= 1u; }
            if (++f == F) { f = 0; phf ^= 1u; }
            continue;
          }
          // with kFoldX the dequant warps already waited for this unit's activation tile before publishing ffull
          if constexpr (!kFoldX)
            ok = mbar_wait_ab(&xfull[sx], phx, a.status, kErrTimeoutFull, abort_flag);
          ok = ok && mbar_wait_ab(&ffull[f], phf, a.status, kErrTimeoutDequant, abort_flag);
          if (!ok) break;
          trace_mark(a, 4, k - u0);
          tc_fence_after();
          // descriptors: start-address fields advance by (byte offset >> 4); no carry leaves the 14-bit field
          const uint64_t bdesc = xdesc0 + (uint64_t)((sx * S::kXSlot) >> 4);
          const uint32_t a_t = tmem + (uint32_t)(S::kAcol + f * S::kAStageCols);
          const uint64_t adesc = wdesc0 + (uint64_t)((f * kW16Bytes) >> 4);
#pragma unroll
          for (int j = 0; j < S::KU; ++j) {
            if (j < ku) {
#pragma unroll
              for (int kk = 0; kk < kBK / 16; ++kk) {
                const int q = j * (kBK / 16) + kk;   // 16-wide K step within the unit
                const uint32_t d = acc_addr;
                const uint32_t en = (!first || q > 0) ? 1u : 0u;
                const uint64_t bd = bdesc + (uint64_t)((j * S::kXSub + kk * 32) >> 4);
                if constexpr (TS) {
                  umma_f16_ts(d, a_t + (uint32_t)(j * 32 + kk * 8), bd, idesc, en);
                } else {
                  umma_f16_ss(d, adesc + (uint64_t)((kk * 32) >> 4), bd, idesc, en);
                }
              }
            }
          }
          umma_commit(&xempty[sx]);
          umma_commit(&fempty[f]);
          first = false;
          if (++sx == RX) { sx = 0; phx ^= 1u; }
          if (++f == F) { f = 0; phf ^= 1u; }
        }
        umma_commit(&afull[acc]);   // every issuer arrives once per segment (count NACC), even with no unit in it
        u = ue;
      }
      umma_commit(mdone);
      mbar_wait(mdone, 0, a.status, kErrTimeoutAccum);
      if (mw == 0) trace_cta(a, 10);
    }
  } else if (warp < kFirstEpiWarp) {
    // ------------------------------------------------------------------ dequant
    // NG independent groups take alternate units (group g: units i = g, g + NG, ...); int8 -> f16 is exact
    // (prmt + f16x2 subtract); the per-row scale is applied once in the epilogue.
    const int64_t n_units = u1 - u0;
    if constexpr (TS) {
      const int dw = warp - kFirstDqWarp;   // 0..7
      const int g = 0;                      // single group: all 8 warps convert every unit
      const int half = dw >> 2;             // warps 2-5 take k-tiles 0, 2 of a unit; warps 6-9 take 1, 3
      const int quad = warp & 3;
      const int r = quad * 32 + lane;       // weight row = TMEM lane
      const bool tracer = lane == 0 && dw == 0;
      const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)S::kAcol;
      auto to_f16 = [](const uint4 (&v)[4], uint32_t (&o)[32]) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          i8x4_to_f16x4(v[c].x, o[8 * c + 0], o[8 * c + 1]);
          i8x4_to_f16x4(v[c].y, o[8 * c + 2], o[8 * c + 3]);
          i8x4_to_f16x4(v[c].z, o[8 * c + 4], o[8 * c + 5]);
          i8x4_to_f16x4(v[c].w, o[8 * c + 6], o[8 * c + 7]);
        }
      };
      {
        // smem image of one k-tile: pre-tiled weights chunk-major ([c][r][16 B], a warp reads 512 contiguous bytes);
        // plain weights as TMA's 64-byte-swizzled rows
        const bool tiled = a.w_tiles != nullptr;
        const int sw64 = (r >> 1) & 3;
        int sw = 0, f = 0, sx = 0;
        uint32_t pw = 0u, pf = 1u, px = 0u;   // wfull parity, fempty parity (first pass free), xfull parity
        for (int64_t i = g; i < n_units; i += NG) {
          if (!mbar_wait_ab(&wfull[sw], pw, a.status, kErrTimeoutFull, abort_flag)) break;
          if (tracer) {
            trace_mark(a, 1, i);
            if (i == 0) trace_cta(a, 9);
          }
          if (!mbar_wait_ab(&fempty[f], pf, a.status, kErrTimeoutEmpty, abort_flag)) break;
          if constexpr (kFoldX) {
            if (!mbar_wait_ab(&xfull[sx], px, a.status, kErrTimeoutFull, abort_flag)) break;
          }
          if (tracer) trace_mark(a, 2, i);
          tc_fence_after();
          for (int j = half; j < ku; j += 2) {
            const uint8_t* sub = wraw + sw * S::kWSlot + j * kWrawBytes;
            uint4 v[4];
#pragma unroll
            for (int c = 0; c < 4; ++c)
              v[c] = *reinterpret_cast<const uint4*>(sub + (tiled ? c * 2048 + r * 16 : r * 64 + ((c ^ sw64) << 4)));
            uint32_t o[32];
            to_f16(v, o);
            tmem_st32u(tl + (uint32_t)(f * S::kAStageCols + j * 32), o);
          }
          mbar_arrive(&wempty[sw]);
          tc_fence_before();
          mbar_arrive(&ffull[f]);
          if (tracer) trace_mark(a, 3, i);
          if (++sw == RW) { sw = 0; pw ^= 1u; }
          if (++f == F) { f = 0; pf ^= 1u; }
          if (++sx == RX) { sx = 0; px ^= 1u; }
        }
      }
    } else {
      const int t = threadIdx.x - kFirstDqWarp * 32;   // 0..255
      const int g = t >> 6;                             // group 0..3
      const int gt = t & 63;                            // thread within group: rows gt and gt + 64
      const bool tiled = a.w_tiles != nullptr;
      for (int64_t i = g; i < n_units; i += NG) {
        const int sw = (int)(i % RW), f = (int)(i % F);
        if (!mbar_wait_ab(&wfull[sw], (uint32_t)(i / RW) & 1u, a.status, kErrTimeoutFull, abort_flag)) break;
        if (gt == 0) trace_mark(a, 1, i);
        uint4 v[2][4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int r = gt + half * 64;
          const uint8_t* slot = wraw + sw * S::kWSlot;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            // tiled weights land chunk-major ([c][r][16 B]); plain weights as TMA's 64-byte-swizzled rows
            const int off = tiled ? c * 2048 + r * 16 : r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
            v[half][c] = *reinterpret_cast<const uint4*>(slot + off);
          }
        }
        mbar_arrive(&wempty[sw]);
        if (!mbar_wait_ab(&fempty[f], ((uint32_t)(i / F) & 1u) ^ 1u, a.status, kErrTimeoutEmpty, abort_flag)) break;
        if (gt == 0) trace_mark(a, 2, i);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int r = gt + half * 64;
          const int sw128 = r & 7;
          uint8_t* dst = w16 + f * kW16Bytes + r * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 o;
            i8x4_to_f16x4(v[half][c].x, o.x, o.y); i8x4_to_f16x4(v[half][c].y, o.z, o.w);
            *reinterpret_cast<uint4*>(dst + (((2 * c) ^ sw128) << 4)) = o;
            i8x4_to_f16x4(v[half][c].z, o.x, o.y); i8x4_to_f16x4(v[half][c].w, o.z, o.w);
            *reinterpret_cast<uint4*>(dst + (((2 * c + 1) ^ sw128) << 4)) = o;
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&ffull[f]);
        if (gt == 0) trace_mark(a, 3, i);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (overlapped)
    const int et = threadIdx.x - kFirstEpiWarp * 32;   // 0..127
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int ep = (EPI == EPI_RESID_AR) ? *reinterpret_cast<volatile int*>(a.epoch) + 1 + a.ep_offset : 0;
    int seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int tile = (int)(u / a.k_tiles);
      const int ka = (int)(u % a.k_tiles);
      const int64_t tile_end = (int64_t)(tile + 1) * a.k_tiles;
      const int64_t ue = tile_end < u1 ? tile_end : u1;
      const bool whole = ka == 0 && ue == tile_end;
      const int n_tile = tile % a.n_tiles, m_tile = tile / a.n_tiles;
      const int acc = seg & 1;
      const uint32_t acc_addr = tmem + (uint32_t)(acc * S::kAccCols) + ((uint32_t)(quad * 32) << 16);
      // partials written in this segment: both issuers when it has >= 2 units, else only the owner of its unit
      const uint32_t valid = (S::NACC == 1 || ue - u >= 2) ? ((1u << S::NACC) - 1u) : (1u << ((u - u0) % S::NACC));
      mbar_wait_ab(&afull[acc], (uint32_t)(seg >> 1) & 1u, a.status, kErrTimeoutAccum, abort_flag);
      if (et == 0) trace_mark(a, 5, seg);
      tc_fence_after();
      if (whole) {
        if (a.in_ssq != nullptr) compute_row_scale<BN>(a, m_tile, inv, et);
        for (int c0 = 0; c0 < BN; c0 += kChunk) {
          float v[kChunk];
          tmem_ld_acc<BN, S::NACC>(acc_addr + (uint32_t)c0, v, valid);
          if (c0 + kChunk >= BN) {   // accumulator fully read: hand it back to the MMA warp early
            tc_fence_before();
            mbar_arrive(&aempty[acc]);
          }
          epilogue_store<BN, EPI>(a, n_tile, m_tile, row, c0, v, stage, et, inv, ssq_red);
        }
      } else {
        // partial segment: write fp32 partial, take a ticket; the last segment of the tile reduces in k order
        const int first = owner_of((int64_t)tile * a.k_tiles, U, G);
        const int nseg = owner_of(tile_end - 1, U, G) - first + 1;
        const int segidx = (int)blockIdx.x - first;
        float* ws_tile = a.ws + (size_t)tile * a.max_seg * (BN * kBM);
        float* mine = ws_tile + (size_t)segidx * (BN * kBM);
        for (int c0 = 0; c0 < BN; c0 += kChunk) {
          float v[kChunk];
          tmem_ld_acc<BN, S::NACC>(acc_addr + (uint32_t)c0, v, valid);
#pragma unroll
          for (int j = 0; j < kChunk; ++j) __stcg(&mine[(c0 + j) * kBM + row], v[j]);
        }
        tc_fence_before();
        mbar_arrive(&aempty[acc]);
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        if (et == 0) {
          const int prev = atomicAdd(&a.counters[tile], 1);
          const int is_last = prev == nseg - 1;
          if (is_last) a.counters[tile] = 0;   // re-arm for the next launch
          *last_flag = is_last;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        const bool is_last = *last_flag != 0;
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        if (is_last) {
          __threadfence();
          if (a.in_ssq != nullptr) compute_row_scale<BN>(a, m_tile, inv, et);
          for (int c0 = 0; c0 < BN; c0 += kChunk) {
            float v[kChunk];
#pragma unroll
            for (int j = 0; j < kChunk; ++j) v[j] = __ldcg(&ws_tile[(c0 + j) * kBM + row]);
            for (int sg = 1; sg < nseg; ++sg) {
              const float* p = ws_tile + (size_t)sg * (BN * kBM);
#pragma unroll
              for (int j = 0; j < kChunk; ++j) v[j] += __ldcg(&p[(c0 + j) * kBM + row]);
            }
            epilogue_store<BN, EPI>(a, n_tile, m_tile, row, c0, v, stage, et, inv, ssq_red);
          }
        }
      }
      if (et == 0) trace_mark(a, 6, seg);
      u = ue;
    }
    if constexpr (EPI == EPI_RESID_AR) ar_oneshot<BN>(a, row, et, ep, ssq_red);
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    trace_mark(a, 7, 1);
    trace_cta(a, 11);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
  if constexpr (EPI == EPI_RESID_AR) {
    if (threadIdx.x == 0) {   // the last CTA to finish advances this rank's epoch for the next launch
      __threadfence();
      if (atomicAdd(&a.launch_ticket[1], 1) == (int)gridDim.x - 1) {
        *reinterpret_cast<volatile int*>(a.epoch) = *reinterpret_cast<volatile int*>(a.epoch) + 1;
        a.launch_ticket[1] = 0;
        __threadfence();
      }
    }
  }
}

// ====================================================================================================== chain
// Persistent multi-phase W8A16 GEMM ("chain"): up to kMaxChainPhases GEMMs in ONE launch, phase p + 1 consuming
// phase p's outputs - the decode layer transition o_proj + residual -> gate/up + SwiGLU -> down + residual -> next
// layer's QKV + RoPE + KV append.  Every phase is partitioned over the same persistent grid exactly as a single
// launch of it would be (stream-K units, k-ordered partial reduction).  Rings, accumulators and the TMEM allocation
// run on across phases, so an SM's weight stream does not stop at a phase boundary: the producer issues phase
// p + 1's first RW weight units (int8 weights depend on no phase) before it waits for the grid barrier that
// publishes phase p's outputs, and only the activation loads wait.  Launch, prologue, pipeline fill and tail are
// paid once per chain instead of once per GEMM.
// Grid barrier: after its last phase-p epilogue store every CTA adds 1 to bar[p] (release); phase p + 1's
// activation loads and its epilogue (which reads the residual and the folded-norm sums) wait for
// bar[p] == gridDim.x (acquire, bounded).  The launch is cooperative - all CTAs co-resident or the launch fails -
// and the last CTA to finish re-arms the counters.  Decode widths (TS pipeline, pre-tiled weights) only.
HRM_DEVINL int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait for a grid barrier counter; on timeout records kErrTimeoutGrid and raises the CTA abort flag.
HRM_DEVINL bool grid_bar_wait(const int* p, int want, int* status, volatile int* abort_flag) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_gpu(p) >= want) return true;
    __nanosleep(128);   // one poller per CTA role, backed off: the counter's L2 slice stays free for the arrivals
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        record_error(status, kErrTimeoutGrid);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// One phase of the overlapped epilogue (the single-GEMM kernel's epilogue loop over this CTA's segments).
template <int BN, int EPI>
HRM_DEVINL void chain_epi_phase(const GemmArgs& a, int64_t u0, int64_t u1, int64_t U, int64_t G, int& seg,
                                uint32_t tmem, uint64_t* afull, uint64_t* aempty, float* stage, float* inv,
                                float* ssq_red, int* last_flag, volatile int* abort_flag, int et, int quad, int row) {
  using S = GemmSmem<BN>;
  static_assert(EPI == EPI_RESID || EPI == EPI_SWIGLU || EPI == EPI_QKV || EPI == EPI_F16 || EPI == EPI_F32 ||
                EPI == EPI_RESID_AR, "chain phase epilogue");
  // the all-reduce epoch of this phase: read before any of its pushes (the kernel advances it only at its end)
  const int ep = (EPI == EPI_RESID_AR) ? *reinterpret_cast<volatile int*>(a.epoch) + 1 + a.ep_offset : 0;
  for (int64_t u = u0; u < u1; ++seg) {
    const int tile = (int)(u / a.k_tiles);
    const int ka = (int)(u % a.k_tiles);
    const int64_t tile_end = (int64_t)(tile + 1) * a.k_tiles;
    const int64_t ue = tile_end < u1 ? tile_end : u1;
    const bool whole = ka == 0 && ue == tile_end;
    const int n_tile = tile % a.n_tiles, m_tile = tile / a.n_tiles;
    const int acc = seg & 1;
    const uint32_t acc_addr = tmem + (uint32_t)(acc * S::kAccCols) + ((uint32_t)(quad * 32) << 16);
    const uint32_t valid = (S::NACC == 1 || ue - u >= 2) ? ((1u << S::NACC) - 1u) : (1u << ((u - u0) % S::NACC));
    mbar_wait_ab(&afull[acc], (uint32_t)(seg >> 1) & 1u, a.status, kErrChainAFull, abort_flag);
    tc_fence_after();
    if (whole) {
      if (a.in_ssq != nullptr) compute_row_scale<BN>(a, m_tile, inv, et);
      for (int c0 = 0; c0 < BN; c0 += kChunk) {
        float v[kChunk];
        tmem_ld_acc<BN, S::NACC>(acc_addr + (uint32_t)c0, v, valid);
        if (c0 + kChunk >= BN) {
          tc_fence_before();
          mbar_arrive(&aempty[acc]);
        }
        epilogue_store<BN, EPI>(a, n_tile, m_tile, row, c0, v, stage, et, inv, ssq_red);
      }
    } else {
      const int first = owner_of((int64_t)tile * a.k_tiles, U, G);
      const int nseg = owner_of(tile_end - 1, U, G) - first + 1;
      const int segidx = (int)blockIdx.x - first;
      float* ws_tile = a.ws + (size_t)tile * a.max_seg * (BN * kBM);
      float* mine = ws_tile + (size_t)segidx * (BN * kBM);
      for (int c0 = 0; c0 < BN; c0 += kChunk) {
        float v[kChunk];
        tmem_ld_acc<BN, S::NACC>(acc_addr + (uint32_t)c0, v, valid);
#pragma unroll
        for (int j = 0; j < kChunk; ++j) __stcg(&mine[(c0 + j) * kBM + row], v[j]);
      }
      tc_fence_before();
      mbar_arrive(&aempty[acc]);
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (et == 0) {
        const int prev = atomicAdd(&a.counters[tile], 1);
        const int is_last = prev == nseg - 1;
        if (is_last) a.counters[tile] = 0;
        *last_flag = is_last;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      const bool is_last = *last_flag != 0;
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (is_last) {
        __threadfence();
        if (a.in_ssq != nullptr) compute_row_scale<BN>(a, m_tile, inv, et);
        for (int c0 = 0; c0 < BN; c0 += kChunk) {
          float v[kChunk];
#pragma unroll
          for (int j = 0; j < kChunk; ++j) v[j] = __ldcg(&ws_tile[(c0 + j) * kBM + row]);
          for (int sg = 1; sg < nseg; ++sg) {
            const float* p = ws_tile + (size_t)sg * (BN * kBM);
#pragma unroll
            for (int j = 0; j < kChunk; ++j) v[j] += __ldcg(&p[(c0 + j) * kBM + row]);
          }
          epilogue_store<BN, EPI>(a, n_tile, m_tile, row, c0, v, stage, et, inv, ssq_red);
        }
      }
    }
    u = ue;
  }
  // tensor-parallel phase: one flag hop, then every CTA reduces its share of the tiles from local memory
  if constexpr (EPI == EPI_RESID_AR) ar_oneshot<BN>(a, row, et, ep, ssq_red);
}

template <int BN, int EPI>
HRM_DEVINL void chain_epi_dispatch(const GemmArgs& a, int64_t u0, int64_t u1, int64_t U, int64_t G, int& seg,
                                   uint32_t tmem, uint64_t* afull, uint64_t* aempty, float* stage, float* inv,
                                   float* ssq_red, int* last_flag, volatile int* abort_flag, int et, int quad,
                                   int row) {
  if constexpr (EPI >= 0)
    chain_epi_phase<BN, EPI>(a, u0, u1, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red, last_flag, abort_flag,
                             et, quad, row);
}

template <int BN, int E0, int E1, int E2, int E3>
__global__ void __launch_bounds__(kThreads, 1)
w8a16_chain_kernel(const __grid_constant__ CUtensorMap tx0, const __grid_constant__ CUtensorMap tx1,
                   const __grid_constant__ CUtensorMap tx2, const __grid_constant__ CUtensorMap tx3,
                   const __grid_constant__ ChainArgs c) {
  using S = GemmSmem<BN>;
  constexpr int RW = S::RW, RX = S::RX, F = S::F, NG = S::NG;
  static_assert(S::TS && NG == 1, "chains run the decode (TS) pipeline");
  constexpr bool kFoldX = RX > F;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = base + S::kXOff;
  uint8_t* wraw = base + S::kWrawOff;
  float* stage = reinterpret_cast<float*>(base + S::kStageOff);
  float* inv = reinterpret_cast<float*>(base + S::kInvOff);
  float* ssq_red = reinterpret_cast<float*>(base + S::kSsqOff);
  uint64_t* wfull = reinterpret_cast<uint64_t*>(base + S::kBarOff);
  uint64_t* wempty = wfull + RW;
  uint64_t* xfull = wempty + RW;
  uint64_t* xempty = xfull + RX;
  uint64_t* ffull = xempty + RX;
  uint64_t* fempty = ffull + F;
  uint64_t* afull = fempty + F;
  uint64_t* aempty = afull + 2;
  uint64_t* mdone = aempty + 2;
  int* misc = reinterpret_cast<int*>(mdone + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  int* last_flag = misc + 1;
  volatile int* abort_flag = misc + 2;
  volatile int* bar_ok = misc + 3;   // epilogue: the grid barrier its poller saw

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t G = gridDim.x;
  const int nph = c.nph;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], S::kGroupThreads);
    }
    for (int s = 0; s < RX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < F; ++s) {
      mbar_init(&ffull[s], S::kGroupThreads);
      mbar_init(&fempty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&afull[s], S::NACC);
      mbar_init(&aempty[s], kEpiThreads);
    }
    mbar_init(mdone, S::NACC);
    *last_flag = 0;
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto tmx = [&](int p) -> const CUtensorMap* { return p == 0 ? &tx0 : p == 1 ? &tx1 : p == 2 ? &tx2 : &tx3; };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      for (int p = 0; p < nph; ++p) tma_prefetch_desc(tmx(p));
      int sw = 0, sx = 0;
      uint32_t pw = 1u, px = 1u;   // producer-side parities of the empty barriers (first pass: free)
      int64_t nw = 0, nx = 0;      // loads issued into each ring over all phases
      bool ok = true;
      for (int p = 0; ok && p < nph; ++p) {
        const GemmArgs& a = c.ph[p];
        const int64_t U = (int64_t)a.tiles * a.k_tiles;
        const int64_t u0 = unit_start(blockIdx.x, U, G), u1 = unit_start(blockIdx.x + 1, U, G);
        const int64_t n = u1 - u0;
        const int ku = a.ku;
        const int kt_total = a.k_tiles * ku;
        auto issue_w = [&](int64_t i) -> bool {
          const int64_t u = u0 + i;
          const int tile = (int)(u / a.k_tiles), kt = (int)(u % a.k_tiles), n_tile = tile % a.n_tiles;
          if (!mbar_wait_ab(&wempty[sw], pw, c.status, kErrChainWEmpty, abort_flag)) return false;
          mbar_arrive_expect_tx(&wfull[sw], (uint32_t)(ku * kWrawBytes));
          bulk_load(wraw + sw * S::kWSlot, a.w_tiles + ((size_t)n_tile * kt_total + (size_t)kt * ku) * kWrawBytes,
                    (uint32_t)(ku * kWrawBytes), &wfull[sw]);
          ++nw;
          if (++sw == RW) { sw = 0; pw ^= 1u; }
          return true;
        };
        // weights of the first units go out before the barrier that publishes this phase's activations
        const int64_t pre = p > 0 ? (n < RW ? n : RW) : 0;
        for (int64_t i = 0; ok && i < pre; ++i) ok = issue_w(i);
        if (ok && p > 0) {
          ok = grid_bar_wait(&c.bar[p - 1], (int)G, c.status, abort_flag);
          fence_proxy_async_global();
        }
        for (int64_t i = 0; ok && i < n; ++i) {
          if (i >= pre && !(ok = issue_w(i))) break;
          const int64_t u = u0 + i;
          const int tile = (int)(u / a.k_tiles), kt = (int)(u % a.k_tiles), m_tile = tile / a.n_tiles;
          if (!(ok = mbar_wait_ab(&xempty[sx], px, c.status, kErrChainXEmpty, abort_flag))) break;
          mbar_arrive_expect_tx(&xfull[sx], (uint32_t)(ku * S::kXSub));
          tma_load_3d(xs + sx * S::kXSlot, tmx(p), &xfull[sx], 0, m_tile * BN, kt * ku);
          ++nx;
          if (++sx == RX) { sx = 0; px ^= 1u; }
        }
      }
      for (int64_t j = (nw > RW ? nw - RW : 0); j < nw; ++j)
        mbar_wait(&wfull[j % RW], (uint32_t)(j / RW) & 1u, c.status, kErrTimeoutFull);
      for (int64_t j = (nx > RX ? nx - RX : 0); j < nx; ++j)
        mbar_wait(&xfull[j % RX], (uint32_t)(j / RX) & 1u, c.status, kErrTimeoutFull);
    }
  } else if (warp == 1 || warp == kMma2Warp) {
    // ------------------------------------------------------------------ MMA issuers
    const int mw = warp == 1 ? 0 : 1;
    if (lane == 0 && mw < S::NACC) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
      const uint64_t xdesc0 = sdesc_sw128(smem_u32(xs));
      int seg = 0;
      bool ok = true;
      int sx = 0, f = 0;
      uint32_t phx = 0u, phf = 0u;
      for (int p = 0; ok && p < nph; ++p) {
        const GemmArgs& a = c.ph[p];
        const int64_t U = (int64_t)a.tiles * a.k_tiles;
        const int64_t u0 = unit_start(blockIdx.x, U, G), u1 = unit_start(blockIdx.x + 1, U, G);
        const int ku = a.ku;
        for (int64_t u = u0; ok && u < u1; ++seg) {
          const int tile = (int)(u / a.k_tiles);
          const int64_t tile_end = (int64_t)(tile + 1) * a.k_tiles;
          const int64_t ue = tile_end < u1 ? tile_end : u1;
          const int acc = seg & 1;
          const uint32_t acc_addr = tmem + (uint32_t)(acc * S::kAccCols + mw * BN);
          ok = mbar_wait_ab(&aempty[acc], ((uint32_t)(seg >> 1) & 1u) ^ 1u, c.status, kErrChainAEmpty, abort_flag);
          tc_fence_after();
          bool first = true;
          for (int64_t k = u; ok && k < ue; ++k) {
            if (((k - u0) % S::NACC) != mw) {
              if (++sx == RX) { sx = 0; phx ^= 1u; }
              if (++f == F) { f = 0; phf ^= 1u; }
              continue;
            }
            if constexpr (!kFoldX) ok = mbar_wait_ab(&xfull[sx], phx, c.status, kErrChainXFull, abort_flag);
            ok = ok && mbar_wait_ab(&ffull[f], phf, c.status, kErrChainFFull, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint64_t bdesc = xdesc0 + (uint64_t)((sx * S::kXSlot) >> 4);
            const uint32_t a_t = tmem + (uint32_t)(S::kAcol + f * S::kAStageCols);
#pragma unroll
            for (int j = 0; j < S::KU; ++j) {
              if (j < ku) {
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                  const int q = j * (kBK / 16) + kk;
                  const uint32_t en = (!first || q > 0) ? 1u : 0u;
                  const uint64_t bd = bdesc + (uint64_t)((j * S::kXSub + kk * 32) >> 4);
                  umma_f16_ts(acc_addr, a_t + (uint32_t)(j * 32 + kk * 8), bd, idesc, en);
                }
              }
            }
            umma_commit(&xempty[sx]);
            umma_commit(&fempty[f]);
            first = false;
            if (++sx == RX) { sx = 0; phx ^= 1u; }
            if (++f == F) { f = 0; phf ^= 1u; }
          }
          umma_commit(&afull[acc]);
          u = ue;
        }
      }
      umma_commit(mdone);
      mbar_wait(mdone, 0, c.status, kErrTimeoutAccum);
    }
  } else if (warp < kFirstEpiWarp) {
    // ------------------------------------------------------------------ dequant (single group, pre-tiled weights)
    const int dw = warp - kFirstDqWarp;
    const int half = dw >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)S::kAcol;
    int sw = 0, f = 0, sx = 0;
    uint32_t pw = 0u, pf = 1u, px = 0u;
    bool ok = true;
    for (int p = 0; ok && p < nph; ++p) {
      const GemmArgs& a = c.ph[p];
      const int64_t U = (int64_t)a.tiles * a.k_tiles;
      const int64_t n = unit_start(blockIdx.x + 1, U, G) - unit_start(blockIdx.x, U, G);
      const int ku = a.ku;
      for (int64_t i = 0; i < n; ++i) {
        if (!(ok = mbar_wait_ab(&wfull[sw], pw, c.status, kErrChainWFull, abort_flag))) break;
        if (!(ok = mbar_wait_ab(&fempty[f], pf, c.status, kErrChainFEmpty, abort_flag))) break;
        if constexpr (kFoldX) {
          if (!(ok = mbar_wait_ab(&xfull[sx], px, c.status, kErrChainXFull, abort_flag))) break;
        }
        tc_fence_after();
        for (int j = half; j < ku; j += 2) {
          const uint8_t* sub = wraw + sw * S::kWSlot + j * kWrawBytes;
          uint4 v[4];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) v[cc] = *reinterpret_cast<const uint4*>(sub + cc * 2048 + r * 16);
          uint32_t o[32];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            i8x4_to_f16x4(v[cc].x, o[8 * cc + 0], o[8 * cc + 1]);
            i8x4_to_f16x4(v[cc].y, o[8 * cc + 2], o[8 * cc + 3]);
            i8x4_to_f16x4(v[cc].z, o[8 * cc + 4], o[8 * cc + 5]);
            i8x4_to_f16x4(v[cc].w, o[8 * cc + 6], o[8 * cc + 7]);
          }
          tmem_st32u(tl + (uint32_t)(f * S::kAStageCols + j * 32), o);
        }
        mbar_arrive(&wempty[sw]);
        tc_fence_before();
        mbar_arrive(&ffull[f]);
        if (++sw == RW) { sw = 0; pw ^= 1u; }
        if (++f == F) { f = 0; pf ^= 1u; }
        if (++sx == RX) { sx = 0; px ^= 1u; }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue, phase by phase
    const int et = threadIdx.x - kFirstEpiWarp * 32;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int seg = 0;
    for (int p = 0; p < nph; ++p) {
      const GemmArgs& a = c.ph[p];
      // the residual and the folded-norm sums this phase reads were written by other CTAs in earlier phases: one
      // thread polls the grid barrier (acquire), the CTA barrier passes the result on, every thread fences
      if (p > 0) {
        if (et == 0) *bar_ok = grid_bar_wait(&c.bar[p - 1], (int)G, c.status, abort_flag) ? 1 : 0;
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        const bool passed = *bar_ok != 0;
        asm volatile("fence.acq_rel.gpu;" ::: "memory");
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");   // bar_ok is rewritten next phase
        if (!passed) break;
      }
      const int64_t U = (int64_t)a.tiles * a.k_tiles;
      const int64_t u0 = unit_start(blockIdx.x, U, G), u1 = unit_start(blockIdx.x + 1, U, G);
      if (p == 0)
        chain_epi_dispatch<BN, E0>(a, u0, u1, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red, last_flag,
                                   abort_flag, et, quad, row);
      else if (p == 1)
        chain_epi_dispatch<BN, E1>(a, u0, u1, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red, last_flag,
                                   abort_flag, et, quad, row);
      else if (p == 2)
        chain_epi_dispatch<BN, E2>(a, u0, u1, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red, last_flag,
                                   abort_flag, et, quad, row);
      else
        chain_epi_dispatch<BN, E3>(a, u0, u1, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red, last_flag,
                                   abort_flag, et, quad, row);
      // publish this CTA's phase-p outputs: every epilogue thread fences its own stores, then one arrival
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (et == 0) {
        __threadfence();
        atomicAdd(&c.bar[p], 1);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
  if (threadIdx.x == 0) {   // the last CTA to finish re-arms the barrier counters for the next launch
    __threadfence();
    if (atomicAdd(&c.bar[kMaxChainPhases], 1) == (int)G - 1) {
      for (int p = 0; p < kMaxChainPhases; ++p) c.bar[p] = 0;
      c.bar[kMaxChainPhases] = 0;
      // tensor-parallel chains: one epoch per all-reduce phase of this launch
      constexpr int n_ar = (E0 == EPI_RESID_AR) + (E1 == EPI_RESID_AR) + (E2 == EPI_RESID_AR) + (E3 == EPI_RESID_AR);
      if constexpr (n_ar > 0) {
        int* epoch = nullptr;
        for (int p = 0; p < nph; ++p)
          if (c.ph[p].epoch != nullptr) epoch = c.ph[p].epoch;
        if (epoch != nullptr) *reinterpret_cast<volatile int*>(epoch) = *reinterpret_cast<volatile int*>(epoch) + n_ar;
      }
      __threadfence();
    }
  }
}

// ====================================================================================================== host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn tmap_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
  return fn;
}

void make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swz) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((row_stride_elems * elem_bytes) % 16 != 0) throw std::runtime_error("TMA row stride must be a multiple of 16B");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tmap_encode_fn()(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

// Per-device bounded-wait status word (device int32), registered once by the Python layer.
static int* g_status[64] = {nullptr};
void set_status_word(int device, int* p) {
  if (device >= 0 && device < 64) g_status[device] = p;
}
static long long* g_trace = nullptr;
void set_gemm_trace(long long* p) { g_trace = p; }

int* status_word() {
  int d = 0;
  cudaGetDevice(&d);
  return (d >= 0 && d < 64) ? g_status[d] : nullptr;
}

int gemm_pick_bn(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

namespace {
int g_pdl = -1;   // -1: not read from the environment yet
}
bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* e = std::getenv("HRM_PDL");
    g_pdl = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return g_pdl != 0;
}
void set_pdl_enabled(bool on) { g_pdl = on ? 1 : 0; }

int gemm_sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

static int owner_host(int64_t x, int64_t U, int64_t G) { return (int)(((x + 1) * G - 1) / U); }

GemmPlan gemm_plan(int M, int N, int K, int force_ctas) {
  GemmPlan p{};
  p.bn = gemm_pick_bn(M);
  p.n_tiles = (N + kBM - 1) / kBM;
  p.m_tiles = (M + p.bn - 1) / p.bn;
  const int kt = K / kBK;
  const int ku_max = p.bn <= 128 ? 4 : 1;   // GemmCfg<BN>::KU
  p.ku = (ku_max >= 4 && kt % 4 == 0) ? 4 : (ku_max >= 2 && kt % 2 == 0) ? 2 : 1;
  p.k_tiles = kt / p.ku;
  p.tiles = p.n_tiles * p.m_tiles;
  const int64_t U = (int64_t)p.tiles * p.k_tiles;
  int64_t G = force_ctas > 0 ? force_ctas : gemm_sm_count();
  if (G > U) G = U;
  if (G < 1) G = 1;
  p.ctas = (int)G;
  // largest number of k-segments any tile is cut into
  int max_seg = 1;
  bool any_split = false;
  for (int t = 0; t < p.tiles; ++t) {
    const int64_t f = (int64_t)t * p.k_tiles, l = f + p.k_tiles - 1;
    const int n = owner_host(l, U, G) - owner_host(f, U, G) + 1;
    max_seg = std::max(max_seg, n);
    any_split |= n > 1;
  }
  p.max_seg = max_seg;
  p.splits = max_seg;
  p.ws_floats = any_split ? (size_t)p.tiles * max_seg * p.bn * kBM : 0;
  p.counters = any_split ? p.tiles : 0;
  return p;
}

template <int BN, int EPI>
static void launch_bn(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, const GemmPlan& p,
                      cudaStream_t stream) {
  using S = GemmSmem<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(w8a16_gemm_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kAlloc);
    attr_set = true;
  }
  launch_maybe_pdl(w8a16_gemm_kernel<BN, EPI>, dim3(p.ctas), dim3(kThreads), (size_t)S::kAlloc, stream, tw, tx, a);
}

template <int EPI>
static void launch_epi(const CUtensorMap& tw, const CUtensorMap& tx, const GemmArgs& a, const GemmPlan& p,
                       cudaStream_t s) {
  switch (p.bn) {
    case 16: launch_bn<16, EPI>(tw, tx, a, p, s); break;
    case 32: launch_bn<32, EPI>(tw, tx, a, p, s); break;
    case 64: launch_bn<64, EPI>(tw, tx, a, p, s); break;
    case 128: launch_bn<128, EPI>(tw, tx, a, p, s); break;
    default: launch_bn<256, EPI>(tw, tx, a, p, s); break;
  }
}

void gemm_w8a16_launch(const void* x, int ldx, const int8_t* w, int epi, GemmArgs a, const GemmPlan& p,
                       cudaStream_t stream) {
  if (a.K % kBK != 0) throw std::runtime_error("w8a16 gemm: K must be a multiple of 64");
  if (epi == EPI_QKV && (kBM % a.head_dim != 0)) throw std::runtime_error("w8a16 gemm: head_dim must divide 128");
  if (epi == EPI_SWIGLU && a.N % kBM != 0) throw std::runtime_error("w8a16 gemm: swiglu N must be a multiple of 128");
  if (p.ws_floats && (a.ws == nullptr || a.counters == nullptr))
    throw std::runtime_error("w8a16 gemm: this shape needs the split-K workspace");
  CUtensorMap tw, tx;
  if (p.ku < 1 || (a.K / kBK) % p.ku != 0) throw std::runtime_error("w8a16 gemm: bad plan (ku)");
  if (a.w_tiles == nullptr) {
    make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.N, a.K, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    std::memset(&tw, 0, sizeof(tw));   // unused: the tiled weights are fetched with bulk copies
    if ((reinterpret_cast<uintptr_t>(a.w_tiles) & 15) != 0) throw std::runtime_error("tiled weights not 16B aligned");
  }
  // activations as a 3-D view (64 k, M rows, K/64 k-tiles) so one TMA box brings a whole unit: [ku][BN][64]
  {
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
    if (((uint64_t)ldx * 2) % 16 != 0) throw std::runtime_error("x row stride must be a multiple of 16 bytes");
    cuuint64_t dims[3] = {(cuuint64_t)kBK, (cuuint64_t)a.M, (cuuint64_t)(a.K / kBK)};
    cuuint64_t strides[2] = {(cuuint64_t)ldx * 2, (cuuint64_t)kBK * 2};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)p.bn, (cuuint32_t)p.ku};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = tmap_encode_fn()(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(x), dims, strides, box, es,
                                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("x tensor map encode failed: " + std::to_string((int)r));
  }
  if (a.status == nullptr) a.status = status_word();
  if (a.trace == nullptr) a.trace = g_trace;
  a.k_tiles = p.k_tiles;
  a.ku = p.ku;
  a.n_tiles = p.n_tiles;
  a.tiles = p.tiles;
  a.max_seg = p.max_seg;
  switch (epi) {
    case EPI_F16: launch_epi<EPI_F16>(tw, tx, a, p, stream); break;
    case EPI_F32: launch_epi<EPI_F32>(tw, tx, a, p, stream); break;
    case EPI_RESID: launch_epi<EPI_RESID>(tw, tx, a, p, stream); break;
    case EPI_SWIGLU: launch_epi<EPI_SWIGLU>(tw, tx, a, p, stream); break;
    case EPI_QKV: launch_epi<EPI_QKV>(tw, tx, a, p, stream); break;
    case EPI_RESID_AR:
      if (p.m_tiles != 1 || p.bn > 64) throw std::runtime_error("w8a16 gemm: fused all-reduce supports M <= 64");
      if (a.N / 128 > a.ar_max_tiles) throw std::runtime_error("w8a16 gemm: too many tiles for the symmetric buffer");
      launch_epi<EPI_RESID_AR>(tw, tx, a, p, stream);
      break;
    default: throw std::runtime_error("w8a16 gemm: bad epilogue");
  }
}

}  // namespace hrm

namespace hrm {

GemmPlan gemm_chain_phase_plan(int M, int N, int K, int ctas) {
  GemmPlan p{};
  p.bn = gemm_pick_bn(M);
  p.n_tiles = (N + kBM - 1) / kBM;
  p.m_tiles = (M + p.bn - 1) / p.bn;
  const int kt = K / kBK;
  p.ku = (kt % 4 == 0) ? 4 : (kt % 2 == 0) ? 2 : 1;
  p.k_tiles = kt / p.ku;
  p.tiles = p.n_tiles * p.m_tiles;
  const int64_t U = (int64_t)p.tiles * p.k_tiles;
  const int64_t G = ctas;
  p.ctas = ctas;
  int max_seg = 1;
  bool any_split = false;
  for (int t = 0; t < p.tiles; ++t) {
    const int64_t f = (int64_t)t * p.k_tiles, l = f + p.k_tiles - 1;
    const int n = owner_host(l, U, G) - owner_host(f, U, G) + 1;
    max_seg = std::max(max_seg, n);
    any_split |= n > 1;
  }
  p.max_seg = max_seg;
  p.splits = max_seg;
  p.ws_floats = any_split ? (size_t)p.tiles * max_seg * p.bn * kBM : 0;
  p.counters = any_split ? p.tiles : 0;
  return p;
}

template <int BN, int E0, int E1, int E2, int E3>
static void launch_chain_bn(const CUtensorMap (&tx)[kMaxChainPhases], const ChainArgs& c, int G, cudaStream_t s) {
  using S = GemmSmem<BN>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(w8a16_chain_kernel<BN, E0, E1, E2, E3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         S::kAlloc);
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = S::kAlloc;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;   // the grid barrier needs every CTA resident
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, w8a16_chain_kernel<BN, E0, E1, E2, E3>, tx[0], tx[1], tx[2], tx[3],
                                           c);
  if (e != cudaSuccess) throw std::runtime_error(std::string("chain launch failed: ") + cudaGetErrorString(e));
}

template <int E0, int E1, int E2, int E3>
static void launch_chain(int bn, const CUtensorMap (&tx)[kMaxChainPhases], const ChainArgs& c, int G,
                         cudaStream_t s) {
  // BN = 64 (M 33..64) runs the unfolded activation pipeline (MMA waits the activation ring itself); its first
  // B200 run timed out on an empty-slot wait, so chains take M <= 32 until that path is fixed.
  switch (bn) {
    case 16: launch_chain_bn<16, E0, E1, E2, E3>(tx, c, G, s); break;
    case 32: launch_chain_bn<32, E0, E1, E2, E3>(tx, c, G, s); break;
    default: throw std::runtime_error("w8a16 chain: M must be <= 32");
  }
}

void gemm_chain_launch(const ChainPhaseDesc* ph, int nph, int* bar, cudaStream_t stream) {
  if (nph < 1 || nph > kMaxChainPhases) throw std::runtime_error("w8a16 chain: 1..4 phases");
  if (bar == nullptr) throw std::runtime_error("w8a16 chain: barrier counters required");
  const int G = gemm_sm_count();
  ChainArgs c{};
  c.nph = nph;
  c.bar = bar;
  c.status = status_word();
  CUtensorMap tx[kMaxChainPhases];
  std::memset(tx, 0, sizeof(tx));
  int bn = 0;
  for (int p = 0; p < nph; ++p) {
    GemmArgs a = ph[p].a;
    const int epi = ph[p].epi;
    if (a.K % kBK != 0) throw std::runtime_error("w8a16 chain: K must be a multiple of 64");
    if (a.w_tiles == nullptr || (reinterpret_cast<uintptr_t>(a.w_tiles) & 15) != 0)
      throw std::runtime_error("w8a16 chain: pre-tiled, 16-byte aligned weights required");
    if (epi == EPI_QKV && (kBM % a.head_dim != 0)) throw std::runtime_error("w8a16 chain: head_dim must divide 128");
    if (epi == EPI_SWIGLU && a.N % kBM != 0) throw std::runtime_error("w8a16 chain: swiglu N must be a multiple of 128");
    const GemmPlan pl = gemm_chain_phase_plan(a.M, a.N, a.K, G);
    if (p == 0) bn = pl.bn;
    if (pl.bn != bn || pl.m_tiles != 1) throw std::runtime_error("w8a16 chain: one token tile (M <= 64) in all phases");
    if (pl.ws_floats && (a.ws == nullptr || a.counters == nullptr))
      throw std::runtime_error("w8a16 chain: this shape needs the split-K workspace");
    const void* x = ph[p].x;
    const int ldx = ph[p].ldx;
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
    if (((uint64_t)ldx * 2) % 16 != 0) throw std::runtime_error("x row stride must be a multiple of 16 bytes");
    cuuint64_t dims[3] = {(cuuint64_t)kBK, (cuuint64_t)a.M, (cuuint64_t)(a.K / kBK)};
    cuuint64_t strides[2] = {(cuuint64_t)ldx * 2, (cuuint64_t)kBK * 2};
    cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)pl.bn, (cuuint32_t)pl.ku};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = tmap_encode_fn()(&tx[p], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(x), dims, strides, box,
                                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("x tensor map encode failed: " + std::to_string((int)r));
    if (epi == EPI_RESID_AR) {
      if (a.N / kBM > a.ar_max_tiles || a.N % kBM != 0) throw std::runtime_error("w8a16 chain: bad all-reduce tiles");
      if ((int64_t)a.M * kBM > a.ar_tile_floats) throw std::runtime_error("w8a16 chain: symmetric slot too small");
      int k = 0;
      for (int q = 0; q < p; ++q) k += ph[q].epi == EPI_RESID_AR;
      a.ep_offset = k;   // the k-th all-reduce of this launch
    }
    if (a.status == nullptr) a.status = c.status;
    a.trace = nullptr;
    a.k_tiles = pl.k_tiles;
    a.ku = pl.ku;
    a.n_tiles = pl.n_tiles;
    a.tiles = pl.tiles;
    a.max_seg = pl.max_seg;
    c.ph[p] = a;
  }
  auto is = [&](int e0, int e1, int e2, int e3) {
    const int want[kMaxChainPhases] = {e0, e1, e2, e3};
    for (int p = 0; p < kMaxChainPhases; ++p)
      if ((p < nph ? ph[p].epi : -1) != want[p]) return false;
    return true;
  };
  if (is(EPI_RESID, EPI_SWIGLU, EPI_RESID, EPI_QKV))
    launch_chain<EPI_RESID, EPI_SWIGLU, EPI_RESID, EPI_QKV>(bn, tx, c, G, stream);
  else if (is(EPI_RESID, EPI_SWIGLU, EPI_RESID, -1))
    launch_chain<EPI_RESID, EPI_SWIGLU, EPI_RESID, -1>(bn, tx, c, G, stream);
  else if (is(EPI_RESID_AR, EPI_SWIGLU, EPI_RESID_AR, EPI_QKV))
    launch_chain<EPI_RESID_AR, EPI_SWIGLU, EPI_RESID_AR, EPI_QKV>(bn, tx, c, G, stream);
  else if (is(EPI_RESID_AR, EPI_SWIGLU, EPI_RESID_AR, -1))
    launch_chain<EPI_RESID_AR, EPI_SWIGLU, EPI_RESID_AR, -1>(bn, tx, c, G, stream);
  else if (is(EPI_F16, EPI_F16, -1, -1))
    launch_chain<EPI_F16, EPI_F16, -1, -1>(bn, tx, c, G, stream);
  else
    throw std::runtime_error("w8a16 chain: unsupported epilogue sequence");
}

}  // namespace hrm
