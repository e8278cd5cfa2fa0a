#include "gemm_w8a16_impl.cuh"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

namespace hrm {

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
// `origin`: the unit of this phase whose running index (see run_par in the kernel) is 0 mod NACC.
template <int BN, int EPI>
HRM_DEVINL void chain_epi_phase(const GemmArgs& a, int64_t u0, int64_t u1, int64_t origin, int64_t U, int64_t G,
                                int& seg,
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
    // a one-unit segment holds only the partial of the issuer that took the unit
    const uint32_t valid = (S::NACC == 1 || ue - u >= 2) ? ((1u << S::NACC) - 1u) : (1u << ((u - origin) % S::NACC));
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
      int nseg, segidx;   // every phase runs on all CTAs, so a phase may have fewer units than CTAs
      tile_segments((int64_t)tile * a.k_tiles, a.k_tiles, u, U, G, nseg, segidx);
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
HRM_DEVINL void chain_epi_dispatch(const GemmArgs& a, int64_t u0, int64_t u1, int64_t origin, int64_t U, int64_t G,
                                   int& seg,
                                   uint32_t tmem, uint64_t* afull, uint64_t* aempty, float* stage, float* inv,
                                   float* ssq_red, int* last_flag, volatile int* abort_flag, int et, int quad,
                                   int row) {
  if constexpr (EPI >= 0)
    chain_epi_phase<BN, EPI>(a, u0, u1, origin, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red, last_flag,
                             abort_flag, et, quad, row);
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
  // The two MMA issuers take alternate units of the CTA's running unit sequence over all phases, so each issuer's
  // previous unit is always NACC units back.  (Alternating per phase would let the gap reach NACC + 1, or more across
  // phases with a single unit: an issuer could then wait on a ring slot whose previous fill - the other issuer's
  // unit - is still pending, and its parity wait would return on the fill before that.)  run_par[p]: the running
  // index of this CTA's first unit of phase p, mod NACC.
  int* run_par = misc + 4;   // [kMaxChainPhases]

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
    int64_t run = 0;
    for (int p = 0; p < c.nph; ++p) {
      run_par[p] = (int)(run % S::NACC);
      const int64_t U = (int64_t)c.ph[p].tiles * c.ph[p].k_tiles;
      run += unit_start(blockIdx.x + 1, U, (int64_t)gridDim.x) - unit_start(blockIdx.x, U, (int64_t)gridDim.x);
    }
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
        const int64_t origin = u0 - run_par[p];   // issuer of unit k: (k - origin) % NACC
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
            if (((k - origin) % S::NACC) != mw) {
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
      const int64_t origin = u0 - run_par[p];
      if (p == 0)
        chain_epi_dispatch<BN, E0>(a, u0, u1, origin, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red,
                                   last_flag, abort_flag, et, quad, row);
      else if (p == 1)
        chain_epi_dispatch<BN, E1>(a, u0, u1, origin, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red,
                                   last_flag, abort_flag, et, quad, row);
      else if (p == 2)
        chain_epi_dispatch<BN, E2>(a, u0, u1, origin, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red,
                                   last_flag, abort_flag, et, quad, row);
      else
        chain_epi_dispatch<BN, E3>(a, u0, u1, origin, U, G, seg, tmem, afull, aempty, stage, inv, ssq_red,
                                   last_flag, abort_flag, et, quad, row);
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
    // with fewer units than CTAs every unit is its own segment (see tile_segments)
    const int n = U >= G ? owner_host(l, U, G) - owner_host(f, U, G) + 1 : p.k_tiles;
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
  ensure_smem_limit<w8a16_chain_kernel<BN, E0, E1, E2, E3>>(S::kAlloc);
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
  // BN = 64 (M 33..64) runs the unfolded activation pipeline: the MMA issuers wait on the two-deep activation ring
  // themselves.  Its first B200 run timed out on a ring wait.  The cause was the issuer alternation restarting every
  // phase (an issuer could wait one fill early on a two-deep ring and pass on the older fill); the alternation now
  // runs over all phases (run_par).  Chains stay at M <= 32 until BN = 64 has run on a B200 again.
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
