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
#include "gemm_w8a16_impl.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace hrm {

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
        TileWalk wk{a.n_tiles, a.tiles / a.n_tiles, a.k_tiles, a.m_fastest, 0, 0, 0};
        wk.start(u0);
        for (int64_t i = 0; i < pre; ++i, wk.next()) {
          uint8_t* dst = wraw + i * S::kWSlot;
          mbar_arrive_expect_tx(&wfull[i], (uint32_t)(ku * kWrawBytes));
          if (a.w_tiles != nullptr) {
            bulk_load(dst, a.w_tiles + ((size_t)wk.n_tile * kt_total + (size_t)wk.kt * ku) * kWrawBytes,
                      (uint32_t)(ku * kWrawBytes), &wfull[i]);
          } else {
            for (int j = 0; j < ku; ++j)
              tma_load_2d(dst + j * kWrawBytes, &tmW, &wfull[i], (wk.kt * ku + j) * kBK, wk.n_tile * kBM);
          }
        }
      }
      pdl_wait();
      pdl_trigger();
      int64_t nw = pre, nx = 0;   // units issued into each ring
      // (n-tile, m-tile, unit-within-tile) of the current unit, advanced incrementally (no divisions in the loop)
      TileWalk wk{a.n_tiles, a.tiles / a.n_tiles, a.k_tiles, a.m_fastest, 0, 0, 0};
      wk.start(u0);
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
            bulk_load(dst, a.w_tiles + ((size_t)wk.n_tile * kt_total + (size_t)wk.kt * ku) * kWrawBytes,
                      (uint32_t)(ku * kWrawBytes), &wfull[sw]);
          } else {
            for (int j = 0; j < ku; ++j)
              tma_load_2d(dst + j * kWrawBytes, &tmW, &wfull[sw], (wk.kt * ku + j) * kBK, wk.n_tile * kBM);
          }
          nw = i + 1;
        }
        if (!mbar_wait_ab(&xempty[sx], px, a.status, kErrTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&xfull[sx], (uint32_t)(ku * S::kXSub));
        tma_load_3d(xs + sx * S::kXSlot, &tmX, &xfull[sx], 0, wk.m_tile * BN, wk.kt * ku);
        nx = i + 1;
        if (++sw == RW) { sw = 0; pw ^= 1u; }
        if (++sx == RX) { sx = 0; px ^= 1u; }
        wk.next();
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
      int n_tile, m_tile;
      TileWalk::coords(tile, a.n_tiles, a.tiles / a.n_tiles, a.m_fastest, n_tile, m_tile);
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
        if constexpr (EPI == EPI_RESID_AR) {
          if (a.ar_ll) ar_tile_finish_ll<BN>(a, n_tile, row, et, ep, ssq_red);
          else ar_tile_finish<BN>(a, n_tile, row, et, ep, ssq_red);
        }
      } else {
        // partial segment: write fp32 partial, take a ticket; the last segment of the tile reduces in k order
        const int first = owner_of((int64_t)tile * a.k_tiles, U, G);
        const int nseg = owner_of(tile_end - 1, U, G) - first + 1;
        const int segidx = (int)blockIdx.x - first;
        // partial of this segment, column-group-major: float4 (row r, tokens 4g..4g+3) at g * 128 + r, so every warp
        // store / load of a token group is 512 contiguous bytes
        float* ws_tile = a.ws + (size_t)tile * a.max_seg * (BN * kBM);
        float* mine = ws_tile + (size_t)segidx * (BN * kBM);
        for (int c0 = 0; c0 < BN; c0 += kChunk) {
          float v[kChunk];
          tmem_ld_acc<BN, S::NACC>(acc_addr + (uint32_t)c0, v, valid);
          float4* dst = reinterpret_cast<float4*>(mine) + (c0 / 4) * kBM + row;
#pragma unroll
          for (int q = 0; q < kChunk / 4; ++q)
            __stcg(dst + q * kBM, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
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
            sum_segments<BN>(ws_tile, nseg, row, c0, v);
            epilogue_store<BN, EPI>(a, n_tile, m_tile, row, c0, v, stage, et, inv, ssq_red);
          }
          if constexpr (EPI == EPI_RESID_AR) {
            if (a.ar_ll) ar_tile_finish_ll<BN>(a, n_tile, row, et, ep, ssq_red);
            else ar_tile_finish<BN>(a, n_tile, row, et, ep, ssq_red);
          }
        }
      }
      if (et == 0) trace_mark(a, 6, seg);
      u = ue;
    }
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


// ====================================================================================================== host

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

static int g_mfast = -1;   // -1: read HRM_GEMM_MFAST on first use

bool gemm_m_fastest() {
  if (g_mfast < 0) {
    const char* e = getenv("HRM_GEMM_MFAST");
    g_mfast = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return g_mfast == 1;
}

void set_gemm_m_fastest(bool on) { g_mfast = on ? 1 : 0; }

int gemm_sm_count() {
  // Per device: a process may drive GPUs with different SM counts.  Without a usable device (host-side planning on
  // a machine with no GPU) the plan is made for a 148-SM B200.
  static std::atomic<int> sms[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();   // clear the sticky-free error this query left behind
    return 148;
  }
  int n = sms[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      throw std::runtime_error("cudaDeviceGetAttribute(multiprocessor count) failed");
    sms[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}


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
  ensure_smem_limit<w8a16_gemm_kernel<BN, EPI>>(S::kAlloc);
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
  a.m_fastest = (p.m_tiles > 1 && epi != EPI_RESID_AR && gemm_m_fastest()) ? 1 : 0;
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
