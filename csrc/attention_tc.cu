// Paged decode attention on tcgen05 tensor cores (one query token per sequence, GQA).
//
// One CTA = (context split, kv head, sequence).  Keys go on the MMA M side ("swap-AB"), the group's query heads
// (padded to 16) on N:
//     S^T[128 keys x 16]  = K_tile[128 x D] . Q^T            (A = K tile, K-major; B = Q, K-major)
//     O^T[D x 16]        += V_tile^T[D x 128] . P^T          (A = V tile, MN-major; B = P^T, K-major)
// so no tensor-core work is wasted on padding rows and every K/V byte is read once per kv head.
//
// K/V tiles of 128 keys (8 paged blocks of 16 tokens) are fetched by TMA from the paged cache viewed as a 4-D tensor
// [num_blocks][Hk][16][D]: one box = 16 tokens x 64 dims (2 KB, 128-byte swizzle), so the smem tile lands directly in
// the canonical UMMA layout (two 64-dim regions of [128 keys][128 B]).  The same layout serves as the K-major
// A operand of S and as the MN-major A operand of O.  A 3-slot ring of 32 KB (K0, V0, K1, V1, ...) keeps loads in
// flight; S is double-buffered in TMEM so the next S MMA overlaps the softmax of the current tile.
//
// Warp roles: warp 0 TMA producer, warp 1 MMA issuer (one thread), warps 2-5 softmax / O rescale / epilogue
// (thread = TMEM lane = key within the tile, or = output dim for O).  Softmax uses exp2 with the scale folded in;
// the running max is exchanged across the 4 warps each tile, row sums stay per thread until the end.  Splits are
// merged by the existing combine kernel (partials stored in natural-log units).
#include "common.cuh"
#include "kernels.h"
#include "gemm_w8a16.h"

#include <stdexcept>

namespace hrm {

namespace {
constexpr int kKeys = 128;              // keys per tile
constexpr int kD = 128;                 // head dim supported by this kernel
constexpr int kN = 16;                  // padded heads per group
constexpr int kSlotBytes = kKeys * kD * 2;   // 32 KB: one K or V tile
constexpr int kSlots = 3;
constexpr int kThreads = 6 * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// Lazy rescale: the running max used for P and O only moves when a tile's max exceeds it by more than this (log2
// units), so P <= 2^8 and O / the row sums stay exact relative to the same reference max.
constexpr float kRescaleLog2 = 8.f;
// In-kernel split merge stages (max, sum) of up to this many (head, split) pairs in the 8 KB of P buffers.
constexpr int kMergeMax = 960;

struct Smem {
  static constexpr int kRing = 0;                                  // kSlots x 32 KB
  static constexpr int kQ = kRing + kSlots * kSlotBytes;           // 2 regions x 16 rows x 128 B = 4 KB
  static constexpr int kP = kQ + 2 * kN * 128;                     // 2 buffers x 4 KB
  static constexpr int kRed = kP + 2 * 2 * kN * 128;               // [3][4 warps][16] floats: 2 max buffers + sums
  static constexpr int kBar = kRed + 3 * 4 * kN * 4;
  static constexpr int kBytes = kBar + 16 * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
};
}  // namespace

// One 128-key x 128-dim K or V tile (8 paged blocks of 16 tokens) into the canonical SW128 K-major image
// [2 dim halves][128 keys][128 B].  When the tile's 8 blocks are consecutive in the pool (the usual case: blocks are
// handed out lowest id first) two TMA boxes of 8 blocks each bring it; otherwise 16 one-block boxes.  TMA issue cost
// per instruction, not bytes, bounds this loop, so the 8-block path moves the same 32 KB with 8x fewer instructions.
HRM_DEVINL void load_kv_tile(uint8_t* dst, const CUtensorMap* m1, const CUtensorMap* m8, uint64_t* bar, const int* btab,
                             int bi0, int max_blocks, int hk, int num_blocks) {
  int blk[kKeys / 16];
  bool run = true;
#pragma unroll
  for (int j = 0; j < kKeys / 16; ++j) {
    const int bi = bi0 + j < max_blocks ? bi0 + j : max_blocks - 1;
    blk[j] = btab[bi];
    run = run && blk[j] == blk[0] + j;
  }
  run = run && blk[0] >= 0 && blk[0] + kKeys / 16 <= num_blocks;
  if (run) {
    tma_load_4d(dst, m8, bar, 0, 0, hk, blk[0]);
    tma_load_4d(dst + 16384, m8, bar, 64, 0, hk, blk[0]);
  } else {
#pragma unroll
    for (int j = 0; j < kKeys / 16; ++j) {
      tma_load_4d(dst + j * 2048, m1, bar, 0, 0, hk, blk[j]);
      tma_load_4d(dst + 16384 + j * 2048, m1, bar, 64, 0, hk, blk[j]);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 2)
attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmK8, const __grid_constant__ CUtensorMap tmV8,
                      const DecodeAttnArgs a, int num_blocks, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base + Smem::kRing;
  uint8_t* qs = base + Smem::kQ;
  uint8_t* ps = base + Smem::kP;
  float* red = reinterpret_cast<float*>(base + Smem::kRed);     // [2][4][16] tile maxima, then [4][16] sums
  uint64_t* full = reinterpret_cast<uint64_t*>(base + Smem::kBar);
  uint64_t* empty = full + kSlots;
  uint64_t* sfull = empty + kSlots;     // [2] S buffer (t & 1) written
  uint64_t* pfull = sfull + 2;          // [2] P buffer (t & 1) written
  uint64_t* pvdone = pfull + 2;         // [2] O MMA of tile t (which read P buffer t & 1) complete
  uint64_t* qready = pvdone + 2;
  uint64_t* mdone = qready + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.Hk;
  const float scale2 = a.scale * kLog2e;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&pfull[i], 128);
      mbar_init(&pvdone[i], 1);
    }
    mbar_init(qready, 128);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 32;
  // With kv_prefetch the caller vouches that the previous grid writes no block table, no context length and no KV
  // entry except the last key of each sequence: the producer then streams the older tiles before pdl_wait().
  const bool early = warp == 0 && lane == 0 && a.kv_prefetch;
  if (!early) {
    pdl_wait();
    pdl_trigger();
  }
  const int ctx = a.context_lens[b];
  const int k0 = split * a.keys_per_split;
  const int k1 = min(ctx, k0 + a.keys_per_split);
  const int nt = k1 > k0 ? (k1 - k0 + kKeys - 1) / kKeys : 0;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    bool waited = !early;
    if (lane == 0 && nt > 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmK8);
      tma_prefetch_desc(&tmV8);
      const int* btab = a.block_tables + (size_t)b * a.max_blocks;
      int issued = 0;
      for (int t = 0; t < nt; ++t) {
        const int key0 = k0 + t * kKeys;
        if (!waited && key0 + kKeys >= ctx) {   // this tile holds the newest key: written by the previous grid
          pdl_wait();
          pdl_trigger();
          waited = true;
        }
        for (int kv = 0; kv < 2; ++kv) {
          const int u = 2 * t + kv, s = u % kSlots;
          const uint32_t ph = (uint32_t)(u / kSlots) & 1u;
          if (!mbar_wait_ab(&empty[s], ph ^ 1u, status, kErrTimeoutEmpty, abort_flag)) goto prod_done;
          mbar_arrive_expect_tx(&full[s], kSlotBytes);
          uint8_t* dst = ring + s * kSlotBytes;
          load_kv_tile(dst, kv ? &tmV : &tmK, kv ? &tmV8 : &tmK8, &full[s], btab, key0 / 16, a.max_blocks, hk,
                       num_blocks);
          ++issued;
        }
      }
  prod_done:
      // drain: every issued TMA must have landed before the CTA may exit
      for (int u = max(0, issued - kSlots); u < issued; ++u)
        mbar_wait(&full[u % kSlots], (uint32_t)(u / kSlots) & 1u, status, kErrTimeoutFull);
    }
    if (!waited) {
      pdl_wait();
      pdl_trigger();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nt > 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kKeys, kN, false);   // A K-major (K tile), B K-major (Q)
      // O^T: A = V tile MN-major (bit 15), B = P^T K-major
      constexpr uint32_t idO = idesc_bf16_f32(kD, kN, false) | (1u << 15);
      bool ok = mbar_wait_ab(qready, 0, status, kErrTimeoutFull, abort_flag);
      const uint32_t qa = smem_u32(qs), pa = smem_u32(ps);
      auto issue_s = [&](int t) -> bool {
        const int u = 2 * t, s = u % kSlots;
        if (!mbar_wait_ab(&full[s], (uint32_t)(u / kSlots) & 1u, status, kErrTimeoutFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(ring + s * kSlotBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t qoff = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + (uint32_t)(t & 1) * 16u, sdesc_sw128(ka + off), sdesc_sw128(qa + qoff), idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(&sfull[t & 1]);
        return true;
      };
      ok = ok && issue_s(0);
      for (int t = 0; ok && t < nt; ++t) {
        if (t + 1 < nt && !issue_s(t + 1)) break;
        if (!mbar_wait_ab(&pfull[t & 1], (uint32_t)(t >> 1) & 1u, status, kErrTimeoutDequant, abort_flag)) break;
        const int u = 2 * t + 1, s = u % kSlots;
        if (!mbar_wait_ab(&full[s], (uint32_t)(u / kSlots) & 1u, status, kErrTimeoutFull, abort_flag)) break;
        tc_fence_after();
        const uint32_t va = smem_u32(ring + s * kSlotBytes);
        const uint32_t pb = pa + (uint32_t)(t & 1) * (2 * kN * 128);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
          umma_f16_ss(tO, sdesc_sw128_mn(va + kk * 2048, 16384), sdesc_sw128(pb + poff), idO,
                      (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(&pvdone[t & 1]);
      }
      // drain: all issued MMAs complete before TMEM is read for the last time / freed
      umma_commit(mdone);
      mbar_wait(mdone, 0, status, kErrTimeoutAccum);
    }
  } else {
    // ------------------------------------------------------------------ softmax / correction / epilogue
    const int t = threadIdx.x - 64;            // 0..127
    const int quad = warp & 3;
    const int row = quad * 32 + lane;          // TMEM lane owned by this thread
    const int w4 = warp - 2;                   // 0..3 index for the cross-warp exchange
    // Q^T operand: row h, dim d -> region d/64, row h, chunk ((d%64)/8) ^ (h%8)
    {
      const int h = t >> 3, c = t & 7;
      for (int reg = 0; reg < 2; ++reg) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (h < G) v = *reinterpret_cast<const uint4*>(a.q + ((size_t)b * a.Hq + hk * G + h) * kD + reg * 64 + c * 8);
        *reinterpret_cast<uint4*>(qs + reg * (kN * 128) + h * 128 + ((c ^ (h & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(qready);
    }
    float lsum[kN];
    float mrun[kN];
#pragma unroll
    for (int h = 0; h < kN; ++h) { lsum[h] = 0.f; mrun[h] = -INFINITY; }
    asm volatile("bar.sync 1, 128;" ::: "memory");

    for (int it = 0; it < nt; ++it) {
      mbar_wait_ab(&sfull[it & 1], (uint32_t)(it >> 1) & 1u, status, kErrTimeoutAccum, abort_flag);
      tc_fence_after();
      float s[kN];
      tmem_ld16(tmem + (uint32_t)(it & 1) * 16u + ((uint32_t)(quad * 32) << 16), s);
      const int key = k0 + it * kKeys + row;
      const bool valid = key < k1;
      float* rbuf = red + (it & 1) * (4 * kN);
#pragma unroll
      for (int h = 0; h < kN; ++h) {
        if (h < G) {                      // padded heads (h >= G) are never output: skip their softmax
          s[h] = valid ? s[h] * scale2 : -INFINITY;
          const float tm = warp_max(s[h]);
          if (lane == 0) rbuf[w4 * kN + h] = tm;
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      float corr[kN];
      bool any_corr = false;
#pragma unroll
      for (int h = 0; h < kN; ++h) {
        corr[h] = 1.f;
        if (h < G) {
          const float tm = fmaxf(fmaxf(rbuf[h], rbuf[kN + h]), fmaxf(rbuf[2 * kN + h], rbuf[3 * kN + h]));
          if (tm > mrun[h] + kRescaleLog2) {        // also taken on the first tile with a finite key (mrun = -inf)
            corr[h] = mrun[h] == -INFINITY ? 0.f : exp2f(mrun[h] - tm);
            any_corr = true;
            mrun[h] = tm;
          }
          const float p = (mrun[h] == -INFINITY) ? 0.f : exp2f(s[h] - mrun[h]);
          s[h] = p;
          lsum[h] = lsum[h] * corr[h] + p;
        }
      }
      // P buffer (it & 1) was last read by the O MMA of tile it - 2
      if (it > 1) mbar_wait_ab(&pvdone[it & 1], (uint32_t)((it - 2) >> 1) & 1u, status, kErrTimeoutAccum, abort_flag);
      // P^T operand: row h, key k=row -> region k/64, chunk ((k%64)/8) ^ (h%8), byte (k%8)*2
      {
        const int reg = row >> 6, kk = row & 63;
        uint8_t* pb = ps + (it & 1) * (2 * kN * 128) + reg * (kN * 128) + ((kk & 7) << 1);
#pragma unroll
        for (int h = 0; h < kN; ++h) {
          if (h < G) {
            __nv_bfloat16 v = __float2bfloat16_rn(s[h]);
            *reinterpret_cast<__nv_bfloat16*>(pb + h * 128 + ((((kk >> 3) ^ (h & 7))) << 4)) = v;
          }
        }
      }
      // any_corr is uniform (every thread saw the same maxima).  O holds tiles < it: rescale after O(it - 1) lands.
      if (it > 0 && any_corr) {
        mbar_wait_ab(&pvdone[(it - 1) & 1], (uint32_t)((it - 1) >> 1) & 1u, status, kErrTimeoutAccum, abort_flag);
        tc_fence_after();
        float o[kN];
        tmem_ld16(tO + ((uint32_t)(quad * 32) << 16), o);
        uint32_t ob[kN];
#pragma unroll
        for (int h = 0; h < kN; ++h) ob[h] = __float_as_uint(o[h] * corr[h]);
        tmem_st16(tO + ((uint32_t)(quad * 32) << 16), ob);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&pfull[it & 1]);
    }

    // ---------------------------------------------------------------- epilogue
    // global row sums: reduce per-thread partial sums over the 128 threads
#pragma unroll
    for (int h = 0; h < kN; ++h) lsum[h] = warp_sum(lsum[h]);
    float* sums = red + 2 * (4 * kN);
    if (lane == 0) {
#pragma unroll
      for (int h = 0; h < kN; ++h) sums[w4 * kN + h] = lsum[h];
    }
    if (nt > 0)
      mbar_wait_ab(&pvdone[(nt - 1) & 1], (uint32_t)((nt - 1) >> 1) & 1u, status, kErrTimeoutAccum, abort_flag);
    tc_fence_after();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    float o[kN];
    if (nt > 0) tmem_ld16(tO + ((uint32_t)(quad * 32) << 16), o);
    const int d = row;
#pragma unroll
    for (int h = 0; h < kN; ++h) {
      if (h >= G) break;
      const float L = sums[h] + sums[kN + h] + sums[2 * kN + h] + sums[3 * kN + h];
      const float A = nt > 0 ? o[h] : 0.f;
      const int hq = hk * G + h;
      if (a.splits == 1) {
        a.out[((size_t)b * a.Hq + hq) * kD + d] = __float2half_rn(L > 0.f ? A / L : 0.f);
      } else {
        float* p = a.ws + (((size_t)b * a.Hq + hq) * a.splits + split) * (kD + 2);
        p[2 + d] = A;
        if (d == 0) {
          p[0] = nt > 0 ? mrun[h] * kLn2 : -INFINITY;
          p[1] = L;
        }
      }
    }
    if (a.splits > 1 && a.tickets != nullptr) {
      // split merge in-kernel: the last CTA of this (sequence, kv head) to publish its partials combines all splits
      // in split order (deterministic whichever CTA is last), same math as decode_combine_kernel
      volatile int* is_last = reinterpret_cast<volatile int*>(red);   // tile maxima are no longer needed
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (t == 0) {
        int* tk = a.tickets + (size_t)b * a.Hk + hk;
        const int prev = atomicAdd(tk, 1);
        *is_last = prev == a.splits - 1;
        if (prev == a.splits - 1) *tk = 0;   // re-arm: every split of this launch has counted
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*is_last) {
        // all loads of a round are independent: stage (m, L) of every (head, split) in the P buffers (free now:
        // the last O MMA has completed), per-head factors next, then each thread (= output dim) sums its column
        __threadfence();
        const int n = G * a.splits;                   // <= kMergeMax (checked on the host)
        float* mst = reinterpret_cast<float*>(ps);    // [n] split maxima -> weights exp(m_s - M)
        float* lst = mst + kMergeMax;                 // [n] split row sums
        float* linv = lst + kMergeMax;                // [G] 1 / merged row sum (0 when empty)
        for (int i = t; i < n; i += 128) {
          const int h = i / a.splits, sp = i - h * a.splits;
          const float* p = a.ws + (((size_t)b * a.Hq + hk * G + h) * a.splits + sp) * (kD + 2);
          mst[i] = __ldcg(p);
          lst[i] = __ldcg(p + 1);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (t < G) {
          float M = -INFINITY;
          for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, mst[t * a.splits + sp]);
          float L = 0.f;
          for (int sp = 0; sp < a.splits; ++sp) {
            const float ms = mst[t * a.splits + sp];
            const float f = (M == -INFINITY || ms == -INFINITY) ? 0.f : __expf(ms - M);
            mst[t * a.splits + sp] = f;
            L += lst[t * a.splits + sp] * f;
          }
          linv[t] = L > 0.f ? 1.f / L : 0.f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        for (int h = 0; h < G; ++h) {
          const int hq = hk * G + h;
          const float* p = a.ws + ((size_t)b * a.Hq + hq) * a.splits * (kD + 2) + 2 + d;
          float A = 0.f;
#pragma unroll 4
          for (int sp = 0; sp < a.splits; ++sp) A += __ldcg(p + sp * (kD + 2)) * mst[h * a.splits + sp];
          a.out[((size_t)b * a.Hq + hq) * kD + d] = __float2half_rn(A * linv[h]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// ------------------------------------------------------------------------------------------------ host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn tmap_encode_fn();

static void make_kv_map(CUtensorMap* m, const void* cache, int num_blocks, int Hk, int bs, int blocks_per_box = 1) {
  if ((reinterpret_cast<uintptr_t>(cache) & 15) != 0) throw std::runtime_error("KV cache must be 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)bs, (cuuint64_t)Hk, (cuuint64_t)num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)kD * 2, (cuuint64_t)bs * kD * 2, (cuuint64_t)Hk * bs * kD * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)bs, 1, (cuuint32_t)blocks_per_box};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = tmap_encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(cache), dims, strides, box,
                                es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("KV tensor map encode failed: " + std::to_string((int)r));
}

int decode_attn_tc_merge_max() { return kMergeMax; }

bool decode_attn_tc_supported(const DecodeAttnArgs& a) {
  return a.D == kD && a.block_size == 16 && a.Hq / a.Hk <= kN && a.keys_per_split % kKeys == 0;
}

void decode_attn_tc_launch(const DecodeAttnArgs& a, int num_blocks, int* status, cudaStream_t s) {
  if (!decode_attn_tc_supported(a)) throw std::runtime_error("tcgen05 decode attention: unsupported shape");
  CUtensorMap tk, tv, tk8, tv8;
  make_kv_map(&tk, a.k_cache, num_blocks, a.Hk, a.block_size);
  make_kv_map(&tv, a.v_cache, num_blocks, a.Hk, a.block_size);
  make_kv_map(&tk8, a.k_cache, num_blocks, a.Hk, a.block_size, kKeys / 16);
  make_kv_map(&tv8, a.v_cache, num_blocks, a.Hk, a.block_size, kKeys / 16);
  ensure_smem_limit<attn_decode_tc_kernel>(Smem::kAlloc);
  dim3 grid(a.splits, a.Hk, a.B);
  if (status == nullptr) status = status_word();
  launch_maybe_pdl(attn_decode_tc_kernel, grid, dim3(kThreads), (size_t)Smem::kAlloc, s, tk, tv, tk8, tv8, a,
                   num_blocks, status);
  if (a.splits > 1 && a.tickets == nullptr) decode_combine_launch(a, s);
}


// ================================================================================================================
// Paged prefill (varlen, causal) flash attention on tcgen05.
//
// One CTA = (query tile, kv head, sequence).  A query tile is 128 MMA rows packing the GQA group: row r is token
// t0 + r / G, head hk*G + r % G, so one K/V tile feeds all heads sharing the kv head (tokens per tile = 128 / G).
//     S[128 rows x 128 keys] = Q_tile . K_tile^T          (A = Q, K-major; B = K tile, K-major)
//     O[128 rows x D]       += P . V_tile                 (A = P, K-major; B = V tile, MN-major)
// Q arrives by one 3-D TMA box per 64 dims (view [T][Hq][D]); K/V tiles come from the paged cache exactly as in
// decode.  Softmax: thread = row (TMEM lane), two TMEM passes per tile (max, then exp2 + P store), lazy rescaling:
// O and the row sum are rescaled only when the row max grows by more than 2^8, so most tiles skip the O round trip.
// S is double-buffered in TMEM (2 x 128 columns) so the next QK^T overlaps the softmax; O uses 128 more columns.
// CTAs are launched heaviest-first (last query tiles see the most keys).
// ================================================================================================================
namespace {
constexpr int kPfRows = 128;
constexpr int kPfThreads = 6 * 32;
constexpr float kRescaleThresh = 8.0f;   // log2 units
struct PfSmem {
  static constexpr int kQ = 0;                                 // 2 regions x [128 rows][128 B] = 32 KB
  static constexpr int kRing = kQ + 2 * kPfRows * 128;         // kSlots x 32 KB
  static constexpr int kP = kRing + kSlots * kSlotBytes;       // 2 regions x 16 KB
  static constexpr int kBar = kP + 2 * kPfRows * 128;
  static constexpr int kBytes = kBar + 16 * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;
};
}  // namespace

__global__ void __launch_bounds__(kPfThreads, 1)
attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmK8,
                       const __grid_constant__ CUtensorMap tmV8, const PrefillAttnArgs a, int tpt, int num_blocks,
                       int* status) {
  const int G = a.Hq / a.Hk;
  const int tile = gridDim.x - 1 - blockIdx.x;   // heaviest (latest) tiles first
  const int hk = blockIdx.y, seq = blockIdx.z;
  const int qo = a.cu_q[seq];
  const int qlen = a.cu_q[seq + 1] - qo;
  const int t0 = tile * tpt;
  if (t0 >= qlen) return;   // uniform exit before any barrier / TMEM allocation
  const int qstart = a.q_start[seq];
  const int ctx = a.context_lens[seq];
  const int tl = min(qlen, t0 + tpt) - 1;
  const int kend = min(ctx, qstart + tl + 1);
  const int nt = (kend + kKeys - 1) / kKeys;
  const float scale2 = a.scale * kLog2e;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = base + PfSmem::kQ;
  uint8_t* ring = base + PfSmem::kRing;
  uint8_t* ps = base + PfSmem::kP;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + PfSmem::kBar);
  uint64_t* empty = full + kSlots;
  uint64_t* sfull = empty + kSlots;   // [2]
  uint64_t* pfull = sfull + 2;
  uint64_t* pvdone = pfull + 1;
  uint64_t* qfull = pvdone + 1;
  uint64_t* mdone = qfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&sfull[0], 1);
    mbar_init(&sfull[1], 1);
    mbar_init(pfull, 128);
    mbar_init(pvdone, 1);
    mbar_init(qfull, 1);
    mbar_init(mdone, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmK8);
      tma_prefetch_desc(&tmV8);
      mbar_arrive_expect_tx(qfull, 2 * 128 * G * tpt);
      tma_load_3d(qs, &tmQ, qfull, 0, hk * G, qo + t0);
      tma_load_3d(qs + kPfRows * 128, &tmQ, qfull, 64, hk * G, qo + t0);
      const int* btab = a.block_tables + (size_t)seq * a.max_blocks;
      int issued = 0;
      for (int t = 0; t < nt; ++t) {
        for (int kv = 0; kv < 2; ++kv) {
          const int u = 2 * t + kv, s = u % kSlots;
          if (!mbar_wait_ab(&empty[s], ((uint32_t)(u / kSlots) & 1u) ^ 1u, status, kErrTimeoutEmpty, abort_flag))
            goto pf_prod_done;
          mbar_arrive_expect_tx(&full[s], kSlotBytes);
          uint8_t* dst = ring + s * kSlotBytes;
          load_kv_tile(dst, kv ? &tmV : &tmK, kv ? &tmV8 : &tmK8, &full[s], btab, t * (kKeys / 16), a.max_blocks, hk,
                       num_blocks);
          ++issued;
        }
      }
    pf_prod_done:
      mbar_wait(qfull, 0, status, kErrTimeoutFull);
      for (int u = max(0, issued - kSlots); u < issued; ++u)
        mbar_wait(&full[u % kSlots], (uint32_t)(u / kSlots) & 1u, status, kErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(kPfRows, kKeys, false);
      constexpr uint32_t idO = idesc_bf16_f32(kPfRows, kD, true);   // B = V tile, MN-major
      const uint32_t qa = smem_u32(qs), pa = smem_u32(ps);
      bool ok = mbar_wait_ab(qfull, 0, status, kErrTimeoutFull, abort_flag);
      auto issue_s = [&](int t) -> bool {
        const int u = 2 * t, s = u % kSlots;
        if (!mbar_wait_ab(&full[s], (uint32_t)(u / kSlots) & 1u, status, kErrTimeoutFull, abort_flag)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(ring + s * kSlotBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tmem + (uint32_t)(t & 1) * 128u, sdesc_sw128(qa + off), sdesc_sw128(ka + off), idS,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(&sfull[t & 1]);
        return true;
      };
      ok = ok && issue_s(0);
      for (int t = 0; ok && t < nt; ++t) {
        if (t + 1 < nt && !issue_s(t + 1)) break;
        if (!mbar_wait_ab(pfull, (uint32_t)t & 1u, status, kErrTimeoutDequant, abort_flag)) break;
        const int u = 2 * t + 1, s = u % kSlots;
        if (!mbar_wait_ab(&full[s], (uint32_t)(u / kSlots) & 1u, status, kErrTimeoutFull, abort_flag)) break;
        tc_fence_after();
        const uint32_t va = smem_u32(ring + s * kSlotBytes);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_f16_ss(tO, sdesc_sw128(pa + poff), sdesc_sw128_mn(va + kk * 2048, 16384), idO,
                      (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        umma_commit(pvdone);
      }
      umma_commit(mdone);
      mbar_wait(mdone, 0, status, kErrTimeoutAccum);
    }
  } else {
    // ------------------------------------------------------------------ softmax (thread = row)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const bool row_ok = r < G * tpt && t0 + r / G < qlen;
    const int pos = qstart + t0 + r / G;
    const int kmax = row_ok ? min(ctx, pos + 1) : 0;   // keys [0, kmax) visible to this row
    float m_used = -INFINITY, l = 0.f;
    for (int it = 0; it < nt; ++it) {
      mbar_wait_ab(&sfull[it & 1], (uint32_t)(it >> 1) & 1u, status, kErrTimeoutAccum, abort_flag);
      tc_fence_after();
      const uint32_t sa = tmem + (uint32_t)(it & 1) * 128u + lane_off;
      const int key0 = it * kKeys;
      float tmax = -INFINITY;
      for (int c = 0; c < kKeys; c += 32) {
        float v[32];
        tmem_ld32(sa + (uint32_t)c, v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (key0 + c + i < kmax) tmax = fmaxf(tmax, v[i]);
      }
      tmax *= scale2;
      float corr = 1.f;
      bool rescale = false;
      if (tmax > m_used + kRescaleThresh || (m_used == -INFINITY && tmax != -INFINITY)) {
        corr = m_used == -INFINITY ? 0.f : exp2f(m_used - tmax);
        rescale = m_used != -INFINITY;
        m_used = tmax;
        l *= corr;
      }
      if (it > 0) mbar_wait_ab(pvdone, (uint32_t)(it - 1) & 1u, status, kErrTimeoutAccum, abort_flag);
      tc_fence_after();
      // tcgen05.ld/st are warp-collective: the rescale runs for the whole warp whenever any of its rows needs it
      // (rows that do not rescale multiply by 1).
      if (__any_sync(0xffffffffu, rescale && it > 0)) {
        const float cf = (rescale && it > 0) ? corr : 1.f;
        for (int c = 0; c < kD; c += 32) {
          float o[32];
          tmem_ld32(tO + lane_off + (uint32_t)c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= cf;
          tmem_st32(tO + lane_off + (uint32_t)c, o);
        }
      }
      // P row: keys [c, c+32) -> region c/64, 16-byte chunks ((c%64)/8 + q) ^ (r%8)
      for (int c = 0; c < kKeys; c += 32) {
        float v[32];
        tmem_ld32(sa + (uint32_t)c, v);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = (key0 + c + i < kmax && m_used != -INFINITY) ? exp2f(v[i] * scale2 - m_used) : 0.f;
          const float p1 = (key0 + c + i + 1 < kmax && m_used != -INFINITY) ? exp2f(v[i + 1] * scale2 - m_used) : 0.f;
          l += p0 + p1;
          __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
          pk[i >> 1] = *reinterpret_cast<uint32_t*>(&b2);
        }
        uint8_t* prow = ps + (c >> 6) * 16384 + r * 128;
        const int cb = (c & 63) >> 3;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(prow + (((cb + q) ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pfull);
    }
    if (nt > 0) mbar_wait_ab(pvdone, (uint32_t)(nt - 1) & 1u, status, kErrTimeoutAccum, abort_flag);
    tc_fence_after();
    {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __half* orow = a.out + ((size_t)(qo + t0 + r / G) * a.Hq + hk * G + r % G) * kD;
      for (int c = 0; c < kD; c += 32) {
        float o[32];
        if (nt > 0) {
          tmem_ld32(tO + lane_off + (uint32_t)c, o);   // warp-collective: every lane loads
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0.f;
        }
        if (!row_ok) continue;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          __half2 h0 = __floats2half2_rn(o[i] * inv, o[i + 1] * inv), h1 = __floats2half2_rn(o[i + 2] * inv, o[i + 3] * inv);
          __half2 h2 = __floats2half2_rn(o[i + 4] * inv, o[i + 5] * inv), h3 = __floats2half2_rn(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4*>(orow + c + i) =
              make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                         *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

bool prefill_attn_tc_supported(const PrefillAttnArgs& a) {
  const int G = a.Hk > 0 ? a.Hq / a.Hk : 0;
  return a.D == kD && a.block_size == 16 && G >= 1 && G <= 128 && a.Hq % a.Hk == 0;
}

void prefill_attn_tc_launch(const PrefillAttnArgs& a, int num_blocks, int total_q, int* status, cudaStream_t s) {
  if (!prefill_attn_tc_supported(a)) throw std::runtime_error("tcgen05 prefill attention: unsupported shape");
  if (a.S == 0 || a.max_q == 0) return;
  const int G = a.Hq / a.Hk;
  const int tpt = kPfRows / G;
  CUtensorMap tq, tk, tv;
  {
    if ((reinterpret_cast<uintptr_t>(a.q) & 15) != 0) throw std::runtime_error("q must be 16-byte aligned");
    cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)a.Hq, (cuuint64_t)total_q};
    cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)a.Hq * kD * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)G, (cuuint32_t)tpt};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = tmap_encode_fn()(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(a.q), dims,
                                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("Q tensor map encode failed: " + std::to_string((int)r));
  }
  make_kv_map(&tk, a.k_cache, num_blocks, a.Hk, a.block_size);
  make_kv_map(&tv, a.v_cache, num_blocks, a.Hk, a.block_size);
  CUtensorMap tk8, tv8;
  make_kv_map(&tk8, a.k_cache, num_blocks, a.Hk, a.block_size, kKeys / 16);
  make_kv_map(&tv8, a.v_cache, num_blocks, a.Hk, a.block_size, kKeys / 16);
  ensure_smem_limit<attn_prefill_tc_kernel>(PfSmem::kAlloc);
  if (status == nullptr) status = status_word();
  dim3 grid((a.max_q + tpt - 1) / tpt, a.Hk, a.S);
  attn_prefill_tc_kernel<<<grid, kPfThreads, PfSmem::kAlloc, s>>>(tq, tk, tv, tk8, tv8, a, tpt, num_blocks, status);
}

}  // namespace hrm
