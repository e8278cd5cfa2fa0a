// W8A16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM, TMA-fed), with fused epilogues.
//
//   Y[m, n] = sum_k X[m, k] * (Wq[n, k] * scale[n])        X: f16 [M, K], Wq: int8 [N, K] (DSI8 row layout)
//
// This replaces the reference's DP4A GEMVs (`gemv_w8_prequant` / `gemv_w8`,
// scripts/deepseek_native_engine.sh:446-529) and the fp16 cuBLAS matmuls of the torch TP path
// (tp/parallel_linear.py:31-35,59-66).
//
// Design ("swap-AB", weight rows on the MMA M side):
//  * one CTA owns 128 weight rows (MMA M = 128) x BN tokens (MMA N = BN in {16..256}) x a K range (split-K);
//  * warp 0 issues TMA loads: the raw int8 weight tile [128 x 64] (64-byte swizzle) and the f16 activation tile
//    [BN x 64] (128-byte swizzle, the UMMA canonical K-major layout);
//  * 8 dequant warps convert int8 -> f16 exactly (prmt + f16x2 subtract) straight into the 128-byte-swizzled
//    canonical layout of the A operand; the per-row scale is applied once in the epilogue;
//  * one thread of warp 1 issues tcgen05.mma (kind::f16, fp32 accumulator in TMEM) and tcgen05.commit frees
//    each stage;
//  * the same 8 warps run the epilogue out of TMEM (tcgen05.ld): plain f16/f32 stores, residual add, SwiGLU over
//    gate/up rows interleaved per tile, or QKV bias + rotate-half RoPE + paged-KV append.
//  * split-K partials go to a caller-provided fp32 workspace; the last CTA of a tile (atomic ticket) sums the
//    partials in split order, so results are bitwise deterministic whatever the CTA scheduling.
#include "common.cuh"
#include "gemm_w8a16.h"

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

namespace hrm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kDqWarps = 8;
constexpr int kFirstDqWarp = 2;
constexpr int kThreads = (kFirstDqWarp + kDqWarps) * 32;
constexpr int kEpiThreads = kDqWarps * 32;
constexpr int kWrawBytes = kBM * kBK;          // int8 tile
constexpr int kW16Bytes = kBM * kBK * 2;       // f16 tile

template <int BN> struct GemmCfg;
template <> struct GemmCfg<16>  { static constexpr int kStages = 4; };
template <> struct GemmCfg<32>  { static constexpr int kStages = 4; };
template <> struct GemmCfg<64>  { static constexpr int kStages = 4; };
template <> struct GemmCfg<128> { static constexpr int kStages = 4; };
template <> struct GemmCfg<256> { static constexpr int kStages = 3; };

template <int BN>
struct GemmSmem {
  static constexpr int kStages = GemmCfg<BN>::kStages;
  static constexpr int kXBytes = BN * kBK * 2;
  static constexpr int kW16Off = 0;
  static constexpr int kXOff = kW16Off + kStages * kW16Bytes;
  static constexpr int kWrawOff = kXOff + kStages * kXBytes;
  static constexpr int kBarOff = kWrawOff + kStages * kWrawBytes;
  static constexpr int kBytes = kBarOff + (3 * kStages + 1) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;   // slack for manual 1024-byte alignment
  static constexpr int kTmemCols = BN < 32 ? 32 : BN;
  static_assert(kStages * (kW16Bytes + kXBytes + kWrawBytes) >= BN * kBM * 4, "staging area too small");
};

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
w8a16_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                  const GemmArgs a) {
  using S = GemmSmem<BN>;
  constexpr int ST = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* w16 = base + S::kW16Off;
  uint8_t* xs = base + S::kXOff;
  uint8_t* wraw = base + S::kWrawOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + S::kBarOff);
  uint64_t* dqf = full + ST;
  uint64_t* empty = dqf + ST;
  uint64_t* accf = empty + ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y, split = blockIdx.z;
  const int kt0 = split * a.tiles_per_split;
  const int kt1 = min(a.k_tiles, kt0 + a.tiles_per_split);
  const int nkt = kt1 - kt0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&dqf[s], kEpiThreads);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *last_flag = 0;
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

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      for (int i = 0; i < nkt; ++i) {
        const int s = i % ST;
        const uint32_t ph = (uint32_t)(i / ST) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, a.status, kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&full[s], kWrawBytes + S::kXBytes);
        const int kx = (kt0 + i) * kBK;
        tma_load_2d(wraw + s * kWrawBytes, &tmW, &full[s], kx, n_tile * kBM);
        tma_load_2d(xs + s * S::kXBytes, &tmX, &full[s], kx, m_tile * BN);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN);
      for (int i = 0; i < nkt; ++i) {
        const int s = i % ST;
        const uint32_t ph = (uint32_t)(i / ST) & 1u;
        if (!mbar_wait(&full[s], ph, a.status, kErrTimeoutFull)) break;
        if (!mbar_wait(&dqf[s], ph, a.status, kErrTimeoutDequant)) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(w16 + s * kW16Bytes);
        const uint32_t b0 = smem_u32(xs + s * S::kXBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          umma_f16_ss(tmem, sdesc_sw128(a0 + kk * 32), sdesc_sw128(b0 + kk * 32), idesc,
                      (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accf);
    }
  } else {
    // ------------------------------------------------------------------ dequant
    const int t = threadIdx.x - kFirstDqWarp * 32;  // 0..255
    const int r = t & (kBM - 1);
    const int h = t >> 7;                           // which 32-element half of the 64-wide K stage
    for (int i = 0; i < nkt; ++i) {
      const int s = i % ST;
      const uint32_t ph = (uint32_t)(i / ST) & 1u;
      if (!mbar_wait(&full[s], ph, a.status, kErrTimeoutFull)) break;
      const uint8_t* src = wraw + s * kWrawBytes + r * 64;
      const int sw64 = (r >> 1) & 3;
      const uint4 v0 = *reinterpret_cast<const uint4*>(src + (((2 * h) ^ sw64) << 4));
      const uint4 v1 = *reinterpret_cast<const uint4*>(src + (((2 * h + 1) ^ sw64) << 4));
      uint8_t* dst = w16 + s * kW16Bytes + r * 128;
      const int sw128 = r & 7;
      uint4 o;
      i8x4_to_f16x4(v0.x, o.x, o.y); i8x4_to_f16x4(v0.y, o.z, o.w);
      *reinterpret_cast<uint4*>(dst + (((4 * h + 0) ^ sw128) << 4)) = o;
      i8x4_to_f16x4(v0.z, o.x, o.y); i8x4_to_f16x4(v0.w, o.z, o.w);
      *reinterpret_cast<uint4*>(dst + (((4 * h + 1) ^ sw128) << 4)) = o;
      i8x4_to_f16x4(v1.x, o.x, o.y); i8x4_to_f16x4(v1.y, o.z, o.w);
      *reinterpret_cast<uint4*>(dst + (((4 * h + 2) ^ sw128) << 4)) = o;
      i8x4_to_f16x4(v1.z, o.x, o.y); i8x4_to_f16x4(v1.w, o.z, o.w);
      *reinterpret_cast<uint4*>(dst + (((4 * h + 3) ^ sw128) << 4)) = o;
      fence_proxy_async_smem();
      mbar_arrive(&dqf[s]);
    }

    // ------------------------------------------------------------------ epilogue
    mbar_wait(accf, 0, a.status, kErrTimeoutAccum);
    tc_fence_after();
    const int quad = warp & 3;                       // TMEM lanes this warp may access
    const int row = quad * 32 + lane;                // tile row == TMEM lane
    const int colgrp = (warp - kFirstDqWarp) >> 2;   // 0 or 1
    constexpr int kColsPerWarp = BN / 2 < 16 ? 16 : BN / 2;
    const int c_begin = colgrp * kColsPerWarp;
    const int c_end = min(BN, c_begin + kColsPerWarp);
    const int n = n_tile * kBM + row;
    const int tile_id = m_tile * gridDim.x + n_tile;
    const bool split_k = a.splits > 1;

    if (split_k) {
      float* my = a.ws + ((size_t)tile_id * a.splits + split) * (size_t)(BN * kBM);
      for (int c0 = c_begin; c0 < c_end; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) __stcg(&my[(c0 + j) * kBM + row], v[j]);
      }
      __threadfence();
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (t == 0) {
        const int prev = atomicAdd(&a.counters[tile_id], 1);
        const int is_last = (prev == a.splits - 1);
        if (is_last) a.counters[tile_id] = 0;      // re-arm for the next launch
        *last_flag = is_last;
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
      if (!*last_flag) goto done;
      __threadfence();
    }

    {
      const float sc = (n < a.N) ? a.scale[n] : 0.f;
      const float bi = (a.bias != nullptr && n < a.N) ? a.bias[n] : 0.f;
      float* stage = reinterpret_cast<float*>(base);   // [BN][128] fp32, reuses the pipeline buffers
      for (int c0 = c_begin; c0 < c_end; c0 += 16) {
        float v[16];
        if (split_k) {
          const float* wsb = a.ws + (size_t)tile_id * a.splits * (size_t)(BN * kBM);
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __ldcg(&wsb[(c0 + j) * kBM + row]);
          for (int sp = 1; sp < a.splits; ++sp) {
            const float* p = wsb + (size_t)sp * (BN * kBM);
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] += __ldcg(&p[(c0 + j) * kBM + row]);
          }
        } else {
          tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m_tile * BN + c0 + j;
          const float y = v[j] * sc + bi;
          if constexpr (EPI == EPI_SWIGLU || EPI == EPI_QKV) {
            stage[(c0 + j) * kBM + row] = y;
          } else {
            if (m < a.M && n < a.N) {
              if constexpr (EPI == EPI_F16) {
                reinterpret_cast<__half*>(a.out)[(size_t)m * a.ldo + n] = __float2half_rn(y);
              } else if constexpr (EPI == EPI_F32) {
                reinterpret_cast<float*>(a.out)[(size_t)m * a.ldo + n] = y;
              } else if constexpr (EPI == EPI_RESID) {
                float* rp = &a.resid[(size_t)m * a.ldr + n];
                *rp = *rp + y;
              }
            }
          }
        }
      }
      if constexpr (EPI == EPI_SWIGLU || EPI == EPI_QKV) {
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        if constexpr (EPI == EPI_SWIGLU) {
          // Tile rows [0,64) are gate rows, [64,128) the matching up rows; output column n_tile*64 + i.
          for (int idx = t; idx < BN * 64; idx += kEpiThreads) {
            const int j = idx >> 6, i = idx & 63;
            const int m = m_tile * BN + j;
            const int oc = n_tile * 64 + i;
            if (m < a.M && oc * 2 < a.N) {
              const float g = stage[j * kBM + i];
              const float u = stage[j * kBM + 64 + i];
              reinterpret_cast<__half*>(a.out)[(size_t)m * a.ldo + oc] = __float2half_rn(silu(g) * u);
            }
          }
        } else {
          const int D = a.head_dim, halfD = D >> 1;
          for (int idx = t; idx < BN * kBM; idx += kEpiThreads) {
            const int j = idx >> 7, rr = idx & (kBM - 1);
            const int m = m_tile * BN + j;
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
              if (d < halfD) y = srow[rr] * c - srow[rr + halfD] * s;
              else y = srow[rr - halfD] * s + srow[rr] * c;
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
      }
    }
  done:;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ====================================================================================================== host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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
  CUresult r = encode_fn()(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
}

int gemm_pick_bn(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

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

GemmPlan gemm_plan(int M, int N, int K, int force_splits) {
  GemmPlan p{};
  p.bn = gemm_pick_bn(M);
  p.n_tiles = (N + kBM - 1) / kBM;
  p.m_tiles = (M + p.bn - 1) / p.bn;
  p.k_tiles = K / kBK;
  const int tiles = p.n_tiles * p.m_tiles;
  int splits = 1;
  if (force_splits > 0) {
    splits = force_splits;
  } else {
    // Up to two 1-CTA-per-SM residents fit per SM for BN <= 64 (<= ~110 KB smem); fill those slots, keep at
    // least 4 K stages per split.
    const int slots = gemm_sm_count() * (p.bn <= 64 ? 2 : 1);
    if (tiles < slots) splits = std::max(1, std::min(slots / tiles, p.k_tiles / 4));
  }
  splits = std::max(1, std::min(splits, p.k_tiles));
  p.tiles_per_split = (p.k_tiles + splits - 1) / splits;
  p.splits = (p.k_tiles + p.tiles_per_split - 1) / p.tiles_per_split;
  p.ws_floats = p.splits > 1 ? (size_t)tiles * p.splits * p.bn * kBM : 0;
  p.counters = p.splits > 1 ? tiles : 0;
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
  dim3 grid(p.n_tiles, p.m_tiles, p.splits);
  w8a16_gemm_kernel<BN, EPI><<<grid, kThreads, S::kAlloc, stream>>>(tw, tx, a);
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
  CUtensorMap tw, tx;
  make_tmap_2d(&tw, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.N, a.K, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_64B);
  make_tmap_2d(&tx, x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.K, a.M, ldx, kBK, p.bn, CU_TENSOR_MAP_SWIZZLE_128B);
  a.k_tiles = p.k_tiles;
  a.tiles_per_split = p.tiles_per_split;
  a.splits = p.splits;
  switch (epi) {
    case EPI_F16: launch_epi<EPI_F16>(tw, tx, a, p, stream); break;
    case EPI_F32: launch_epi<EPI_F32>(tw, tx, a, p, stream); break;
    case EPI_RESID: launch_epi<EPI_RESID>(tw, tx, a, p, stream); break;
    case EPI_SWIGLU: launch_epi<EPI_SWIGLU>(tw, tx, a, p, stream); break;
    case EPI_QKV: launch_epi<EPI_QKV>(tw, tx, a, p, stream); break;
    default: throw std::runtime_error("w8a16 gemm: bad epilogue");
  }
}

}  // namespace hrm
