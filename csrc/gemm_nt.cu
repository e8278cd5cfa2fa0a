// Dense "NT" GEMM on the 5th-generation tensor cores for the experiments plane (training and chat of the reversible
// LM):  C[m, n] = sum_k A[m, k] * B[n, k]   (A [M, K] and B [N, K] row-major, bf16 or f16; C [M, N] fp32).
//
// Counterpart of the reference trainer's WMMA GEMM (`wmma_gemm`, llm_engine.cu:471-524: f16 operands, fp32
// accumulate, C = A . Btr^T), which its forward, input-gradient and weight-gradient products all go through after
// transposing operands into the "both K-major" form.  Here one CTA computes a 128 x 128 output tile: a TMA producer
// thread streams 128 x 64 tiles of A and B (128-byte swizzle, the canonical K-major layout) through a 3-stage ring,
// one thread issues tcgen05.mma (M = 128, N = 128, K = 16 per instruction) into a TMEM accumulator and releases ring
// slots with tcgen05.commit, and four epilogue warps read the accumulator back (thread = row = TMEM lane) and store
// fp32 rows.  Rows, columns and k beyond the matrix come in as zeros from the TMA fill and are not stored, so no
// dimension needs padding.  Every wait is bounded (2 s): a timeout records an error code in the status word, drains
// the issued copies and frees TMEM.
#include "common.cuh"
#include "gemm_w8a16.h"
#include "kernels.h"

#include <stdexcept>
#include <string>

namespace hrm {
namespace {

constexpr int kNtBM = 128, kNtBN = 128, kNtBK = 64, kNtStages = 3;
constexpr int kNtThreads = 6 * 32;                // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kNtTile = kNtBM * kNtBK * 2;        // 16 KB per operand tile (BN == BM)
struct NtSmem {
  static constexpr int kA = 0;
  static constexpr int kB = kA + kNtStages * kNtTile;
  static constexpr int kBar = kB + kNtStages * kNtTile;      // full[S], empty[S], acc
  static constexpr int kBytes = kBar + (2 * kNtStages + 1) * 8 + 16;
  static constexpr int kAlloc = kBytes + 1024;                // 1024-byte alignment of the swizzled tiles
};
static_assert(2 * NtSmem::kAlloc <= 227 * 1024, "two CTAs per SM");

}  // namespace

template <bool BF16>
__global__ void __launch_bounds__(kNtThreads, 2)
gemm_nt_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, float* __restrict__ C,
               int M, int N, int K, int ldc, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = base + NtSmem::kA;
  uint8_t* sb = base + NtSmem::kB;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + NtSmem::kBar);
  uint64_t* empty = full + kNtStages;
  uint64_t* acc = empty + kNtStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kNtBM, n0 = blockIdx.x * kNtBN;
  const int kt_n = (K + kNtBK - 1) / kNtBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNtStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kNtBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&ta);
      tma_prefetch_desc(&tb);
      int issued = 0;
      for (int kt = 0; kt < kt_n; ++kt) {
        const int s = kt % kNtStages;
        const uint32_t ph = ((uint32_t)(kt / kNtStages) & 1u) ^ 1u;   // slots start free
        if (!mbar_wait_ab(&empty[s], ph, status, kErrTimeoutEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], 2u * kNtTile);
        tma_load_2d(sa + s * kNtTile, &ta, &full[s], kt * kNtBK, m0);
        tma_load_2d(sb + s * kNtTile, &tb, &full[s], kt * kNtBK, n0);
        ++issued;
      }
      // drain: every issued copy has landed before the CTA can exit (consumed ones have, hence the bounded wait)
      for (int j = issued > kNtStages ? issued - kNtStages : 0; j < issued; ++j)
        mbar_wait(&full[j % kNtStages], (uint32_t)(j / kNtStages) & 1u, status, kErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = BF16 ? idesc_bf16_f32(kNtBM, kNtBN) : idesc_f16_f32(kNtBM, kNtBN);
      for (int kt = 0; kt < kt_n; ++kt) {
        const int s = kt % kNtStages;
        if (!mbar_wait_ab(&full[s], (uint32_t)(kt / kNtStages) & 1u, status, kErrTimeoutFull, abort_flag)) break;
        tc_fence_after();
        const uint64_t ad = sdesc_sw128(smem_u32(sa + s * kNtTile));
        const uint64_t bd = sdesc_sw128(smem_u32(sb + s * kNtTile));
#pragma unroll
        for (int kk = 0; kk < kNtBK / 16; ++kk)   // K = 16 per instruction: 32 bytes along the 128-byte row
          umma_f16_ss(tmem, ad + (uint64_t)((kk * 32) >> 4), bd + (uint64_t)((kk * 32) >> 4), idesc,
                      (kt > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);   // the slot is free once these MMAs have read it
      }
      umma_commit(acc);           // accumulator complete (also after an abort: arrives when issued MMAs finish)
    }
  } else {
    // ---------------------------------------------------------------- epilogue: thread = row = TMEM lane
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int m = m0 + row;
    const bool ok = mbar_wait_ab(acc, 0u, status, kErrTimeoutAccum, abort_flag);
    tc_fence_after();
    for (int c0 = 0; c0 < kNtBN; c0 += 16) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);   // warp-collective: every lane runs it
      if (!ok || m >= M) continue;
      float* crow = C + (size_t)m * ldc + n0 + c0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (n0 + c0 + 4 * q < N)   // N is a multiple of 4
          *reinterpret_cast<float4*>(crow + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kNtBN);
  }
}

void gemm_nt_launch(const void* A, int lda, const void* B, int ldb, float* C, int ldc, int M, int N, int K,
                    bool bf16, int* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return;
  if (N % 4 != 0 || ldc % 4 != 0) throw std::runtime_error("gemm_nt: N and ldc must be multiples of 4");
  if (lda % 8 != 0 || ldb % 8 != 0) throw std::runtime_error("gemm_nt: lda / ldb must be multiples of 8 elements");
  if ((reinterpret_cast<uintptr_t>(C) & 15) != 0) throw std::runtime_error("gemm_nt: C must be 16-byte aligned");
  const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  make_tmap_2d(&ta, A, dt, 2, (uint64_t)K, (uint64_t)M, (uint64_t)lda, kNtBK, kNtBM, CU_TENSOR_MAP_SWIZZLE_128B);
  make_tmap_2d(&tb, B, dt, 2, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, kNtBK, kNtBN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (status == nullptr) status = status_word();
  const dim3 grid((N + kNtBN - 1) / kNtBN, (M + kNtBM - 1) / kNtBM);
  if (grid.y > 65535u) throw std::runtime_error("gemm_nt: M too large");
  if (bf16) {
    ensure_smem_limit<gemm_nt_kernel<true>>(NtSmem::kAlloc);
    gemm_nt_kernel<true><<<grid, kNtThreads, NtSmem::kAlloc, stream>>>(ta, tb, C, M, N, K, ldc, status);
  } else {
    ensure_smem_limit<gemm_nt_kernel<false>>(NtSmem::kAlloc);
    gemm_nt_kernel<false><<<grid, kNtThreads, NtSmem::kAlloc, stream>>>(ta, tb, C, M, N, K, ldc, status);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("gemm_nt launch failed: ") + cudaGetErrorString(e));
}

}  // namespace hrm
