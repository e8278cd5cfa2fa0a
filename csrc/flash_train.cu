// Causal flash attention forward and backward for the experiments plane's reversible LM (head dim 16 or 32, fp32).
//
// Counterpart of the reference trainer's kernels `flash_fwd_hf` / `flash_bwd_dq_hf` / `flash_bwd_dkv_hf`
// (llm_engine.cu:856-1146): tiled causal attention that never materialises the T x T probability matrix, keeps the
// per-row log-sum-exp from the forward, and splits the backward into a dQ pass (one CTA per query tile) and a dK/dV
// pass (one CTA per key tile) so that no gradient needs an atomic and the result is deterministic.
//
// Design.  With a head dimension of 16 a score costs 16 multiply-adds for Q.K and 16 for P.V, and a 128 x 128 x 16
// tensor-core tile is a single instruction whose scores must then pass through registers for the softmax anyway; the
// work per score is dominated by the softmax and the shared-memory traffic, not by the products.  So these kernels run
// on the CUDA cores in fp32: a thread owns one query row (forward, dQ) or one key row (dK/dV) in registers, the other
// operand streams through shared memory in 64-row tiles and is read as same-address broadcasts, and the scores of a
// tile stay in registers (online softmax, one rescale per tile).  Scores are kept in base-2 units
// (s2 = q.k * scale * log2(e)) so every exponential is one exp2f; `lse` holds m2 + log2(l) per row.
//
// Layout: q, k, v, o and their gradients are [B, T, H, D] (row stride H * D); lse is [B, H, T].  No padding is
// needed: rows beyond T load as zeros and are not stored.
#include "kernels.h"

#include <cmath>
#include <stdexcept>
#include <string>

namespace hrm {
namespace {

constexpr int kRowsPerCta = 128;   // thread = row
constexpr int kTile = 64;          // rows of the streamed operand per shared-memory tile
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
__device__ __forceinline__ void load_row(float (&r)[D], const float* p, float mul, bool ok) {
#pragma unroll
  for (int c = 0; c < D / 4; ++c) {
    const float4 x = ok ? reinterpret_cast<const float4*>(p)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    r[4 * c] = x.x * mul;
    r[4 * c + 1] = x.y * mul;
    r[4 * c + 2] = x.z * mul;
    r[4 * c + 3] = x.w * mul;
  }
}

template <int D>
__device__ __forceinline__ float dot_smem(const float (&r)[D], const float4* s) {
  float a = 0.f;
#pragma unroll
  for (int c = 0; c < D / 4; ++c) {
    const float4 x = s[c];
    a = fmaf(r[4 * c], x.x, a);
    a = fmaf(r[4 * c + 1], x.y, a);
    a = fmaf(r[4 * c + 2], x.z, a);
    a = fmaf(r[4 * c + 3], x.w, a);
  }
  return a;
}

template <int D>
__device__ __forceinline__ void axpy_smem(float (&acc)[D], float a, const float4* s) {
#pragma unroll
  for (int c = 0; c < D / 4; ++c) {
    const float4 x = s[c];
    acc[4 * c] = fmaf(a, x.x, acc[4 * c]);
    acc[4 * c + 1] = fmaf(a, x.y, acc[4 * c + 1]);
    acc[4 * c + 2] = fmaf(a, x.z, acc[4 * c + 2]);
    acc[4 * c + 3] = fmaf(a, x.w, acc[4 * c + 3]);
  }
}

// Stage rows [r0, r0 + kTile) of two [B, T, H, D] tensors (this (b, h)) in shared memory; rows >= T are zeros.
template <int D>
__device__ __forceinline__ void stage_pair(float4 (*sa)[D / 4], float4 (*sb)[D / 4], const float* a, const float* b,
                                           int r0, int T, size_t rs) {
  for (int e = threadIdx.x; e < kTile * (D / 4); e += kRowsPerCta) {
    const int r = e / (D / 4), c = e % (D / 4), t = r0 + r;
    const bool ok = t < T;
    sa[r][c] = ok ? reinterpret_cast<const float4*>(a + (size_t)t * rs)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    sb[r][c] = ok ? reinterpret_cast<const float4*>(b + (size_t)t * rs)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

}  // namespace

// Forward: one CTA = 128 queries of one (b, h); thread = query row.  Heaviest (latest) query tiles launch first.
template <int D>
__global__ void __launch_bounds__(kRowsPerCta)
flash_train_fwd_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                       float* __restrict__ o, float* __restrict__ lse, int T, int H, float scale2) {
  __shared__ float4 sk[kTile][D / 4];
  __shared__ float4 sv[kTile][D / 4];
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kRowsPerCta;
  const int i = q0 + threadIdx.x;
  const size_t rs = (size_t)H * D;
  const size_t base = (size_t)b * T * rs + (size_t)h * D;

  float qr[D], acc[D];
  load_row<D>(qr, q + base + (size_t)i * rs, scale2, i < T);
#pragma unroll
  for (int d = 0; d < D; ++d) acc[d] = 0.f;
  float m = -INFINITY, l = 0.f;

  const int kend = min(T, q0 + kRowsPerCta);
  for (int k0 = 0; k0 < kend; k0 += kTile) {
    __syncthreads();
    stage_pair<D>(sk, sv, k + base, v + base, k0, T, rs);
    __syncthreads();
    float s[kTile];
    float tmax = -INFINITY;
#pragma unroll
    for (int r = 0; r < kTile; ++r) {
      const float x = dot_smem<D>(qr, sk[r]);
      const int j = k0 + r;
      s[r] = (j <= i && j < T) ? x : -INFINITY;
      tmax = fmaxf(tmax, s[r]);
    }
    const float mnew = fmaxf(m, tmax);
    if (mnew != -INFINITY) {   // else: no key of this tile is visible to this row (and none before it)
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - mnew);
      l *= alpha;
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] *= alpha;
#pragma unroll
      for (int r = 0; r < kTile; ++r) {
        const float p = exp2f(s[r] - mnew);   // masked scores: exp2(-inf) = 0
        l += p;
        axpy_smem<D>(acc, p, sv[r]);
      }
      m = mnew;
    }
  }
  if (i < T) {
    const float inv = 1.f / l;
    float4* orow = reinterpret_cast<float4*>(o + base + (size_t)i * rs);
#pragma unroll
    for (int c = 0; c < D / 4; ++c)
      orow[c] = make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv, acc[4 * c + 3] * inv);
    lse[((size_t)b * H + h) * T + i] = m + log2f(l);
  }
}

// dQ: one CTA = 128 queries; thread = query row.  dQ_i = scale * sum_j P_ij (dO_i . v_j - D_i) k_j with
// D_i = dO_i . O_i computed in the thread.
template <int D>
__global__ void __launch_bounds__(kRowsPerCta)
flash_train_dq_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                      const float* __restrict__ o, const float* __restrict__ lse, const float* __restrict__ dout,
                      float* __restrict__ dq, int T, int H, float scale, float scale2) {
  __shared__ float4 sk[kTile][D / 4];
  __shared__ float4 sv[kTile][D / 4];
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kRowsPerCta;
  const int i = q0 + threadIdx.x;
  const bool live = i < T;
  const size_t rs = (size_t)H * D;
  const size_t base = (size_t)b * T * rs + (size_t)h * D;

  float qr[D], dor[D], acc[D];
  load_row<D>(qr, q + base + (size_t)i * rs, scale2, live);
  load_row<D>(dor, dout + base + (size_t)i * rs, 1.f, live);
  float delta = 0.f;
  {
    float orow[D];
    load_row<D>(orow, o + base + (size_t)i * rs, 1.f, live);
#pragma unroll
    for (int d = 0; d < D; ++d) delta = fmaf(dor[d], orow[d], delta);
  }
  const float lrow = live ? lse[((size_t)b * H + h) * T + i] : INFINITY;
#pragma unroll
  for (int d = 0; d < D; ++d) acc[d] = 0.f;

  const int kend = min(T, q0 + kRowsPerCta);
  for (int k0 = 0; k0 < kend; k0 += kTile) {
    __syncthreads();
    stage_pair<D>(sk, sv, k + base, v + base, k0, T, rs);
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < kTile; ++r) {
      const int j = k0 + r;
      const float s = dot_smem<D>(qr, sk[r]);
      const float p = (j <= i && j < T && live) ? exp2f(s - lrow) : 0.f;
      const float dp = dot_smem<D>(dor, sv[r]);
      axpy_smem<D>(acc, p * (dp - delta), sk[r]);
    }
  }
  if (live) {
    float4* row = reinterpret_cast<float4*>(dq + base + (size_t)i * rs);
#pragma unroll
    for (int c = 0; c < D / 4; ++c)
      row[c] = make_float4(acc[4 * c] * scale, acc[4 * c + 1] * scale, acc[4 * c + 2] * scale, acc[4 * c + 3] * scale);
  }
}

// dK / dV: one CTA = 128 keys; thread = key row.  Query rows i >= j stream through shared memory with their dO,
// log-sum-exp and D_i (computed while staging).  dV_j = sum_i P_ij dO_i, dK_j = scale * sum_i dS_ij q_i.
template <int D>
__global__ void __launch_bounds__(kRowsPerCta)
flash_train_dkv_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                       const float* __restrict__ o, const float* __restrict__ lse, const float* __restrict__ dout,
                       float* __restrict__ dk, float* __restrict__ dv, int T, int H, float scale, float scale2) {
  __shared__ float4 sq[kTile][D / 4];
  __shared__ float4 sdo[kTile][D / 4];
  __shared__ float slse[kTile];
  __shared__ float sdelta[kTile];
  const int b = blockIdx.z, h = blockIdx.y;
  const int k0 = blockIdx.x * kRowsPerCta;
  const int j = k0 + threadIdx.x;
  const bool live = j < T;
  const size_t rs = (size_t)H * D;
  const size_t base = (size_t)b * T * rs + (size_t)h * D;
  const float* lse_bh = lse + ((size_t)b * H + h) * T;

  float kr[D], vr[D], ak[D], av[D];
  load_row<D>(kr, k + base + (size_t)j * rs, scale2, live);
  load_row<D>(vr, v + base + (size_t)j * rs, 1.f, live);
#pragma unroll
  for (int d = 0; d < D; ++d) ak[d] = av[d] = 0.f;

  for (int q0 = k0; q0 < T; q0 += kTile) {   // queries before the CTA's first key see none of its keys
    __syncthreads();
    stage_pair<D>(sq, sdo, q + base, dout + base, q0, T, rs);
    if (threadIdx.x < kTile) {
      const int t = q0 + threadIdx.x;
      float dl = 0.f;
      if (t < T) {
        const float4* orow = reinterpret_cast<const float4*>(o + base + (size_t)t * rs);
        const float4* grow = reinterpret_cast<const float4*>(dout + base + (size_t)t * rs);
#pragma unroll
        for (int c = 0; c < D / 4; ++c) {
          const float4 x = orow[c], y = grow[c];
          dl = fmaf(x.x, y.x, fmaf(x.y, y.y, fmaf(x.z, y.z, fmaf(x.w, y.w, dl))));
        }
      }
      sdelta[threadIdx.x] = dl;
      slse[threadIdx.x] = t < T ? lse_bh[t] : INFINITY;   // p = exp2(s - inf) = 0 for rows past the end
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < kTile; ++r) {
      const int i = q0 + r;
      const float s = dot_smem<D>(kr, sq[r]);
      const float p = (i >= j && live) ? exp2f(s - slse[r]) : 0.f;
      const float dp = dot_smem<D>(vr, sdo[r]);
      axpy_smem<D>(av, p, sdo[r]);
      axpy_smem<D>(ak, p * (dp - sdelta[r]), sq[r]);
    }
  }
  if (live) {
    float4* krow = reinterpret_cast<float4*>(dk + base + (size_t)j * rs);
    float4* vrow = reinterpret_cast<float4*>(dv + base + (size_t)j * rs);
#pragma unroll
    for (int c = 0; c < D / 4; ++c) {
      krow[c] = make_float4(ak[4 * c] * scale, ak[4 * c + 1] * scale, ak[4 * c + 2] * scale, ak[4 * c + 3] * scale);
      vrow[c] = make_float4(av[4 * c], av[4 * c + 1], av[4 * c + 2], av[4 * c + 3]);
    }
  }
}

// ------------------------------------------------------------------------------------------------ two rows per thread
// The same three kernels with every thread owning two rows (64 threads per 128-row tile): each shared-memory read of
// the streamed operand feeds both rows, which halves the shared loads per multiply-add of the one-row kernels (those
// are issue-bound: the loads and the per-pair mask took about as many issue slots as the FMAs), and tiles that lie
// wholly below the causal diagonal run without per-pair masks.
namespace {
constexpr int kRpt = 2;
constexpr int kThreads2 = kRowsPerCta / kRpt;

template <int D, int NT, int ROWS>
__device__ __forceinline__ void stage_rows(float4 (*sa)[D / 4], float4 (*sb)[D / 4], const float* a, const float* b,
                                           int r0, int T, size_t rs) {
  for (int e = threadIdx.x; e < ROWS * (D / 4); e += NT) {
    const int r = e / (D / 4), c = e % (D / 4), t = r0 + r;
    const bool ok = t < T;
    sa[r][c] = ok ? reinterpret_cast<const float4*>(a + (size_t)t * rs)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    sb[r][c] = ok ? reinterpret_cast<const float4*>(b + (size_t)t * rs)[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

template <int D>
__device__ __forceinline__ void load_vec(float4 (&r)[D / 4], const float4* s) {
#pragma unroll
  for (int c = 0; c < D / 4; ++c) r[c] = s[c];
}

template <int D>
__device__ __forceinline__ float dot_reg(const float (&a)[D], const float4 (&b)[D / 4]) {
  float x = 0.f;
#pragma unroll
  for (int c = 0; c < D / 4; ++c) {
    x = fmaf(a[4 * c], b[c].x, x);
    x = fmaf(a[4 * c + 1], b[c].y, x);
    x = fmaf(a[4 * c + 2], b[c].z, x);
    x = fmaf(a[4 * c + 3], b[c].w, x);
  }
  return x;
}

template <int D>
__device__ __forceinline__ void axpy_reg(float (&acc)[D], float a, const float4 (&b)[D / 4]) {
#pragma unroll
  for (int c = 0; c < D / 4; ++c) {
    acc[4 * c] = fmaf(a, b[c].x, acc[4 * c]);
    acc[4 * c + 1] = fmaf(a, b[c].y, acc[4 * c + 1]);
    acc[4 * c + 2] = fmaf(a, b[c].z, acc[4 * c + 2]);
    acc[4 * c + 3] = fmaf(a, b[c].w, acc[4 * c + 3]);
  }
}

constexpr int kFwdTile2 = 32;   // keys per forward tile (the scores of both rows stay in registers)

// One key tile of the two-row forward: scores, one rescale per row, P.V.  MASK: the tile touches the diagonal.
template <int D, bool MASK>
__device__ __forceinline__ void fwd2_tile(const float4 (*sk)[D / 4], const float4 (*sv)[D / 4], int k0, int T,
                                          const int (&ii)[kRpt], const float (&qr)[kRpt][D], float (&acc)[kRpt][D],
                                          float (&m)[kRpt], float (&l)[kRpt]) {
  float s[kRpt][kFwdTile2];
  float tmax[kRpt];
#pragma unroll
  for (int u = 0; u < kRpt; ++u) tmax[u] = -INFINITY;
#pragma unroll
  for (int r = 0; r < kFwdTile2; ++r) {
    float4 kk[D / 4];
    load_vec<D>(kk, sk[r]);
#pragma unroll
    for (int u = 0; u < kRpt; ++u) {
      float x = dot_reg<D>(qr[u], kk);
      if constexpr (MASK) {
        const int j = k0 + r;
        x = (j <= ii[u] && j < T) ? x : -INFINITY;
      }
      s[u][r] = x;
      tmax[u] = fmaxf(tmax[u], x);
    }
  }
  float mu[kRpt];
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    const float mnew = fmaxf(m[u], tmax[u]);
    const float alpha = (m[u] == -INFINITY) ? 0.f : exp2f(m[u] - mnew);
    l[u] *= alpha;
#pragma unroll
    for (int d = 0; d < D; ++d) acc[u][d] *= alpha;
    m[u] = mnew;
    mu[u] = mnew == -INFINITY ? 0.f : mnew;   // a row with no visible key yet keeps p = exp2(-inf) = 0
  }
#pragma unroll
  for (int r = 0; r < kFwdTile2; ++r) {
    float4 vv[D / 4];
    load_vec<D>(vv, sv[r]);
#pragma unroll
    for (int u = 0; u < kRpt; ++u) {
      const float p = exp2f(s[u][r] - mu[u]);
      l[u] += p;
      axpy_reg<D>(acc[u], p, vv);
    }
  }
}

}  // namespace

template <int D>
__global__ void __launch_bounds__(kThreads2)
flash_train_fwd2_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                        float* __restrict__ o, float* __restrict__ lse, int T, int H, float scale2) {
  __shared__ float4 sk[kFwdTile2][D / 4];
  __shared__ float4 sv[kFwdTile2][D / 4];
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kRowsPerCta;
  const size_t rs = (size_t)H * D;
  const size_t base = (size_t)b * T * rs + (size_t)h * D;
  int ii[kRpt];
  float qr[kRpt][D], acc[kRpt][D], m[kRpt], l[kRpt];
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    ii[u] = q0 + threadIdx.x + u * kThreads2;
    load_row<D>(qr[u], q + base + (size_t)ii[u] * rs, scale2, ii[u] < T);
#pragma unroll
    for (int d = 0; d < D; ++d) acc[u][d] = 0.f;
    m[u] = -INFINITY;
    l[u] = 0.f;
  }
  const int kend = min(T, q0 + kRowsPerCta);
  for (int k0 = 0; k0 < kend; k0 += kFwdTile2) {
    __syncthreads();
    stage_rows<D, kThreads2, kFwdTile2>(sk, sv, k + base, v + base, k0, T, rs);
    __syncthreads();
    if (k0 + kFwdTile2 <= q0)   // every key of the tile precedes every row of the CTA (and is < T)
      fwd2_tile<D, false>(sk, sv, k0, T, ii, qr, acc, m, l);
    else
      fwd2_tile<D, true>(sk, sv, k0, T, ii, qr, acc, m, l);
  }
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    if (ii[u] >= T) continue;
    const float inv = 1.f / l[u];
    float4* orow = reinterpret_cast<float4*>(o + base + (size_t)ii[u] * rs);
#pragma unroll
    for (int c = 0; c < D / 4; ++c)
      orow[c] = make_float4(acc[u][4 * c] * inv, acc[u][4 * c + 1] * inv, acc[u][4 * c + 2] * inv,
                            acc[u][4 * c + 3] * inv);
    lse[((size_t)b * H + h) * T + ii[u]] = m[u] + log2f(l[u]);
  }
}

namespace {

// One key tile of the two-row dQ pass.
template <int D, bool MASK>
__device__ __forceinline__ void dq2_tile(const float4 (*sk)[D / 4], const float4 (*sv)[D / 4], int k0, int T,
                                         const int (&ii)[kRpt], const float (&qr)[kRpt][D],
                                         const float (&dor)[kRpt][D], const float (&delta)[kRpt],
                                         const float (&lrow)[kRpt], float (&acc)[kRpt][D]) {
#pragma unroll 4
  for (int r = 0; r < kTile; ++r) {
    float4 kk[D / 4], vv[D / 4];
    load_vec<D>(kk, sk[r]);
    load_vec<D>(vv, sv[r]);
#pragma unroll
    for (int u = 0; u < kRpt; ++u) {
      float p = exp2f(dot_reg<D>(qr[u], kk) - lrow[u]);   // rows past T: lrow = +inf, p = 0
      if constexpr (MASK) {
        const int j = k0 + r;
        p = (j <= ii[u] && j < T) ? p : 0.f;
      }
      const float dp = dot_reg<D>(dor[u], vv);
      axpy_reg<D>(acc[u], p * (dp - delta[u]), kk);
    }
  }
}

// One query tile of the two-row dK / dV pass.
template <int D, bool MASK>
__device__ __forceinline__ void dkv2_tile(const float4 (*sq)[D / 4], const float4 (*sdo)[D / 4], const float* slse,
                                          const float* sdelta, int q0, const int (&jj)[kRpt],
                                          const float (&kr)[kRpt][D], const float (&vr)[kRpt][D],
                                          float (&ak)[kRpt][D], float (&av)[kRpt][D]) {
#pragma unroll 4
  for (int r = 0; r < kTile; ++r) {
    float4 qq[D / 4], dd[D / 4];
    load_vec<D>(qq, sq[r]);
    load_vec<D>(dd, sdo[r]);
    const float lr = slse[r], dl = sdelta[r];
#pragma unroll
    for (int u = 0; u < kRpt; ++u) {
      float p = exp2f(dot_reg<D>(kr[u], qq) - lr);   // query rows past T: lse = +inf, p = 0
      if constexpr (MASK) p = (q0 + r >= jj[u]) ? p : 0.f;
      const float dp = dot_reg<D>(vr[u], dd);
      axpy_reg<D>(av[u], p, dd);
      axpy_reg<D>(ak[u], p * (dp - dl), qq);
    }
  }
}

}  // namespace

template <int D>
__global__ void __launch_bounds__(kThreads2)
flash_train_dq2_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                       const float* __restrict__ o, const float* __restrict__ lse, const float* __restrict__ dout,
                       float* __restrict__ dq, int T, int H, float scale, float scale2) {
  __shared__ float4 sk[kTile][D / 4];
  __shared__ float4 sv[kTile][D / 4];
  const int b = blockIdx.z, h = blockIdx.y;
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kRowsPerCta;
  const size_t rs = (size_t)H * D;
  const size_t base = (size_t)b * T * rs + (size_t)h * D;
  int ii[kRpt];
  float qr[kRpt][D], dor[kRpt][D], acc[kRpt][D], delta[kRpt], lrow[kRpt];
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    ii[u] = q0 + threadIdx.x + u * kThreads2;
    const bool live = ii[u] < T;
    load_row<D>(qr[u], q + base + (size_t)ii[u] * rs, scale2, live);
    load_row<D>(dor[u], dout + base + (size_t)ii[u] * rs, 1.f, live);
    float orow[D];
    load_row<D>(orow, o + base + (size_t)ii[u] * rs, 1.f, live);
    delta[u] = 0.f;
#pragma unroll
    for (int d = 0; d < D; ++d) delta[u] = fmaf(dor[u][d], orow[d], delta[u]);
    lrow[u] = live ? lse[((size_t)b * H + h) * T + ii[u]] : INFINITY;
#pragma unroll
    for (int d = 0; d < D; ++d) acc[u][d] = 0.f;
  }
  const int kend = min(T, q0 + kRowsPerCta);
  for (int k0 = 0; k0 < kend; k0 += kTile) {
    __syncthreads();
    stage_rows<D, kThreads2, kTile>(sk, sv, k + base, v + base, k0, T, rs);
    __syncthreads();
    if (k0 + kTile <= q0)
      dq2_tile<D, false>(sk, sv, k0, T, ii, qr, dor, delta, lrow, acc);
    else
      dq2_tile<D, true>(sk, sv, k0, T, ii, qr, dor, delta, lrow, acc);
  }
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    if (ii[u] >= T) continue;
    float4* row = reinterpret_cast<float4*>(dq + base + (size_t)ii[u] * rs);
#pragma unroll
    for (int c = 0; c < D / 4; ++c)
      row[c] = make_float4(acc[u][4 * c] * scale, acc[u][4 * c + 1] * scale, acc[u][4 * c + 2] * scale,
                           acc[u][4 * c + 3] * scale);
  }
}

template <int D>
__global__ void __launch_bounds__(kThreads2)
flash_train_dkv2_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                        const float* __restrict__ o, const float* __restrict__ lse, const float* __restrict__ dout,
                        float* __restrict__ dk, float* __restrict__ dv, int T, int H, float scale, float scale2) {
  static_assert(kThreads2 == kTile, "one staging thread per query row of a tile");
  __shared__ float4 sq[kTile][D / 4];
  __shared__ float4 sdo[kTile][D / 4];
  __shared__ float slse[kTile];
  __shared__ float sdelta[kTile];
  const int b = blockIdx.z, h = blockIdx.y;
  const int k0 = blockIdx.x * kRowsPerCta;
  const size_t rs = (size_t)H * D;
  const size_t base = (size_t)b * T * rs + (size_t)h * D;
  const float* lse_bh = lse + ((size_t)b * H + h) * T;
  int jj[kRpt];
  float kr[kRpt][D], vr[kRpt][D], ak[kRpt][D], av[kRpt][D];
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    jj[u] = k0 + threadIdx.x + u * kThreads2;
    load_row<D>(kr[u], k + base + (size_t)jj[u] * rs, scale2, jj[u] < T);
    load_row<D>(vr[u], v + base + (size_t)jj[u] * rs, 1.f, jj[u] < T);
#pragma unroll
    for (int d = 0; d < D; ++d) ak[u][d] = av[u][d] = 0.f;
  }
  for (int q0 = k0; q0 < T; q0 += kTile) {
    __syncthreads();
    stage_rows<D, kThreads2, kTile>(sq, sdo, q + base, dout + base, q0, T, rs);
    {
      const int t = q0 + threadIdx.x;
      float dl = 0.f;
      if (t < T) {
        const float4* orow = reinterpret_cast<const float4*>(o + base + (size_t)t * rs);
        const float4* grow = reinterpret_cast<const float4*>(dout + base + (size_t)t * rs);
#pragma unroll
        for (int c = 0; c < D / 4; ++c) {
          const float4 x = orow[c], y = grow[c];
          dl = fmaf(x.x, y.x, fmaf(x.y, y.y, fmaf(x.z, y.z, fmaf(x.w, y.w, dl))));
        }
      }
      sdelta[threadIdx.x] = dl;
      slse[threadIdx.x] = t < T ? lse_bh[t] : INFINITY;
    }
    __syncthreads();
    if (q0 >= k0 + kRowsPerCta)   // every query row of the tile follows every key of the CTA
      dkv2_tile<D, false>(sq, sdo, slse, sdelta, q0, jj, kr, vr, ak, av);
    else
      dkv2_tile<D, true>(sq, sdo, slse, sdelta, q0, jj, kr, vr, ak, av);
  }
#pragma unroll
  for (int u = 0; u < kRpt; ++u) {
    if (jj[u] >= T) continue;
    float4* krow = reinterpret_cast<float4*>(dk + base + (size_t)jj[u] * rs);
    float4* vrow = reinterpret_cast<float4*>(dv + base + (size_t)jj[u] * rs);
#pragma unroll
    for (int c = 0; c < D / 4; ++c) {
      krow[c] = make_float4(ak[u][4 * c] * scale, ak[u][4 * c + 1] * scale, ak[u][4 * c + 2] * scale,
                            ak[u][4 * c + 3] * scale);
      vrow[c] = make_float4(av[u][4 * c], av[u][4 * c + 1], av[u][4 * c + 2], av[u][4 * c + 3]);
    }
  }
}

namespace {

void check_flash_args(int B, int T, int H, int D) {
  if (D != 16 && D != 32) throw std::runtime_error("flash_train: head dim must be 16 or 32");
  if (B <= 0 || T <= 0 || H <= 0 || H > 65535 || B > 65535)
    throw std::runtime_error("flash_train: bad shape");
}

void check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + " launch failed: " + cudaGetErrorString(e));
}

}  // namespace

void flash_train_fwd_launch(const float* q, const float* k, const float* v, float* o, float* lse, int B, int T, int H,
                            int D, int rpt, cudaStream_t s) {
  check_flash_args(B, T, H, D);
  const float scale2 = (float)(kLog2e / std::sqrt((double)D));
  const dim3 grid((T + kRowsPerCta - 1) / kRowsPerCta, H, B);
  if (D == 16 && rpt == 2)
    flash_train_fwd2_kernel<16><<<grid, kThreads2, 0, s>>>(q, k, v, o, lse, T, H, scale2);
  else if (D == 16)
    flash_train_fwd_kernel<16><<<grid, kRowsPerCta, 0, s>>>(q, k, v, o, lse, T, H, scale2);
  else
    flash_train_fwd_kernel<32><<<grid, kRowsPerCta, 0, s>>>(q, k, v, o, lse, T, H, scale2);
  check_launch("flash_train_fwd");
}

void flash_train_bwd_launch(const float* q, const float* k, const float* v, const float* o, const float* lse,
                            const float* dout, float* dq, float* dk, float* dv, int B, int T, int H, int D, int rpt,
                            cudaStream_t s) {
  check_flash_args(B, T, H, D);
  const float scale = (float)(1.0 / std::sqrt((double)D));
  const float scale2 = scale * kLog2e;
  const dim3 grid((T + kRowsPerCta - 1) / kRowsPerCta, H, B);
  if (D == 16 && rpt == 2) {
    flash_train_dq2_kernel<16><<<grid, kThreads2, 0, s>>>(q, k, v, o, lse, dout, dq, T, H, scale, scale2);
    flash_train_dkv2_kernel<16><<<grid, kThreads2, 0, s>>>(q, k, v, o, lse, dout, dk, dv, T, H, scale, scale2);
  } else if (D == 16) {
    flash_train_dq_kernel<16><<<grid, kRowsPerCta, 0, s>>>(q, k, v, o, lse, dout, dq, T, H, scale, scale2);
    flash_train_dkv_kernel<16><<<grid, kRowsPerCta, 0, s>>>(q, k, v, o, lse, dout, dk, dv, T, H, scale, scale2);
  } else {
    flash_train_dq_kernel<32><<<grid, kRowsPerCta, 0, s>>>(q, k, v, o, lse, dout, dq, T, H, scale, scale2);
    flash_train_dkv_kernel<32><<<grid, kRowsPerCta, 0, s>>>(q, k, v, o, lse, dout, dk, dv, T, H, scale, scale2);
  }
  check_launch("flash_train_bwd");
}

}  // namespace hrm
