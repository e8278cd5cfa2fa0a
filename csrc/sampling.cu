// Top-k support for sampled decoding: the k-th largest value of every row, and each row's top-k candidate values.
//
// The reference engine decodes greedily only (its distributed pick is an argmax, engine/llama_tp.py:317-335).  This
// library adds temperature / top-k sampling on the same path: the argmax kernel turns every kept logit into
// v / T + Gumbel(seed, position, token id) and keeps its max (Gumbel-max: the argmax of the perturbed values is a
// sample of softmax(v / T) over the kept tokens), and "kept" means v >= the row's k-th largest logit.  Under tensor
// parallelism a rank sees one vocabulary shard, so the global k-th largest comes from the union of every rank's
// local top-k values: each rank writes its candidates (values above its local threshold, padded with the threshold
// itself up to k), the candidates are gathered, and the same selection runs over the gathered rows.
//
// Selection: one CTA per row, radix select over the order-preserving 32-bit image of the floats, 8 bits per pass
// (4 passes over the row), a 256-bin shared histogram fed through warp-aggregated atomics (lanes with the same bin
// add once), so a row whose values share their top bits does not serialise on one bin.
#include "common.cuh"
#include "kernels.h"

#include <stdexcept>
#include <string>

namespace hrm {
namespace {
constexpr int kSelThreads = 512;
}

// out[row] = k-th largest of x[row, 0:n] (k = kvec[row]); -inf when k <= 0 or k >= n (no restriction).
__global__ void __launch_bounds__(kSelThreads)
kth_largest_kernel(const float* __restrict__ x, int n, int ld, const int* __restrict__ kvec, float* __restrict__ out) {
  __shared__ unsigned int hist[256];
  __shared__ unsigned int s_prefix, s_remaining;
  const int row = blockIdx.x;
  const int k = kvec[row];
  if (k <= 0 || k >= n) {
    if (threadIdx.x == 0) out[row] = -INFINITY;
    return;
  }
  const float* xr = x + (size_t)row * ld;
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0u, mask = 0u;
  uint32_t remaining = (uint32_t)k;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0u;
    __syncthreads();
    // every thread of a warp runs the same number of iterations, so the warp-wide match below is well formed
    for (int base = 0; base < n; base += blockDim.x) {
      const int i = base + threadIdx.x;
      bool take = false;
      uint32_t bin = 0u;
      if (i < n) {
        const uint32_t o = float_order(xr[i]);
        take = (o & mask) == prefix;
        bin = (o >> shift) & 255u;
      }
      const unsigned active = __ballot_sync(0xffffffffu, take);
      if (take) {
        const unsigned peers = __match_any_sync(active, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (unsigned)__popc(peers));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t above = 0u, b = 255u;
      for (;; --b) {   // the bin holding the remaining-th largest of the values under the current prefix
        if (above + hist[b] >= remaining || b == 0u) break;
        above += hist[b];
      }
      s_prefix = prefix | (b << shift);
      s_remaining = remaining - above;
    }
    __syncthreads();
    prefix = s_prefix;
    remaining = s_remaining;
    mask |= 255u << shift;
    __syncthreads();   // hist is cleared by the next pass
  }
  if (threadIdx.x == 0) out[row] = order_to_float(prefix);
}

// cand[row, 0:kmax] = the values of x[row] above thresh[row], then thresh[row] up to k slots, then -inf.  With no
// restriction (thresh = -inf: k >= n) every value is a candidate.  Rows with k <= 0 get -inf throughout.
__global__ void __launch_bounds__(kSelThreads)
topk_candidates_kernel(const float* __restrict__ x, int n, int ld, const float* __restrict__ thresh,
                       const int* __restrict__ kvec, int kmax, float* __restrict__ cand) {
  __shared__ unsigned int count;
  const int row = blockIdx.x;
  const int k = min(kvec[row], kmax);
  float* cr = cand + (size_t)row * kmax;
  if (threadIdx.x == 0) count = 0u;
  __syncthreads();
  if (k > 0) {
    const float t = thresh[row];
    const float* xr = x + (size_t)row * ld;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float v = xr[i];
      if (v > t) {
        const unsigned slot = atomicAdd(&count, 1u);
        if (slot < (unsigned)kmax) cr[slot] = v;
      }
    }
  }
  __syncthreads();
  const int filled = k > 0 ? (int)min(count, (unsigned)kmax) : 0;
  const float t = k > 0 ? thresh[row] : -INFINITY;
  for (int i = filled + threadIdx.x; i < kmax; i += blockDim.x) cr[i] = (i < k && t != -INFINITY) ? t : -INFINITY;
}

void kth_largest_launch(const float* x, int rows, int n, int ld, const int* k, float* out, cudaStream_t s) {
  if (rows <= 0) return;
  if (n <= 0 || ld < n) throw std::runtime_error("kth_largest: bad row length / stride");
  kth_largest_kernel<<<rows, kSelThreads, 0, s>>>(x, n, ld, k, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("kth_largest launch failed: ") + cudaGetErrorString(e));
}

void topk_candidates_launch(const float* x, int rows, int n, int ld, const float* thresh, const int* k, int kmax,
                            float* cand, cudaStream_t s) {
  if (rows <= 0) return;
  if (n <= 0 || ld < n || kmax <= 0) throw std::runtime_error("topk_candidates: bad row length / stride / kmax");
  topk_candidates_kernel<<<rows, kSelThreads, 0, s>>>(x, n, ld, thresh, k, kmax, cand);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("topk_candidates launch failed: ") + cudaGetErrorString(e));
}

}  // namespace hrm
