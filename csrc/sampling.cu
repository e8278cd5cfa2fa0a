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
// Selection: radix select over the order-preserving 32-bit image of the floats in three passes (11 / 11 / 10 bits),
// each pass spread over many CTAs per row so a decode batch of a few rows still uses the whole GPU.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace hrm {
namespace {
constexpr int kSelThreads = 512;
}

// Multi-CTA radix select of the k-th largest value of every row, three digits of 11 / 11 / 10 bits over the
// order-preserving image of the floats.  Per row, a state record { prefix, mask, remaining, pad, hist[2048] } lives
// in global scratch; each pass is a histogram launch (grid: chunks x rows, every CTA counts the elements that match
// the row's prefix in a shared histogram and adds its non-zero bins to the row's) followed by a select launch (one
// CTA per row: finds the bin holding the remaining-th largest, extends the prefix and clears the histogram).
constexpr int kRadixBins = 2048;
constexpr int kRadixState = 4 + kRadixBins;   // u32 words per row
constexpr int kHistThreads = 256;

HRM_DEVINL void radix_digit(int pass, int& shift, uint32_t& digit) {
  shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
  digit = pass == 2 ? 0x3FFu : 0x7FFu;
}

__global__ void __launch_bounds__(kHistThreads)
radix_init_kernel(const int* __restrict__ kvec, int n, uint32_t* __restrict__ state) {
  uint32_t* st = state + (size_t)blockIdx.x * kRadixState;
  const int k = kvec[blockIdx.x];
  for (int i = threadIdx.x; i < kRadixState; i += blockDim.x) st[i] = 0u;
  if (threadIdx.x == 0 && k > 0 && k < n) st[2] = (uint32_t)k;   // remaining; 0 marks "no restriction"
}

__global__ void __launch_bounds__(kHistThreads)
radix_hist_kernel(const float* __restrict__ x, int n, int ld, int chunk, uint32_t* __restrict__ state, int pass) {
  __shared__ uint32_t sh[kRadixBins];
  const int row = blockIdx.y;
  uint32_t* st = state + (size_t)row * kRadixState;
  if (st[2] == 0u) return;   // row without a top-k restriction (uniform over the CTA)
  const uint32_t prefix = st[0], mask = st[1];
  int shift;
  uint32_t digit;
  radix_digit(pass, shift, digit);
  for (int b = threadIdx.x; b < kRadixBins; b += blockDim.x) sh[b] = 0u;
  __syncthreads();
  const float* xr = x + (size_t)row * ld;
  const int i0 = blockIdx.x * chunk, i1 = min(n, i0 + chunk);
  for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const uint32_t o = float_order(xr[i]);
    if ((o & mask) == prefix) atomicAdd(&sh[(o >> shift) & digit], 1u);
  }
  __syncthreads();
  for (int b = threadIdx.x; b <= (int)digit; b += blockDim.x)
    if (sh[b] != 0u) atomicAdd(&st[4 + b], sh[b]);
}

// One warp per row: lane l sums a block of the bins (highest bins first), a warp scan over the block sums finds the
// block that crosses `remaining`, and that lane walks its block.
__global__ void __launch_bounds__(32)
radix_select_kernel(uint32_t* __restrict__ state, int pass, float* __restrict__ out) {
  const int row = blockIdx.x, lane = threadIdx.x;
  uint32_t* st = state + (size_t)row * kRadixState;
  const uint32_t remaining = st[2];
  if (remaining == 0u) {
    if (pass == 2 && lane == 0) out[row] = -INFINITY;
    return;
  }
  int shift;
  uint32_t digit;
  radix_digit(pass, shift, digit);
  const int nb = (int)digit + 1, per = nb / 32;     // 64 or 32 bins per lane
  const int hi = nb - 1 - lane * per;               // lane's block: bins hi, hi - 1, ..., hi - per + 1
  uint32_t sum = 0u;
  for (int j = 0; j < per; ++j) sum += st[4 + hi - j];
  uint32_t incl = sum;                              // inclusive scan from the top bins down
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const uint32_t excl = incl - sum;
  const unsigned hit = __ballot_sync(0xffffffffu, excl < remaining && incl >= remaining);
  const int owner = hit != 0u ? __ffs(hit) - 1 : 31;
  if (lane == owner) {
    uint32_t above = excl;
    int b = hi;
    for (int j = 0; j < per - 1; ++j, --b) {
      const uint32_t c = st[4 + b];
      if (above + c >= remaining) break;
      above += c;
    }
    const uint32_t prefix = st[0] | ((uint32_t)b << shift);
    st[0] = prefix;
    st[1] |= digit << shift;
    st[2] = remaining - above;
    if (pass == 2) out[row] = order_to_float(prefix);
  }
  __syncwarp();
  for (int b = lane; b < kRadixBins; b += 32) st[4 + b] = 0u;
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

int kth_largest_state_words(int rows) { return rows * kRadixState; }

void kth_largest_launch(const float* x, int rows, int n, int ld, const int* k, float* out, uint32_t* state, int sms,
                        cudaStream_t s) {
  if (rows <= 0) return;
  if (n <= 0 || ld < n) throw std::runtime_error("kth_largest: bad row length / stride");
  if (rows > 65535) throw std::runtime_error("kth_largest: more than 65535 rows");
  // about two CTAs per SM over all rows, at least 2048 elements per CTA
  int chunks = std::max(1, std::min((2 * sms + rows - 1) / rows, (n + 2047) / 2048));
  const int chunk = (n + chunks - 1) / chunks;
  chunks = (n + chunk - 1) / chunk;
  radix_init_kernel<<<rows, kHistThreads, 0, s>>>(k, n, state);
  for (int pass = 0; pass < 3; ++pass) {
    radix_hist_kernel<<<dim3(chunks, rows), kHistThreads, 0, s>>>(x, n, ld, chunk, state, pass);
    radix_select_kernel<<<rows, 32, 0, s>>>(state, pass, out);
  }
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
