// Optimizer kernels of the experiments-plane trainer, over one flat fp32 parameter buffer.
//
// Reference: `reduce_sumsq_1/2` + `adamw` (llm_engine.cu:1188-1221) with the host reading the squared norm back
// (:1486-1493).  Here the global-norm clip factor is computed on the device (deterministic fixed-grid two-pass sum,
// non-finite terms skipped), and AdamW reads the clip factor and the step counter from device memory, so the whole
// optimizer step can sit inside a captured CUDA graph with no host round trip.
#include "kernels.h"

namespace hrm {

constexpr int kSumsqBlocks = 1024;
constexpr int kSumsqThreads = 256;

__global__ void __launch_bounds__(kSumsqThreads) sumsq_partial_kernel(const float* __restrict__ g, long long n,
                                                                     float* __restrict__ partial) {
  __shared__ float red[kSumsqThreads];
  float s = 0.f;
  for (long long i = (long long)blockIdx.x * kSumsqThreads + threadIdx.x; i < n; i += (long long)kSumsqBlocks * kSumsqThreads) {
    const float x = g[i];
    if (isfinite(x)) s += x * x;
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int k = kSumsqThreads / 2; k > 0; k >>= 1) {
    if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

// scalars[0] = global grad norm, scalars[1] = clip factor (1 when the norm is non-finite or within the limit)
__global__ void __launch_bounds__(kSumsqThreads) clip_factor_kernel(const float* __restrict__ partial, float clip,
                                                                   float* __restrict__ scalars) {
  __shared__ float red[kSumsqThreads];
  float s = 0.f;
  for (int i = threadIdx.x; i < kSumsqBlocks; i += kSumsqThreads) s += partial[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int k = kSumsqThreads / 2; k > 0; k >>= 1) {
    if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float norm = sqrtf(red[0]);
    scalars[0] = norm;
    scalars[1] = (!isfinite(norm) || norm <= 0.f || clip <= 0.f || norm <= clip) ? 1.f : clip / norm;
  }
}

// Decoupled AdamW; step[0] is the 1-based step of this update (bias corrections), advanced by the last block.
__global__ void adamw_flat_kernel(float* __restrict__ w, float* __restrict__ m, float* __restrict__ v,
                                  const float* __restrict__ g, long long n, float lr, float wd, float b1, float b2,
                                  float eps, const int* __restrict__ step, const float* __restrict__ scalars) {
  const float t = (float)step[0];
  const float inv_b1t = 1.f / (1.f - powf(b1, t)), inv_b2t = 1.f / (1.f - powf(b2, t));
  const float cs = scalars[1];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float gi = g[i] * cs;
    if (!isfinite(gi)) gi = 0.f;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    w[i] -= lr * ((mi * inv_b1t) / (sqrtf(vi * inv_b2t) + eps) + wd * w[i]);
  }
}

__global__ void step_advance_kernel(int* step) { step[0] += 1; }

void grad_clip_factor_launch(const float* g, long long n, float clip, float* partial, float* scalars, cudaStream_t s) {
  sumsq_partial_kernel<<<kSumsqBlocks, kSumsqThreads, 0, s>>>(g, n, partial);
  clip_factor_kernel<<<1, kSumsqThreads, 0, s>>>(partial, clip, scalars);
}

void adamw_flat_launch(float* w, float* m, float* v, const float* g, long long n, float lr, float wd, float b1,
                       float b2, float eps, int* step, const float* scalars, int sm_count, cudaStream_t s) {
  long long blocks = (n + 255) / 256;
  if (blocks > (long long)sm_count * 16) blocks = (long long)sm_count * 16;
  adamw_flat_kernel<<<(int)blocks, 256, 0, s>>>(w, m, v, g, n, lr, wd, b1, b2, eps, step, scalars);
  step_advance_kernel<<<1, 1, 0, s>>>(step);
}

}  // namespace hrm
