// RMSNorm, residual-add + RMSNorm, int8 embedding lookup, SwiGLU (standalone form).
//
// Reference kernels replaced: `rmsnorm_quant` (deepseek_native_engine.sh:392-443, per-token, <<<1,256>>>),
// `add_inplace` (:666-669), `embed_lookup` (:672-677), `silu_gate_mul` (:607-613) and the torch RMSNorm
// (tp/norm.py:17-20, fp16 math).  Here the statistics and math are fp32; the normalised output is written as f16
// because it only feeds the W8A16 GEMM's f16 operand.
#include "common.cuh"
#include "kernels.h"

namespace hrm {

template <int THREADS>
HRM_DEVINL float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < THREADS / 32) ? red[l] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

// out_h[m] = f16(x[m] * rsqrt(mean(x^2) + eps) * w);  optionally x += delta first (residual add), written back.
template <int THREADS, bool ADD>
__global__ void __launch_bounds__(THREADS) rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                          const float* __restrict__ w, __half* __restrict__ out,
                                                          int H, float eps) {
  __shared__ float red[32];
  const size_t row = blockIdx.x;
  float* xr = x + row * H;
  const float* dr = ADD ? delta + row * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < H; i += THREADS * 4) {
    float4 v = *reinterpret_cast<float4*>(xr + i);
    if (ADD) {
      const float4 d = *reinterpret_cast<const float4*>(dr + i);
      v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
      *reinterpret_cast<float4*>(xr + i) = v;
    }
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  const float tot = block_sum<THREADS>(ss, red);
  const float inv = rsqrtf(tot / (float)H + eps);
  __half* orow = out + row * H;
  for (int i = threadIdx.x * 4; i < H; i += THREADS * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(w + i);
    __half2 a = __floats2half2_rn(v.x * inv * g.x, v.y * inv * g.y);
    __half2 b = __floats2half2_rn(v.z * inv * g.z, v.w * inv * g.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(orow + i) = pk;
  }
}

void rmsnorm_launch(float* x, const float* delta, const float* w, __half* out, int M, int H, float eps,
                    cudaStream_t s) {
  if (M == 0) return;
  if (delta)
    rmsnorm_kernel<256, true><<<M, 256, 0, s>>>(x, delta, w, out, H, eps);
  else
    rmsnorm_kernel<256, false><<<M, 256, 0, s>>>(x, nullptr, w, out, H, eps);
}

// out[m, :] = q[ids[m] - vocab_start, :] * scale[...]  if the id is in this rank's range, else 0.
__global__ void embed_q8_kernel(const int64_t* __restrict__ ids, const int8_t* __restrict__ q,
                                const float* __restrict__ scale, float* __restrict__ out, int H, int vocab_start,
                                int vocab_local) {
  const int m = blockIdx.x;
  const int64_t id = ids[m] - vocab_start;
  float* orow = out + (size_t)m * H;
  const bool in = id >= 0 && id < vocab_local;
  const float sc = in ? scale[id] : 0.f;
  const int8_t* qr = in ? q + (size_t)id * H : nullptr;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (in) {
      const char4 c = *reinterpret_cast<const char4*>(qr + i);
      o = make_float4(c.x * sc, c.y * sc, c.z * sc, c.w * sc);
    }
    *reinterpret_cast<float4*>(orow + i) = o;
  }
}

void embed_q8_launch(const int64_t* ids, const int8_t* q, const float* scale, float* out, int M, int H,
                     int vocab_start, int vocab_local, cudaStream_t s) {
  if (M == 0) return;
  embed_q8_kernel<<<M, 256, 0, s>>>(ids, q, scale, out, H, vocab_start, vocab_local);
}

}  // namespace hrm

namespace hrm {

// Device-side decode bookkeeping so that a captured decode step needs no host input between steps:
//   prepare: slots[b] = table[b][pos/bs]*bs + pos%bs (or -1 if inactive), context_lens[b] = pos + 1
//   advance: ids[b] = tokens[b], positions[b] += 1
__global__ void decode_prepare_kernel(const int* __restrict__ positions, const int* __restrict__ tables, int maxb,
                                      int bs, const int* __restrict__ active, int* __restrict__ slots,
                                      int* __restrict__ context_lens, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int pos = positions[b];
  const bool on = active == nullptr || active[b] != 0;
  const int blk = pos / bs;
  slots[b] = (on && blk < maxb) ? tables[(size_t)b * maxb + blk] * bs + (pos - blk * bs) : -1;
  context_lens[b] = pos + 1;
}

__global__ void decode_advance_kernel(const int64_t* __restrict__ tokens, int64_t* __restrict__ ids,
                                      int* __restrict__ positions, const int* __restrict__ active, int B) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (active == nullptr || active[b] != 0) {
    ids[b] = tokens[b];
    positions[b] += 1;
  }
}

void decode_prepare_launch(const int* positions, const int* tables, int maxb, int bs, const int* active, int* slots,
                           int* context_lens, int B, cudaStream_t s) {
  if (B == 0) return;
  decode_prepare_kernel<<<(B + 127) / 128, 128, 0, s>>>(positions, tables, maxb, bs, active, slots, context_lens, B);
}

void decode_advance_launch(const int64_t* tokens, int64_t* ids, int* positions, const int* active, int B,
                           cudaStream_t s) {
  if (B == 0) return;
  decode_advance_kernel<<<(B + 127) / 128, 128, 0, s>>>(tokens, ids, positions, active, B);
}

}  // namespace hrm

namespace hrm {

// RMSNorm preparation without normalising: optionally x += delta, then
//   xg[m, n] = f16(x[m, n] * gamma[n])          (the next GEMM's operand, gamma folded in)
//   ssq[t * M + m] = sum_{n in [128t, 128t+128)} x[m, n]^2
// The consuming GEMM multiplies token m's outputs by rsqrt(sum_t ssq[t*M+m] / H + eps).  One CTA per row; each
// thread owns 32 consecutive columns, 4 threads per 128-column tile.
__global__ void __launch_bounds__(256) norm_prep_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                        const float* __restrict__ gamma, __half* __restrict__ xg,
                                                        float* __restrict__ ssq, int M, int H) {
  const int m = blockIdx.x;
  float* xr = x + (size_t)m * H;
  // every thread runs the same number of iterations so the 4-lane shuffles below always see full warps
  for (int base = 0; base < H; base += blockDim.x * 32) {
    const int c0 = base + threadIdx.x * 32;
    const bool act = c0 < H;   // H % 128 == 0: the 4 threads of one tile are all active or all idle
    float s = 0.f;
    if (act) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 v = *reinterpret_cast<float4*>(xr + c0 + i);
        if (delta) {
          const float4 d = *reinterpret_cast<const float4*>(delta + (size_t)m * H + c0 + i);
          v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
          *reinterpret_cast<float4*>(xr + c0 + i) = v;
        }
        s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        const float4 g = *reinterpret_cast<const float4*>(gamma + c0 + i);
        __half2 a = __floats2half2_rn(v.x * g.x, v.y * g.y), b = __floats2half2_rn(v.z * g.z, v.w * g.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&a);
        pk.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(xg + (size_t)m * H + c0 + i) = pk;
      }
    }
    // 4 consecutive threads cover one 128-column tile
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (act && (threadIdx.x & 3) == 0) ssq[(size_t)(c0 / 128) * M + m] = s;
  }
}

void norm_prep_launch(float* x, const float* delta, const float* gamma, __half* xg, float* ssq, int M, int H,
                      cudaStream_t s) {
  if (M == 0) return;
  norm_prep_kernel<<<M, 256, 0, s>>>(x, delta, gamma, xg, ssq, M, H);
}

}  // namespace hrm
