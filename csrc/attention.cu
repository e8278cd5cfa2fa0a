// Paged attention over block tables (block size 16, layout [num_blocks, Hk, bs, D], bf16), GQA head // group.
//
// Replaces the reference's `attn_decode` (deepseek_native_engine.sh:562-604: one block per head walking every
// position serially, GQA as head % KVH) and the sm_75 paged flash kernels (csrc/flash_attn_sm75.cu:89-425,
// per-sequence contiguous pages).
//
// decode: flash-decode split-K.  One CTA per (split, kv head, sequence) serves all `group` query heads that share
//         the kv head, so each K/V byte is read once per kv head.  Warps walk whole 16-token blocks; partial
//         (max, sum, acc) per split are merged by a second kernel in split order (deterministic).
// prefill: causal flash attention over varlen query chunks whose keys (including the chunk itself) are already
//          in the paged cache; absolute positions give the causal bound.
// argmax: packed 64-bit (order(value), ~index) row maximum; identical tie rule to the distributed exchange.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <stdexcept>

namespace hrm {

constexpr int kMaxGroup = 8;

template <int D>
__global__ void __launch_bounds__(128) decode_attn_kernel(const DecodeAttnArgs a) {
  constexpr int E = D / 32;        // output elements per lane
  constexpr int HALF = D / 2;
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.Hk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ctx = a.context_lens[b];
  const int k0 = split * a.keys_per_split;
  const int k1 = min(ctx, k0 + a.keys_per_split);

  __shared__ float qs[kMaxGroup][D];
  __shared__ float cm[4][kMaxGroup], cl[4][kMaxGroup];
  __shared__ float cacc[4][kMaxGroup][D];

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    qs[g][d] = __bfloat162float(a.q[((size_t)b * a.Hq + hk * G + g) * D + d]) * a.scale;
  }
  __syncthreads();

  float m[kMaxGroup], l[kMaxGroup], acc[kMaxGroup][E];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
  }

  const int key_in_blk = lane & 15, half = lane >> 4;
  const int* btab = a.block_tables + (size_t)b * a.max_blocks;
  const int bs = a.block_size;
  for (int blk_start = (k0 / bs + warp) * bs; blk_start < k1; blk_start += 4 * bs) {
    const int blk = btab[blk_start / bs];
    const size_t base = ((size_t)blk * a.Hk + hk) * bs * D;
    const int kidx = blk_start + key_in_blk;
    const bool valid = kidx >= k0 && kidx < k1 && key_in_blk < bs;
    float s[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) s[g] = 0.f;
    if (key_in_blk < bs) {
      const __nv_bfloat16* kr = a.k_cache + base + (size_t)key_in_blk * D + half * HALF;
#pragma unroll
      for (int c = 0; c < HALF; c += 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(kr + c);
        const __nv_bfloat162* kp = reinterpret_cast<const __nv_bfloat162*>(&raw);
        float kv[8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 f = __bfloat1622float2(kp[u]);
          kv[2 * u] = f.x;
          kv[2 * u + 1] = f.y;
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
          if (g < G) {
#pragma unroll
            for (int u = 0; u < 8; ++u) s[g] += kv[u] * qs[g][half * HALF + c + u];
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g >= G) break;
      float sc = s[g] + __shfl_xor_sync(0xffffffffu, s[g], 16);
      sc = valid ? sc : -INFINITY;
      const float mx = warp_max(sc);
      const float mn = fmaxf(m[g], mx);
      float p = 0.f, corr = 1.f;
      if (mn != -INFINITY) {
        corr = __expf(m[g] - mn);
        p = valid ? __expf(sc - mn) : 0.f;
      }
      const float ps = warp_sum(half == 0 ? p : 0.f);
      l[g] = l[g] * corr + ps;
      m[g] = mn;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[g][e] *= corr;
      s[g] = p;   // reuse: lane j (< 16) holds p of key j
    }
    // P.V: lane owns output elements [lane*E, lane*E+E)
    for (int j = 0; j < bs && j < 16; ++j) {
      const __nv_bfloat16* vr = a.v_cache + base + (size_t)j * D + lane * E;
      float vv[E];
      if constexpr (E == 4) {
        const uint2 raw = *reinterpret_cast<const uint2*>(vr);
        const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(&raw);
        const float2 f0 = __bfloat1622float2(vp[0]), f1 = __bfloat1622float2(vp[1]);
        vv[0] = f0.x; vv[1] = f0.y; vv[2] = f1.x; vv[3] = f1.y;
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) vv[e] = __bfloat162float(vr[e]);
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g >= G) break;
        const float pj = __shfl_sync(0xffffffffu, s[g], j);
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] += pj * vv[e];
      }
    }
  }

  // merge the 4 warps
  if (lane == 0) {
    for (int g = 0; g < G; ++g) { cm[warp][g] = m[g]; cl[warp][g] = l[g]; }
  }
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= G) break;
#pragma unroll
    for (int e = 0; e < E; ++e) cacc[warp][g][lane * E + e] = acc[g][e];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    const int g = i / D, d = i % D;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, cm[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int w = 0; w < 4; ++w) {
        const float f = __expf(cm[w][g] - M);
        L += cl[w][g] * f;
        A += cacc[w][g][d] * f;
      }
    }
    const int h = hk * G + g;
    if (a.splits == 1) {
      a.out[((size_t)b * a.Hq + h) * D + d] = __float2half_rn(L > 0.f ? A / L : 0.f);
    } else {
      float* p = a.ws + (((size_t)b * a.Hq + h) * a.splits + split) * (D + 2);
      p[2 + d] = A;
      if (d == 0) { p[0] = M; p[1] = L; }
    }
  }
}

template <int D>
__global__ void decode_combine_kernel(const DecodeAttnArgs a) {
  pdl_wait();      // partials come from the attention grid launched just before
  pdl_trigger();
  const int bh = blockIdx.x;
  const int d = threadIdx.x;
  const float* p = a.ws + (size_t)bh * a.splits * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, p[s * (D + 2)]);
  float L = 0.f, A = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < a.splits; ++s) {
      const float ms = p[s * (D + 2)];
      if (ms == -INFINITY) continue;
      const float f = __expf(ms - M);
      L += p[s * (D + 2) + 1] * f;
      A += p[s * (D + 2) + 2 + d] * f;
    }
  }
  a.out[(size_t)bh * D + d] = __float2half_rn(L > 0.f ? A / L : 0.f);
}

void decode_combine_launch(const DecodeAttnArgs& a, cudaStream_t s) {
  if (a.D == 128) launch_maybe_pdl(decode_combine_kernel<128>, dim3(a.B * a.Hq), dim3(128), 0, s, a);
  else launch_maybe_pdl(decode_combine_kernel<64>, dim3(a.B * a.Hq), dim3(64), 0, s, a);
}

size_t decode_attn_ws_floats(int B, int Hq, int D, int splits) { return (size_t)B * Hq * splits * (D + 2); }

void decode_attn_launch(const DecodeAttnArgs& a, cudaStream_t s) {
  if (a.Hq / a.Hk > kMaxGroup) throw std::runtime_error("decode attention: group size > 8 unsupported");
  if (a.block_size > 16 || a.keys_per_split % a.block_size) throw std::runtime_error("decode attention: bad split");
  dim3 grid(a.splits, a.Hk, a.B);
  if (a.D == 128) {
    decode_attn_kernel<128><<<grid, 128, 0, s>>>(a);
    if (a.splits > 1) decode_combine_kernel<128><<<a.B * a.Hq, 128, 0, s>>>(a);
  } else if (a.D == 64) {
    decode_attn_kernel<64><<<grid, 128, 0, s>>>(a);
    if (a.splits > 1) decode_combine_kernel<64><<<a.B * a.Hq, 64, 0, s>>>(a);
  } else {
    throw std::runtime_error("decode attention: head_dim must be 64 or 128");
  }
}

// ------------------------------------------------------------------------------------------------ prefill
constexpr int kPfQ = 64;    // queries per CTA (2 threads per query)
constexpr int kPfK = 32;    // keys per smem tile

template <int D>
__global__ void __launch_bounds__(128) prefill_attn_kernel(const PrefillAttnArgs a) {
  constexpr int HALF = D / 2;
  const int seq = blockIdx.z, h = blockIdx.y;
  const int G = a.Hq / a.Hk;
  const int hk = h / G;
  const int qo = a.cu_q[seq];
  const int qlen = a.cu_q[seq + 1] - qo;
  const int qt0 = blockIdx.x * kPfQ;
  if (qt0 >= qlen) return;
  const int t = threadIdx.x;
  const int qi = qt0 + (t >> 1), half = t & 1;
  const bool qvalid = qi < qlen;
  const int pos = a.q_start[seq] + qi;
  const int ctx = a.context_lens[seq];
  const int kend = min(ctx, a.q_start[seq] + min(qlen, qt0 + kPfQ));

  __shared__ __align__(16) __nv_bfloat16 Ks[kPfK][D];
  __shared__ __align__(16) __nv_bfloat16 Vs[kPfK][D];

  float q[HALF], acc[HALF];
  {
    const __nv_bfloat16* qr = a.q + ((size_t)(qo + (qvalid ? qi : 0)) * a.Hq + h) * D + half * HALF;
#pragma unroll
    for (int i = 0; i < HALF; ++i) {
      q[i] = __bfloat162float(qr[i]) * a.scale;
      acc[i] = 0.f;
    }
  }
  float m = -INFINITY, l = 0.f;
  const int* btab = a.block_tables + (size_t)seq * a.max_blocks;
  for (int kt = 0; kt < kend; kt += kPfK) {
    __syncthreads();
    // cooperative load of kPfK keys (16-byte chunks)
    constexpr int CH = D / 8;
    for (int c = t; c < kPfK * CH; c += 128) {
      const int j = c / CH, cc = c % CH;
      const int key = kt + j;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (key < kend) {
        const int blk = btab[key / a.block_size];
        const size_t off = (((size_t)blk * a.Hk + hk) * a.block_size + key % a.block_size) * D + cc * 8;
        kv = *reinterpret_cast<const uint4*>(a.k_cache + off);
        vv = *reinterpret_cast<const uint4*>(a.v_cache + off);
      }
      *reinterpret_cast<uint4*>(&Ks[j][cc * 8]) = kv;
      *reinterpret_cast<uint4*>(&Vs[j][cc * 8]) = vv;
    }
    __syncthreads();
    float s[kPfK];
    float tmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPfK; ++j) {
      float d0 = 0.f;
      const __nv_bfloat162* kr = reinterpret_cast<const __nv_bfloat162*>(&Ks[j][half * HALF]);
#pragma unroll
      for (int i = 0; i < HALF / 2; ++i) {
        const float2 f = __bfloat1622float2(kr[i]);
        d0 += q[2 * i] * f.x + q[2 * i + 1] * f.y;
      }
      d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
      const int key = kt + j;
      s[j] = (key <= pos && key < kend && qvalid) ? d0 : -INFINITY;
      tmax = fmaxf(tmax, s[j]);
    }
    const float mn = fmaxf(m, tmax);
    if (mn == -INFINITY) continue;
    const float corr = __expf(m - mn);
    l *= corr;
#pragma unroll
    for (int i = 0; i < HALF; ++i) acc[i] *= corr;
#pragma unroll
    for (int j = 0; j < kPfK; ++j) {
      const float p = __expf(s[j] - mn);
      l += p;
      const __nv_bfloat162* vr = reinterpret_cast<const __nv_bfloat162*>(&Vs[j][half * HALF]);
#pragma unroll
      for (int i = 0; i < HALF / 2; ++i) {
        const float2 f = __bfloat1622float2(vr[i]);
        acc[2 * i] += p * f.x;
        acc[2 * i + 1] += p * f.y;
      }
    }
    m = mn;
  }
  if (qvalid) {
    __half* orow = a.out + ((size_t)(qo + qi) * a.Hq + h) * D + half * HALF;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < HALF; i += 2) {
      *reinterpret_cast<__half2*>(orow + i) = __floats2half2_rn(acc[i] * inv, acc[i + 1] * inv);
    }
  }
}

void prefill_attn_launch(const PrefillAttnArgs& a, cudaStream_t s) {
  if (a.S == 0 || a.max_q == 0) return;
  dim3 grid((a.max_q + kPfQ - 1) / kPfQ, a.Hq, a.S);
  if (a.D == 128) prefill_attn_kernel<128><<<grid, 128, 0, s>>>(a);
  else if (a.D == 64) prefill_attn_kernel<64><<<grid, 128, 0, s>>>(a);
  else throw std::runtime_error("prefill attention: head_dim must be 64 or 128");
}

// ------------------------------------------------------------------------------------------------ argmax
// Greedy pick over a row of logits, split over gridDim.x CTAs per row so a decode batch of a few rows still
// streams the [M, V] logits with the whole GPU (one 1024-thread CTA per row took ~60 us for 16 x 128256).  Each CTA
// reduces its slice to one packed key (order-preserving float bits, then ~index: larger value wins, ties go to the
// lower id); slices meet in atomicMax on the row's accumulator, which is order independent, so the result is
// deterministic.  The CTA that takes the last ticket publishes the key / token and re-arms accumulator and ticket
// (both start at zero).
// Tensor-parallel exchange of one row's key (XCHG), run by the row's final CTA, thread 0: see ArgmaxXchg.
HRM_DEVINL unsigned long long argmax_exchange_row(const ArgmaxXchg& x, int row, int M, unsigned long long mine) {
  // this launch's epoch: every row's final thread reads it before taking a row ticket, and the counter only moves
  // once all M rows have taken theirs
  const int ep = *reinterpret_cast<volatile int*>(x.epoch) + 1;
  const size_t slot = ((size_t)(ep & 1) * x.world + x.rank) * x.max_rows + row;
  for (int d = 0; d < x.world; ++d) {
    char* base = reinterpret_cast<char*>(x.peers[d]);
    reinterpret_cast<unsigned long long*>(base + x.off_keys)[slot] = mine;
  }
  fence_acq_rel_sys();   // release pattern: the key stores above are visible before any of the flags below
  for (int d = 0; d < x.world; ++d) {
    char* base = reinterpret_cast<char*>(x.peers[d]);
    st_relaxed_sys(reinterpret_cast<int*>(base + x.off_flags) + ((size_t)x.rank * x.max_rows + row) * 32, ep);
  }
  char* own = reinterpret_cast<char*>(x.peers[x.rank]);
  const int* flags = reinterpret_cast<const int*>(own + x.off_flags);
  const unsigned long long* slots = reinterpret_cast<const unsigned long long*>(own + x.off_keys);
  unsigned long long best = 0ull;
  for (int r = 0; r < x.world; ++r) {   // max is order independent; rank order only fixes the reads
    if (!wait_flag_acquire(flags + ((size_t)r * x.max_rows + row) * 32, ep, x.status)) continue;
    const unsigned long long k = __ldcg(slots + ((size_t)(ep & 1) * x.world + r) * x.max_rows + row);
    best = k > best ? k : best;
  }
  __threadfence();
  if (atomicAdd(x.row_ticket, 1) == M - 1) {   // last row of the launch: re-arm and advance the epoch
    *x.row_ticket = 0;
    *reinterpret_cast<volatile int*>(x.epoch) = ep;
    __threadfence();
  }
  return best;
}

// Key of one logit: the plain argmax key, or (SAMPLE) the key of v / T + Gumbel noise for logits at or above the
// row's top-k threshold (0, i.e. never the maximum, below it); a row with inv_temp == 0 stays greedy.
template <bool SAMPLE>
HRM_DEVINL unsigned long long pick_key(float v, uint32_t id, float it, float th, unsigned long long rk) {
  if constexpr (!SAMPLE) {
    return argmax_key(v, id);
  } else {
    if (it == 0.f) return argmax_key(v, id);
    if (!(v >= th)) return 0ull;
    return argmax_key(fmaf(v, it, gumbel_noise(rk, id)), id);
  }
}

template <bool XCHG, bool SAMPLE>
__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, int V, int ld, int chunk,
                                                     int vocab_start, unsigned long long* acc,
                                                     unsigned long long* ticket, unsigned long long* keys,
                                                     int64_t* tokens, const ArgmaxXchg x, const SampleArgs sp) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.y;
  const float* lr = logits + (size_t)row * ld;
  const int i0 = blockIdx.x * chunk, i1 = min(V, i0 + chunk);
  float it = 0.f, th = -INFINITY;
  unsigned long long rk = 0ull;
  if constexpr (SAMPLE) {
    it = sp.inv_temp[row];
    th = sp.thresh != nullptr ? sp.thresh[row] : -INFINITY;
    rk = sample_row_key(sp.seed[row], sp.pos[row]);
  }
  unsigned long long best = 0ull;
  const bool vec = ((reinterpret_cast<uintptr_t>(lr + i0) & 15) == 0) && (chunk % 4 == 0);
  if (vec) {
    const int n4 = (i1 - i0) >> 2;
    const float4* l4 = reinterpret_cast<const float4*>(lr + i0);
    for (int j = threadIdx.x; j < n4; j += blockDim.x) {
      const float4 v = l4[j];
      const uint32_t id = (uint32_t)(vocab_start + i0 + 4 * j);
      unsigned long long k = pick_key<SAMPLE>(v.x, id, it, th, rk);
      unsigned long long t = pick_key<SAMPLE>(v.y, id + 1, it, th, rk);
      k = t > k ? t : k;
      t = pick_key<SAMPLE>(v.z, id + 2, it, th, rk);
      k = t > k ? t : k;
      t = pick_key<SAMPLE>(v.w, id + 3, it, th, rk);
      k = t > k ? t : k;
      best = k > best ? k : best;
    }
    for (int i = i0 + 4 * n4 + threadIdx.x; i < i1; i += blockDim.x) {
      const unsigned long long k = pick_key<SAMPLE>(lr[i], (uint32_t)(vocab_start + i), it, th, rk);
      best = k > best ? k : best;
    }
  } else {
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
      const unsigned long long k = pick_key<SAMPLE>(lr[i], (uint32_t)(vocab_start + i), it, th, rk);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
  if (gridDim.x > 1) {
    atomicMax(&acc[row], best);
    __threadfence();
    if (atomicAdd(&ticket[row], 1ull) != (unsigned long long)(gridDim.x - 1)) return;
    __threadfence();
    best = atomicExch(&acc[row], 0ull);
    ticket[row] = 0ull;
  }
  if constexpr (XCHG) best = argmax_exchange_row(x, row, (int)gridDim.y, best);
  if (keys) keys[row] = best ^ (1ull << 63);   // signed-int64 order == unsigned key order
  if (tokens) tokens[row] = (int64_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFull));
}

int argmax_chunks(int M, int V, int sms) {
  if (M > kArgmaxMaxRows) return 1;
  int c = (2 * sms + M - 1) / M;
  c = std::min(c, std::max(1, V / 2048));
  return std::max(1, c);
}

void argmax_launch(const float* logits, int M, int V, int ld, int vocab_start, unsigned long long* keys,
                   int64_t* tokens, unsigned long long* scratch, int sms, cudaStream_t s) {
  if (M == 0) return;
  const int c = scratch != nullptr ? argmax_chunks(M, V, sms) : 1;
  int chunk = (V + c - 1) / c;
  chunk = (chunk + 3) & ~3;
  const int grid_x = (V + chunk - 1) / chunk;
  unsigned long long* acc = scratch;
  unsigned long long* ticket = scratch != nullptr ? scratch + kArgmaxMaxRows : nullptr;
  launch_maybe_pdl(argmax_kernel<false, false>, dim3(grid_x, M), dim3(256), 0, s, logits, V, ld, chunk, vocab_start,
                   acc, ticket, keys, tokens, ArgmaxXchg{}, SampleArgs{});
}

void argmax_xchg_launch(const float* logits, int M, int V, int ld, int vocab_start, unsigned long long* keys,
                        int64_t* tokens, unsigned long long* scratch, int sms, const ArgmaxXchg& x, cudaStream_t s) {
  if (M == 0) return;
  if (M > x.max_rows) throw std::runtime_error("argmax exchange: more rows than the symmetric key slots hold");
  if (x.peers == nullptr || x.epoch == nullptr || x.row_ticket == nullptr || x.world < 1 || x.rank < 0 ||
      x.rank >= x.world)
    throw std::runtime_error("argmax exchange: bad peer table / counters");
  const int c = scratch != nullptr ? argmax_chunks(M, V, sms) : 1;
  int chunk = (V + c - 1) / c;
  chunk = (chunk + 3) & ~3;
  const int grid_x = (V + chunk - 1) / chunk;
  unsigned long long* acc = scratch;
  unsigned long long* ticket = scratch != nullptr ? scratch + kArgmaxMaxRows : nullptr;
  launch_maybe_pdl(argmax_kernel<true, false>, dim3(grid_x, M), dim3(256), 0, s, logits, V, ld, chunk, vocab_start,
                   acc, ticket, keys, tokens, x, SampleArgs{});
}

void argmax_sample_launch(const float* logits, int M, int V, int ld, int vocab_start, unsigned long long* keys,
                          int64_t* tokens, unsigned long long* scratch, int sms, const SampleArgs& sp,
                          const ArgmaxXchg* x, cudaStream_t s) {
  if (M == 0) return;
  if (sp.inv_temp == nullptr || sp.seed == nullptr || sp.pos == nullptr)
    throw std::runtime_error("sampled argmax: inv_temp, seed and pos are required");
  if (x != nullptr) {
    if (M > x->max_rows) throw std::runtime_error("argmax exchange: more rows than the symmetric key slots hold");
    if (x->peers == nullptr || x->epoch == nullptr || x->row_ticket == nullptr || x->world < 1 || x->rank < 0 ||
        x->rank >= x->world)
      throw std::runtime_error("argmax exchange: bad peer table / counters");
  }
  const int c = scratch != nullptr ? argmax_chunks(M, V, sms) : 1;
  int chunk = (V + c - 1) / c;
  chunk = (chunk + 3) & ~3;
  const int grid_x = (V + chunk - 1) / chunk;
  unsigned long long* acc = scratch;
  unsigned long long* ticket = scratch != nullptr ? scratch + kArgmaxMaxRows : nullptr;
  if (x != nullptr)
    launch_maybe_pdl(argmax_kernel<true, true>, dim3(grid_x, M), dim3(256), 0, s, logits, V, ld, chunk, vocab_start,
                     acc, ticket, keys, tokens, *x, sp);
  else
    launch_maybe_pdl(argmax_kernel<false, true>, dim3(grid_x, M), dim3(256), 0, s, logits, V, ld, chunk,
                     vocab_start, acc, ticket, keys, tokens, ArgmaxXchg{}, sp);
}

}  // namespace hrm
