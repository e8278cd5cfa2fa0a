// PHO-id record scoring for the PHO index prototype.
//
// Reference: `score_kernel` in experiments/pho_index_cuda.sh:159-175 (one thread per record; score = number of
// (record id, query id) equal pairs minus 0.05 * |record length - query length|), run there on at most 256
// candidates copied to the GPU per query.  Here every record of the index stays resident in HBM (a record is 32
// bytes of ids + a length, so even 10^9 records fit), the query ids sit in shared memory, each thread reads its
// record's eight ids with two 16-byte loads, and the kernel is a pure streaming pass over the index.
#include "kernels.h"

namespace hrm {

constexpr int kPhoMaxIds = 8;    // ids stored per record
constexpr int kPhoMaxQuery = 32;

__global__ void __launch_bounds__(256) pho_score_kernel(const uint4* __restrict__ rec_ids,
                                                        const uint32_t* __restrict__ rec_len,
                                                        const uint32_t* __restrict__ q, int q_len,
                                                        float* __restrict__ scores, long long n) {
  __shared__ uint32_t qs[kPhoMaxQuery];
  if (threadIdx.x < kPhoMaxQuery) qs[threadIdx.x] = threadIdx.x < q_len ? q[threadIdx.x] : 0u;
  __syncthreads();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const uint4 a = __ldg(&rec_ids[2 * i]), b = __ldg(&rec_ids[2 * i + 1]);
    const uint32_t ids[kPhoMaxIds] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const uint32_t len = min(__ldg(&rec_len[i]), (uint32_t)kPhoMaxIds);
    int hits = 0;
#pragma unroll
    for (int j = 0; j < kPhoMaxIds; ++j) {
      if (j < (int)len) {
        for (int t = 0; t < q_len; ++t) hits += ids[j] == qs[t];
      }
    }
    scores[i] = (float)hits - 0.05f * (float)abs((int)len - q_len);
  }
}

void pho_score_launch(const uint32_t* rec_ids, const uint32_t* rec_len, const uint32_t* q, int q_len, float* scores,
                      long long n, int sm_count, cudaStream_t s) {
  if (n <= 0) return;
  long long blocks = (n + 255) / 256;
  const long long cap = (long long)sm_count * 8;
  if (blocks > cap) blocks = cap;
  pho_score_kernel<<<(int)blocks, 256, 0, s>>>(reinterpret_cast<const uint4*>(rec_ids), rec_len, q,
                                               q_len < kPhoMaxQuery ? q_len : kPhoMaxQuery, scores, n);
}

}  // namespace hrm
