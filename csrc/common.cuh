// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits, TMA tile loads, tcgen05 (UMMA)
// descriptors / MMA / TMEM access, and small numeric helpers.  Written against the public PTX ISA for sm_100a.
//
// Rules enforced here for every kernel of this library:
//  * every spin-wait is bounded; on timeout it records an error code in a global status word and returns
//    (no __trap, no device assert);
//  * TMA loads never use cluster multicast (loads are CTA-local);
//  * tcgen05.mma operands are f16 x f16 (kind::f16) - A and B always share one type.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>
#include <stdexcept>
#include <string>
#include <utility>

#define HRM_DEVINL __device__ __forceinline__

namespace hrm {

// Error codes written to the kernel status word (0 = ok).
enum : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,
  kErrTimeoutEmpty = 2,
  kErrTimeoutDequant = 3,
  kErrTimeoutAccum = 4,
  kErrTimeoutPeer = 5,
  kErrBadShape = 6,
  kErrTimeoutGrid = 7,   // grid-wide barrier of a persistent multi-phase kernel
  // multi-phase GEMM chain: which ring wait gave up first (the status word keeps the first error)
  kErrChainWEmpty = 8, kErrChainXEmpty = 9, kErrChainFEmpty = 10, kErrChainWFull = 11, kErrChainXFull = 12,
  kErrChainFFull = 13, kErrChainAEmpty = 14, kErrChainAFull = 15,
};

// Every wait is bounded in time: 2 s of %globaltimer, far above any legitimate wait in these kernels (the longest
// is an epilogue warp waiting for a prefill mainloop of a few tens of milliseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;
HRM_DEVINL uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

HRM_DEVINL uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

HRM_DEVINL void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------- programmatic dependent launch
// A grid launched with the programmatic-serialization attribute may start while the previous kernel in its stream
// is still running.  Its threads must pass pdl_wait() (griddepcontrol.wait: the previous grid has completed and its
// memory is visible) before touching anything that grid, or an earlier one, may write.  pdl_trigger()
// (griddepcontrol.launch_dependents) lets the NEXT grid be scheduled early.  Rules of this library: a kernel
// triggers only after its own pdl_wait(), so when a dependent starts, every grid before its direct predecessor has
// completed; before pdl_wait() a kernel only sets up shared memory / TMEM and reads data that no kernel of the
// inference step writes (int8 weights), or data the caller vouches for (older KV entries).  Both are no-ops for a
// grid launched without the attribute.
HRM_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HRM_DEVINL void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier
HRM_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
HRM_DEVINL void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

HRM_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
// Relaxed arrive: unlike the default (release) form it does not wait for this thread's outstanding global loads to
// complete, so a thread can keep a deep register prefetch in flight across its arrivals.  Only for barriers whose
// payload is ordered by other means (tcgen05.wait::st + tcgen05.fence for tensor-memory stores).
HRM_DEVINL void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.relaxed.cta.shared::cta.b64 st, [%0];\n\t}"
               ::"r"(smem_u32(bar)) : "memory");
}
HRM_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
HRM_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a thread whose phase is not complete yet is parked (it stops competing for issue
// slots with the working warps of its SM sub-partition) until the phase completes or the hint expires.
constexpr uint32_t kSuspendHintNs = 1000000u;   // 1 ms
HRM_DEVINL bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs) : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false (and records `code`) when the time limit is hit.
HRM_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  record_error(status, code);
  return false;
}
// Bounded wait with a CTA-wide abort flag in shared memory: once any thread of the CTA timed out, every other wait
// returns false at once, so the CTA drains quickly (callers keep uniform control flow and skip issuing new work).
HRM_DEVINL bool mbar_wait_ab(uint64_t* bar, uint32_t parity, int* status, int code, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  *abort_flag = 1;
  record_error(status, code);
  return false;
}

// ---------------------------------------------------------------- TMA (no multicast)
HRM_DEVINL void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
HRM_DEVINL void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
HRM_DEVINL void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z),
        "r"(w) : "memory");
}
HRM_DEVINL void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// Streaming 16-byte global load (read-only path, no L1 allocation, 256-byte L2 fetch granule).
HRM_DEVINL uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// Contiguous global -> shared bulk copy (bytes a multiple of 16, both addresses 16-byte aligned), CTA-local.
HRM_DEVINL void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
HRM_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Orders this thread's earlier (generic-proxy) acquires before its later async-proxy (TMA / bulk) global reads.
HRM_DEVINL void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05 / TMEM
HRM_DEVINL void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(smem_slot)), "r"(ncols) : "memory");
}
HRM_DEVINL void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
HRM_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
HRM_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
HRM_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, fp32 accumulate; single issuing thread.
HRM_DEVINL void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 with the A operand read from tensor memory: for M = 128, row m
// of A sits in TMEM lane m and its 16-bit elements are packed two per 32-bit column in K order (low half = even k).
HRM_DEVINL void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread have completed.
HRM_DEVINL void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// Instruction descriptor, kind::f16: D = f32, A = B = f16, both K-major, shape M x N.
HRM_DEVINL constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4)                      // D format: f32
       | (0u << 7) | (0u << 10)         // A, B format: f16
       | (0u << 15) | (0u << 16)        // K-major A and B
       | ((uint32_t)(N >> 3) << 17)
       | ((uint32_t)(M >> 4) << 24);
}
// Same with bf16 operands (used by attention where Q/K/V are bf16).
HRM_DEVINL constexpr uint32_t idesc_bf16_f32(int M, int N, bool b_mn_major = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | ((b_mn_major ? 1u : 0u) << 16)
       | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major operand stored in the 128-byte-swizzled canonical layout:
// rows of 128 bytes, 8-row groups 1024 bytes apart (SBO = 1024), atom base 1024-byte aligned.  Advancing along
// K inside the 128-byte row is done by adding the byte offset to the start address.
HRM_DEVINL uint64_t sdesc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);      // start address
  d |= (uint64_t)(16u >> 4) << 16;                  // LBO (ignored for swizzled K-major; canonical value 1)
  d |= (uint64_t)(1024u >> 4) << 32;                // SBO
  d |= (uint64_t)1 << 46;                           // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                           // SWIZZLE_128B
  return d;
}
// MN-major operand in the 128-byte-swizzled canonical layout: 64 MN-elements (128 bytes) per row, rows along K,
// 8-row (8 K) groups 1024 bytes apart; consecutive 64-element MN blocks are LBO bytes apart.
HRM_DEVINL uint64_t sdesc_sw128_mn(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
HRM_DEVINL void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 32 bit, 32 consecutive columns per thread.
HRM_DEVINL void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
HRM_DEVINL void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread (store into TMEM).
HRM_DEVINL void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns per thread (raw 32-bit words); waits for the store to complete.
HRM_DEVINL void tmem_st32u(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- numerics
// Four signed int8 (one 32-bit word) -> two f16x2, exact.  Each byte is biased to unsigned (xor 0x80), placed
// in the mantissa of the f16 1024.0 (0x6400 | u gives 1024 + u, exact for u < 1024), then 1024 + 128 is
// subtracted.
HRM_DEVINL void i8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  asm("prmt.b32 %0, %1, %2, 0x4140;" : "=r"(lo) : "r"(u), "r"(0x64646464u));
  asm("prmt.b32 %0, %1, %2, 0x4342;" : "=r"(hi) : "r"(u), "r"(0x64646464u));
  const uint32_t bias = 0x64806480u;  // f16x2 (1152, 1152)
  asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(lo), "r"(bias));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(hi), "r"(bias));
}

HRM_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
HRM_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

HRM_DEVINL float silu(float x) { return x / (1.0f + __expf(-x)); }

// Monotone float -> uint32 map (total order) and the packed 64-bit argmax key: larger value wins, then the
// lower index (the low word stores ~idx).
HRM_DEVINL uint32_t float_order(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
HRM_DEVINL unsigned long long argmax_key(float v, uint32_t idx) {
  return ((unsigned long long)float_order(v) << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
HRM_DEVINL float order_to_float(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o);
}

// Sampling noise.  A counter-based generator: the SplitMix64 output mix (Steele, Lea and Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014) applied to a per-(seed, position) key plus the golden-ratio step
// times the global token id, so every rank of a tensor-parallel group draws the same noise for a token id whatever
// its vocabulary shard, and a request's draw depends only on its seed and position (not on the batch it is in).
constexpr unsigned long long kGoldenGamma = 0x9E3779B97F4A7C15ull;
HRM_DEVINL unsigned long long mix64(unsigned long long z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
HRM_DEVINL unsigned long long sample_row_key(unsigned long long seed, int pos) {
  return mix64(seed + kGoldenGamma * (unsigned long long)((long long)pos + 1));
}
// Standard Gumbel variate -log(-log(u)) for token `id` under row key `rk`; u in (0, 1) from the top 23 bits.
HRM_DEVINL float gumbel_noise(unsigned long long rk, uint32_t id) {
  const unsigned long long h = mix64(rk + kGoldenGamma * ((unsigned long long)id + 1ull));
  const float u = ((float)(h >> 41) + 0.5f) * (1.0f / 8388608.0f);
  return -logf(-logf(u));
}

// ---------------------------------------------------------------- peer-memory (NVLink) flags
// Used by the fused all-reduce GEMM epilogue and the distributed argmax exchange.
// Relaxed system-scope flag accesses and the fence that turns them into release / acquire patterns: a writer
// fences once after its data stores (and after the named barrier that orders its CTA's other stores before the
// fence) and then stores the flag relaxed; a reader polls relaxed and fences once after it sees the flag.
HRM_DEVINL void st_relaxed_sys(int* p, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HRM_DEVINL int ld_relaxed_sys(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
HRM_DEVINL void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// 64-bit relaxed system-scope accesses: an aligned 64-bit access is single-copy atomic, so a word that carries its
// own epoch next to its payload is either wholly old or wholly new to a peer that reads it.
HRM_DEVINL void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
HRM_DEVINL unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Bounded relaxed poll for a flag to reach `want` (epochs only grow), then one acquire fence.  Records
// kErrTimeoutPeer on timeout and returns false.
HRM_DEVINL bool wait_flag_acquire(const int* p, int want, int* status) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_relaxed_sys(p) - want >= 0) {
      fence_acq_rel_sys();
      return true;
    }
    __nanosleep(32);   // back off: the flag's line stays free for the peer's store
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      record_error(status, kErrTimeoutPeer);
      return false;
    }
  }
}
HRM_DEVINL void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
HRM_DEVINL int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded wait for a peer flag to reach `want` (epochs only grow).  Records kErrTimeoutPeer on timeout.
HRM_DEVINL bool wait_peer_flag(const int* p, int want, int* status) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (ld_acquire_sys(p) - want >= 0) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      record_error(status, kErrTimeoutPeer);
      return false;
    }
  }
}

// ---------------------------------------------------------------- host: per-device set-up
// cudaFuncSetAttribute acts on the CURRENT device only, so a process that drives several GPUs must raise a kernel's
// dynamic shared-memory limit once on each of them.  One flag per device and per kernel: the kernel symbol is the
// template argument, so every kernel (every template instantiation of one) has its own flags.  The flags are
// atomics because launches may come from several host threads; a racing second cudaFuncSetAttribute is harmless
// (same value), so no lock is needed.
constexpr int kMaxDevices = 64;

inline int current_device_or_throw() {
  int d = 0;
  const cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaGetDevice failed: ") + cudaGetErrorString(e));
  if (d < 0 || d >= kMaxDevices) throw std::runtime_error("device ordinal beyond the supported 64 devices");
  return d;
}

template <auto Kernel>
inline void ensure_smem_limit(int bytes) {
  static std::atomic<bool> done[kMaxDevices];   // zero-initialised (static storage), one set per kernel symbol
  const int d = current_device_or_throw();
  if (done[d].load(std::memory_order_acquire)) return;
  const cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("cudaFuncSetAttribute(max dynamic shared memory) failed: ") +
                             cudaGetErrorString(e));
  done[d].store(true, std::memory_order_release);
}

// ---------------------------------------------------------------- host: launches
// Programmatic dependent launch of the decode-path kernels (on unless HRM_PDL=0 in the environment, or turned off
// with set_pdl_enabled; defined with the GEMM host code).
bool pdl_enabled();
void set_pdl_enabled(bool on);

// Launches `kern` (throws std::runtime_error when the launch is rejected, so a kernel never silently goes missing).
template <typename... KArgs, typename... Args>
inline void launch_maybe_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("kernel launch failed: ") + cudaGetErrorString(e));
}

}  // namespace hrm
