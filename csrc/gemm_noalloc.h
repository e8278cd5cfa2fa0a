// C entry point of the W8A16 GEMM (f16 output) that allocates no device memory.
//
// This entry point has no counterpart in the reference: the reference's int8 GEMVs use no scratch memory, and its
// engine always runs inside a process that owns a device allocator.
//
// Who needs it: callers that reach the GEMM through a plain C ABI and have no device allocator of their own (a C or
// C++ host program that loads this library without PyTorch, so there is no caching allocator to draw scratch from),
// and callers that fix every device buffer up front and must not allocate afterwards (a serving loop whose memory
// plan is frozen, where a cudaMalloc would synchronise the device and could fail mid-request). The ordinary entry
// point takes its stream-K scratch from a PyTorch tensor; this one takes it from fixed-size arrays in the module's
// static device memory, which every GPU that loads the library holds until the process exits.
//
// Contract:
//  * out[m, n] = f16( sum_k x[m, k] * w[n, k] * scale[n] ); x f16 [M, ldx], w int8 [N, K] row-major, scale f32 [N],
//    out f16 [M, ldo]. All pointers are device pointers on the current device; x and w must be 16-byte aligned,
//    ldx a multiple of 8 elements, K a multiple of 64.
//  * The first call on a device (made with that device current) does the per-device set-up: it looks up where that
//    device keeps the static scratch. Make that first call before any stream capture begins.
//  * Scratch limit: the stream-K plan of (M, N, K) may need at most HRM_NOALLOC_MAX_WS_FLOATS floats of partial sums
//    and HRM_NOALLOC_MAX_TILES output tiles; larger plans are rejected with HRM_NOALLOC_ERR_TOO_BIG and a message.
//    On a 148-SM B200 every decode GEMM of a 70B-class model fits for M <= 16 tokens (the widest, the 128256-row
//    lm_head at K = 8192, needs 4,104,192 floats).  From M = 17 the token tile doubles (32 columns) and that
//    lm_head needs about 8.2M floats, so it is rejected; the hidden-size projections still fit up to M = 64.
//  * What must start at zero: the per-tile tickets. They live in static storage, which is zero when the module
//    loads, and every launch returns each ticket it used to zero. The partial-sum scratch needs no initial value
//    (every partial is written before it is read). A launch that gave up on a bounded wait can leave tickets
//    non-zero: hrm_w8a16_noalloc_check() reports that and re-zeroes them.
//  * Every call shares the same scratch. Calls that overlap on the GPU (two streams, or two host threads, on one
//    device) race and give wrong results; serialise them.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HRM_NOALLOC_MAX_WS_FLOATS (4u * 1024u * 1024u)   // 16 MiB of fp32 partial sums per device
#define HRM_NOALLOC_MAX_TILES 4096                       // 16 KiB of tickets per device

enum {
  HRM_NOALLOC_OK = 0,
  HRM_NOALLOC_ERR_ARG = 1,       // null pointer, bad shape, stride or alignment
  HRM_NOALLOC_ERR_TOO_BIG = 2,   // the plan needs more scratch than the static arrays hold
  HRM_NOALLOC_ERR_SETUP = 3,     // per-device set-up failed (no current device, symbol lookup failed)
  HRM_NOALLOC_ERR_LAUNCH = 4,    // the runtime refused the launch
};

// Launch on `stream`; returns an HRM_NOALLOC_* code. Nothing is allocated on the device.
int hrm_w8a16_gemm_f16_noalloc(const void* x, int ldx, const int8_t* w, const float* scale, void* out, int ldo,
                               int M, int N, int K, cudaStream_t stream);

// Message for the last non-zero code returned on this host thread ("" if none).
const char* hrm_w8a16_noalloc_last_error(void);

// Synchronises the current device, stores this entry point's bounded-wait status word in *code (0 = no wait gave
// up) and, if it is non-zero, re-zeroes the status word and every ticket. Returns an HRM_NOALLOC_* code.
int hrm_w8a16_noalloc_check(int* code);

#ifdef __cplusplus
}
#endif
