// No-allocation C entry point of the W8A16 GEMM: the same persistent stream-K kernel as the PyTorch entry point,
// with its partial-sum scratch, tickets and status word in this file's static device arrays instead of tensors.
// The contract (limits, what starts at zero, overlapping calls) is written beside the declarations.
#include "gemm_noalloc.h"
#include "gemm_w8a16.h"

#include <cstdio>
#include <exception>
#include <mutex>

namespace {

constexpr int kMaxDevices = 64;

// Static device storage: one copy on every device that loads the module, held until the process exits. Sized for
// the stream-K plan of every decode GEMM of a 70B-class model at up to 16 tokens (the widest, a 128256-row lm_head,
// needs 4,104,192 floats on 148 SMs). In host code these names are host-side stand-ins, never device addresses:
// the kernel only ever receives the addresses that cudaGetSymbolAddress returns below.
static __device__ __align__(256) float g_noalloc_ws[HRM_NOALLOC_MAX_WS_FLOATS];
static __device__ __align__(256) int g_noalloc_tickets[HRM_NOALLOC_MAX_TILES];
static __device__ __align__(256) int g_noalloc_status[4];

struct DeviceScratch {
  bool ready = false;
  float* ws = nullptr;
  int* tickets = nullptr;
  int* status = nullptr;
};

DeviceScratch g_scratch[kMaxDevices];
std::mutex g_setup_mu;
thread_local char g_err[256] = {0};

int fail(int code, const char* msg) {
  std::snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

// Per-device set-up, run with `dev` current: find where this device keeps the static arrays.
int setup_device(int dev, DeviceScratch** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(HRM_NOALLOC_ERR_SETUP, "device index out of range");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceScratch& s = g_scratch[dev];
  if (!s.ready) {
    const cudaError_t e1 = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.ws), g_noalloc_ws);
    const cudaError_t e2 = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.tickets), g_noalloc_tickets);
    const cudaError_t e3 = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.status), g_noalloc_status);
    if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess) {
      const cudaError_t e = e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3);
      std::snprintf(g_err, sizeof(g_err), "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return HRM_NOALLOC_ERR_SETUP;
    }
    s.ready = true;
  }
  *out = &s;
  return HRM_NOALLOC_OK;
}

}  // namespace

extern "C" int hrm_w8a16_gemm_f16_noalloc(const void* x, int ldx, const int8_t* w, const float* scale, void* out,
                                          int ldo, int M, int N, int K, cudaStream_t stream) {
  g_err[0] = 0;
  if (!x || !w || !scale || !out) return fail(HRM_NOALLOC_ERR_ARG, "null pointer argument");
  if (M < 0 || N <= 0 || K <= 0) return fail(HRM_NOALLOC_ERR_ARG, "M must be >= 0, N and K > 0");
  if (K % 64 != 0) return fail(HRM_NOALLOC_ERR_ARG, "K must be a multiple of 64");
  if (ldx < K || ldx % 8 != 0) return fail(HRM_NOALLOC_ERR_ARG, "ldx must be >= K and a multiple of 8");
  if (ldo < N) return fail(HRM_NOALLOC_ERR_ARG, "ldo must be >= N");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return fail(HRM_NOALLOC_ERR_ARG, "x and w must be 16-byte aligned");
  if (M == 0) return HRM_NOALLOC_OK;

  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(HRM_NOALLOC_ERR_SETUP, "no current CUDA device");
  DeviceScratch* s = nullptr;
  if (const int rc = setup_device(dev, &s)) return rc;

  hrm::GemmPlan p{};
  try {
    p = hrm::gemm_plan(M, N, K, 0);
  } catch (const std::exception& e) {
    return fail(HRM_NOALLOC_ERR_SETUP, e.what());
  }
  if (p.ws_floats > HRM_NOALLOC_MAX_WS_FLOATS || p.counters > HRM_NOALLOC_MAX_TILES) {
    std::snprintf(g_err, sizeof(g_err),
                  "shape M=%d N=%d K=%d needs %zu scratch floats and %d tickets; the static limits are %u and %d",
                  M, N, K, p.ws_floats, p.counters, HRM_NOALLOC_MAX_WS_FLOATS, HRM_NOALLOC_MAX_TILES);
    return HRM_NOALLOC_ERR_TOO_BIG;
  }
  hrm::GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.scale = scale;
  a.out = out;
  a.ldo = ldo;
  a.ws = s->ws;
  a.counters = s->tickets;
  a.status = s->status;
  try {
    hrm::gemm_w8a16_launch(x, ldx, w, hrm::EPI_F16, a, p, stream);
  } catch (const std::exception& e) {
    return fail(HRM_NOALLOC_ERR_LAUNCH, e.what());
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HRM_NOALLOC_ERR_LAUNCH, cudaGetErrorString(e));
  return HRM_NOALLOC_OK;
}

extern "C" const char* hrm_w8a16_noalloc_last_error(void) { return g_err; }

extern "C" int hrm_w8a16_noalloc_check(int* code) {
  g_err[0] = 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(HRM_NOALLOC_ERR_SETUP, "no current CUDA device");
  DeviceScratch* s = nullptr;
  if (const int rc = setup_device(dev, &s)) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(HRM_NOALLOC_ERR_LAUNCH, "device synchronise failed");
  int v = 0;
  if (cudaMemcpy(&v, s->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(HRM_NOALLOC_ERR_LAUNCH, "status read failed");
  if (code) *code = v;
  if (v != 0) {
    if (cudaMemset(s->status, 0, 4 * sizeof(int)) != cudaSuccess ||
        cudaMemset(s->tickets, 0, HRM_NOALLOC_MAX_TILES * sizeof(int)) != cudaSuccess)
      return fail(HRM_NOALLOC_ERR_LAUNCH, "re-zeroing the tickets failed");
  }
  return HRM_NOALLOC_OK;
}
