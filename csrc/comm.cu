// Symmetric-memory plumbing: each rank cudaMalloc's one buffer, exports a CUDA IPC handle, and maps every peer's
// buffer into its own address space (NVLink P2P through NVSwitch).  The handles travel over the
// torch.distributed store/process group; the device sees a table of peer base pointers.
//
// This replaces the reference's `cudaDeviceEnablePeerAccess` + `cudaMemcpy` hand-offs
// (deepseek_native_engine.sh:909-921,1046,1102) and the ring of `cudaMemcpyPeerAsync` (llm_engine.cu:1522-1594):
// peers are read and written directly by kernels instead of by copy engines.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "comm.h"

namespace hrm {
namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Allocate `bytes` of zeroed device memory on the current device; returns (ptr, ipc_handle_bytes).
pybind11::tuple symm_alloc(int64_t bytes) {
  void* p = nullptr;
  ck(cudaMalloc(&p, (size_t)bytes), "cudaMalloc");
  ck(cudaMemset(p, 0, (size_t)bytes), "cudaMemset");
  cudaIpcMemHandle_t h;
  ck(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  return pybind11::make_tuple((int64_t)(uintptr_t)p,
                              pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t symm_open(pybind11::bytes handle) {
  std::string s = handle;
  if (s.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return (int64_t)(uintptr_t)p;
}

void symm_close(int64_t ptr) { ck(cudaIpcCloseMemHandle(reinterpret_cast<void*>((uintptr_t)ptr)), "cudaIpcCloseMemHandle"); }
void symm_free(int64_t ptr) { ck(cudaFree(reinterpret_cast<void*>((uintptr_t)ptr)), "cudaFree"); }

bool can_access_peer(int64_t dev, int64_t peer) {
  int ok = 0;
  ck(cudaDeviceCanAccessPeer(&ok, (int)dev, (int)peer), "cudaDeviceCanAccessPeer");
  return ok != 0;
}

// Non-owning tensor view over a raw device pointer (the symmetric heap owns the memory).
at::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, (int)device));
  return torch::from_blob(reinterpret_cast<void*>((uintptr_t)ptr), shape, [](void*) {}, opts);
}

}  // namespace

void register_comm_bindings(pybind11::module& m) {
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("can_access_peer", &can_access_peer);
  m.def("tensor_from_ptr", &tensor_from_ptr);
}

}  // namespace hrm
