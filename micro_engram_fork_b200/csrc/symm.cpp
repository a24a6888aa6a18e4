// Symmetric device buffers over NVLink peer memory (the native comm substrate).
//
// Each rank allocates one device buffer with cudaMalloc and exports a CUDA IPC handle; the
// Python side exchanges the 64-byte handles through the process group's store, and every
// rank opens its peers' handles. The result is a table of per-rank base addresses that
// kernels index directly: a row owned by rank r at byte offset o is at ptr[r] + o, read or
// written with plain loads / stores / atomics over NVLink 5 through NVSwitch. Buffers have
// the same layout on every rank, so offsets are shared.
//
// No multicast objects here: peer access is plain P2P, which is what the engram fetch, the
// row-gradient push and the P2P all-reduce use.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <string>
#include <vector>

#define ME_CUDA_CHECK(x)                                                               \
  do {                                                                                 \
    cudaError_t e_ = (x);                                                              \
    TORCH_CHECK(e_ == cudaSuccess, #x, " failed: ", cudaGetErrorString(e_));           \
  } while (0)

// Allocate `nbytes` on the current device; returns the device address (int64).
int64_t symm_alloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  ME_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  ME_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  ME_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

// The IPC handle of an allocation made by symm_alloc, as bytes.
py::bytes symm_export(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  ME_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

// Map a peer's allocation into this process; returns its address here.
int64_t symm_import(py::bytes handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  ME_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  ME_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

// A non-owning tensor view of device memory (the owner keeps the allocation alive).
torch::Tensor symm_view(int64_t ptr, std::vector<int64_t> shape, torch::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {}, opts);
}

bool can_access_peer(int64_t dev, int64_t peer) {
  int ok = 0;
  ME_CUDA_CHECK(cudaDeviceCanAccessPeer(&ok, (int)dev, (int)peer));
  return ok != 0;
}
