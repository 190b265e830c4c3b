// symm.cpp -- symmetric peer memory over NVLink for the fused collectives.
//
// Every rank allocates the same-sized buffer, exports a CUDA IPC handle, and
// the handles are exchanged through torch.distributed (host side, Python).
// Opening a peer's handle maps that GPU's buffer into this process, so a
// kernel can load from and store to it directly (P2P over NVLink/NVSwitch).
// No collective library is involved in the data path.
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>
#include <cstring>
#include <string>

namespace {

void check(cudaError_t e, const char *what) {
  TORCH_CHECK(e == cudaSuccess, "symm: ", what, ": ", cudaGetErrorString(e));
}

}  // namespace

// Allocate `bytes` of device memory on the current device (zeroed).
// Returns (device pointer, ipc handle bytes).
std::tuple<int64_t, py::bytes> symm_alloc(int64_t bytes) {
  void *p = nullptr;
  check(cudaMalloc(&p, (size_t)bytes), "cudaMalloc");
  check(cudaMemset(p, 0, (size_t)bytes), "cudaMemset");
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  return {reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char *>(&h), sizeof(h))};
}

// Map a peer's buffer from its handle; returns the local address of it.
int64_t symm_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "symm: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void *p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t peer_ptr) {
  if (peer_ptr) cudaIpcCloseMemHandle(reinterpret_cast<void *>(peer_ptr));
}

void symm_free(int64_t ptr) {
  if (ptr) cudaFree(reinterpret_cast<void *>(ptr));
}

// Whether this device can address `peer` directly (NVLink / PCIe P2P).
bool symm_can_access(int64_t device, int64_t peer) {
  int ok = 0;
  cudaDeviceCanAccessPeer(&ok, (int)device, (int)peer);
  return ok != 0;
}

// A non-owning uint8 tensor over this rank's own buffer (for inspection:
// the slab a fused collective left behind). The buffer must outlive it.
at::Tensor symm_view(int64_t ptr, int64_t bytes, int64_t device) {
  TORCH_CHECK(ptr != 0 && bytes > 0, "symm: null or empty view");
  return torch::from_blob(reinterpret_cast<void *>(ptr), {bytes},
                          at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (int)device));
}

void register_symm(py::module &m) {
  m.def("symm_view", &symm_view);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_free", &symm_free);
  m.def("symm_can_access", &symm_can_access);
}
