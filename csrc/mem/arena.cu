// Flat state arenas: one cudaMalloc per arena (so each is exactly one CUDA IPC allocation), exported and
// imported with cudaIpcGetMemHandle / cudaIpcOpenMemHandle.  Imported peer mappings are cached per handle
// for the life of the process.
#include <cuda_runtime.h>
#include <ATen/ATen.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "../include/common.cuh"

namespace emb {

std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}
int64_t launch_count() { return launch_counter().load(); }
void reset_launch_count() { launch_counter().store(0); }

at::Tensor arena_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0);
  int prev;
  EMB_CUDA_CHECK(cudaGetDevice(&prev));
  EMB_CUDA_CHECK(cudaSetDevice((int)device));
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)nbytes);
  cudaSetDevice(prev);
  TORCH_CHECK(e == cudaSuccess, "arena cudaMalloc(", nbytes, ") failed: ", cudaGetErrorString(e));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, (int)device);
  return at::from_blob(p, {nbytes}, [](void* ptr) { cudaFree(ptr); }, opts);
}

at::Tensor ipc_get_handle(at::Tensor arena) {
  TORCH_CHECK(arena.is_cuda());
  cudaIpcMemHandle_t h;
  EMB_CUDA_CHECK(cudaIpcGetMemHandle(&h, arena.data_ptr()));
  auto out = at::empty({(int64_t)sizeof(h)}, at::kByte);
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

static std::mutex g_mu;
static std::map<std::string, uint64_t> g_open;

// Map a peer allocation; returns its device address in this process (cached per handle).
int64_t ipc_open(at::Tensor handle) {
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t));
  std::string key((const char*)handle.data_ptr(), sizeof(cudaIpcMemHandle_t));
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_open.find(key);
  if (it != g_open.end()) return (int64_t)it->second;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  EMB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  g_open[key] = (uint64_t)p;
  return (int64_t)(uint64_t)p;
}

// Unmap one peer allocation previously mapped with ipc_open (no-op if it is not mapped).
bool ipc_close(at::Tensor handle) {
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t));
  std::string key((const char*)handle.data_ptr(), sizeof(cudaIpcMemHandle_t));
  std::lock_guard<std::mutex> g(g_mu);
  auto it = g_open.find(key);
  if (it == g_open.end()) return false;
  cudaIpcCloseMemHandle((void*)it->second);
  g_open.erase(it);
  return true;
}

void ipc_close_all() {
  std::lock_guard<std::mutex> g(g_mu);
  for (auto& kv : g_open) cudaIpcCloseMemHandle((void*)kv.second);
  g_open.clear();
}

int64_t ipc_open_count() {
  std::lock_guard<std::mutex> g(g_mu);
  return (int64_t)g_open.size();
}

}  // namespace emb
