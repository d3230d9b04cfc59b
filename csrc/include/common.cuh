// Shared helpers for the sm_100a kernels of elasticmegatron_b200.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <atomic>
#include <mutex>

#include <c10/cuda/CUDAStream.h>
#include <ATen/ATen.h>

namespace emb {

// Host-side count of kernel launches issued by this extension (read by the benchmark).
std::atomic<long long>& launch_counter();
inline void count_launch(long long n = 1) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

#define EMB_CUDA_CHECK(expr)                                                                  \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__,  \
                ":", __LINE__);                                                               \
  } while (0)

#define EMB_LAUNCH_CHECK() EMB_CUDA_CHECK(cudaGetLastError())

// Device-side error words of the kernels with bounded waits: one zero-initialised int per (device, slot),
// allocated on first use on each device and kept until exit, so a timeout or abort code recorded on one
// device is never dropped when another device becomes current.
enum ErrSlot { kErrGemm = 0, kErrAttnFwd = 1, kErrAttnBwd = 2, kErrComm = 3, kErrSlots = 8 };
constexpr int kMaxDevices = 64;
inline int* device_err_flag(int slot) {
  static std::mutex mu;
  static int* flags[kMaxDevices] = {};
  int dev = 0;
  EMB_CUDA_CHECK(cudaGetDevice(&dev));
  TORCH_CHECK(dev >= 0 && dev < kMaxDevices && slot >= 0 && slot < kErrSlots, "device_err_flag: bad device/slot");
  std::lock_guard<std::mutex> g(mu);
  if (!flags[dev]) {
    int* f = nullptr;
    EMB_CUDA_CHECK(cudaMalloc(&f, kErrSlots * sizeof(int)));
    EMB_CUDA_CHECK(cudaMemset(f, 0, kErrSlots * sizeof(int)));
    flags[dev] = f;
  }
  return flags[dev] + slot;
}

inline cudaStream_t cur_stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

inline int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum; `sh` needs 32 floats.  All threads receive the result.
__device__ __forceinline__ float block_sum(float v, float* sh) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  int nw = (blockDim.x + 31) >> 5;
  float r = (threadIdx.x < nw) ? sh[threadIdx.x] : 0.f;
  if (w == 0) r = warp_sum(r);
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  return sh[0];
}

__device__ __forceinline__ float block_max(float v, float* sh) {
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) sh[w] = v;
  __syncthreads();
  int nw = (blockDim.x + 31) >> 5;
  float r = (threadIdx.x < nw) ? sh[threadIdx.x] : -INFINITY;
  if (w == 0) r = warp_max(r);
  if (threadIdx.x == 0) sh[0] = r;
  __syncthreads();
  return sh[0];
}

// 8 x bf16 packed in 16 bytes
struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

inline void check_cuda_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace emb
