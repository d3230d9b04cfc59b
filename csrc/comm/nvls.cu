// All-reduce of fp32 buffers through NVSwitch multicast (NVLS) with a peer-memory fallback.
//
// Both kernels work on a symmetric staging buffer that every rank of the group maps (one allocation per rank,
// the same size and offset everywhere).  The host reduces a tensor in two stream-ordered barriers
// (`sym_barrier` over a signal area at the head of the buffer):
//   copy in -> barrier -> [this kernel: rank r reduces slice r] -> barrier -> copy out.
//
// * `nvls_allreduce_f32`: the buffer is bound to an NVLink multicast object.  For every 16-byte vector of its
//   slice a thread issues `multimem.ld_reduce ... add.v4.f32` on the multicast address - the switch reads the
//   vector from every GPU of the group and returns the sum - and `multimem.st ... v4.f32` of that sum, which the
//   switch writes into every GPU's buffer.  Per GPU this moves its slice in (the reduced values) plus the other
//   slices' results, about one buffer in each direction, against 2 (n - 1) / n buffers each way for a ring.
// * `p2p_allreduce_f32` (no multicast object): rank r reads slice r of every peer's buffer (unicast NVLink
//   loads, fixed rank order so every rank computes bit-identical sums), and stores the sum into slice r of every
//   peer's buffer.
//
// The multimem reductions run in the switch; the order in which it adds the n contributions is not specified,
// so results can differ in the last bit from the fixed-order P2P path (both are exact for n = 2).
// Neither kernel waits on anything: ordering comes entirely from the barriers around them.
#include "../include/common.cuh"

namespace emb {

namespace {

struct Ptrs8 {
  uint64_t p[8];
};

__device__ __forceinline__ void mm_ld_reduce_v4(const float* a, float4& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(a)
               : "memory");
}
__device__ __forceinline__ void mm_st_v4(float* a, const float4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_ld_reduce_f32(const float* a, float& v) {
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(a) : "memory");
}
__device__ __forceinline__ void mm_st_f32(float* a, float v) {
  asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(a), "f"(v) : "memory");
}

// mc: multicast address of the slice's first float; n4 vectors of 4 floats then `tail` scalars.
__global__ void nvls_allreduce_kernel(float* mc, int64_t n4, int tail) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v;
    mm_ld_reduce_v4(mc + 4 * i, v);
    mm_st_v4(mc + 4 * i, v);
  }
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t < tail) {
    float v;
    mm_ld_reduce_f32(mc + 4 * n4 + t, v);
    mm_st_f32(mc + 4 * n4 + t, v);
  }
  // the stores above are visible system-wide before anything this thread does next (the barrier kernel that
  // follows on the stream also fences; this keeps the kernel correct on its own)
  __threadfence_system();
}

// bufs: every rank's staging base; off: byte offset of this rank's slice; count floats.
__global__ void p2p_allreduce_kernel(Ptrs8 bufs, int n, uint64_t off, int64_t count) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool vec = ((off | (uint64_t)count * 4) & 15) == 0;
  if (vec) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count / 4; i += stride) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < n; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(bufs.p[r] + off) + i);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      for (int r = 0; r < n; ++r) __stcg(reinterpret_cast<float4*>(bufs.p[r] + off) + i, acc);
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += stride) {
      float acc = 0.f;
      for (int r = 0; r < n; ++r) acc += __ldcg(reinterpret_cast<const float*>(bufs.p[r] + off) + i);
      for (int r = 0; r < n; ++r) __stcg(reinterpret_cast<float*>(bufs.p[r] + off) + i, acc);
    }
  }
  __threadfence_system();
}

int grid_for(int64_t bytes) {
  const int64_t want = (bytes + 32767) / 32768;  // ~32 KiB of slice per CTA
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)num_sms() * 4));
}

}  // namespace

// mc_slice: multicast address of this rank's slice (16-byte aligned for the vector path); count floats.
void nvls_allreduce_f32(int64_t mc_slice, int64_t count) {
  TORCH_CHECK(mc_slice != 0 && (mc_slice & 3) == 0, "nvls_allreduce_f32: bad multicast address");
  TORCH_CHECK(count >= 0);
  if (count == 0) return;
  int64_t n4 = 0;
  int tail = (int)count;
  if ((mc_slice & 15) == 0) {
    n4 = count / 4;
    tail = (int)(count - 4 * n4);
  } else {
    TORCH_CHECK(count <= (1 << 20), "nvls_allreduce_f32: unaligned slices must be small");
  }
  const int threads = 256;
  int grid = grid_for(count * 4);
  if (n4 == 0) grid = (tail + threads - 1) / threads;
  nvls_allreduce_kernel<<<grid, threads, 0, cur_stream()>>>(reinterpret_cast<float*>(mc_slice), n4, tail);
  EMB_LAUNCH_CHECK();
  count_launch();
}

// bufs: int64 CPU [n] staging base of every rank as mapped here; off: byte offset of this rank's slice.
void p2p_allreduce_f32(at::Tensor bufs, int64_t off, int64_t count) {
  TORCH_CHECK(!bufs.is_cuda() && bufs.scalar_type() == at::kLong, "bufs: int64 CPU tensor");
  const int n = (int)bufs.numel();
  TORCH_CHECK(n >= 1 && n <= 8 && off >= 0 && (off & 3) == 0 && count >= 0);
  if (count == 0) return;
  Ptrs8 p{};
  auto c = bufs.contiguous();
  for (int i = 0; i < n; ++i) p.p[i] = (uint64_t)c.data_ptr<int64_t>()[i];
  p2p_allreduce_kernel<<<grid_for(count * 4 * n), 256, 0, cur_stream()>>>(p, n, (uint64_t)off, count);
  EMB_LAUNCH_CHECK();
  count_launch();
}

}  // namespace emb
