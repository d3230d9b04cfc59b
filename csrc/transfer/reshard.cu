// K1: the reshard transfer kernel.
//
// One launch executes every copy a rank is responsible for in a switch.  Each task is a strided 2-D
// (optionally 3-plane) byte copy whose source and/or destination may be another GPU's memory mapped into this
// process through CUDA IPC; loads and stores to peer memory travel over NVLink / NVSwitch.  The host splits
// the planner's descriptors into tasks of at most ~1 MiB so every SM gets work, and the kernel is persistent
// (grid = a multiple of the SM count).  Within a task each warp walks rows; lanes move 16-byte vectors with
// several loads in flight before the stores (peer reads are latency-bound, so bytes in flight matter).
// Unaligned tasks fall back to 2-byte moves (every element type here is >= 2 bytes).
//
// There is no spin-wait in this kernel: ordering against the peers' previous and next work is provided by
// stream-ordered NCCL barriers issued around the launch by the host.
#include "../include/common.cuh"

namespace emb {

struct CopyTask {
  uint64_t src, dst;          // byte addresses
  uint64_t src_stride, dst_stride;  // bytes between rows
  uint64_t src_plane, dst_plane;    // bytes between planes
  uint32_t rows, row_bytes;
  uint32_t planes, flags;     // flags bit0: 16-byte aligned
};
static_assert(sizeof(CopyTask) == 64, "task layout");

template <int UNROLL>
__device__ __forceinline__ void copy_row_vec(const uint4* __restrict__ s, uint4* __restrict__ d, uint32_t nvec,
                                             int lane) {
  uint32_t i = lane;
  for (; i + 32 * (UNROLL - 1) < nvec; i += 32 * UNROLL) {
    uint4 v[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) v[u] = __ldcg(s + i + 32 * u);
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) __stcg(d + i + 32 * u, v[u]);
  }
  for (; i < nvec; i += 32) __stcg(d + i, __ldcg(s + i));
}

__global__ void __launch_bounds__(512) reshard_copy_kernel(const CopyTask* __restrict__ tasks, int ntasks) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  for (int t = blockIdx.x; t < ntasks; t += gridDim.x) {
    const CopyTask tk = tasks[t];
    const uint32_t units = tk.planes * tk.rows;
    if (tk.flags & 1u) {
      const uint32_t nvec = tk.row_bytes >> 4;
      for (uint32_t u = warp; u < units; u += nwarps) {
        uint32_t p = u / tk.rows, r = u - p * tk.rows;
        const uint4* s = reinterpret_cast<const uint4*>(tk.src + p * tk.src_plane + r * tk.src_stride);
        uint4* d = reinterpret_cast<uint4*>(tk.dst + p * tk.dst_plane + r * tk.dst_stride);
        copy_row_vec<4>(s, d, nvec, lane);
      }
    } else {
      const uint32_t nh = tk.row_bytes >> 1;
      for (uint32_t u = warp; u < units; u += nwarps) {
        uint32_t p = u / tk.rows, r = u - p * tk.rows;
        const uint16_t* s = reinterpret_cast<const uint16_t*>(tk.src + p * tk.src_plane + r * tk.src_stride);
        uint16_t* d = reinterpret_cast<uint16_t*>(tk.dst + p * tk.dst_plane + r * tk.dst_stride);
        for (uint32_t i = lane; i < nh; i += 32) d[i] = s[i];
      }
    }
  }
}

// tasks: uint8 CUDA tensor holding ntasks * 64 bytes of CopyTask records.
void reshard_copy(at::Tensor tasks, int64_t ntasks, int64_t grid) {
  TORCH_CHECK(tasks.is_cuda() && tasks.scalar_type() == at::kByte && tasks.numel() >= ntasks * 64);
  if (ntasks == 0) return;
  if (grid <= 0) grid = std::min<int64_t>(ntasks, (int64_t)num_sms() * 4);
  reshard_copy_kernel<<<(int)grid, 512, 0, cur_stream()>>>(reinterpret_cast<const CopyTask*>(tasks.data_ptr()),
                                                          (int)ntasks);
  EMB_LAUNCH_CHECK();
  count_launch();
}

int64_t copy_task_bytes() { return sizeof(CopyTask); }

}  // namespace emb
