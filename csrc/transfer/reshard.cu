// K1: the reshard transfer kernel.
//
// One launch executes every copy a rank is responsible for in a switch.  Each task is a strided 2-D
// (optionally 3-plane) byte copy whose source and/or destination may be another GPU's memory mapped into this
// process through CUDA IPC; loads and stores to peer memory travel over NVLink / NVSwitch.  The host splits
// the planner's descriptors into tasks of at most ~1 MiB so every SM gets work, and the kernel is persistent
// (grid = a multiple of the SM count).  Within a task the work units are (plane, row, 8 KiB segment of the
// row), handed to the CTA's warps round-robin, so a task that is one long row (a ZeRO-sharded flat range)
// still keeps every warp busy; lanes move 16-byte vectors with several loads in flight before the stores
// (peer reads are latency-bound, so bytes in flight matter).
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

constexpr uint32_t SEG_BYTES = 8192;  // bytes of one warp work unit

__global__ void __launch_bounds__(512) reshard_copy_kernel(const CopyTask* __restrict__ tasks, int ntasks) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  for (int t = blockIdx.x; t < ntasks; t += gridDim.x) {
    const CopyTask tk = tasks[t];
    const uint32_t nseg = (tk.row_bytes + SEG_BYTES - 1) / SEG_BYTES;
    const uint32_t rows_total = tk.planes * tk.rows;
    const uint64_t units = (uint64_t)rows_total * nseg;
    const bool vec = (tk.flags & 1u) != 0;
    for (uint64_t u = warp; u < units; u += nwarps) {
      const uint32_t pr = (uint32_t)(u / nseg), sg = (uint32_t)(u - (uint64_t)pr * nseg);
      const uint32_t p = pr / tk.rows, r = pr - p * tk.rows;
      const uint32_t off = sg * SEG_BYTES;
      const uint32_t len = min(SEG_BYTES, tk.row_bytes - off);
      const uint64_t sa = tk.src + p * tk.src_plane + r * tk.src_stride + off;
      const uint64_t da = tk.dst + p * tk.dst_plane + r * tk.dst_stride + off;
      if (vec) {
        copy_row_vec<4>(reinterpret_cast<const uint4*>(sa), reinterpret_cast<uint4*>(da), len >> 4, lane);
      } else {
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(sa);
        uint16_t* d16 = reinterpret_cast<uint16_t*>(da);
        for (uint32_t i = lane; i < (len >> 1); i += 32) d16[i] = s16[i];
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
