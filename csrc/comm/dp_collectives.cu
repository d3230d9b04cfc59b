// K6 / K7: data-parallel gradient reduce-scatter and parameter all-gather over NVLink peer memory.
//
// Every rank of a ZeRO shard group maps its peers' gradient and parameter arenas (CUDA IPC) and a small
// symmetric flag array.  A bucket's collective is a pull:
//   * reduce-scatter (fp32 gradients): rank z reads its shard's slice of the bucket from every rank r in the
//     fixed order r = 0..n-1, sums, and writes the sum in place into its own arena (the slice nobody else reads);
//   * all-gather (parameters): rank z copies every peer r's own shard of the bucket into its arena.
// Readiness is a flag per (collective, bucket, source rank) holding the step's epoch: `dp_signal` stores it
// (release, system scope, after a system fence) into that slot of every peer's flag array once the source's
// data is final on its stream; a pulling CTA waits (acquire, bounded by wall clock) for the flags of every
// source before it reads.  A pull never waits on another pull, and the fixed summation order makes the reduced
// gradients identical run to run.  Reuse of the arenas is ordered by one barrier over the same flag memory
// after a step's reduce-scatters (`sym_barrier`), issued by the host.
//
// On a timeout the kernel records 0x6000 | source rank in the device error flag and skips the bucket (no trap).
#include "../include/common.cuh"

namespace emb {

namespace {

struct Ptrs8 {
  uint64_t p[8];
};

__device__ __forceinline__ uint64_t gtime_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait until flags[slot * n + r] >= epoch (wrap-safe) for every r in [0, n); false on timeout.
__device__ bool wait_sources(const uint32_t* flags, int slot, int n, uint32_t epoch, uint64_t limit_ns, int* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = gtime_ns();
    for (int r = 0; r < n && ok; ++r) {
      const uint32_t* f = flags + (size_t)slot * n + r;
      for (uint64_t it = 0;; ++it) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if ((int32_t)(v - epoch) >= 0) break;
        if ((it & 255) == 255 && gtime_ns() - t0 > limit_ns) {
          atomicCAS(err, 0, 0x6000 | r);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  return ok != 0;
}

__global__ void dp_signal_kernel(Ptrs8 flags, int n, int me, int slot0, int nslots, uint32_t epoch) {
  // every write issued on this stream before the signal (gradient accumulation, optimizer emit) is visible
  // system-wide before any peer can observe the flag
  __threadfence_system();
  for (int i = threadIdx.x; i < nslots * n; i += blockDim.x) {
    const int s = slot0 + i / n, d = i % n;
    uint32_t* f = reinterpret_cast<uint32_t*>(flags.p[d]) + (size_t)s * n + me;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(epoch) : "memory");
  }
}

// out[i] = sum_r src_r[i] for i < count (fp32, 16-byte vectors when aligned); src_r = peers[r] + off.
__global__ void dp_rs_pull_kernel(Ptrs8 peers, int n, int me, uint64_t off, int64_t count, const uint32_t* flags,
                                  int slot, uint32_t epoch, uint64_t limit_ns, int* err) {
  if (!wait_sources(flags, slot, n, epoch, limit_ns, err)) return;
  float* out = reinterpret_cast<float*>(peers.p[me] + off);
  const bool vec = ((off | (uint64_t)count * 4) & 15) == 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    const int64_t nv = count / 4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += stride) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < n; ++r) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(peers.p[r] + off) + i);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
      reinterpret_cast<float4*>(out)[i] = acc;
    }
  } else {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += stride) {
      float acc = 0.f;
      for (int r = 0; r < n; ++r) acc += __ldcg(reinterpret_cast<const float*>(peers.p[r] + off) + i);
      out[i] = acc;
    }
  }
}

// For every source r != me: bytes [off + r * shard_bytes, +shard_bytes) of peers[r] -> the same bytes locally.
__global__ void dp_ag_pull_kernel(Ptrs8 peers, int n, int me, uint64_t off, uint64_t shard_bytes,
                                  const uint32_t* flags, int slot, uint32_t epoch, uint64_t limit_ns, int* err) {
  if (!wait_sources(flags, slot, n, epoch, limit_ns, err)) return;
  const bool vec = ((off | shard_bytes) & 15) == 0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int r = 0; r < n; ++r) {
    if (r == me) continue;
    const uint64_t o = off + (uint64_t)r * shard_bytes;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(peers.p[r] + o);
    uint8_t* dst = reinterpret_cast<uint8_t*>(peers.p[me] + o);
    if (vec) {
      const int64_t nv = shard_bytes / 16;
      for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += stride)
        reinterpret_cast<uint4*>(dst)[i] = __ldcg(reinterpret_cast<const uint4*>(src) + i);
    } else {
      for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)shard_bytes; i += stride)
        dst[i] = src[i];
    }
  }
}

Ptrs8 to_ptrs(const at::Tensor& t, int n) {
  TORCH_CHECK(!t.is_cuda() && t.scalar_type() == at::kLong && t.numel() == n && n >= 1 && n <= 8,
              "peer pointers: int64 CPU tensor of 1..8 entries");
  Ptrs8 p{};
  auto c = t.contiguous();
  for (int i = 0; i < n; ++i) p.p[i] = (uint64_t)c.data_ptr<int64_t>()[i];
  return p;
}

int pull_grid(int64_t bytes) {
  const int64_t want = (bytes + 65535) / 65536;  // ~64 KiB per CTA
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)num_sms() * 2));
}

}  // namespace

// flags: int64 [n] flag-array base of every rank (as mapped here); slots [slot0, slot0 + nslots) are signalled.
void dp_signal(at::Tensor flags, int64_t me, int64_t slot0, int64_t nslots, int64_t epoch) {
  const int n = (int)flags.numel();
  Ptrs8 f = to_ptrs(flags, n);
  dp_signal_kernel<<<1, 256, 0, cur_stream()>>>(f, n, (int)me, (int)slot0, (int)nslots, (uint32_t)epoch);
  EMB_LAUNCH_CHECK();
  count_launch();
}

// peers: int64 [n] gradient-arena base of every rank; reduces count fp32 elements at byte offset off.
void dp_rs_pull(at::Tensor peers, int64_t me, int64_t off, int64_t count, at::Tensor flags, int64_t slot,
                int64_t epoch, int64_t timeout_ms) {
  const int n = (int)peers.numel();
  Ptrs8 p = to_ptrs(peers, n);
  Ptrs8 f = to_ptrs(flags, n);
  TORCH_CHECK(me >= 0 && me < n && off >= 0 && count >= 0);
  if (count == 0) return;
  dp_rs_pull_kernel<<<pull_grid(count * 4 * n), 256, 0, cur_stream()>>>(
      p, n, (int)me, (uint64_t)off, count, reinterpret_cast<const uint32_t*>(f.p[me]), (int)slot,
      (uint32_t)epoch, (uint64_t)std::max<int64_t>(1, timeout_ms) * 1000000ull, device_err_flag(kErrComm));
  EMB_LAUNCH_CHECK();
  count_launch();
}

// peers: int64 [n] parameter-arena base of every rank; the bucket starts at byte off, shard r at off + r * shard.
void dp_ag_pull(at::Tensor peers, int64_t me, int64_t off, int64_t shard_bytes, at::Tensor flags, int64_t slot,
                int64_t epoch, int64_t timeout_ms) {
  const int n = (int)peers.numel();
  Ptrs8 p = to_ptrs(peers, n);
  Ptrs8 f = to_ptrs(flags, n);
  TORCH_CHECK(me >= 0 && me < n && off >= 0 && shard_bytes >= 0);
  if (shard_bytes == 0 || n == 1) return;
  dp_ag_pull_kernel<<<pull_grid(shard_bytes * (n - 1)), 256, 0, cur_stream()>>>(
      p, n, (int)me, (uint64_t)off, (uint64_t)shard_bytes, reinterpret_cast<const uint32_t*>(f.p[me]), (int)slot,
      (uint32_t)epoch, (uint64_t)std::max<int64_t>(1, timeout_ms) * 1000000ull, device_err_flag(kErrComm));
  EMB_LAUNCH_CHECK();
  count_launch();
}

}  // namespace emb
