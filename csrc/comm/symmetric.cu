// Symmetric-memory signalling between the GPUs of one NVSwitch domain.
//
// Every rank of a group owns one arena whose first bytes are a signal array (one uint32 slot per peer) and
// maps every peer's arena (CUDA IPC).  `sym_barrier` is a stream-ordered barrier over that memory: rank `me`
// stores the epoch into slot `me` of every peer's signal array (release, system scope) and waits until every
// peer has stored an epoch >= its own into the corresponding slot of its own array (acquire, system scope).
// It replaces a 1-element NCCL all-reduce used as a barrier between fused GEMM/collective launches at a
// fraction of its latency (one small block, no NCCL proxy, no reduction).
//
// The wait is bounded by a wall-clock limit read from %globaltimer (and an iteration cap as a backstop): on
// expiry the kernel records 0x5000 | peer in the device error flag and returns, so the context stays usable
// and the host sees the failure at its next check.
#include "../include/common.cuh"

namespace emb {

namespace {

struct SigPtrs {
  uint32_t* p[8];
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void sym_barrier_kernel(SigPtrs sig, int me, int tp, uint32_t epoch, uint64_t limit_ns, int* err) {
  const int j = threadIdx.x;
  if (j < tp && j != me) {
    // make every write this GPU issued before the barrier (earlier kernels on the stream, peer stores
    // included) visible system-wide before the peer can observe the signal
    __threadfence_system();
    uint32_t* remote = sig.p[j] + me;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
    const uint32_t* mine = sig.p[me] + j;
    const uint64_t t0 = globaltimer_ns();
    for (uint64_t it = 0;; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
      if ((int32_t)(v - epoch) >= 0) break;
      if ((it & 255) == 255 && (globaltimer_ns() - t0 > limit_ns || it > (1ull << 34))) {
        atomicCAS(err, 0, 0x5000 | j);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
}

int* comm_err_flag() { return device_err_flag(kErrComm); }

}  // namespace

// sig_ptrs: int64 CPU [tp] - signal-array base address of every rank as mapped in this process (own first
// bytes of the local arena at index `me`).  epoch: strictly increasing per barrier on this group.
void sym_barrier(at::Tensor sig_ptrs, int64_t me, int64_t epoch, int64_t timeout_ms) {
  TORCH_CHECK(!sig_ptrs.is_cuda() && sig_ptrs.scalar_type() == at::kLong, "sig_ptrs: int64 CPU tensor");
  const int64_t tp = sig_ptrs.numel();
  TORCH_CHECK(tp >= 1 && tp <= 8 && me >= 0 && me < tp, "sym_barrier: 1 <= tp <= 8, 0 <= me < tp");
  if (tp == 1) return;
  SigPtrs s{};
  auto pc = sig_ptrs.contiguous();
  for (int64_t i = 0; i < tp; ++i) {
    s.p[i] = reinterpret_cast<uint32_t*>(pc.data_ptr<int64_t>()[i]);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(s.p[i]) & 3) == 0, "signal array must be 4-byte aligned");
  }
  sym_barrier_kernel<<<1, 32, 0, cur_stream()>>>(s, (int)me, (int)tp, (uint32_t)epoch,
                                                 (uint64_t)std::max<int64_t>(1, timeout_ms) * 1000000ull,
                                                 comm_err_flag());
  EMB_LAUNCH_CHECK();
  count_launch();
}

int64_t comm_error_flag() {
  int v = 0;
  EMB_CUDA_CHECK(cudaMemcpy(&v, comm_err_flag(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void comm_clear_error() { EMB_CUDA_CHECK(cudaMemset(comm_err_flag(), 0, sizeof(int))); }

}  // namespace emb
