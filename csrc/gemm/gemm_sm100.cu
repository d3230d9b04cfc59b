// K3: dense bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   C[M, N] (=|+=) A[M, K] * B[K, N]      A, B bf16;  C bf16 (store) or fp32 (store / accumulate)
//
// Operand layouts (per the torch-style call gemm(a, b, trans_a, trans_b)):
//   A is K-major when a is [M, K] row-major, MN-major when a is [K, M] row-major (trans_a);
//   B is K-major when b is [N, K] row-major (trans_b), MN-major when b is [K, N] row-major.
// So fprop (x @ W^T), dgrad (dy @ W) and wgrad (dy^T @ x, accumulated into the fp32 main_grad) all run
// without a transpose copy.
//
// Structure: persistent kernel, one CTA per SM, 192 threads, warp-specialised:
//   warp 0      - TMA producer: one elected thread streams 128x64 A and 256x64 B tiles (128-byte swizzle)
//                 into a 4-stage shared-memory ring, completing on per-stage mbarriers;
//   warp 1      - allocates 512 TMEM columns (two 128x256 fp32 accumulators) and one elected thread issues
//                 tcgen05.mma (M=128, N=256, K=16) with shared-memory descriptors, committing each stage back
//                 to the producer and each finished accumulator to the epilogue;
//   warps 2..5  - epilogue: tcgen05.ld 32x32b from their TMEM lane quarter, convert, store to global memory,
//                 while the MMA warp already accumulates the next tile into the other TMEM buffer.
// No TMA multicast is used anywhere (this kernel also runs inside multi-GPU jobs).
//
// Every mbarrier wait is bounded; on a timeout the kernel records an error code in a device flag that the
// host checks, and the waiting role stops issuing work (no trap).
#include <cudaTypedefs.h>

#include <cstdlib>

#include <atomic>

#include "../include/common.cuh"

namespace emb {
namespace gk {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KiB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KiB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t WAIT_LIMIT = 1u << 28;  // ~seconds of polling before giving up

// ------------------------------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and records `code` in *err) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(32);
  }
  atomicExch(err, code);
  return false;
}
__device__ __forceinline__ uint64_t gtimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the roles on the main loop's critical path (TMA producer, MMA issuer): polls without
// __nanosleep, whose wake-up granularity otherwise lands in the producer -> MMA -> commit -> producer ring on
// every stage.  Gives up after ~4 s of wall clock (read every 4096 polls), recording `code` in *err.
__device__ __forceinline__ bool mbar_wait_hot(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = gtimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 4095) == 0 && gtimer_ns() - t0 > 4000000000ull) break;
  }
  atomicExch(err, code);
  return false;
}
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm100 "version 1"), 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16: bf16 x bf16 -> fp32, M=128, N=256.
__host__ __device__ constexpr uint32_t make_idesc(bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                     // D = F32
         | (1u << 7)                   // A = BF16
         | (1u << 10)                  // B = BF16
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define TMEM_LD_32(taddr, r)                                                                                        \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19," \
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                                    \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),      \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),     \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                   \
      : "r"(taddr))

struct Params {
  void* C;
  int M, N, K;
  int ldc;
  int out_fp32;    // C is fp32 (else bf16)
  int accumulate;  // C += (fp32 only)
  int a_mn, b_mn;  // operand majorness
  int* err;
  int split_tail;  // 2-SM kernel: run the last partial wave as 256 x 128 half tiles when they fit in one wave
  int m_fast;      // measurement only (EMB_GEMM_RASTER=m): m blocks vary fastest whatever the shape
  int no_store;    // 2-SM kernel, measurement only: read the accumulators but write no output
  int c_tma;       // 2-SM kernel: C is written (or add-reduced) through the tensor map tmC, one 32-row block per
                   // epilogue warp and bulk operation (else row by row)
  int probe;       // 2-SM kernel, measurement only: bit 0 issues no MMAs, bit 1 loads no operands (the
                   // pipeline's barriers still run), isolating the main loop's feed from its math
  // grouped GEMM (1-SM kernel; MoE experts).  group_mode 1: A rows come in per-group segments padded to BM,
  // group_info[m tile] = group of that tile (-1: skip); B holds every group's matrix stacked along its row
  // coordinate, group g's rows start at g * group_b_stride.  group_mode 2 (weight gradient): group g reduces
  // over rows [group_info[g], group_info[g + 1]) of A and B (multiples of BK) into C + g * group_c_stride.
  int group_mode;
  const int* group_info;
  int groups;
  int group_b_stride;
  long long group_c_stride;
  // reduce-scatter epilogue (2-SM kernel only): when scatter != 0, output row `row` belongs to TP rank
  // owner = row / rows_per_rank and is written (bf16) into that rank's staging buffer peer_out[owner] at slot
  // `my_slot`: peer_out[owner] + (my_slot * rows_per_rank + row % rows_per_rank) * ldc + col.
  int scatter;
  int rows_per_rank;
  int my_slot;
  void* peer_out[8];
  // all-gather prologue (2-SM kernel, AG template only), push mode.  A = ag_local [M, K] (K-major), chunk c =
  // rows [c*rows_per_rank, (c+1)*rows_per_rank) coming from TP rank c.  This rank's own chunk is already in
  // place; its copy warps store this rank's shard (ag_shard, [rows_per_rank, K] contiguous) into every peer's
  // buffer (ag_dst[peer], same layout) in units of AG_UNIT_ROWS rows and after each unit set the peer's flag
  // ag_flags[peer][my_slot * ag_units_max + unit] = ag_epoch (release, system scope).  The producer of a tile
  // whose rows come from chunk c waits for the flags of those rows in its own array ag_flags[my_slot].
  // ready[0] hands out units (zeroed by the host before the launch).
  void* ag_dst[8];
  uint32_t* ag_flags[8];
  const void* ag_shard;
  void* ag_local;
  int* ready;
  int ag_tp;
  int ag_units_max;
  uint32_t ag_epoch;
};

struct TileInfo {
  int m0, n0, kb0, kb1, b_off;
  long long c_off;
};

// Output tile t of the persistent schedule (the dimension with fewer tiles fastest; m fastest in the grouped
// modes, whose per-tile group lookup is by m block); false when the tile has no work (grouped modes).
__device__ __forceinline__ bool tile_info(const Params& p, int t, int tiles_m, int tiles_n, int nk, TileInfo& ti) {
  if (p.group_mode == 2) {
    const int per = tiles_m * tiles_n;
    const int g = t / per, r = t - g * per;
    ti.m0 = (r % tiles_m) * BM;
    ti.n0 = (r / tiles_m) * BN;
    ti.kb0 = p.group_info[g] / BK;
    ti.kb1 = p.group_info[g + 1] / BK;
    ti.b_off = 0;
    ti.c_off = (long long)g * p.group_c_stride;
    return ti.kb1 > ti.kb0;
  }
  if (p.group_mode == 0 && tiles_n < tiles_m && !p.m_fast) {
    ti.m0 = (t / tiles_n) * BM;
    ti.n0 = (t % tiles_n) * BN;
  } else {
    ti.m0 = (t % tiles_m) * BM;
    ti.n0 = (t / tiles_m) * BN;
  }
  ti.kb0 = 0;
  ti.kb1 = nk;
  ti.b_off = 0;
  ti.c_off = 0;
  if (p.group_mode == 1) {
    const int g = p.group_info[t % tiles_m];
    if (g < 0) return false;
    ti.b_off = g * p.group_b_stride;
  }
  return true;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles_m = (p.M + BM - 1) / BM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n * (p.group_mode == 2 ? p.groups : 1);
  const int nk = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // one arrive per epilogue warp
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        TileInfo ti;
        if (!tile_info(p, t, tiles_m, tiles_n, nk, ti)) continue;
        const int m0 = ti.m0, n0 = ti.n0;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_hot(&empty[s], ph ^ 1, p.err, 1) || *abort_flag) { ok = false; *abort_flag = 1; break; }
          mbar_expect_tx(&full[s], STAGE_BYTES);
          uint8_t* a_dst = sA + s * A_STAGE_BYTES;
          uint8_t* b_dst = sB + s * B_STAGE_BYTES;
          const int k0 = kb * BK;
          if (!p.a_mn) {
            tma_load_2d(a_dst, &tmA, &full[s], k0, m0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[s], m0, k0);
            tma_load_2d(a_dst + 8192, &tmA, &full[s], m0 + 64, k0);
          }
          if (!p.b_mn) {
            tma_load_2d(b_dst, &tmB, &full[s], k0, n0 + ti.b_off);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_2d(b_dst + j * 8192, &tmB, &full[s], n0 + 64 * j, k0 + ti.b_off);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(p.a_mn, p.b_mn);
      // per-K16-step descriptor advance and LBO/SBO for each operand layout
      const uint32_t a_lbo = p.a_mn ? 8192 : 16, a_sbo = 1024, a_step = p.a_mn ? 2048 : 32;
      const uint32_t b_lbo = p.b_mn ? 8192 : 16, b_sbo = 1024, b_step = p.b_mn ? 2048 : 32;
      int it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        TileInfo ti;
        if (!tile_info(p, t, tiles_m, tiles_n, nk, ti)) continue;
        const int buf = local & 1;
        const uint32_t tph = (local >> 1) & 1;
        ++local;
        if (!mbar_wait_hot(&tempty[buf], tph ^ 1, p.err, 2) || *abort_flag) { ok = false; *abort_flag = 1; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait_hot(&full[s], ph, p.err, 3) || *abort_flag) { ok = false; *abort_flag = 1; break; }
          // (no tcgen05 fence here: the TMA -> MMA hand-off is ordered by the mbarrier alone)
          const uint32_t a_addr = smem_u32(sA + s * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sB + s * B_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = smem_desc(a_addr + k * a_step, a_lbo, a_sbo);
            const uint64_t bd = smem_desc(b_addr + k * b_step, b_lbo, b_sbo);
            mma_bf16(d_tmem, ad, bd, idesc, ((kb - ti.kb0) | k) != 0);
          }
          mma_commit(&empty[s]);  // frees the smem stage once these MMAs have read it
        }
        if (ok) mma_commit(&tfull[buf]);  // accumulator ready for the epilogue
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      TileInfo ti;
      if (!tile_info(p, t, tiles_m, tiles_n, nk, ti)) continue;
      const int buf = local & 1;
      const uint32_t tph = (local >> 1) & 1;
      ++local;
      if (!mbar_wait(&tfull[buf], tph, p.err, 4) || *abort_flag) { *abort_flag = 1; break; }
      tc_fence_after();
      const int m0 = ti.m0;
      const int n0 = ti.n0;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN + c * 32;
        TMEM_LD_32(taddr, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= p.N) continue;
        const int ncols = min(32, p.N - col0);
        if (p.out_fp32) {
          float* dst = reinterpret_cast<float*>(p.C) + ti.c_off + (size_t)row * p.ldc + col0;
          if (ncols == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
              float4* d4 = reinterpret_cast<float4*>(dst) + v;
              if (p.accumulate) {
                float4 old = *d4;
                o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
              }
              *d4 = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < ncols) {
                float v = __uint_as_float(r[j]);
                dst[j] = p.accumulate ? dst[j] + v : v;
              }
            }
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + ti.c_off + (size_t)row * p.ldc + col0;
          if (ncols == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[8 * v + j]);
              reinterpret_cast<uint4*>(dst)[v] = pack8(f);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

}  // namespace gk

// ------------------------------------------------------------------------------------------ 2-SM variant
// A cluster of two CTAs on two SMs computes a 256x256 tile with tcgen05.mma.cta_group::2 (M=256, N=256):
// CTA r loads rows [128r, 128r+128) of the A tile and rows [128r, 128r+128) of the B tile (N-half) into its
// own shared memory, so each SM streams 32 KiB per 64-deep k-block instead of 48 KiB for the same MMA work,
// and each SM's TMEM holds its 128 rows x 256 columns of the accumulator.  Protocol:
//   full[s]   - leader CTA only; its producer arms it with the bytes of both CTAs; both CTAs' TMA loads
//               complete on it (cta_group::2 form, barrier addressed in the leader through mapa);
//   empty[s]  - in both CTAs; the leader's MMA commit arrives on both (multicast to the pair, mask 0b11);
//   tfull[b]  - in both CTAs; the leader's commit after the last k-block of a tile arrives on both;
//   tempty[b] - leader only; all 8 epilogue warps of the pair arrive (remote arrive from the peer).
// TMA loads never use cluster multicast.
namespace gk2 {
// Cycle counters of the main-loop roles (probe bit 2, measurement only), read by gemm_debug_counters().
__device__ unsigned long long g_dbg[16];
__device__ __forceinline__ unsigned long long clk() {
  unsigned long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}
constexpr int BM = 256, BN = 256;
// K depth of a pipeline stage: 64 (5 stages of 32 KiB per CTA) or 128 (3 stages of 64 KiB, half as many
// barrier round trips and MMA-issue loop iterations per unit of tensor work).
template <int BK_>
struct Cfg {
  static constexpr int BK = BK_;
  static constexpr int STAGES = BK_ == 64 ? 5 : 3;
  static constexpr int A_HALF = 128 * BK_ * 2;  // per CTA
  static constexpr int B_HALF = 128 * BK_ * 2;
  static constexpr int STAGE_BYTES = A_HALF + B_HALF;
  static constexpr int EPI_BUFS = BK_ == 64 ? 2 : 1;
};
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 192;
constexpr int NUM_THREADS_AG = 256;  // + 2 copy warps for the all-gather prologue
constexpr int AG_UNIT_ROWS = 32;     // rows per pushed unit (one readiness flag each)
constexpr int EPI_STRIDE = 144;  // 128-byte rows padded to 144 B: a warp's 16-byte writes hit 4-way banks
// Epilogue staging: two 16 KiB buffers of four 32-row x 128-byte warp blocks (tensor-map path), which also hold
// EPI_BUFS padded 128-row buffers for the row-by-row path.
template <int BK_>
constexpr int epi_bytes() {
  return Cfg<BK_>::EPI_BUFS * 128 * EPI_STRIDE > 32768 ? Cfg<BK_>::EPI_BUFS * 128 * EPI_STRIDE : 32768;
}
template <int BK_>
constexpr int smem_bytes() {
  return Cfg<BK_>::STAGES * Cfg<BK_>::STAGE_BYTES + epi_bytes<BK_>() + 1024 + 256;
}
static_assert(smem_bytes<64>() <= 232448 && smem_bytes<128>() <= 232448, "2-SM GEMM shared memory");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(cta));
  return r;
}
__device__ __forceinline__ void remote_arrive(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(gk::smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          gk::smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}
__host__ __device__ constexpr uint32_t make_idesc2(bool a_mn, bool b_mn, int n = BN) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// bounded acquire-wait until the flag written by a peer GPU reaches `epoch` (wrap-safe); false on timeout
__device__ __forceinline__ bool wait_epoch(const uint32_t* flag, uint32_t epoch, int* err, int code) {
  for (uint32_t i = 0; i < gk::WAIT_LIMIT; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if ((int32_t)(v - epoch) >= 0) {
      asm volatile("fence.proxy.async.global;" ::: "memory");  // the TMA reads that follow see the pushed rows
      return true;
    }
    __nanosleep(64);
  }
  atomicExch(err, code);
  return false;
}

template <bool AG, int BK_>
__global__ void __launch_bounds__(AG ? NUM_THREADS_AG : NUM_THREADS, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, gk::Params p) {
  using namespace gk;
  constexpr int BK = BK_, STAGES = Cfg<BK_>::STAGES, A_HALF = Cfg<BK_>::A_HALF, B_HALF = Cfg<BK_>::B_HALF;
  constexpr int STAGE_BYTES = Cfg<BK_>::STAGE_BYTES, EPI_BUFS = Cfg<BK_>::EPI_BUFS;
  constexpr int EPI_BYTES = epi_bytes<BK_>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_HALF;
  uint8_t* sEpi = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES + EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;  // [2]
  uint64_t* tempty = tfull + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int tiles_m = (p.M + BM - 1) / BM;
  const int tiles_n = (p.N + BN - 1) / BN;
  const int num_tiles = tiles_m * tiles_n;
  const int nk = (p.K + BK - 1) / BK;
  // tile -> (m block, n block).  The dimension with fewer tiles varies fastest, so the tiles in flight at once
  // share few panels of the long operand and those panels stay in L2 while every tile that needs them runs
  // (a 32000 x 4096 weight gradient with m fastest streamed each 2 MB A panel from DRAM once per n block:
  // 0.75x of cuBLAS).  With the all-gather prologue, n varies fastest and m blocks start at this rank's own
  // chunk, so the first tiles never wait for a peer's rows.
  const int my_chunk = AG ? p.my_slot : 0;
  const int mt_per_chunk = AG ? p.rows_per_rank / BM : 1;
  const bool n_fast = AG || (tiles_n < tiles_m && !p.m_fast);
  auto tile_m = [&](int t) -> int {
    if (AG) return (t / tiles_n + my_chunk * mt_per_chunk) % tiles_m;
    return n_fast ? t / tiles_n : t % tiles_m;
  };
  auto tile_n = [&](int t) -> int { return n_fast ? t % tiles_n : t / tiles_m; };
  // Tail split (not with the all-gather prologue): when the tiles of the last, partial wave could run as twice
  // as many 256 x 128 halves in one wave, they do - the last wave then takes half as long (4096 x 4096
  // outputs: 256 tiles on 74 clusters = 3 full waves + 34 tiles -> 3.5 wave-times instead of 4).  Work unit u
  // maps to tile unit_tile(u); unit_half(u) is -1 for a whole tile, else which 128-column half.
  const int tail = AG ? 0 : num_tiles % num_clusters;
  const bool split_tail = !AG && p.split_tail && tail > 0 && 2 * tail <= num_clusters;
  const int full_tiles = split_tail ? num_tiles - tail : num_tiles;
  const int num_units = split_tail ? full_tiles + 2 * tail : num_tiles;
  auto unit_tile = [&](int u) -> int { return u < full_tiles ? u : full_tiles + ((u - full_tiles) >> 1); };
  auto unit_half = [&](int u) -> int { return u < full_tiles ? -1 : ((u - full_tiles) & 1); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const bool timing = (p.probe & 4) != 0;
  if (warp == 0) {
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      unsigned long long t_begin = timing ? clk() : 0, t_wait = 0, t_issue = 0;
      for (int u = cluster_id; u < num_units && ok; u += num_clusters) {
        const int t = unit_tile(u), hf = unit_half(u);
        const int m0 = tile_m(t) * BM + 128 * rank;
        // each CTA supplies half of the tile's B columns: 128 of a whole tile, 64 of a half tile (the loaded box
        // stays 128 rows; the MMA reads its first 64)
        const int n0 = tile_n(t) * BN + (hf > 0 ? 128 : 0) + (hf >= 0 ? 64 : 128) * rank;
        if (AG) {
          const int c = m0 / p.rows_per_rank;
          if (c != my_chunk) {
            const int u0 = (m0 - c * p.rows_per_rank) / AG_UNIT_ROWS;
            const uint32_t* f = p.ag_flags[my_chunk] + c * p.ag_units_max;
            bool got = true;
            for (int u = u0; u < u0 + 128 / AG_UNIT_ROWS && got; ++u) got = wait_epoch(f + u, p.ag_epoch, p.err, 15);
            if (!got) { ok = false; *abort_flag = 1; break; }
          }
        }
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const unsigned long long t0 = timing ? clk() : 0;
          if (!mbar_wait_hot(&empty[s], ph ^ 1, p.err, 11) || *abort_flag) { ok = false; *abort_flag = 1; break; }
          const unsigned long long t1 = timing ? clk() : 0;
          t_wait += t1 - t0;
          const uint32_t bar = mapa(smem_u32(&full[s]), 0);
          if (p.probe & 2) {
            if (leader) mbar_arrive(&full[s]);
            continue;
          }
          if (leader) mbar_expect_tx(&full[s], 2 * STAGE_BYTES);
          uint8_t* a_dst = sA + s * A_HALF;
          uint8_t* b_dst = sB + s * B_HALF;
          const int k0 = kb * BK;
          // K-major: 64-wide K panels of 128 rows, 16 KiB apart.  MN-major: 64-wide M (N) panels of BK K-rows,
          // BK * 128 bytes apart, one {64, BK} box each (the MN-major tensor maps have BK-row boxes).
          if (!p.a_mn) {
#pragma unroll
            for (int h = 0; h < BK / 64; ++h) tma_load_2d_pair(a_dst + h * 16384, &tmA, bar, k0 + 64 * h, m0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, bar, m0, k0);
            tma_load_2d_pair(a_dst + BK * 128, &tmA, bar, m0 + 64, k0);
          }
          if (!p.b_mn) {
#pragma unroll
            for (int h = 0; h < BK / 64; ++h) tma_load_2d_pair(b_dst + h * 16384, &tmB, bar, k0 + 64 * h, n0);
          } else {
            tma_load_2d_pair(b_dst, &tmB, bar, n0, k0);
            tma_load_2d_pair(b_dst + BK * 128, &tmB, bar, n0 + 64, k0);
          }
          if (timing) t_issue += clk() - t1;
        }
      }
      if (timing && leader) {
        atomicAdd(&g_dbg[4], t_wait);
        atomicAdd(&g_dbg[5], t_issue);
        atomicAdd(&g_dbg[6], clk() - t_begin);
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      const uint32_t idesc_full = make_idesc2(p.a_mn, p.b_mn);
      const uint32_t idesc_half = make_idesc2(p.a_mn, p.b_mn, BN / 2);
      // descriptors of stage 0 at k-step 0; a k-step / stage advances the 14-bit start-address field only
      const uint64_t a_desc0 = smem_desc(smem_u32(sA), p.a_mn ? BK * 128 : 16, 1024);
      const uint64_t b_desc0 = smem_desc(smem_u32(sB), p.b_mn ? BK * 128 : 16, 1024);
      auto kstep = [&](bool mn, int k) -> uint32_t {  // byte offset of k-step k (16 deep) inside a stage
        return mn ? (uint32_t)k * 2048u : (uint32_t)(k >> 2) * 16384u + (uint32_t)(k & 3) * 32u;
      };
      int it = 0, local = 0;
      bool ok = true;
      unsigned long long t_begin = timing ? clk() : 0, t_wf = 0, t_is = 0, t_wt = 0, nkb = 0;
      for (int u = cluster_id; u < num_units && ok; u += num_clusters, ++local) {
        const uint32_t idesc = unit_half(u) >= 0 ? idesc_half : idesc_full;
        const int buf = local & 1;
        const uint32_t tph = (local >> 1) & 1;
        const unsigned long long ta = timing ? clk() : 0;
        if (!mbar_wait_hot(&tempty[buf], tph ^ 1, p.err, 12) || *abort_flag) { ok = false; *abort_flag = 1; break; }
        if (timing) t_wt += clk() - ta;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const unsigned long long t0 = timing ? clk() : 0;
          if (!mbar_wait_hot(&full[s], ph, p.err, 13) || *abort_flag) { ok = false; *abort_flag = 1; break; }
          const unsigned long long t1 = timing ? clk() : 0;
          t_wf += t1 - t0;
          // (no tcgen05 fence here: the TMA -> MMA hand-off is ordered by the mbarrier alone)
          const uint64_t a_s = a_desc0 + (uint64_t)((s * A_HALF) >> 4);
          const uint64_t b_s = b_desc0 + (uint64_t)((s * B_HALF) >> 4);
          if (!(p.probe & 1)) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              mma_pair(d_tmem, a_s + (kstep(p.a_mn, k) >> 4), b_s + (kstep(p.b_mn, k) >> 4), idesc, (kb | k) != 0);
            }
          }
          commit_pair(&empty[s]);
          if (timing) { t_is += clk() - t1; ++nkb; }
        }
        if (ok) commit_pair(&tfull[buf]);
      }
      if (timing) {
        atomicAdd(&g_dbg[0], t_wf);
        atomicAdd(&g_dbg[1], t_is);
        atomicAdd(&g_dbg[2], t_wt);
        atomicAdd(&g_dbg[3], clk() - t_begin);
        atomicAdd(&g_dbg[9], nkb);
        atomicAdd(&g_dbg[10], 1ull);
      }
    }
  } else if (AG && warp >= 6) {
    // ------------------------------------------------------------------ all-gather push warps
    // Units (peer d, AG_UNIT_ROWS rows of this rank's shard) are claimed through one atomic counter by the
    // copy warps of every CTA (so resident CTAs finish all pushes even if others are not yet scheduled).
    // Peers are served in the order in which they consume this rank's chunk (rank me-1 first).  A unit is
    // read from local HBM and stored into the peer's buffer over NVLink (posted writes), then the peer's flag
    // for the unit is released at system scope.
    __shared__ int claimed;
    const int ct = threadIdx.x - 192;  // 0..63
    const size_t row_bytes = (size_t)p.K * 2;
    const int units = p.rows_per_rank / AG_UNIT_ROWS;
    const int total = (p.ag_tp - 1) * units;
    const size_t nv = (size_t)AG_UNIT_ROWS * row_bytes / 16;
    while (true) {
      if (ct == 0) claimed = atomicAdd(p.ready, 1);
      asm volatile("bar.sync 2, 64;" ::: "memory");
      const int u = claimed;
      asm volatile("bar.sync 2, 64;" ::: "memory");
      if (u >= total) break;
      const int d = u / units, j = u % units;
      const int dest = (my_chunk - 1 - d + 2 * p.ag_tp) % p.ag_tp;
      const size_t src_off = (size_t)j * AG_UNIT_ROWS * row_bytes;
      const size_t dst_off = ((size_t)my_chunk * p.rows_per_rank + (size_t)j * AG_UNIT_ROWS) * row_bytes;
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.ag_shard) + src_off);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.ag_dst[dest]) + dst_off);
      size_t v = ct;
      for (; v + 64 * 7 < nv; v += 64 * 8) {
        uint4 x[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) x[q] = src[v + 64 * q];
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[v + 64 * q] = x[q];
      }
      for (; v < nv; v += 64) dst[v] = src[v];
      __threadfence_system();
      asm volatile("bar.sync 2, 64;" ::: "memory");
      if (ct == 0) {
        uint32_t* f = p.ag_flags[dest] + my_chunk * p.ag_units_max + j;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(p.ag_epoch) : "memory");
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row_in_half = quarter * 32 + lane;
    int local = 0;
    uint32_t epi_n = 0;  // bulk groups issued by this thread (selects the staging buffer)
    unsigned long long e_begin = timing ? clk() : 0, e_wait = 0;
    for (int u = cluster_id; u < num_units; u += num_clusters, ++local) {
      const int t = unit_tile(u), hf = unit_half(u);
      const int buf = local & 1;
      const uint32_t tph = (local >> 1) & 1;
      const unsigned long long ta = timing ? clk() : 0;
      if (!mbar_wait(&tfull[buf], tph, p.err, 14) || *abort_flag) { *abort_flag = 1; break; }
      if (timing) e_wait += clk() - ta;
      tc_fence_after();
      const int row = tile_m(t) * BM + 128 * rank + row_in_half;
      const int n0 = tile_n(t) * BN + (hf > 0 ? BN / 2 : 0);
      const int n_chunks = (hf >= 0 ? BN / 2 : BN) / 32;
      const bool row_ok = row < p.M;
      if (p.c_tma && !p.no_store) {
        // Each warp stages its 32 rows x 128 bytes (32 fp32 or 64 bf16 columns) in a 128-byte-swizzled block
        // (16-byte chunk j of row r at chunk j ^ (r & 7): conflict-free writes) and one lane hands the block to
        // the TMA unit: a tensor store, or an fp32 add-reduction into C for the accumulating weight gradient.
        // Out-of-range rows / columns are clipped by the tensor map.
        const int row0 = tile_m(t) * BM + 128 * rank + quarter * 32;
        const int cols = p.out_fp32 ? 32 : 64;
        const int steps = (hf >= 0 ? BN / 2 : BN) / cols;
#pragma unroll 1
        for (int c = 0; c < steps; ++c) {
          uint32_t r[64];
          // (a half tile's MMA ran with N = 128 into columns [0, 128) of the buffer, whichever half it is)
          const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN + c * cols;
          TMEM_LD_32(taddr, r);
          if (!p.out_fp32) TMEM_LD_32(taddr + 32, (r + 32));
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
          uint8_t* wbuf = sEpi + (epi_n & 1) * 16384 + quarter * 4096;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
          uint8_t* myrow = wbuf + lane * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 v;
            if (p.out_fp32) {
              v = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            } else {
              float f[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) f[q] = __uint_as_float(r[8 * j + q]);
              v = pack8(f);
            }
            *reinterpret_cast<uint4*>(myrow + ((j ^ (lane & 7)) << 4)) = v;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            const int x = n0 + c * cols;
            if (p.accumulate) {
              asm volatile(
                  "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                      reinterpret_cast<uint64_t>(&tmC)),
                  "r"(x), "r"(row0), "r"(smem_u32(wbuf))
                  : "memory");
            } else {
              asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                               reinterpret_cast<uint64_t>(&tmC)),
                           "r"(x), "r"(row0), "r"(smem_u32(wbuf))
                           : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          ++epi_n;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) remote_arrive(mapa(smem_u32(&tempty[buf]), 0));
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < n_chunks; ++c) {
        uint32_t r[32];
        const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + buf * BN + c * 32;
        TMEM_LD_32(taddr, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int col0 = n0 + c * 32;
        if (!row_ok || col0 >= p.N || p.no_store) continue;
        const int ncols = min(32, p.N - col0);
        void* gdst;
        if (p.scatter) {
          // fused reduce-scatter: this partial row chunk goes straight to its owner's staging slot (peer memory
          // over NVLink), handed to the bulk-copy engine below so the epilogue warps move on to the next chunk
          const int owner = row / p.rows_per_rank;
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.peer_out[owner]) +
                               ((size_t)p.my_slot * p.rows_per_rank + (row - owner * p.rows_per_rank)) * p.ldc + col0;
          if (ncols != 32 || (reinterpret_cast<uintptr_t>(dst) & 15) != 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
            continue;
          }
          gdst = dst;
        } else {
          gdst = p.out_fp32 ? (void*)(reinterpret_cast<float*>(p.C) + (size_t)row * p.ldc + col0)
                            : (void*)(reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col0);
        }
        if (ncols == 32 && ((reinterpret_cast<uintptr_t>(gdst) & 15) == 0)) {
          // stage the row chunk in shared memory and hand it to the bulk-copy engine: a plain store, or an
          // fp32 add-reduction into C (the wgrad accumulate), without the read-modify-write round trip
          uint8_t* srow = sEpi + (epi_n % EPI_BUFS) * (128 * EPI_STRIDE) + row_in_half * EPI_STRIDE;
          if constexpr (EPI_BUFS == 2) {
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          } else {
            asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
          }
          uint32_t bytes;
          if (p.out_fp32) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              *reinterpret_cast<float4*>(srow + v * 16) =
                  make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                              __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            }
            bytes = 128;
          } else {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[8 * v + j]);
              *reinterpret_cast<uint4*>(srow + v * 16) = pack8(f);
            }
            bytes = 64;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          if (p.accumulate) {
            asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(gdst),
                         "r"(smem_u32(srow)), "r"(bytes)
                         : "memory");
          } else {
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
                         "r"(smem_u32(srow)), "r"(bytes)
                         : "memory");
          }
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          ++epi_n;
          continue;
        }
        if (p.out_fp32) {
          float* dst = reinterpret_cast<float*>(p.C) + (size_t)row * p.ldc + col0;
          if (ncols == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              float4 o = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                     __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
              float4* d4 = reinterpret_cast<float4*>(dst) + v;
              if (p.accumulate) {
                float4 old = *d4;
                o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
              }
              *d4 = o;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < ncols) {
                float v = __uint_as_float(r[j]);
                dst[j] = p.accumulate ? dst[j] + v : v;
              }
            }
          }
        } else {
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + (size_t)row * p.ldc + col0;
          if (ncols == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[8 * v + j]);
              reinterpret_cast<uint4*>(dst)[v] = pack8(f);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols) dst[j] = __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(mapa(smem_u32(&tempty[buf]), 0));
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (timing && leader && warp == 2 && lane == 0) {
      atomicAdd(&g_dbg[7], e_wait);
      atomicAdd(&g_dbg[8], clk() - e_begin);
    }
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}
}  // namespace gk2

namespace gk {
// ------------------------------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    EMB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [rows, cols] (cols contiguous), box {box_cols, box_rows}.
static CUtensorMap make_map(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

static int* err_flag() { return device_err_flag(kErrGemm); }

}  // namespace gk

// Output through a tensor map in the 2-SM kernel (EMB_GEMM_C_TMA=0 selects the row-by-row epilogue).
static int raster_m_fast() {
  static int v = [] {
    const char* e = std::getenv("EMB_GEMM_RASTER");
    return (e && e[0] == 'm') ? 1 : 0;
  }();
  return v;
}

static bool c_tma_enabled() {
  static bool on = [] {
    const char* e = std::getenv("EMB_GEMM_C_TMA");
    return !(e && std::atoi(e) == 0);
  }();
  return on;
}

// Stage depth of the 2-SM kernel unless a variant asks otherwise (EMB_GEMM_BK=64 or 128 overrides).
static int gemm2_default_bk() {
  static int bk = [] {
    const char* e = std::getenv("EMB_GEMM_BK");
    return (e && std::atoi(e) == 64) ? 64 : 128;
  }();
  return bk;
}

namespace gk2 {
// Launch the 2-SM kernel on `clusters` CTA pairs with stage depth `bk` (64 or 128); sets the kernel's
// shared-memory limit on each device the first time it is used there.
template <bool AG>
static void launch(int bk, const CUtensorMap& tA, const CUtensorMap& tB, const CUtensorMap& tC, const gk::Params& p,
                   int clusters) {
  static bool attr_set[2][kMaxDevices] = {};
  int dev = 0;
  EMB_CUDA_CHECK(cudaGetDevice(&dev));
  const int which = bk == 128 ? 1 : 0;
  auto kern = which ? gemm2_kernel<AG, 128> : gemm2_kernel<AG, 64>;
  const int smem = which ? smem_bytes<128>() : smem_bytes<64>();
  if (!attr_set[which][dev]) {
    EMB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set[which][dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(AG ? NUM_THREADS_AG : NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = cur_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  EMB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tA, tB, tC, p));
}
}  // namespace gk2

static bool ok_2d(const at::Tensor& t) {
  return t.dim() == 2 && t.stride(1) == 1 && t.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0;
}

// The 1-SM kernel's dynamic shared-memory limit, raised once per device (a function attribute belongs to the
// device's context).
static void gemm1_smem_attr() {
  static bool done[kMaxDevices] = {};
  int dev = 0;
  EMB_CUDA_CHECK(cudaGetDevice(&dev));
  if (!done[dev]) {
    EMB_CUDA_CHECK(cudaFuncSetAttribute(gk::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gk::SMEM_BYTES));
    done[dev] = true;
  }
}

bool gemm_tc_supported(at::Tensor a, at::Tensor b, bool trans_a, bool trans_b, c10::optional<at::Tensor> out,
                       bool accumulate) {
  if (!a.is_cuda() || a.scalar_type() != at::kBFloat16 || b.scalar_type() != at::kBFloat16) return false;
  if (!ok_2d(a) || !ok_2d(b)) return false;
  if (out.has_value() && out->defined()) {
    auto& c = *out;
    if (c.dim() != 2 || c.stride(1) != 1) return false;
    if (c.scalar_type() != at::kFloat && c.scalar_type() != at::kBFloat16) return false;
    if (accumulate && c.scalar_type() != at::kFloat) return false;
  }
  return true;
}

at::Tensor gemm_tc(at::Tensor a, at::Tensor b, bool trans_a, bool trans_b, c10::optional<at::Tensor> out,
                      bool accumulate, int64_t variant) {
  using namespace gk;
  TORCH_CHECK(gemm_tc_supported(a, b, trans_a, trans_b, out, accumulate), "gemm_tc: unsupported operands");
  const int64_t M = trans_a ? a.size(1) : a.size(0);
  const int64_t K = trans_a ? a.size(0) : a.size(1);
  const int64_t N = trans_b ? b.size(0) : b.size(1);
  TORCH_CHECK((trans_b ? b.size(1) : b.size(0)) == K, "gemm: inner dimensions differ");
  at::Tensor C;
  if (out.has_value() && out->defined()) {
    C = *out;
    TORCH_CHECK(C.size(0) == M && C.size(1) == N, "gemm: bad output shape");
  } else {
    C = at::empty({M, N}, a.options());
  }
  if (M == 0 || N == 0) return C;
  if (K == 0) {
    if (!accumulate) C.zero_();
    return C;
  }
  const bool a_mn = trans_a, b_mn = !trans_b;
  CUtensorMap tA = a_mn ? make_map(a.data_ptr(), K, M, a.stride(0), 64, 64) : make_map(a.data_ptr(), M, K, a.stride(0), 64, BM);
  CUtensorMap tB = b_mn ? make_map(b.data_ptr(), K, N, b.stride(0), 64, 64) : make_map(b.data_ptr(), N, K, b.stride(0), 64, BN);
  Params p{};
  p.m_fast = raster_m_fast();
  p.C = C.data_ptr();
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldc = (int)C.stride(0);
  p.out_fp32 = C.scalar_type() == at::kFloat;
  p.accumulate = accumulate ? 1 : 0;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.err = err_flag();
  const int64_t tiles2 = ((M + 255) / 256) * ((N + 255) / 256);
  // variant: 0 auto, 1 one-SM tiles, 2 two-SM tiles, 3 two-SM tiles without the tail split (for comparison)
  // variant 9: variant 2 without output stores (epilogue cost measurement; the result is not written)
  // variants 10 / 11 / 12: variant 9 without MMAs / without operand loads / without either (main-loop probes)
  // variants 13 / 14: variant 2 / 11 with per-role cycle counters (gemm_debug_counters)
  // variants 4 / 5: variant 2 with 64-deep / 128-deep stages (variant 2 itself uses the default depth);
  // variant 15: variant 13 with 128-deep stages
  const bool pair = (variant >= 2 && variant <= 5) || (variant >= 9 && variant <= 15) ||
                    (variant <= 0 && tiles2 >= num_sms() / 2);
  const int bk = variant == 4 ? 64 : (variant == 5 || variant == 15) ? 128
                 : (variant >= 9 && variant <= 14) ? 64 : gemm2_default_bk();
  if (variant == 15) variant = 13;
  if (variant == 4 || variant == 5) variant = 2;
  p.split_tail = variant == 3 ? 0 : 1;
  p.no_store = (variant >= 9 && variant != 13) ? 1 : 0;
  p.probe = variant == 13 ? 4 : variant == 14 ? 6 : (variant >= 10 ? variant - 9 : 0);
  if (pair) {
    // 2-SM clusters: each CTA loads a 128-row half of the A tile and of the B tile
    CUtensorMap tA2 = a_mn ? make_map(a.data_ptr(), K, M, a.stride(0), 64, bk) : make_map(a.data_ptr(), M, K, a.stride(0), 64, 128);
    CUtensorMap tB2 = b_mn ? make_map(b.data_ptr(), K, N, b.stride(0), 64, bk) : make_map(b.data_ptr(), N, K, b.stride(0), 64, 128);
    // C through a tensor map when its rows are 16-byte aligned: 32-row boxes of 128 bytes, 128-byte swizzle
    CUtensorMap tC = tA2;
    const int esz = p.out_fp32 ? 4 : 2;
    if (((uintptr_t)C.data_ptr() % 16) == 0 && (C.stride(0) * esz) % 16 == 0 && p.no_store == 0) {
      cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
      cuuint64_t strides[1] = {(cuuint64_t)(C.stride(0) * esz)};
      cuuint32_t box[2] = {(cuuint32_t)(128 / esz), 32};
      cuuint32_t estr[2] = {1, 1};
      CUresult r = get_encode()(&tC, p.out_fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                C.data_ptr(), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled(C) failed: ", (int)r);
      p.c_tma = c_tma_enabled() ? 1 : 0;
    }
    const int clusters = (int)std::min<int64_t>(tiles2, num_sms() / 2);
    gk2::launch<false>(bk, tA2, tB2, tC, p, clusters);
  } else {
    gemm1_smem_attr();
    const int tiles = (int)(((M + BM - 1) / BM) * ((N + BN - 1) / BN));
    const int grid = std::min(tiles, num_sms());
    gemm_kernel<<<grid, NUM_THREADS, SMEM_BYTES, cur_stream()>>>(tA, tB, p);
  }
  EMB_LAUNCH_CHECK();
  count_launch();
  return C;
}

// Grouped GEMM over per-group row segments (MoE experts), 1-SM tcgen05 kernel.
//   y [R, N] = a [R, K] @ op(w[g]) for every 128-row tile whose tile_group entry is g >= 0 (other tiles are
//   skipped and their rows of y left unwritten).  w: [G, N, K] (trans_b) or [G, K, N] (!trans_b; K % 64 == 0 so
//   that a k-block never reaches into the next group's rows).
at::Tensor gemm_grouped(at::Tensor a, at::Tensor w, bool trans_b, at::Tensor tile_group) {
  using namespace gk;
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && a.dim() == 2 &&
              w.dim() == 3 && a.is_contiguous() && w.is_contiguous(), "gemm_grouped: bf16 a [R, K], w [G, ., .]");
  TORCH_CHECK(tile_group.is_cuda() && tile_group.scalar_type() == at::kInt);
  const int64_t R = a.size(0), K = a.size(1), G = w.size(0);
  const int64_t N = trans_b ? w.size(1) : w.size(2);
  TORCH_CHECK((trans_b ? w.size(2) : w.size(1)) == K, "gemm_grouped: inner dimensions differ");
  TORCH_CHECK(R % BM == 0 && tile_group.numel() >= R / BM, "gemm_grouped: rows must be whole 128-row tiles");
  TORCH_CHECK(K % 8 == 0 && N % 8 == 0 && (trans_b || K % BK == 0), "gemm_grouped: unsupported sizes");
  auto C = at::empty({R, N}, a.options());
  if (R == 0 || N == 0) return C;
  CUtensorMap tA = make_map(a.data_ptr(), R, K, K, 64, BM);
  CUtensorMap tB = trans_b ? make_map(w.data_ptr(), G * N, K, K, 64, BN) : make_map(w.data_ptr(), G * K, N, N, 64, 64);
  Params p{};
  p.m_fast = raster_m_fast();
  p.C = C.data_ptr();
  p.M = (int)R;
  p.N = (int)N;
  p.K = (int)K;
  p.ldc = (int)N;
  p.a_mn = 0;
  p.b_mn = !trans_b;
  p.err = err_flag();
  p.group_mode = 1;
  p.group_info = tile_group.data_ptr<int>();
  p.groups = (int)G;
  p.group_b_stride = (int)(trans_b ? N : K);
  gemm1_smem_attr();
  const int tiles = (int)((R / BM) * ((N + BN - 1) / BN));
  gemm_kernel<<<std::min(tiles, num_sms()), NUM_THREADS, SMEM_BYTES, cur_stream()>>>(tA, tB, p);
  EMB_LAUNCH_CHECK();
  count_launch();
  return C;
}

// Grouped weight gradient: out[g] (+)= dy[seg[g]:seg[g+1]]^T @ x[seg[g]:seg[g+1]] for g < G, with dy [R, M],
// x [R, N] bf16, seg int32 [G + 1] (device, multiples of 64), out fp32 [G, M, N].
void gemm_grouped_wgrad(at::Tensor dy, at::Tensor x, at::Tensor seg, at::Tensor out, bool accumulate) {
  using namespace gk;
  TORCH_CHECK(dy.is_cuda() && dy.scalar_type() == at::kBFloat16 && x.scalar_type() == at::kBFloat16 &&
              dy.is_contiguous() && x.is_contiguous() && dy.size(0) == x.size(0), "gemm_grouped_wgrad: operands");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.dim() == 3 && out.is_contiguous() && seg.scalar_type() == at::kInt);
  const int64_t R = dy.size(0), M = dy.size(1), N = x.size(1), G = out.size(0);
  TORCH_CHECK(out.size(1) == M && out.size(2) == N && seg.numel() == G + 1, "gemm_grouped_wgrad: shapes");
  TORCH_CHECK(M % 8 == 0 && N % 8 == 0, "gemm_grouped_wgrad: sizes must be multiples of 8");
  if (R == 0 || G == 0) {
    if (!accumulate) out.zero_();
    return;
  }
  if (!accumulate) out.zero_();  // groups without rows are skipped by the kernel
  CUtensorMap tA = make_map(dy.data_ptr(), R, M, M, 64, 64);
  CUtensorMap tB = make_map(x.data_ptr(), R, N, N, 64, 64);
  Params p{};
  p.m_fast = raster_m_fast();
  p.C = out.data_ptr();
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)R;
  p.ldc = (int)N;
  p.out_fp32 = 1;
  p.accumulate = 1;
  p.a_mn = 1;
  p.b_mn = 1;
  p.err = err_flag();
  p.group_mode = 2;
  p.group_info = seg.data_ptr<int>();
  p.groups = (int)G;
  p.group_c_stride = (long long)M * N;
  gemm1_smem_attr();
  const int64_t tiles = G * ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  gemm_kernel<<<(int)std::min<int64_t>(tiles, num_sms()), NUM_THREADS, SMEM_BYTES, cur_stream()>>>(tA, tB, p);
  EMB_LAUNCH_CHECK();
  count_launch();
}

// out_local[i, n] = sum_s stage[s, i, n] over the TP slots (bf16 in, fp32 sum, bf16 out)
__global__ void rs_reduce_kernel(const __nv_bfloat16* __restrict__ stage, __nv_bfloat16* __restrict__ out,
                                 int64_t slot_elems, int tp) {
  const int64_t nv = slot_elems / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int sl = 0; sl < tp; ++sl) {
      float f[8];
      unpack8(reinterpret_cast<const uint4*>(stage + sl * slot_elems)[i], f);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += f[k];
    }
    reinterpret_cast<uint4*>(out)[i] = pack8(acc);
  }
}

// Fused GEMM -> reduce-scatter over `tp` ranks: op(a) @ op(b) = [M, N] partial, M = tp * rows_per_rank; row
// block `o` is written into rank o's staging buffer (peer pointers `peers`, int64 [tp]) at slot `my_slot`.
// The caller orders it with barriers and then runs rs_reduce on its own staging buffer.
void gemm_rs(at::Tensor a, at::Tensor b, bool trans_a, bool trans_b, at::Tensor peers, int64_t my_slot,
             int64_t rows_per_rank) {
  using namespace gk;
  TORCH_CHECK(gemm_tc_supported(a, b, trans_a, trans_b, c10::nullopt, false), "gemm_rs: unsupported operands");
  const int64_t M = trans_a ? a.size(1) : a.size(0);
  const int64_t K = trans_a ? a.size(0) : a.size(1);
  const int64_t N = trans_b ? b.size(0) : b.size(1);
  const int64_t tp = peers.numel();
  TORCH_CHECK(tp >= 1 && tp <= 8 && M == tp * rows_per_rank && N % 8 == 0,
              "gemm_rs: M must equal tp * rows_per_rank, tp <= 8, N % 8 == 0");
  auto pc = peers.to(at::kCPU).contiguous();
  const bool a_mn = trans_a, b_mn = !trans_b;
  const int bk2 = gemm2_default_bk();
  CUtensorMap tA = a_mn ? make_map(a.data_ptr(), K, M, a.stride(0), 64, bk2) : make_map(a.data_ptr(), M, K, a.stride(0), 64, 128);
  CUtensorMap tB = b_mn ? make_map(b.data_ptr(), K, N, b.stride(0), 64, bk2) : make_map(b.data_ptr(), N, K, b.stride(0), 64, 128);
  Params p{};
  p.m_fast = raster_m_fast();
  p.C = nullptr;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldc = (int)N;
  p.a_mn = a_mn;
  p.b_mn = b_mn;
  p.err = err_flag();
  p.scatter = 1;
  p.split_tail = 1;
  p.rows_per_rank = (int)rows_per_rank;
  p.my_slot = (int)my_slot;
  for (int64_t i = 0; i < tp; ++i) p.peer_out[i] = reinterpret_cast<void*>(pc.data_ptr<int64_t>()[i]);
  const int64_t tiles2 = ((M + 255) / 256) * ((N + 255) / 256);
  const int clusters = (int)std::min<int64_t>(tiles2, num_sms() / 2);
  gk2::launch<false>(gemm2_default_bk(), tA, tB, tA /* unused */, p, clusters);
  count_launch();
}

// Fused all-gather -> GEMM: C[M, N] = A_full @ op(b) where A_full [M, K] = concat over tp ranks of their
// [rows_per_rank, K] shards.  `local` is this rank's gather buffer (its own chunk already in place); `peers`
// (int64 [tp]) are the peers' gather buffers (CUDA-IPC mapped, same layout) into which this kernel pushes
// `shard`; `flags` (int64 [tp]) are the ranks' readiness-flag arrays (units_max uint32 per chunk), set to
// `epoch` when a unit lands; `claim` is an int32 counter zeroed before the launch.
at::Tensor gemm_ag(at::Tensor local, at::Tensor b, bool trans_b, at::Tensor peers, int64_t my_slot,
                   int64_t rows_per_rank, at::Tensor claim, at::Tensor shard, at::Tensor flags, int64_t epoch,
                   int64_t units_max) {
  using namespace gk;
  TORCH_CHECK(gemm_tc_supported(local, b, false, trans_b, c10::nullopt, false), "gemm_ag: unsupported operands");
  const int64_t M = local.size(0), K = local.size(1);
  const int64_t N = trans_b ? b.size(0) : b.size(1);
  const int64_t tp = peers.numel();
  TORCH_CHECK(tp >= 1 && tp <= 8 && M == tp * rows_per_rank && rows_per_rank % 256 == 0 && (K * 2) % 16 == 0,
              "gemm_ag: rows per rank must be a multiple of 256, tp <= 8");
  TORCH_CHECK(flags.numel() == tp && rows_per_rank / gk2::AG_UNIT_ROWS <= units_max, "gemm_ag: flag array too small");
  TORCH_CHECK(claim.is_cuda() && claim.scalar_type() == at::kInt && claim.numel() >= 1);
  TORCH_CHECK(shard.is_cuda() && shard.is_contiguous() && shard.scalar_type() == at::kBFloat16 &&
                  shard.size(0) == rows_per_rank && shard.size(1) == K,
              "gemm_ag: shard must be a contiguous bf16 [rows_per_rank, K] tensor");
  auto pc = peers.to(at::kCPU).contiguous();
  auto fc = flags.to(at::kCPU).contiguous();
  const bool b_mn = !trans_b;
  CUtensorMap tA = make_map(local.data_ptr(), M, K, local.stride(0), 64, 128);
  CUtensorMap tB = b_mn ? make_map(b.data_ptr(), K, N, b.stride(0), 64, gemm2_default_bk())
                        : make_map(b.data_ptr(), N, K, b.stride(0), 64, 128);
  auto C = at::empty({M, N}, local.options());
  Params p{};
  p.m_fast = raster_m_fast();
  p.C = C.data_ptr();
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldc = (int)N;
  p.a_mn = 0;
  p.b_mn = b_mn;
  p.err = err_flag();
  p.rows_per_rank = (int)rows_per_rank;
  p.my_slot = (int)my_slot;
  p.ag_local = local.data_ptr();
  p.ag_shard = shard.data_ptr();
  p.ready = claim.data_ptr<int>();
  p.ag_tp = (int)tp;
  p.ag_units_max = (int)units_max;
  p.ag_epoch = (uint32_t)epoch;
  for (int64_t i = 0; i < tp; ++i) {
    p.ag_dst[i] = reinterpret_cast<void*>(pc.data_ptr<int64_t>()[i]);
    p.ag_flags[i] = reinterpret_cast<uint32_t*>(fc.data_ptr<int64_t>()[i]);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(p.ag_dst[i]) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.ag_flags[i]) & 3) == 0,
                "gemm_ag: misaligned peer buffer");
  }
  const int64_t tiles2 = ((M + 255) / 256) * ((N + 255) / 256);
  const int clusters = (int)std::min<int64_t>(tiles2, num_sms() / 2);
  gk2::launch<true>(gemm2_default_bk(), tA, tB, tA /* unused */, p, clusters);
  count_launch();
  return C;
}

at::Tensor rs_reduce(at::Tensor stage, int64_t tp, int64_t rows, int64_t n) {
  TORCH_CHECK(stage.is_cuda() && stage.scalar_type() == at::kBFloat16 && stage.numel() >= tp * rows * n);
  TORCH_CHECK(n % 8 == 0);
  auto out = at::empty({rows, n}, stage.options());
  const int64_t slot = rows * n;
  const int64_t nv = slot / 8;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((nv + 255) / 256, (int64_t)num_sms() * 8));
  rs_reduce_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<const __nv_bfloat16*>(stage.data_ptr()),
                                                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), slot, (int)tp);
  EMB_LAUNCH_CHECK();
  count_launch();
  return out;
}

int64_t gemm_error_flag() {
  int v = 0;
  EMB_CUDA_CHECK(cudaMemcpy(&v, gk::err_flag(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

// Role cycle counters of the last timed GEMM launches (variants 13 / 14), then reset.
std::vector<int64_t> gemm_debug_counters() {
  unsigned long long h[16];
  EMB_CUDA_CHECK(cudaMemcpyFromSymbol(h, gk2::g_dbg, sizeof(h)));
  unsigned long long z[16] = {0};
  EMB_CUDA_CHECK(cudaMemcpyToSymbol(gk2::g_dbg, z, sizeof(z)));
  return std::vector<int64_t>(h, h + 16);
}

void gemm_clear_error() { EMB_CUDA_CHECK(cudaMemset(gk::err_flag(), 0, sizeof(int))); }

// Library fallback for operands the tensor-core kernel does not take (e.g. fp32 inputs or unaligned strides).
// Calls of gemm() that the tcgen05 kernels could not take (dtype, layout or a row stride that breaks TMA's
// 16-byte rule) and that therefore ran on at::matmul; the first one also prints a warning.
static std::atomic<int64_t> g_gemm_fallbacks{0};
int64_t gemm_fallback_count() { return g_gemm_fallbacks.load(); }

at::Tensor gemm(at::Tensor a, at::Tensor b, bool trans_a, bool trans_b, c10::optional<at::Tensor> out,
                   bool accumulate) {
  if (gemm_tc_supported(a, b, trans_a, trans_b, out, accumulate)) return gemm_tc(a, b, trans_a, trans_b, out, accumulate, 0);
  g_gemm_fallbacks.fetch_add(1);
  TORCH_WARN_ONCE("gemm: operands the tcgen05 kernels cannot take (dtype, layout or a row stride that is not a "
                  "multiple of 16 bytes) run on at::matmul; gemm_fallback_count() counts them");
  auto A = trans_a ? a.t() : a;
  auto B = trans_b ? b.t() : b;
  if (out.has_value() && out->defined()) {
    auto C = *out;
    if (accumulate) {
      C.add_(at::matmul(A.to(C.scalar_type()), B.to(C.scalar_type())));
    } else {
      C.copy_(at::matmul(A, B));
    }
    return C;
  }
  return at::matmul(A, B);
}

}  // namespace emb
