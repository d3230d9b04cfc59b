// K10 (backward): causal GQA flash attention backward on tcgen05 / TMEM / TMA, sm_100a, head dim 128.
//
// One CTA = one (128-row key/value tile j, batch, query group g).  K_j and V_j stay in shared memory; the CTA
// walks every head of the group and every query tile i >= j (causal), so dK_j and dV_j accumulate in TMEM
// across all of them and are written once, with no atomics.  Per (head, query tile) step:
//   S^T  = K_j Q_i^T          (TMEM cols   0..127; later reused for dQ)
//   dP^T = V_j dO_i^T         (TMEM cols 128..255)
//   one thread per key row:   P^T = exp(S^T * scale - lse) written back as packed bf16 into TMEM cols 0..63,
//                             dS^T = P^T * (dP^T - Delta) * scale as a bf16 128-byte-swizzled shared tile
//   dV  += P^T dO_i            (cols 256..383; P^T from TMEM as the A operand, dO as an MN-major operand)
//   dK  += dS^T Q_i            (cols 384..511; Q as an MN-major operand)
//   dQ_i = dS K_j              (cols 128..255, where dP^T was; dS^T read as an MN-major A operand, K_j MN-major B)
//   one thread per query row adds its dQ row into an fp32 accumulator with bulk tensor add-reductions.
// Q tiles are double-buffered, so the next step's Q arrives while this step runs, and S^T of the next step is
// issued right after this step's MMAs (its columns hold only P^T, which the dV MMA before it has read): it
// overlaps the dQ read-out, and only dP^T of the next step waits for that read-out (it overwrites dQ).
// Delta = rowsum(dO * O) comes from a small preprocessing kernel; a finishing kernel casts the dQ accumulator
// into the query slots of dqkv.  Waits are bounded (error flag); no TMA multicast.
#include <cudaTypedefs.h>

#include "../include/common.cuh"

namespace emb {
namespace fa {
CUtensorMap qkv_map(const at::Tensor& qkv);
}

namespace fab {

constexpr int D = 128, T = 128;
constexpr int TILE = 128 * 128 * 2;
constexpr int DQ_STAGE = 4 * 2 * 4096;  // dQ staging: per softmax warp two 32-row x 128-byte blocks
constexpr int SMEM_BYTES = 6 * TILE + DQ_STAGE + 1024 /*lse, delta*/ + 1024 /*align*/ + 256 /*barriers*/;  // K V Q0 Q1 dO dS
static_assert(SMEM_BYTES <= 232448, "flash_bwd_kernel shared memory above the 227 KiB per-block limit");
constexpr uint32_t WAIT_LIMIT = 1u << 26;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int* err, int code) {
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (i > 64) __nanosleep(64);
  }
  atomicExch(err, code);
  return false;
}
__device__ __forceinline__ void tma4(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int slot, int bb, int s) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(slot), "r"(bb), "r"(s), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ uint64_t desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__host__ __device__ constexpr uint32_t idesc(bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
// A from tensor memory (128 lanes x 16 bf16 packed in 8 columns), B from shared memory
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ float ex2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
#define FAB_LD32(taddr, r)                                                                                          \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19," \
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                                    \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),      \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),     \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                   \
      : "r"(taddr))

#define FAB_ST16(taddr, r)                                                                                          \
  asm volatile(                                                                                                     \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"( \
          taddr),                                                                                                   \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])                                       \
      : "memory")

__device__ __forceinline__ uint32_t swz_off(int row, int col) {
  const int panel = col >> 6, c = col & 63;
  return panel * 16384 + row * 128 + (((c >> 3) ^ (row & 7)) << 4) + (c & 7) * 2;
}

struct Params {
  const float* lse;    // [b, H, s]
  const float* delta;  // [b, H, s]
  float* dq_acc;       // [s, b, H, d] fp32, zero-initialised
  __nv_bfloat16* dqkv; // [s, b, G, hpg + 2, d]
  int s, b, G, hpg;
  float scale, scale_log2;
  int causal;
  int* err;
};

__global__ void __launch_bounds__(192, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tqkv, const __grid_constant__ CUtensorMap tdo,
                     const __grid_constant__ CUtensorMap tdq, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = sm;
  uint8_t* sV = sm + TILE;
  uint8_t* sQ = sm + 2 * TILE;   // [2]: Q of steps n (n even) and n (n odd)
  uint8_t* sdO = sm + 4 * TILE;
  uint8_t* sdS = sm + 5 * TILE;  // dS^T [key rows x query cols]
  uint8_t* sdq = sm + 6 * TILE;  // [4 warps][2][32 rows x 128 B], 128-byte swizzle
  float* s_lse = reinterpret_cast<float*>(sm + 6 * TILE + DQ_STAGE);
  float* s_delta = s_lse + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 6 * TILE + DQ_STAGE + 1024);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;   // [2]
  uint64_t* q_empty = bars + 3;  // [2]
  uint64_t* do_full = bars + 5;
  uint64_t* do_empty = bars + 6;
  uint64_t* s_full = bars + 7;
  uint64_t* ds_full = bars + 8;
  uint64_t* mma2_done = bars + 9;
  uint64_t* dq_empty = bars + 10;
  uint64_t* stats_full = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.s / T;
  const int jt = blockIdx.x;  // key/value tile
  const int bg = blockIdx.y;
  const int bidx = bg / p.G, g = bg % p.G;
  const int H = p.G * p.hpg;
  const int slots = p.hpg + 2;
  const int k_slot = g * slots + p.hpg, v_slot = k_slot + 1;
  const int i0 = p.causal ? jt : 0;
  const int nsteps = p.hpg * (nq - i0);

  if (threadIdx.x == 0) {
    bar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      bar_init(&q_full[i], 1);
      bar_init(&q_empty[i], 1);
    }
    bar_init(do_full, 1);
    bar_init(do_empty, 1);
    bar_init(s_full, 1);
    bar_init(ds_full, 4);
    bar_init(mma2_done, 1);
    bar_init(dq_empty, 4);
    bar_init(stats_full, 4);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)), "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      bar_expect(kv_full, 2 * TILE);
      tma4(sK, &tqkv, kv_full, 0, k_slot, bidx, jt * T);
      tma4(sK + 16384, &tqkv, kv_full, 64, k_slot, bidx, jt * T);
      tma4(sV, &tqkv, kv_full, 0, v_slot, bidx, jt * T);
      tma4(sV + 16384, &tqkv, kv_full, 64, v_slot, bidx, jt * T);
      for (int n = 0; n < nsteps; ++n) {
        const int hj = n / (nq - i0), it = i0 + n % (nq - i0);
        const int h = g * p.hpg + hj;
        const int qb = n & 1;
        // Q(n) goes into the buffer step n - 2 used (free once that step's MMAs completed)
        if (!bar_wait(&q_empty[qb], ((n >> 1) & 1) ^ 1, p.err, 41) || *abort_flag) { *abort_flag = 1; break; }
        bar_expect(&q_full[qb], TILE);
        tma4(sQ + qb * TILE, &tqkv, &q_full[qb], 0, g * slots + hj, bidx, it * T);
        tma4(sQ + qb * TILE + 16384, &tqkv, &q_full[qb], 64, g * slots + hj, bidx, it * T);
        // dO(n) into the single dO buffer once step n - 1's MMAs completed
        if (!bar_wait(do_empty, (n & 1) ^ 1, p.err, 50) || *abort_flag) { *abort_flag = 1; break; }
        bar_expect(do_full, TILE);
        tma4(sdO, &tdo, do_full, 0, h, bidx, it * T);
        tma4(sdO + 16384, &tdo, do_full, 64, h, bidx, it * T);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_kk = idesc(false, false), id_kmn = idesc(false, true), id_mnmn = idesc(true, true);
      const uint32_t aK = su32(sK), aV = su32(sV), adO = su32(sdO), adS = su32(sdS);
      bool ok = bar_wait(kv_full, 0, p.err, 42) && !*abort_flag;
      for (int n = 0; n < nsteps && ok; ++n) {
        const uint32_t ph = n & 1;
        const int qb = n & 1;
        const uint32_t aQ = su32(sQ + qb * TILE);
        // S^T = K Q^T (cols 0..127): needs only this step's Q; its columns last held P^T(n - 1), which the
        // dV MMA of step n - 1, issued before on this thread, has read (the tensor pipe runs them in order)
        if (!bar_wait(&q_full[qb], (n >> 1) & 1, p.err, 43) || *abort_flag) { ok = false; break; }
        fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // reduce over d: K-major panels of the K / Q tiles
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma(tmem + 0, desc(aK + off, 16, 1024), desc(aQ + off, 16, 1024), id_kk, k != 0);
        }
        // dP^T = V dO^T (cols 128..255): needs dO(n) and dQ(n - 1) read out of these columns
        if (!bar_wait(do_full, ph, p.err, 51) || !bar_wait(dq_empty, ph ^ 1, p.err, 44) || *abort_flag) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma(tmem + 128, desc(aV + off, 16, 1024), desc(adO + off, 16, 1024), id_kk, k != 0);
        }
        commit(s_full);
        if (!bar_wait(ds_full, ph, p.err, 45) || *abort_flag) { ok = false; break; }
        fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // reduce over the query index
          const uint32_t offa = (k >> 2) * 16384 + (k & 3) * 32;  // dS^T as K-major A (rows = keys)
          const uint32_t offb = k * 2048;                          // dO / Q as MN-major B (rows = queries)
          // P^T from TMEM: 16 queries of bf16 pairs = 8 columns per k-step
          mma_ts(tmem + 256, tmem + k * 8, desc(adO + offb, 16384, 1024), id_kmn, (n | k) != 0);
          mma(tmem + 384, desc(adS + offa, 16, 1024), desc(aQ + offb, 16384, 1024), id_kmn, (n | k) != 0);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {  // dQ = dS K: reduce over keys; dS^T tile as MN-major A, K tile MN-major B
          mma(tmem + 128, desc(adS + k * 2048, 16384, 1024), desc(aK + k * 2048, 16384, 1024), id_mnmn, k != 0);
        }
        commit(&q_empty[qb]);
        commit(do_empty);
        commit(mma2_done);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // TMEM lane: key row for S^T/dP^T/dK/dV, query row for dQ
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int kpos = jt * T + r;
    bool ok = true;
    uint32_t dq_n = 0;  // dQ blocks this warp has handed to the bulk-copy engine (selects the staging buffer)
    for (int n = 0; n < nsteps; ++n) {
      const int hj = n / (nq - i0), it = i0 + n % (nq - i0);
      const int h = g * p.hpg + hj;
      const uint32_t ph = n & 1;
      // per-query statistics of this step (the previous step's readers finished before dq_empty completed)
      if (n > 0 && (!bar_wait(dq_empty, ph ^ 1, p.err, 46) || *abort_flag)) { ok = false; break; }
      {
        const size_t base = ((size_t)bidx * H + h) * p.s + it * T;
        s_lse[r] = p.lse[base + r] * 1.4426950408889634f;
        s_delta[r] = p.delta[base + r];
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!bar_wait(s_full, ph, p.err, 47) || *abort_flag) { ok = false; break; }
      fence_after();
      const bool diag = p.causal && it == jt;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32], dv[32];
        FAB_LD32(tmem + lane_base + c * 32, sv);
        FAB_LD32(tmem + lane_base + 128 + c * 32, dv);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float df[32];
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float pr2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int q = c * 32 + i + e;
            const int qpos = it * T + q;
            float pr = ex2f_approx(fmaf(__uint_as_float(sv[i + e]), p.scale_log2, -s_lse[q]));
            if (diag && qpos < kpos) pr = 0.f;
            pr2[e] = pr;
            df[i + e] = pr * (__uint_as_float(dv[i + e]) - s_delta[q]) * p.scale;
          }
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pk[i >> 1]) : "f"(pr2[1]), "f"(pr2[0]));
        }
        // P^T chunk c -> TMEM columns [16 c, 16 c + 16) of S^T: columns this thread has already read
        FAB_ST16(tmem + lane_base + c * 16, pk);
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8)
          *reinterpret_cast<uint4*>(sdS + swz_off(r, c * 32 + v8 * 8)) = pack8(df + v8 * 8);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      fence_before();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) bar_arrive(ds_full);
      // dQ tile (TMEM cols 0..127, lane = query row) -> fp32 accumulator in global memory: each warp stages its
      // 32 rows x 32 columns in a 128-byte-swizzled block and one lane adds it with a bulk tensor reduction
      // (atomic per element against the other key tiles' CTAs), double-buffered per warp
      if (!bar_wait(mma2_done, ph, p.err, 48) || *abort_flag) { ok = false; break; }
      fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t qv[32];
        FAB_LD32(tmem + lane_base + 128 + c * 32, qv);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        uint8_t* wbuf = sdq + quarter * 8192 + (dq_n & 1) * 4096;
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
        uint8_t* myrow = wbuf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<uint4*>(myrow + ((j ^ (lane & 7)) << 4)) =
              make_uint4(qv[4 * j], qv[4 * j + 1], qv[4 * j + 2], qv[4 * j + 3]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          asm volatile(
              "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                  reinterpret_cast<uint64_t>(&tdq)),
              "r"(c * 32), "r"(bidx * H + h), "r"(it * T + quarter * 32), "r"(su32(wbuf))
              : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        ++dq_n;
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(dq_empty);
    }
    if (!ok) {
      *abort_flag = 1;
    } else if (nsteps > 0) {
      // dK (cols 384..) and dV (cols 256..) rows of this key tile -> dqkv key / value slots
      if (!bar_wait(dq_empty, ((nsteps - 1) & 1), p.err, 49)) { *abort_flag = 1; }
      fence_after();
      __nv_bfloat16* dk = p.dqkv + ((((size_t)kpos * p.b + bidx) * p.G + g) * slots + p.hpg) * D;
      __nv_bfloat16* dvp = dk + D;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t kv[32], vv[32];
        FAB_LD32(tmem + lane_base + 384 + c * 32, kv);
        FAB_LD32(tmem + lane_base + 256 + c * 32, vv);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float kf[32], vf[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          kf[i] = __uint_as_float(kv[i]);
          vf[i] = __uint_as_float(vv[i]);
        }
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          reinterpret_cast<uint4*>(dk + c * 32)[v8] = pack8(kf + v8 * 8);
          reinterpret_cast<uint4*>(dvp + c * 32)[v8] = pack8(vf + v8 * 8);
        }
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // staging reads / reductions done
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

// delta[b, h, q] = sum_d dO[q, b, h, d] * O[q, b, h, d]; one warp per row
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ dO, const __nv_bfloat16* __restrict__ O,
                             float* __restrict__ delta, int s, int b, int H) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= s * b * H) return;
  const int q = row / (b * H), rem = row % (b * H), bi = rem / H, h = rem % H;
  const __nv_bfloat16* a = dO + (size_t)row * D;
  const __nv_bfloat16* c = O + (size_t)row * D;
  float acc = 0.f;
  for (int i = lane; i < D; i += 32) acc += bf2f(a[i]) * bf2f(c[i]);
  acc = warp_sum(acc);
  if (lane == 0) delta[((size_t)bi * H + h) * s + q] = acc;
}

// dqkv query slots <- bf16(dq_acc)
__global__ void dq_cast_kernel(const float* __restrict__ dq, __nv_bfloat16* __restrict__ dqkv, int s, int b, int G,
                               int hpg) {
  const int64_t n = (int64_t)s * b * G * hpg * (D / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (D / 8);
    const int v = (int)(i % (D / 8));
    const int hj = (int)(row % hpg);
    const int64_t tg = row / hpg;  // (token, group)
    const float* src = dq + row * D + v * 8;
    float f[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = src[k];
    __nv_bfloat16* dst = dqkv + (tg * (hpg + 2) + hj) * D + v * 8;
    *reinterpret_cast<uint4*>(dst) = pack8(f);
  }
}

static int* err_flag() { return device_err_flag(kErrAttnBwd); }

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    EMB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// {d, head, b, s} view of dO [s, b, H*d].
static CUtensorMap do_map(const at::Tensor& dO, int64_t s, int64_t b, int64_t H) {
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)b, (cuuint64_t)s};
  cuuint64_t strides[3] = {(cuuint64_t)(D * 2), (cuuint64_t)(H * D * 2), (cuuint64_t)(b * H * D * 2)};
  cuuint32_t box[4] = {64, 1, 1, 128};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, dO.data_ptr(), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled(dO) failed: ", (int)r);
  return m;
}

}  // namespace fab

// dqkv [s, b, G, hpg + 2, d] for the causal attention whose forward returned (o, lse).
at::Tensor attn_bwd(at::Tensor dO, at::Tensor qkv, at::Tensor o, at::Tensor lse, int64_t hpg, bool causal) {
  using namespace fab;
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.size(4) == D &&
                  qkv.size(0) % T == 0,
              "attn_bwd: needs contiguous bf16 [s, b, G, hpg+2, 128] with s % 128 == 0");
  TORCH_CHECK(dO.is_contiguous() && o.is_contiguous() && dO.scalar_type() == at::kBFloat16);
  const int64_t s = qkv.size(0), b = qkv.size(1), G = qkv.size(2), H = G * hpg;
  auto dqkv = at::empty_like(qkv);
  auto dq = at::zeros({s, b, H, D}, qkv.options().dtype(at::kFloat));
  auto delta = at::empty({b, H, s}, qkv.options().dtype(at::kFloat));
  auto st = cur_stream();
  const int rows = (int)(s * b * H);
  delta_kernel<<<(rows + 7) / 8, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dO.data_ptr()),
                                               reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()),
                                               delta.data_ptr<float>(), (int)s, (int)b, (int)H);
  CUtensorMap tq = fa::qkv_map(qkv);
  CUtensorMap td = do_map(dO, s, b, H);
  CUtensorMap tdq;
  {
    // {d, (b, head), s} view of the fp32 dQ accumulator [s, b, H, d]: 32-column x 32-row boxes of 128 bytes
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)(b * H), (cuuint64_t)s};
    cuuint64_t strides[2] = {(cuuint64_t)(D * 4), (cuuint64_t)(b * H * D * 4)};
    cuuint32_t box[3] = {32, 1, 32};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = encode_fn()(&tdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq.data_ptr(), dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled(dq) failed: ", (int)r);
  }
  Params p;
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq.data_ptr<float>();
  p.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  p.s = (int)s;
  p.b = (int)b;
  p.G = (int)G;
  p.hpg = (int)hpg;
  p.scale = (float)(1.0 / std::sqrt((double)D));
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
  p.causal = causal ? 1 : 0;
  p.err = err_flag();
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  EMB_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr[dev]) {
    EMB_CUDA_CHECK(cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr[dev] = true;
  }
  dim3 grid((unsigned)(s / T), (unsigned)(b * G));
  flash_bwd_kernel<<<grid, 192, SMEM_BYTES, st>>>(tq, td, tdq, p);
  const int64_t n = s * b * G * hpg * (D / 8);
  dq_cast_kernel<<<(int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms() * 8), 256, 0, st>>>(
      dq.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), (int)s, (int)b, (int)G, (int)hpg);
  EMB_LAUNCH_CHECK();
  count_launch(3);
  return dqkv;
}

int64_t attn_bwd_error_flag() {
  int v = 0;
  EMB_CUDA_CHECK(cudaMemcpy(&v, fab::err_flag(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

}  // namespace emb
