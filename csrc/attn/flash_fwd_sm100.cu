// K10 (forward): causal GQA flash attention on tcgen05 / TMEM / TMA, sm_100a, head dim 128.
//
// Input is the fused QKV activation of the model, [s, b, G, hpg + 2, d] bf16 (per query group: hpg query
// heads, one key, one value); it is read in place through one 4-D TMA tensor map {d, slot, b, s}.  Output
// o [s, b, H, d] bf16 and the per-row log-sum-exp lse [b, H, s] fp32 (natural log of the scaled scores) for
// the backward pass.
//
// One CTA = two 128-row query tiles (Q0 = rows [256 p, 256 p + 128), Q1 = the next 128) of one (batch, head);
// both share every K / V tile the CTA loads.  320 threads (10 warps):
//   warp 0        - TMA: Q0 and Q1 once, then K_j and V_j into 2-deep rings;
//   warp 1        - TMEM owner (512 columns: S0 | S1 | O0 | O1, 128 fp32 columns each) and MMA issuer (one
//                   thread), in the order  PV0(j), S0(j+1), PV1(j), S1(j+1):  while softmax group 0 works on
//                   S0(j+1) the tensor core runs tile 1's work and vice versa (ping-pong);
//   warps 2..5    - softmax group 0 (one thread per row of Q0 = TMEM lane; warp w reads lane quarter w % 4),
//   warps 6..9    - softmax group 1 (Q1):
//                   read the row of S from TMEM, online max with a lazy rescale (the running max moves only when
//                   a row's max grows by more than 2^8; then that warp rescales its O rows in TMEM), p = 2^(s*c - m)
//                   summed in fp32 and written back as packed bf16 INTO the S columns, from where the PV MMA reads
//                   P as its A operand (tcgen05.mma with A in tensor memory): no shared-memory round trip for P.
//                   After the last tile the group divides O by the row sum and stores o and lse.
// Ordering relies on the tensor pipe executing one thread's MMAs in issue order: the commit after S_i(j+1)
// also covers PV_i(j), so a softmax group that sees S_i(j+1) may rescale O_i, and S_i(j+1) (which overwrites
// P_i(j)) is issued only after PV_i(j).  Causal masking touches only the diagonal tile of each query tile.
// All mbarrier waits are bounded (error flag + early exit); no TMA multicast.
#include <cudaTypedefs.h>

#include <cstdlib>

#include "../include/common.cuh"

namespace emb {
namespace fa {

constexpr int D = 128, BQ = 128, BKV = 128;
constexpr int TILE_BYTES = 128 * 128 * 2;  // one 128 x 128 bf16 tile = two 16 KiB swizzle panels
constexpr int SMEM_BYTES = 6 * TILE_BYTES + 1024 + 256;
constexpr int NUM_THREADS = 320;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P values stay below 2^8 between rescales

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
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait without sleeping (every wait here is on the pipeline's critical path): gives up after ~4 s of
// wall clock, recording `code` in *err.
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity, int* err, int code) {
  if (bar_try(b, parity)) return true;
  const uint64_t t0 = gtimer();
  for (uint32_t i = 1;; ++i) {
    if (bar_try(b, parity)) return true;
    if ((i & 4095) == 0 && gtimer() - t0 > 4000000000ull) break;
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
// bf16 x bf16 -> fp32, M=128, N=128; b_mn selects an MN-major B operand.
__host__ __device__ constexpr uint32_t idesc(bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(128 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}
// A and B from shared memory
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
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
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x on the FMA pipe, for a share of the softmax exponentials (the MUFU unit alone would be as busy as the
// tensor core).  Range reduction x = j + f with j = round(x) taken from the float adder (adding 1.5 * 2^23
// leaves round(x) in the low mantissa bits), f in [-1/2, 1/2]; 2^f by a cubic whose coefficients are a
// relative-error least-squares fit of 2^f on Chebyshev nodes of [-1/2, 1/2] computed for this kernel (max
// relative error 7.5e-5 in fp32, below the bf16 rounding of P); 2^j is added to the exponent field.  Inputs
// below -125 are clamped (their result, < 2^-124, is negligible next to the row maximum's 1, and the
// exponent field stays >= 1).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -125.f);
  const float t = x + 12582912.f;  // 1.5 * 2^23
  const float f = x - (t - 12582912.f);
  float q = fmaf(0.0551716648042202f, f, 0.2426111251115799f);
  q = fmaf(q, f, 0.6932609677314758f);
  q = fmaf(q, f, 0.9999280571937561f);
  return __int_as_float(__float_as_int(q) + (__float_as_int(t) << 23));
}

// Packed fp32 pairs (one 64-bit register) for the f32x2 instructions of sm_100: half the issue slots of
// scalar arithmetic in the softmax, whose instruction count bounds how quickly it hands P to the tensor core.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// ex2_poly on a packed pair (same method and coefficients)
__device__ __forceinline__ uint64_t ex2_poly2(uint64_t x2) {
  float x0, x1;
  up2(x2, x0, x1);
  x2 = pk2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t magic = pk2(12582912.f, 12582912.f);
  const uint64_t t = add2(x2, magic);
  const uint64_t f = sub2(x2, sub2(t, magic));
  uint64_t q = fma2(pk2(0.0551716648042202f, 0.0551716648042202f), f, pk2(0.2426111251115799f, 0.2426111251115799f));
  q = fma2(q, f, pk2(0.6932609677314758f, 0.6932609677314758f));
  q = fma2(q, f, pk2(0.9999280571937561f, 0.9999280571937561f));
  float q0, q1, t0, t1;
  up2(q, q0, q1);
  up2(t, t0, t1);
  return pk2(__int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23)),
             __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23)));
}

#define FA_TMEM_LD_32(taddr, r)                                                                                     \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19," \
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                                    \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),      \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),     \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                   \
      : "r"(taddr))
#define FA_TMEM_ST_32(taddr, r)                                                                                     \
  asm volatile(                                                                                                     \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                                     \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),  \
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),   \
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                                                                \
      : "memory")
#define FA_TMEM_LD_16(taddr, r)                                                                                     \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"      \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])                    \
      : "r"(taddr))
#define FA_TMEM_ST_16(taddr, r)                                                                                     \
  asm volatile(                                                                                                     \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"( \
          taddr),                                                                                                   \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])                                       \
      : "memory")

static_assert(SMEM_BYTES <= 232448, "flash_fwd_kernel shared memory above the 227 KiB per-block limit");

struct Params {
  __nv_bfloat16* o;
  float* lse;
  int s, b, G, hpg;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  int* err;
  int timing;  // measurement only: accumulate per-role cycle counters into g_fa_dbg
};
__device__ unsigned long long g_fa_dbg[16];
__device__ __forceinline__ unsigned long long clk64() {
  unsigned long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;                   // [2]: Q0, Q1
  uint8_t* sK = sm + 2 * TILE_BYTES;  // [2]
  uint8_t* sV = sm + 4 * TILE_BYTES;  // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 6 * TILE_BYTES);
  uint64_t* q_full = bars;        // [2]
  uint64_t* k_full = bars + 2;    // [2]
  uint64_t* k_empty = bars + 4;   // [2]
  uint64_t* v_full = bars + 6;    // [2]
  uint64_t* v_empty = bars + 8;   // [2]
  uint64_t* s_full = bars + 10;   // [2] per query tile
  uint64_t* p_full = bars + 12;   // [2] per query tile
  uint64_t* o_final = bars + 14;  // [2] per query tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npairs = (p.s / BQ + 1) / 2;
  const int pr = npairs - 1 - (int)blockIdx.y;  // heavy (late) query tiles first
  const int H = p.G * p.hpg;
  const int bh = blockIdx.x;
  const int bidx = bh / H, h = bh % H;
  const int g = h / p.hpg, hj = h % p.hpg;
  const int slots = p.hpg + 2;
  const int q_slot = g * slots + hj, k_slot = g * slots + p.hpg, v_slot = g * slots + p.hpg + 1;
  const int qt0 = 2 * pr, qt1 = 2 * pr + 1;
  const int nkv = p.s / BKV;
  const bool has1 = qt1 < nkv;              // an odd tile count leaves the last CTA one query tile
  const int n0 = p.causal ? qt0 + 1 : nkv;  // KV tiles query tile 0 needs
  const int n1 = has1 ? (p.causal ? qt1 + 1 : nkv) : 0;  // ... tile 1
  const int nl = n1 > n0 ? n1 : n0;         // KV tiles the CTA loads

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      bar_init(&q_full[i], 1);
      bar_init(&k_full[i], 1);
      bar_init(&k_empty[i], 1);
      bar_init(&v_full[i], 1);
      bar_init(&v_empty[i], 1);
      bar_init(&s_full[i], 1);
      bar_init(&p_full[i], 4);
      bar_init(&o_final[i], 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm)) : "memory");
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
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      for (int i = 0; i < (has1 ? 2 : 1); ++i) {
        bar_expect(&q_full[i], TILE_BYTES);
        const int row = (i ? qt1 : qt0) * BQ;
        tma4(sQ + i * TILE_BYTES, &tm, &q_full[i], 0, q_slot, bidx, row);
        tma4(sQ + i * TILE_BYTES + 16384, &tm, &q_full[i], 64, q_slot, bidx, row);
      }
      for (int j = 0; j < nl; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!bar_wait(&k_empty[st], ph ^ 1, p.err, 21) || *abort_flag) { *abort_flag = 1; break; }
        bar_expect(&k_full[st], TILE_BYTES);
        tma4(sK + st * TILE_BYTES, &tm, &k_full[st], 0, k_slot, bidx, j * BKV);
        tma4(sK + st * TILE_BYTES + 16384, &tm, &k_full[st], 64, k_slot, bidx, j * BKV);
        if (!bar_wait(&v_empty[st], ph ^ 1, p.err, 22) || *abort_flag) { *abort_flag = 1; break; }
        bar_expect(&v_full[st], TILE_BYTES);
        tma4(sV + st * TILE_BYTES, &tm, &v_full[st], 0, v_slot, bidx, j * BKV);
        tma4(sV + st * TILE_BYTES + 16384, &tm, &v_full[st], 64, v_slot, bidx, j * BKV);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc(false), id_pv = idesc(true);
      bool ok = true;
      unsigned long long t_v = 0, t_p = 0, t_start = p.timing ? clk64() : 0;
      // S_i(j) = Q_i K_j^T into columns [128 i, 128 i + 128)
      // Descriptors are built once; a k-step (or stage) only adds to the 14-bit start-address field, which never
      // carries (shared-memory offsets < 2^18 bytes).  K-major Q / K tiles: k-step k at panel k / 4, 32 bytes
      // per step inside the 128-byte swizzle row; MN-major V: 16 key rows (2048 bytes) per step.
      const uint64_t q_d0 = desc(su32(sQ), 16, 1024);
      const uint64_t k_d0 = desc(su32(sK), 16, 1024);
      const uint64_t v_d0 = desc(su32(sV), 16384, 1024);
      constexpr uint32_t TILE16 = TILE_BYTES >> 4;
      auto qk = [&](int i, int j) {
        const uint64_t qd = q_d0 + (uint64_t)(i * TILE16), kd = k_d0 + (uint64_t)((j & 1) * TILE16);
        const uint32_t d = tmem + i * 128;
        mma_ss(d, qd, kd, id_qk, 0);
#pragma unroll
        for (int k = 1; k < 8; ++k) {
          const uint32_t off = (k >> 2) * 1024 + (k & 3) * 2;
          mma_ss(d, qd + off, kd + off, id_qk, 1);
        }
        commit(&s_full[i]);
      };
      // O_i += P_i(j) V_j: P from the first 64 columns of S_i (packed bf16), V as an MN-major B operand
      auto pv = [&](int i, int j) {
        const uint64_t vd = v_d0 + (uint64_t)((j & 1) * TILE16);
        const uint32_t d = tmem + 256 + i * 128, a = tmem + i * 128;
        mma_ts(d, a, vd, id_pv, j != 0);
#pragma unroll
        for (int k = 1; k < 8; ++k) mma_ts(d, a + k * 8, vd + k * 128, id_pv, 1);
      };
      auto wait_k = [&](int j) -> bool {
        return bar_wait(&k_full[j & 1], (j >> 1) & 1, p.err, 23) && !*abort_flag;
      };
      ok = bar_wait(&q_full[0], 0, p.err, 24) && (!has1 || bar_wait(&q_full[1], 0, p.err, 24)) && wait_k(0);
      if (ok) {
        fence_after();
        qk(0, 0);
        if (has1) qk(1, 0);
        commit(&k_empty[0]);
      }
      for (int j = 0; j < nl && ok; ++j) {
        const uint32_t ph = j & 1;
        unsigned long long t0 = p.timing ? clk64() : 0;
        if (!bar_wait(&v_full[j & 1], (j >> 1) & 1, p.err, 25)) { ok = false; break; }
        if (p.timing) { const unsigned long long t1 = clk64(); t_v += t1 - t0; t0 = t1; }
        if (j < n0) {
          if (!bar_wait(&p_full[0], ph, p.err, 26) || *abort_flag) { ok = false; break; }
          if (p.timing) { const unsigned long long t1 = clk64(); t_p += t1 - t0; t0 = t1; }
          fence_after();
          pv(0, j);
          if (j + 1 < n0) {
            if (!wait_k(j + 1)) { ok = false; break; }
            qk(0, j + 1);
          }
        }
        if (j < n1) {
          if (p.timing) t0 = clk64();
          if (!bar_wait(&p_full[1], ph, p.err, 27) || *abort_flag) { ok = false; break; }
          if (p.timing) t_p += clk64() - t0;
          fence_after();
          pv(1, j);
        }
        commit(&v_empty[j & 1]);
        if (j + 1 < nl) {
          if (!wait_k(j + 1)) { ok = false; break; }
          if (j + 1 < n1) qk(1, j + 1);
          commit(&k_empty[(j + 1) & 1]);
        }
      }
      if (p.timing) {
        atomicAdd(&g_fa_dbg[0], t_v);
        atomicAdd(&g_fa_dbg[1], t_p);
        atomicAdd(&g_fa_dbg[2], clk64() - t_start);
        atomicAdd(&g_fa_dbg[3], 1ull);
      }
      if (ok) {
        commit(&o_final[0]);
        if (has1) commit(&o_final[1]);
      } else {
        *abort_flag = 1;
      }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------------ softmax groups
    const int grp = (warp - 2) >> 2;  // query tile
    const int quarter = warp & 3;     // TMEM lane quarter
    const int row = quarter * 32 + lane;
    const int qt = grp ? qt1 : qt0;
    const int n = grp ? n1 : n0;
    const bool active = grp == 0 || has1;
    const int qpos = qt * BQ + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_cols = tmem + lane_base + grp * 128;
    const uint32_t o_cols = tmem + lane_base + 256 + grp * 128;
    const float c = p.scale_log2;
    float m_run = -INFINITY, l = 0.f;
    bool ok = true;
    unsigned long long sw_wait = 0, sw_work = 0, sw_max = 0, sw_resc = 0, sw_exp = 0;
    for (int j = 0; j < n; ++j) {
      const unsigned long long ta = p.timing ? clk64() : 0;
      if (!bar_wait(&s_full[grp], j & 1, p.err, 31) || *abort_flag) { ok = false; break; }
      const unsigned long long tb = p.timing ? clk64() : 0;
      sw_wait += tb - ta;
      fence_after();
      const bool diag = p.causal && j == qt;
      uint32_t r[128];
      FA_TMEM_LD_32(s_cols, r);
      FA_TMEM_LD_32(s_cols + 32, (r + 32));
      FA_TMEM_LD_32(s_cols + 64, (r + 64));
      FA_TMEM_LD_32(s_cols + 96, (r + 96));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (diag) {
        const int lim = qpos - j * BKV;  // keys with index > lim are masked
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > lim) r[i] = __float_as_uint(-INFINITY);
      }
      float mx4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) mx4[k] = fmaxf(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
#pragma unroll
      for (int i = 8; i < 128; i += 2) {
        mx4[(i >> 1) & 3] = max3(mx4[(i >> 1) & 3], __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float m_new = mx * c;
      const unsigned long long tmx = p.timing ? clk64() : 0;
      if (p.timing) sw_max += tmx - tb;
      // lazy rescale: keep the running max unless this row's max grew by more than the threshold
      const bool need = m_new > m_run + RESCALE_THRESHOLD;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        if (p.timing && lane == 0) atomicAdd(&g_fa_dbg[7], 1ull);
        // PV_grp(j - 1) has completed: it was issued before S_grp(j), whose commit we just waited on
        const float alpha = need ? ex2(m_run - m_new) : 1.f;
#pragma unroll 1
        for (int q8 = 0; q8 < 8; ++q8) {
          uint32_t o[16];
          FA_TMEM_LD_16(o_cols + q8 * 16, o);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          FA_TMEM_ST_16(o_cols + q8 * 16, o);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        if (need) {
          l *= alpha;
          m_run = m_new;
        }
      } else if (need) {
        m_run = m_new;  // first tile (O is not read by PV(0)) or no rescale needed in this warp
        l = 0.f;
      }
      // Row sum in fp32, P packed to bf16 pairs into the first 64 columns of S (the PV MMA's A operand).
      const unsigned long long tex = p.timing ? clk64() : 0;
      if (p.timing) sw_resc += tex - tmx;
      const uint64_t cc = pk2(c, c), nmm = pk2(-m_run, -m_run);
      uint64_t sum2[2] = {0ull, 0ull};
      // S is read again from TMEM one 32-column chunk at a time (the row held whole only for the max), so the
      // exponent pass needs few registers; P chunk h2 goes to columns [16 h2, 16 h2 + 16), all already read.
#pragma unroll
      for (int h2 = 0; h2 < 4; ++h2) {
        uint32_t x[32];
        FA_TMEM_LD_32(s_cols + h2 * 32, x);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (diag) {
          const int lim = qpos - j * BKV - h2 * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i > lim) x[i] = __float_as_uint(-INFINITY);
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint64_t x2 = fma2(pk2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), cc, nmm);
          uint64_t e2;
          if ((i % 3) == 2) {
            e2 = ex2_poly2(x2);
          } else {
            float x0, x1;
            up2(x2, x0, x1);
            e2 = pk2(ex2(x0), ex2(x1));
          }
          sum2[i & 1] = add2(sum2[i & 1], e2);
          float e0, e1;
          up2(e2, e0, e1);
          asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(pk[i]) : "f"(e1), "f"(e0));
        }
        FA_TMEM_ST_16(s_cols + h2 * 16, pk);
      }
      {
        const uint64_t t2 = add2(sum2[0], sum2[1]);
        float s0, s1;
        up2(t2, s0, s1);
        l += s0 + s1;
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&p_full[grp]);
      if (p.timing) {
        const unsigned long long te = clk64();
        sw_work += te - tb;
        sw_exp += te - tex;
      }
    }
    if (p.timing && lane == 0) {
      atomicAdd(&g_fa_dbg[4], sw_wait);
      atomicAdd(&g_fa_dbg[5], sw_work);
      atomicAdd(&g_fa_dbg[6], 1ull);
      atomicAdd(&g_fa_dbg[8], sw_max);
      atomicAdd(&g_fa_dbg[9], sw_resc);
      atomicAdd(&g_fa_dbg[10], sw_exp);
      atomicAdd(&g_fa_dbg[11], (unsigned long long)n);
    }
    if (ok && active) ok = bar_wait(&o_final[grp], 0, p.err, 32) && !*abort_flag;
    if (!active) {
      // no second query tile in this CTA
    } else if (!ok) {
      *abort_flag = 1;
    } else {
      fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* dst = p.o + (((size_t)qpos * p.b + bidx) * H + h) * D;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t o[32];
        FA_TMEM_LD_32(o_cols + q4 * 32, o);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(o[v8 * 8 + i]) * inv;
          reinterpret_cast<uint4*>(dst + q4 * 32)[v8] = pack8(f);
        }
      }
      p.lse[((size_t)bidx * H + h) * p.s + qpos] = (m_run + __log2f(l)) * 0.6931471805599453f;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

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

static int* err_flag() { return device_err_flag(kErrAttnFwd); }

// {d, slot, b, s} view of the fused QKV activation with 128-row x 64-column boxes.
CUtensorMap qkv_map(const at::Tensor& qkv) {
  const int64_t s = qkv.size(0), b = qkv.size(1), G = qkv.size(2), S = qkv.size(3), d = qkv.size(4);
  CUtensorMap m;
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)(G * S), (cuuint64_t)b, (cuuint64_t)s};
  cuuint64_t strides[3] = {(cuuint64_t)(d * 2), (cuuint64_t)(G * S * d * 2), (cuuint64_t)(b * G * S * d * 2)};
  cuuint32_t box[4] = {64, 1, 1, 128};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, qkv.data_ptr(), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled(qkv) failed: ", (int)r);
  return m;
}

}  // namespace fa

bool attn_supported(at::Tensor qkv) {
  return qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous() && qkv.dim() == 5 &&
         qkv.size(4) == 128 && qkv.size(0) % 128 == 0 &&
         (reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16) == 0;
}

// Returns (o [s, b, H*d] bf16, lse [b, H, s] fp32).
std::vector<at::Tensor> attn_fwd(at::Tensor qkv, int64_t hpg, bool causal) {
  using namespace fa;
  TORCH_CHECK(attn_supported(qkv), "attn_fwd: needs contiguous bf16 [s, b, G, hpg+2, 128] with s % 128 == 0");
  const int64_t s = qkv.size(0), b = qkv.size(1), G = qkv.size(2);
  TORCH_CHECK(qkv.size(3) == hpg + 2, "attn_fwd: slot count must be hpg + 2");
  const int64_t H = G * hpg;
  auto o = at::empty({s, b, H * D}, qkv.options());
  auto lse = at::empty({b, H, s}, qkv.options().dtype(at::kFloat));
  CUtensorMap m = qkv_map(qkv);
  Params p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.s = (int)s;
  p.b = (int)b;
  p.G = (int)G;
  p.hpg = (int)hpg;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
  p.causal = causal ? 1 : 0;
  p.err = err_flag();
  static const int timing = [] {
    const char* e = std::getenv("EMB_ATTN_TIMING");
    return (e && std::atoi(e) == 1) ? 1 : 0;
  }();
  p.timing = timing;
  static bool attr[kMaxDevices] = {};
  int dev = 0;
  EMB_CUDA_CHECK(cudaGetDevice(&dev));
  if (!attr[dev]) {
    EMB_CUDA_CHECK(cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr[dev] = true;
  }
  dim3 grid((unsigned)(b * H), (unsigned)((s / BQ + 1) / 2));
  flash_fwd_kernel<<<grid, NUM_THREADS, SMEM_BYTES, cur_stream()>>>(m, p);
  EMB_LAUNCH_CHECK();
  count_launch();
  return {o, lse};
}

namespace fa {
// scalar and packed forms: even elements through ex2_poly2 in pairs, an odd tail through ex2_poly
__global__ void exp2_emulated_kernel(const float* x, float* y, int64_t n) {
  for (int64_t i = 2 * (blockIdx.x * (int64_t)blockDim.x + threadIdx.x); i < n; i += 2 * (int64_t)gridDim.x * blockDim.x) {
    if (i + 1 < n) {
      float a, b;
      up2(ex2_poly2(pk2(x[i], x[i + 1])), a, b);
      y[i] = a;
      y[i + 1] = b;
    } else {
      y[i] = ex2_poly(x[i]);
    }
  }
}
}  // namespace fa

// The softmax's FMA-pipe 2^x on a float tensor (accuracy tests against exp2).
at::Tensor attn_exp2_emulated(at::Tensor x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous());
  auto y = at::empty_like(x);
  const int64_t n = x.numel();
  if (n) {
    fa::exp2_emulated_kernel<<<(int)std::min<int64_t>((n + 255) / 256, 4096), 256, 0, cur_stream()>>>(
        x.data_ptr<float>(), y.data_ptr<float>(), n);
    EMB_LAUNCH_CHECK();
    count_launch();
  }
  return y;
}

// Per-role cycle counters of the forward kernel when EMB_ATTN_TIMING=1 (measurement only), then reset:
// [MMA waits for V, MMA waits for P, MMA total, MMA threads, softmax waits for S, softmax work, softmax warps,
//  rescales].
std::vector<int64_t> attn_debug_counters() {
  unsigned long long h[16];
  EMB_CUDA_CHECK(cudaMemcpyFromSymbol(h, fa::g_fa_dbg, sizeof(h)));
  unsigned long long z[16] = {0};
  EMB_CUDA_CHECK(cudaMemcpyToSymbol(fa::g_fa_dbg, z, sizeof(z)));
  return std::vector<int64_t>(h, h + 16);
}

int64_t attn_error_flag() {
  int v = 0;
  EMB_CUDA_CHECK(cudaMemcpy(&v, fa::err_flag(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

}  // namespace emb
