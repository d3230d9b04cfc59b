// K10 (forward): causal GQA flash attention on tcgen05 / TMEM / TMA, sm_100a, head dim 128.
//
// Input is the fused QKV activation of the model, [s, b, G, hpg + 2, d] bf16 (per query group: hpg query
// heads, one key, one value); it is read in place through one 4-D TMA tensor map {d, slot, b, s}.  Output
// o [s, b, H, d] bf16 and the per-row log-sum-exp lse [b, H, s] fp32 (natural log of the scaled scores) for
// the backward pass.
//
// One CTA = one (128-row query tile, batch, head); 192 threads:
//   warp 0      - TMA: Q once (2 boxes of 128 x 64), then K_j and V_j into 2-deep rings;
//   warp 1      - TMEM owner (512 columns: S0, S1, O) and MMA issuer (one thread):
//                 S_j = Q K_j^T (M=128, N=128, K=128) into S[j % 2], and O_j = P_j V_j (P from shared memory,
//                 V as an MN-major operand) one step behind, so S_{j+1} is computed while row j is in softmax;
//   warps 2..5  - one thread per query row: read S_j from TMEM (two passes: max, then exp2), online-softmax
//                 statistics in registers, P_j written as bf16 into a 128-byte-swizzled K-major tile (the
//                 layout the MMA reads), then the previous O tile folded into a 128-float register
//                 accumulator with its rescale factor.  The final O / l is stored straight from registers.
// Causal masking only touches the diagonal tile (equal 128 tiles for queries and keys).
// All mbarrier waits are bounded (error flag + early exit); no TMA multicast.
#include <cudaTypedefs.h>

#include "../include/common.cuh"

namespace emb {
namespace fa {

constexpr int D = 128, BQ = 128, BKV = 128;
constexpr int TILE_BYTES = 128 * 128 * 2;  // one 128 x 128 bf16 tile = two 16 KiB swizzle panels
constexpr int SMEM_BYTES = 7 * TILE_BYTES + 1024 + 256;
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
// bf16 x bf16 -> fp32, M=128, N=128; b_mn selects an MN-major B operand.
__host__ __device__ constexpr uint32_t idesc(bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(128 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
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

struct Params {
  __nv_bfloat16* o;
  float* lse;
  int s, b, G, hpg;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  int* err;
};

// Smem K-major 128 x 128 bf16 tile with 128-byte swizzle: two 64-column panels of 16 KiB.
__device__ __forceinline__ uint32_t swz_off(int row, int col) {
  const int panel = col >> 6, c = col & 63;
  const int g = (c >> 3) ^ (row & 7);
  return panel * 16384 + row * 128 + g * 16 + (c & 7) * 2;
}

__global__ void __launch_bounds__(192, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = sm;
  uint8_t* sK = sm + TILE_BYTES;      // [2]
  uint8_t* sV = sm + 3 * TILE_BYTES;  // [2]
  uint8_t* sP = sm + 5 * TILE_BYTES;  // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 7 * TILE_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]
  uint64_t* s_empty = bars + 11; // [2]
  uint64_t* p_full = bars + 13;  // [2]
  uint64_t* p_empty = bars + 15; // [2]
  uint64_t* o_full = bars + 17;
  uint64_t* o_empty = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 20);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.s / BQ;
  const int qt = nq - 1 - blockIdx.x;  // heavy (late) query tiles first
  const int H = p.G * p.hpg;
  const int bh = blockIdx.y;
  const int bidx = bh / H, h = bh % H;
  const int g = h / p.hpg, hj = h % p.hpg;
  const int slots = p.hpg + 2;
  const int q_slot = g * slots + hj, k_slot = g * slots + p.hpg, v_slot = g * slots + p.hpg + 1;
  const int nkv = p.causal ? qt + 1 : p.s / BKV;

  if (threadIdx.x == 0) {
    bar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      bar_init(&k_full[i], 1);
      bar_init(&k_empty[i], 1);
      bar_init(&v_full[i], 1);
      bar_init(&v_empty[i], 1);
      bar_init(&s_full[i], 1);
      bar_init(&s_empty[i], 4);
      bar_init(&p_full[i], 4);
      bar_init(&p_empty[i], 1);
    }
    bar_init(o_full, 1);
    bar_init(o_empty, 4);
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
    if (lane == 0) {
      bar_expect(q_full, TILE_BYTES);
      tma4(sQ, &tm, q_full, 0, q_slot, bidx, qt * BQ);
      tma4(sQ + 16384, &tm, q_full, 64, q_slot, bidx, qt * BQ);
      for (int j = 0; j < nkv; ++j) {
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
    if (lane == 0) {
      const uint32_t id_qk = idesc(false), id_pv = idesc(true);
      bool ok = bar_wait(q_full, 0, p.err, 23) && !*abort_flag;
      const uint32_t q_addr = su32(sQ);
      auto pv = [&](int jj) -> bool {
        const int st = jj & 1;
        const uint32_t ph = (jj >> 1) & 1;
        if (!bar_wait(&v_full[st], ph, p.err, 24) || !bar_wait(&p_full[st], ph, p.err, 25) ||
            !bar_wait(o_empty, (jj & 1) ^ 1, p.err, 26) || *abort_flag)
          return false;
        fence_after();
        const uint32_t pa = su32(sP + st * TILE_BYTES), va = su32(sV + st * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          // A = P (K-major over the key index), B = V as MN-major (rows = keys, 64-wide d panels 16 KiB apart)
          mma(tmem + 256, desc(pa + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024), desc(va + k * 2048, 16384, 1024),
              id_pv, k != 0);
        }
        commit(&v_empty[st]);
        commit(&p_empty[st]);
        commit(o_full);
        return true;
      };
      for (int j = 0; j < nkv && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!bar_wait(&k_full[st], ph, p.err, 27) || !bar_wait(&s_empty[st], ph ^ 1, p.err, 28) || *abort_flag) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t ka = su32(sK + st * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          mma(tmem + st * 128, desc(q_addr + off, 16, 1024), desc(ka + off, 16, 1024), id_qk, k != 0);
        }
        commit(&k_empty[st]);
        commit(&s_full[st]);
        if (j >= 1) ok = pv(j - 1);
      }
      if (ok) ok = pv(nkv - 1);
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------------ softmax / correction warps
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // row of the query tile == TMEM lane
    const int qpos = qt * BQ + row;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float oacc[D];
#pragma unroll
    for (int i = 0; i < D; ++i) oacc[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool ok = true;
    auto correct = [&](int jj, float alpha) -> bool {
      if (!bar_wait(o_full, jj & 1, p.err, 31) || *abort_flag) return false;
      fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        FA_TMEM_LD_32(tmem + lane_base + 256 + c * 32, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 32; ++i) oacc[c * 32 + i] = oacc[c * 32 + i] * alpha + __uint_as_float(r[i]);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(o_empty);
      return true;
    };
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!bar_wait(&s_full[st], ph, p.err, 32) || *abort_flag) { ok = false; break; }
      fence_after();
      const bool diag = p.causal && j == qt;
      const uint32_t sbase = tmem + lane_base + st * 128;
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        FA_TMEM_LD_32(sbase + c * 32, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kpos = j * BKV + c * 32 + i;
          const float v = (diag && kpos > qpos) ? -INFINITY : __uint_as_float(r[i]) * p.scale_log2;
          mx = fmaxf(mx, v);
        }
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = exp2f(m - m_new);
      // P buffer of this stage must have been consumed by the PV MMA two tiles ago
      if (!bar_wait(&p_empty[st], ph ^ 1, p.err, 33) || *abort_flag) { ok = false; break; }
      uint8_t* pbuf = sP + st * TILE_BYTES;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        FA_TMEM_LD_32(sbase + c * 32, r);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        float pv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kpos = j * BKV + c * 32 + i;
          const float v = (diag && kpos > qpos) ? -INFINITY : __uint_as_float(r[i]) * p.scale_log2;
          pv[i] = exp2f(v - m_new);
          sum += pv[i];
        }
#pragma unroll
        for (int v8 = 0; v8 < 4; ++v8) {
          *reinterpret_cast<uint4*>(pbuf + swz_off(row, c * 32 + v8 * 8)) = pack8(pv + v8 * 8);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive(&s_empty[st]);
      // make the generic-proxy writes of P visible to the tensor core before signalling the MMA warp
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) bar_arrive(&p_full[st]);
      l = l * alpha + sum;
      m = m_new;
      if (j >= 1) {
        if (!correct(j - 1, alpha_prev)) { ok = false; break; }
      }
      alpha_prev = alpha;
    }
    if (ok) ok = correct(nkv - 1, alpha_prev);
    if (!ok) *abort_flag = 1;
    if (ok) {
      const float inv = 1.f / l;
      __nv_bfloat16* dst = p.o + (((size_t)qpos * p.b + bidx) * H + h) * D;
#pragma unroll
      for (int v8 = 0; v8 < D / 8; ++v8) {
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = oacc[v8 * 8 + i] * inv;
        reinterpret_cast<uint4*>(dst)[v8] = pack8(f);
      }
      p.lse[((size_t)bidx * H + h) * p.s + qpos] = (m + log2f(l)) * 0.6931471805599453f;
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
  static bool attr = false;
  if (!attr) {
    EMB_CUDA_CHECK(cudaFuncSetAttribute(flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    attr = true;
  }
  dim3 grid((unsigned)(s / BQ), (unsigned)(b * H));
  flash_fwd_kernel<<<grid, 192, SMEM_BYTES, cur_stream()>>>(m, p);
  EMB_LAUNCH_CHECK();
  count_launch();
  return {o, lse};
}

int64_t attn_error_flag() {
  int v = 0;
  EMB_CUDA_CHECK(cudaMemcpy(&v, fa::err_flag(), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

}  // namespace emb
