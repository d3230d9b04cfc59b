// RMSNorm (fwd/bwd), SwiGLU (fwd/bwd) and RoPE on the fused QKV layout; bf16 I/O, fp32 math.
// Memory-bound kernels: 16-byte vector loads/stores, one CTA per row for the norms, persistent CTAs with
// per-CTA fp32 partials (reduced in a fixed order, so results are deterministic) for the weight gradient.
#include "../include/common.cuh"

namespace emb {

// ------------------------------------------------------------------------------------------ RMSNorm fwd
template <int VPT>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int H, float eps) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      uint4 u = xr[i];
      unpack8(u, v[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[k][j] * v[k][j];
    }
  }
  ss = block_sum(ss, sh);
  const float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd_out[row] = r;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * H);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float wf[8], o[8];
      unpack8(wr[i], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[k][j] * r * wf[j];
      yr[i] = pack8(o);
    }
  }
}

// Residual add fused into the norm that follows it: h = x + o (rounded to bf16, the residual stream's type),
// y = RMSNorm(h) * w.  One read of x and o, one write of h and y: the unfused pair reads h back.
template <int VPT>
__global__ void add_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ o,
                                       const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ h,
                                       __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int H, float eps) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  const uint4* orow = reinterpret_cast<const uint4*>(o + (size_t)row * H);
  uint4* hr = reinterpret_cast<uint4*>(h + (size_t)row * H);
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float a[8], b[8];
      unpack8(xr[i], a);
      unpack8(orow[i], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
      const uint4 u = pack8(a);
      hr[i] = u;
      unpack8(u, v[k]);  // the norm sees the rounded residual, as the unfused pair does
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[k][j] * v[k][j];
    }
  }
  ss = block_sum(ss, sh);
  const float r = rsqrtf(ss / H + eps);
  if (threadIdx.x == 0) rstd_out[row] = r;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * H);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float wf[8], t[8];
      unpack8(wr[i], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] = v[k][j] * r * wf[j];
      yr[i] = pack8(t);
    }
  }
}

// threads per row so that each thread holds at most 4 16-byte vectors of the row in registers
static int pick_threads(int nvec, int& vpt) {
  int t = ((nvec + 3) / 4 + 31) / 32 * 32;
  t = std::max(32, std::min(1024, t));
  vpt = (nvec + t - 1) / t;
  return t;
}

std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(w, "w");
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 4 * 1024, "hidden size must be a multiple of 8 and <= 32768");
  auto y = at::empty_like(x);
  auto rstd = at::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {y, rstd};
  int vpt;
  int threads = pick_threads((int)(H / 8), vpt);
  auto st = cur_stream();
#define L(V) rmsnorm_fwd_kernel<V><<<T, threads, 0, st>>>((const __nv_bfloat16*)x.data_ptr(),          \
      (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)y.data_ptr(), rstd.data_ptr<float>(), (int)H, \
      (float)eps)
  if (vpt <= 1) L(1); else if (vpt == 2) L(2); else if (vpt == 3) L(3); else L(4);
#undef L
  EMB_LAUNCH_CHECK();
  count_launch();
  return {y, rstd};
}

// Returns (h = x + o, y = RMSNorm(h) * w, rstd).
std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, at::Tensor o, at::Tensor w, double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(o, "o");
  check_cuda_bf16(w, "w");
  TORCH_CHECK(x.sizes() == o.sizes() && x.dim() == 2, "add_rmsnorm_fwd: x and o must be equal [T, H]");
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 4 * 1024, "hidden size must be a multiple of 8 and <= 32768");
  auto h = at::empty_like(x);
  auto y = at::empty_like(x);
  auto rstd = at::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {h, y, rstd};
  int vpt;
  int threads = pick_threads((int)(H / 8), vpt);
  auto st = cur_stream();
#define L(V) add_rmsnorm_fwd_kernel<V><<<T, threads, 0, st>>>((const __nv_bfloat16*)x.data_ptr(),                 \
      (const __nv_bfloat16*)o.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), (__nv_bfloat16*)h.data_ptr(),      \
      (__nv_bfloat16*)y.data_ptr(), rstd.data_ptr<float>(), (int)H, (float)eps)
  if (vpt <= 1) L(1); else if (vpt == 2) L(2); else if (vpt == 3) L(3); else L(4);
#undef L
  EMB_LAUNCH_CHECK();
  count_launch();
  return {h, y, rstd};
}

// ------------------------------------------------------------------------------------------ RMSNorm bwd
// Persistent CTAs, several per SM (rows_in_flight), each walking rows r, r + grid, ...  A row is read twice: the
// first pass forms the dot product the second needs (and the fp32 dw partial), the second - served from L1, where
// the first pass left the row's 2 x H bf16 values - writes dx.  Holding only w and the dw partial in registers
// keeps the CTA small enough for four per SM, so four rows' loads are in flight per SM instead of two.
template <int VPT>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   __nv_bfloat16* __restrict__ dx, float* __restrict__ dw_part, int T, int H,
                                   const __nv_bfloat16* __restrict__ dres = nullptr) {
  __shared__ float sh[32];
  const int nvec = H / 8;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  float wf[VPT][8], acc[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
    if (i < nvec) unpack8(wr[i], wf[k]);
  }
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
    const uint4* dr = reinterpret_cast<const uint4*>(dy + (size_t)row * H);
    const float r = rstd[row];
    float dot = 0.f;
    uint4 xv[VPT], dv[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        xv[k] = xr[i];
        dv[k] = dr[i];
      }
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        float xf[8], d[8];
        unpack8(xv[k], xf);
        unpack8(dv[k], d);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = xf[j] * r;
          dot += d[j] * wf[k][j] * xh;
          acc[k][j] += d[j] * xh;
        }
      }
    }
    dot = block_sum(dot, sh) / H;
    uint4* o = reinterpret_cast<uint4*>(dx + (size_t)row * H);
    // dres: the residual stream's gradient, added here when the forward fused the residual add into the norm
    const uint4* rr = dres ? reinterpret_cast<const uint4*>(dres + (size_t)row * H) : nullptr;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        float xf[8], d[8], t[8];
        unpack8(xr[i], xf);  // second read of the row: an L1 hit
        unpack8(dr[i], d);
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = r * (d[j] * wf[k][j] - xf[j] * r * dot);
        if (rr) {
          float a[8];
          unpack8(rr[i], a);
#pragma unroll
          for (int j = 0; j < 8; ++j) t[j] += a[j];
        }
        o[i] = pack8(t);
      }
    }
  }
  float* part = dw_part + (size_t)blockIdx.x * H;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float4* p4 = reinterpret_cast<float4*>(part + i * 8);
      p4[0] = make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]);
      p4[1] = make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]);
    }
  }
}

// Rows in flight per SM for the norm backward kernels (persistent grid = SMs x this, at most T).
constexpr int kNormBwdCtasPerSm = 4;
static int64_t norm_bwd_grid(int64_t T) {
  return std::max<int64_t>(1, std::min<int64_t>(T, (int64_t)num_sms() * kNormBwdCtasPerSm));
}

// dw[h] = sum_b part[b, h] in a fixed order (warp w adds rows w, w + 8, ...; then the 8 warp sums in order);
// optionally accumulated into an fp32 target.  32 columns per CTA.
__global__ void colsum_kernel(const float* __restrict__ part, float* __restrict__ out, int nb, int H, int accumulate) {
  __shared__ float sm[8][33];
  const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
  const int h = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (h < H)
    for (int b = wp; b < nb; b += 8) s += part[(size_t)b * H + h];
  sm[wp][lane] = s;
  __syncthreads();
  if (wp == 0 && h < H) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += sm[k][lane];
    out[h] = accumulate ? out[h] + t : t;
  }
}
static void launch_colsum(const float* part, float* out, int nb, int H, int accumulate, cudaStream_t st) {
  colsum_kernel<<<(H + 31) / 32, 256, 0, st>>>(part, out, nb, H, accumulate);
}

std::vector<at::Tensor> rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd,
                                       c10::optional<at::Tensor> dw_accum, c10::optional<at::Tensor> dres) {
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(x, "x");
  const int64_t T = x.size(0), H = x.size(1);
  const bool has_res = dres.has_value() && dres->defined();
  if (has_res) {
    check_cuda_bf16(*dres, "dres");
    TORCH_CHECK(dres->sizes() == x.sizes(), "rmsnorm_bwd: dres must match x");
  }
  auto dx = at::empty_like(x);
  int vpt;
  int threads = pick_threads((int)(H / 8), vpt);
  const int grid = (int)norm_bwd_grid(T);
  auto part = at::empty({grid, H}, x.options().dtype(at::kFloat));
  auto st = cur_stream();
  const __nv_bfloat16* rp = has_res ? (const __nv_bfloat16*)dres->data_ptr() : nullptr;
#define L(V) rmsnorm_bwd_kernel<V><<<grid, threads, 0, st>>>((const __nv_bfloat16*)dy.data_ptr(),                  \
      (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), rstd.data_ptr<float>(),               \
      (__nv_bfloat16*)dx.data_ptr(), part.data_ptr<float>(), (int)T, (int)H, rp)
  if (vpt <= 1) L(1); else if (vpt == 2) L(2); else if (vpt == 3) L(3); else L(4);
#undef L
  EMB_LAUNCH_CHECK();
  at::Tensor dw;
  bool acc = dw_accum.has_value() && dw_accum->defined();
  if (acc) {
    dw = *dw_accum;
    TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.numel() == H);
  } else {
    dw = at::empty({H}, x.options().dtype(at::kFloat));
  }
  launch_colsum(part.data_ptr<float>(), dw.data_ptr<float>(), grid, (int)H, acc, st);
  EMB_LAUNCH_CHECK();
  count_launch(2);
  return {dx, dw};
}

// ------------------------------------------------------------------------------------------ LayerNorm
// Megatron's LayerNorm (weight and bias) over the last dimension, bf16 I/O, fp32 statistics: one CTA per row
// in the forward; the backward runs persistent CTAs that keep per-CTA fp32 partials of dw and db (reduced in
// a fixed order by colsum_kernel, so the result is deterministic), like the RMSNorm backward.
template <int VPT>
__global__ void layernorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                     const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ y,
                                     float* __restrict__ mean_out, float* __restrict__ rstd_out, int H, float eps) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
  float v[VPT][8];
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      unpack8(xr[i], v[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) sum += v[k][j];
    }
  }
  const float mu = block_sum(sum, sh) / H;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[k][j] - mu;
        ss += d * d;
      }
    }
  }
  const float r = rsqrtf(block_sum(ss, sh) / H + eps);
  if (threadIdx.x == 0) {
    mean_out[row] = mu;
    rstd_out[row] = r;
  }
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  const uint4* br = reinterpret_cast<const uint4*>(bias);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)row * H);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float wf[8], bf[8], o[8];
      unpack8(wr[i], wf);
      unpack8(br[i], bf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[k][j] - mu) * r * wf[j] + bf[j];
      yr[i] = pack8(o);
    }
  }
}

template <int VPT>
__global__ void layernorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                     const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean,
                                     const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                     float* __restrict__ dw_part, float* __restrict__ db_part, int T, int H) {
  __shared__ float sh[32];
  const int nvec = H / 8;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  float wf[VPT][8], accw[VPT][8], accb[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) accw[k][j] = accb[k][j] = 0.f;
    if (i < nvec) unpack8(wr[i], wf[k]);
  }
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)row * H);
    const uint4* dr = reinterpret_cast<const uint4*>(dy + (size_t)row * H);
    const float mu = mean[row], r = rstd[row];
    float xh[VPT][8], g[VPT][8];
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        float d[8];
        unpack8(xr[i], xh[k]);
        unpack8(dr[i], d);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[k][j] = (xh[k][j] - mu) * r;
          g[k][j] = d[j] * wf[k][j];
          sg += g[k][j];
          sgx += g[k][j] * xh[k][j];
          accw[k][j] += d[j] * xh[k][j];
          accb[k][j] += d[j];
        }
      }
    }
    // dx = r * (g - mean(g) - xhat * mean(g * xhat))
    const float mg = block_sum(sg, sh) / H;
    const float mgx = block_sum(sgx, sh) / H;
    uint4* o = reinterpret_cast<uint4*>(dx + (size_t)row * H);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = r * (g[k][j] - mg - xh[k][j] * mgx);
        o[i] = pack8(t);
      }
    }
  }
  float* pw = dw_part + (size_t)blockIdx.x * H;
  float* pb = db_part + (size_t)blockIdx.x * H;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      float4* w4 = reinterpret_cast<float4*>(pw + i * 8);
      float4* b4 = reinterpret_cast<float4*>(pb + i * 8);
      w4[0] = make_float4(accw[k][0], accw[k][1], accw[k][2], accw[k][3]);
      w4[1] = make_float4(accw[k][4], accw[k][5], accw[k][6], accw[k][7]);
      b4[0] = make_float4(accb[k][0], accb[k][1], accb[k][2], accb[k][3]);
      b4[1] = make_float4(accb[k][4], accb[k][5], accb[k][6], accb[k][7]);
    }
  }
}

// Returns (y, mean, rstd).
std::vector<at::Tensor> layernorm_fwd(at::Tensor x, at::Tensor w, at::Tensor b, double eps) {
  check_cuda_bf16(x, "x");
  check_cuda_bf16(w, "w");
  check_cuda_bf16(b, "b");
  TORCH_CHECK(x.dim() == 2, "layernorm_fwd: x must be [T, H]");
  const int64_t T = x.size(0), H = x.size(1);
  TORCH_CHECK(H % 8 == 0 && H <= 8 * 4 * 1024, "hidden size must be a multiple of 8 and <= 32768");
  auto y = at::empty_like(x);
  auto mean = at::empty({T}, x.options().dtype(at::kFloat));
  auto rstd = at::empty({T}, x.options().dtype(at::kFloat));
  if (T == 0) return {y, mean, rstd};
  int vpt;
  int threads = pick_threads((int)(H / 8), vpt);
  auto st = cur_stream();
#define L(V) layernorm_fwd_kernel<V><<<T, threads, 0, st>>>((const __nv_bfloat16*)x.data_ptr(),                  \
      (const __nv_bfloat16*)w.data_ptr(), (const __nv_bfloat16*)b.data_ptr(), (__nv_bfloat16*)y.data_ptr(),      \
      mean.data_ptr<float>(), rstd.data_ptr<float>(), (int)H, (float)eps)
  if (vpt <= 1) L(1); else if (vpt == 2) L(2); else if (vpt == 3) L(3); else L(4);
#undef L
  EMB_LAUNCH_CHECK();
  count_launch();
  return {y, mean, rstd};
}

// Returns (dx, dw, db); dw / db are fp32 and, when given, accumulated into dw_accum / db_accum.
std::vector<at::Tensor> layernorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor mean, at::Tensor rstd,
                                      c10::optional<at::Tensor> dw_accum, c10::optional<at::Tensor> db_accum) {
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(x, "x");
  check_cuda_bf16(w, "w");
  const int64_t T = x.size(0), H = x.size(1);
  auto dx = at::empty_like(x);
  int vpt;
  int threads = pick_threads((int)(H / 8), vpt);
  int grid = (int)std::min<int64_t>(std::max<int64_t>(T, 1), (int64_t)num_sms() * 2);
  auto part = at::zeros({2, grid, H}, x.options().dtype(at::kFloat));
  auto st = cur_stream();
  if (T > 0) {
#define L(V) layernorm_bwd_kernel<V><<<grid, threads, 0, st>>>((const __nv_bfloat16*)dy.data_ptr(),                \
      (const __nv_bfloat16*)x.data_ptr(), (const __nv_bfloat16*)w.data_ptr(), mean.data_ptr<float>(),              \
      rstd.data_ptr<float>(), (__nv_bfloat16*)dx.data_ptr(), part.data_ptr<float>(),                                \
      part.data_ptr<float>() + (size_t)grid * H, (int)T, (int)H)
    if (vpt <= 1) L(1); else if (vpt == 2) L(2); else if (vpt == 3) L(3); else L(4);
#undef L
    EMB_LAUNCH_CHECK();
  }
  at::Tensor dw, db;
  const bool aw = dw_accum.has_value() && dw_accum->defined(), ab = db_accum.has_value() && db_accum->defined();
  dw = aw ? *dw_accum : at::empty({H}, x.options().dtype(at::kFloat));
  db = ab ? *db_accum : at::empty({H}, x.options().dtype(at::kFloat));
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.numel() == H);
  TORCH_CHECK(db.scalar_type() == at::kFloat && db.is_contiguous() && db.numel() == H);
  launch_colsum(part.data_ptr<float>(), dw.data_ptr<float>(), grid, (int)H, aw, st);
  launch_colsum(part.data_ptr<float>() + (size_t)grid * H, db.data_ptr<float>(), grid, (int)H, ab, st);
  EMB_LAUNCH_CHECK();
  count_launch(T > 0 ? 3 : 2);
  return {dx, dw, db};
}

// ------------------------------------------------------------------------------------------ SwiGLU
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ h, __nv_bfloat16* __restrict__ y, int64_t T,
                                  int F) {
  const int fv = F / 8;
  const int64_t n = T * fv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i / fv;
    int j = (int)(i - t * fv);
    const uint4* hr = reinterpret_cast<const uint4*>(h + t * 2 * F);
    float g[8], u[8], o[8];
    unpack8(hr[j], g);
    unpack8(hr[fv + j], u);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = g[k] / (1.f + __expf(-g[k])) * u[k];
    reinterpret_cast<uint4*>(y + t * F)[j] = pack8(o);
  }
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ h,
                                  __nv_bfloat16* __restrict__ dh, int64_t T, int F) {
  const int fv = F / 8;
  const int64_t n = T * fv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i / fv;
    int j = (int)(i - t * fv);
    const uint4* hr = reinterpret_cast<const uint4*>(h + t * 2 * F);
    float g[8], u[8], d[8], dg[8], du[8];
    unpack8(hr[j], g);
    unpack8(hr[fv + j], u);
    unpack8(reinterpret_cast<const uint4*>(dy + t * F)[j], d);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float s = 1.f / (1.f + __expf(-g[k]));
      float silu = g[k] * s;
      dg[k] = d[k] * u[k] * (s * (1.f + g[k] * (1.f - s)));
      du[k] = d[k] * silu;
    }
    uint4* o = reinterpret_cast<uint4*>(dh + t * 2 * F);
    o[j] = pack8(dg);
    o[fv + j] = pack8(du);
  }
}

static int ew_grid(int64_t n) {
  int64_t g = (n + 255) / 256;
  int64_t cap = (int64_t)num_sms() * 8;
  return (int)std::max<int64_t>(1, std::min(g, cap));
}

at::Tensor swiglu_fwd(at::Tensor h) {
  check_cuda_bf16(h, "h");
  const int64_t T = h.numel() / h.size(-1);
  const int F = (int)(h.size(-1) / 2);
  TORCH_CHECK(F % 8 == 0, "ffn size must be a multiple of 8");
  auto sizes = h.sizes().vec();
  sizes.back() = F;
  auto y = at::empty(sizes, h.options());
  if (T == 0) return y;
  swiglu_fwd_kernel<<<ew_grid(T * F / 8), 256, 0, cur_stream()>>>((const __nv_bfloat16*)h.data_ptr(),
                                                                  (__nv_bfloat16*)y.data_ptr(), T, F);
  EMB_LAUNCH_CHECK();
  count_launch();
  return y;
}

at::Tensor swiglu_bwd(at::Tensor dy, at::Tensor h) {
  check_cuda_bf16(dy, "dy");
  check_cuda_bf16(h, "h");
  const int64_t T = h.numel() / h.size(-1);
  const int F = (int)(h.size(-1) / 2);
  auto dh = at::empty_like(h);
  if (T == 0) return dh;
  swiglu_bwd_kernel<<<ew_grid(T * F / 8), 256, 0, cur_stream()>>>((const __nv_bfloat16*)dy.data_ptr(),
                                                                  (const __nv_bfloat16*)h.data_ptr(),
                                                                  (__nv_bfloat16*)dh.data_ptr(), T, F);
  EMB_LAUNCH_CHECK();
  count_launch();
  return dh;
}

// ------------------------------------------------------------------------------------------ RoPE
// qkv: [s, b, G, S, d] bf16; slots [0, nrot) are rotated (rotate-half pairs (i, i + d/2)); others copied.
// cos/sin: [s, d/2] fp32.  inverse: rotate by -angle (the backward pass).
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out,
                            const float* __restrict__ cosv, const float* __restrict__ sinv, int64_t S_tok, int B,
                            int GS, int S, int d, int nrot, int inverse) {
  const int half = d / 2;
  const int pv = half / 8;  // 8-pair vectors per slot
  const int64_t n = S_tok * B * GS * pv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / pv;
    int v = (int)(i - r * pv);
    int slot = (int)(r % GS) % S;
    int64_t tok = r / GS;  // s * B + b
    int64_t s = tok / B;
    const __nv_bfloat16* src = in + r * d;
    __nv_bfloat16* dst = out + r * d;
    uint4 a = reinterpret_cast<const uint4*>(src)[v];
    uint4 b = reinterpret_cast<const uint4*>(src + half)[v];
    if (slot < nrot) {
      float x1[8], x2[8], o1[8], o2[8];
      unpack8(a, x1);
      unpack8(b, x2);
      const float* cp = cosv + s * half + v * 8;
      const float* sp = sinv + s * half + v * 8;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float c = cp[k], sn = inverse ? -sp[k] : sp[k];
        o1[k] = x1[k] * c - x2[k] * sn;
        o2[k] = x2[k] * c + x1[k] * sn;
      }
      a = pack8(o1);
      b = pack8(o2);
    }
    reinterpret_cast<uint4*>(dst)[v] = a;
    reinterpret_cast<uint4*>(dst + half)[v] = b;
  }
}

at::Tensor rope_fwd(at::Tensor qkv, at::Tensor cosv, at::Tensor sinv, int64_t nrot, bool inverse) {
  check_cuda_bf16(qkv, "qkv");
  TORCH_CHECK(qkv.dim() == 5, "qkv must be [s, b, G, slots, d]");
  const int64_t s = qkv.size(0), b = qkv.size(1), G = qkv.size(2), S = qkv.size(3), d = qkv.size(4);
  TORCH_CHECK(d % 16 == 0, "head dim must be a multiple of 16");
  TORCH_CHECK(cosv.is_cuda() && cosv.scalar_type() == at::kFloat && cosv.size(0) == s && cosv.size(1) == d / 2);
  auto out = at::empty_like(qkv);
  int64_t n = s * b * G * S * (d / 16);
  if (n == 0) return out;
  rope_kernel<<<ew_grid(n), 256, 0, cur_stream()>>>((const __nv_bfloat16*)qkv.data_ptr(),
                                                    (__nv_bfloat16*)out.data_ptr(), cosv.data_ptr<float>(),
                                                    sinv.data_ptr<float>(), s, (int)b, (int)(G * S), (int)S, (int)d,
                                                    (int)nrot, inverse ? 1 : 0);
  EMB_LAUNCH_CHECK();
  count_launch();
  return out;
}

}  // namespace emb

// ------------------------------------------------------------------------------------------ allocation-free
// RMSNorm backward for callers that cannot allocate device memory (see csrc/include/noalloc.h): the per-CTA
// weight-gradient partials go to a fixed file-scope device array instead of a per-call allocation.
#include "../include/noalloc.h"

#include <climits>
#include <cstdio>
#include <mutex>

namespace emb {
namespace {

static __device__ __align__(256) float g_noalloc_scratch[EMB_NOALLOC_SCRATCH_FLOATS];

float* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of the scratch array for the current device (looked up once per device).
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace emb

extern "C" int emb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx,
                                       float* dw, int64_t T, int64_t H, int accumulate, cudaStream_t stream) {
  using namespace emb;
  if (T < 0 || T > INT_MAX || H <= 0 || H % 8 != 0 || H > 8 * 4 * 1024 || H > EMB_NOALLOC_SCRATCH_FLOATS) {
    std::fprintf(stderr,
                 "emb_rmsnorm_bwd_noalloc: unsupported shape T=%lld H=%lld (need 0 <= T <= INT_MAX, H %% 8 == 0, "
                 "0 < H <= 32768)\n",
                 (long long)T, (long long)H);
    return EMB_NOALLOC_EBADSIZE;
  }
  if (T == 0) return 0;
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  int vpt;
  const int threads = pick_threads((int)(H / 8), vpt);
  int64_t grid = norm_bwd_grid(T);
  grid = std::min<int64_t>(grid, EMB_NOALLOC_SCRATCH_FLOATS / H);
  if (grid < 1) grid = 1;
  const __nv_bfloat16* dyp = static_cast<const __nv_bfloat16*>(dy);
  const __nv_bfloat16* xp = static_cast<const __nv_bfloat16*>(x);
  const __nv_bfloat16* wp = static_cast<const __nv_bfloat16*>(w);
  __nv_bfloat16* dxp = static_cast<__nv_bfloat16*>(dx);
#define L(V) rmsnorm_bwd_kernel<V><<<(int)grid, threads, 0, stream>>>(dyp, xp, wp, rstd, dxp, scratch, (int)T, (int)H)
  if (vpt <= 1) L(1); else if (vpt == 2) L(2); else if (vpt == 3) L(3); else L(4);
#undef L
  launch_colsum(scratch, dw, (int)grid, (int)H, accumulate ? 1 : 0, stream);
  e = cudaGetLastError();
  count_launch(2);
  return (int)e;
}
