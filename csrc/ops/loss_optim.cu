// Vocab-parallel cross-entropy pieces, vocab-parallel embedding, segmented fused AdamW and the segmented
// gradient sum of squares.  All memory-bound: 16-byte vectors, fp32 math.
#include "../include/common.cuh"

namespace emb {

// ------------------------------------------------------------------------------------------ cross-entropy
// One CTA per token row.  logits: [T, V] bf16 (V % 8 == 0).
__global__ void ce_max_kernel(const __nv_bfloat16* __restrict__ logits, float* __restrict__ out, int V) {
  __shared__ float sh[32];
  const uint4* r = reinterpret_cast<const uint4*>(logits + (size_t)blockIdx.x * V);
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V / 8; i += blockDim.x) {
    float f[8];
    unpack8(r[i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) m = fmaxf(m, f[k]);
  }
  m = block_max(m, sh);
  if (threadIdx.x == 0) out[blockIdx.x] = m;
}

__global__ void ce_stats_kernel(const __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ labels,
                                const float* __restrict__ lmax, float* __restrict__ stats, int T, int V,
                                int64_t vstart) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  const uint4* r = reinterpret_cast<const uint4*>(logits + (size_t)row * V);
  const float m = lmax[row];
  float s = 0.f;
  for (int i = threadIdx.x; i < V / 8; i += blockDim.x) {
    float f[8];
    unpack8(r[i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) s += __expf(f[k] - m);
  }
  s = block_sum(s, sh);
  if (threadIdx.x == 0) {
    stats[row] = s;
    int64_t loc = labels[row] - vstart;
    stats[T + row] = (loc >= 0 && loc < V) ? (bf2f(logits[(size_t)row * V + loc]) - m) : 0.f;
  }
}

__global__ void ce_bwd_kernel(const __nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ labels,
                              const float* __restrict__ lmax, const float* __restrict__ sumexp,
                              const float* __restrict__ dloss, __nv_bfloat16* __restrict__ dlogits, int V,
                              int64_t vstart) {
  const int row = blockIdx.x;
  const uint4* r = reinterpret_cast<const uint4*>(logits + (size_t)row * V);
  uint4* o = reinterpret_cast<uint4*>(dlogits + (size_t)row * V);
  const float m = lmax[row], inv = 1.f / sumexp[row], g = dloss[row];
  const int64_t loc = labels[row] - vstart;
  for (int i = threadIdx.x; i < V / 8; i += blockDim.x) {
    float f[8];
    unpack8(r[i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float p = __expf(f[k] - m) * inv;
      if ((int64_t)(i * 8 + k) == loc) p -= 1.f;
      f[k] = p * g;
    }
    o[i] = pack8(f);
  }
}

at::Tensor ce_local_max(at::Tensor logits) {
  check_cuda_bf16(logits, "logits");
  const int64_t T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0);
  auto out = at::empty({T}, logits.options().dtype(at::kFloat));
  if (T) ce_max_kernel<<<T, 256, 0, cur_stream()>>>((const __nv_bfloat16*)logits.data_ptr(), out.data_ptr<float>(),
                                                     (int)V);
  EMB_LAUNCH_CHECK();
  count_launch();
  return out;
}

at::Tensor ce_local_stats(at::Tensor logits, at::Tensor labels, at::Tensor lmax, int64_t vstart) {
  check_cuda_bf16(logits, "logits");
  const int64_t T = logits.size(0), V = logits.size(1);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == T);
  auto stats = at::empty({2, T}, logits.options().dtype(at::kFloat));
  if (T) ce_stats_kernel<<<T, 256, 0, cur_stream()>>>((const __nv_bfloat16*)logits.data_ptr(),
                                                       labels.data_ptr<int64_t>(), lmax.data_ptr<float>(),
                                                       stats.data_ptr<float>(), (int)T, (int)V, vstart);
  EMB_LAUNCH_CHECK();
  count_launch();
  return stats;
}

at::Tensor ce_bwd(at::Tensor logits, at::Tensor labels, at::Tensor lmax, at::Tensor sumexp,
                     at::Tensor dloss, int64_t vstart) {
  check_cuda_bf16(logits, "logits");
  const int64_t T = logits.size(0), V = logits.size(1);
  auto d = at::empty_like(logits);
  auto sx = sumexp.contiguous();
  auto dl = dloss.to(at::kFloat).contiguous();
  if (T) ce_bwd_kernel<<<T, 256, 0, cur_stream()>>>((const __nv_bfloat16*)logits.data_ptr(),
                                                     labels.data_ptr<int64_t>(), lmax.data_ptr<float>(),
                                                     sx.data_ptr<float>(), dl.data_ptr<float>(),
                                                     (__nv_bfloat16*)d.data_ptr(), (int)V, vstart);
  EMB_LAUNCH_CHECK();
  count_launch();
  return d;
}

// ------------------------------------------------------------------------------------------ embedding
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ w,
                                 __nv_bfloat16* __restrict__ out, int H, int64_t V, int64_t vstart) {
  const int64_t t = blockIdx.x;
  const int64_t loc = ids[t] - vstart;
  uint4* o = reinterpret_cast<uint4*>(out + t * H);
  const bool in = loc >= 0 && loc < V;
  const uint4* r = reinterpret_cast<const uint4*>(w + (in ? loc : 0) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) o[i] = in ? r[i] : make_uint4(0, 0, 0, 0);
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dy,
                                 float* __restrict__ target, int H, int64_t V, int64_t vstart) {
  const int64_t t = blockIdx.x;
  const int64_t loc = ids[t] - vstart;
  if (loc < 0 || loc >= V) return;
  const uint4* d = reinterpret_cast<const uint4*>(dy + t * H);
  float* row = target + loc * H;
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    float f[8];
    unpack8(d[i], f);
#pragma unroll
    for (int k = 0; k < 8; ++k) atomicAdd(row + i * 8 + k, f[k]);
  }
}

at::Tensor embedding_fwd(at::Tensor ids, at::Tensor w, int64_t vstart) {
  check_cuda_bf16(w, "w");
  auto idc = ids.contiguous();
  const int64_t T = idc.numel(), V = w.size(0), H = w.size(1);
  TORCH_CHECK(H % 8 == 0);
  auto out = at::empty({T, H}, w.options());
  if (T) embed_fwd_kernel<<<T, 128, 0, cur_stream()>>>(idc.data_ptr<int64_t>(), (const __nv_bfloat16*)w.data_ptr(),
                                                       (__nv_bfloat16*)out.data_ptr(), (int)H, V, vstart);
  EMB_LAUNCH_CHECK();
  count_launch();
  return out;
}

void embedding_bwd(at::Tensor ids, at::Tensor dy, at::Tensor target, int64_t vstart) {
  check_cuda_bf16(dy, "dy");
  TORCH_CHECK(target.scalar_type() == at::kFloat && target.is_contiguous());
  auto idc = ids.contiguous();
  const int64_t T = idc.numel(), V = target.size(0), H = target.size(1);
  if (T) embed_bwd_kernel<<<T, 128, 0, cur_stream()>>>(idc.data_ptr<int64_t>(), (const __nv_bfloat16*)dy.data_ptr(),
                                                       target.data_ptr<float>(), (int)H, V, vstart);
  EMB_LAUNCH_CHECK();
  count_launch();
}

// ------------------------------------------------------------------------------------------ AdamW
// chunks: [n, 5] int64 rows (grad/param arena offset, optimizer offset, length, weight_decay flag, counted).
// O: [3, n_opt] fp32 (master, exp_avg, exp_avg_sq).  The clip coefficient is computed on the device from the
// all-reduced sum of squares, so the step needs no host synchronisation.
template <typename PT>
__device__ __forceinline__ void store_param(PT* p, int64_t i, float v);
template <>
__device__ __forceinline__ void store_param<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void store_param<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}

struct AdamHyper {
  float lr, b1, b2, eps, wd, bc1, bc2, grad_scale, max_norm;
};

template <typename PT>
__global__ void adam_kernel(float* __restrict__ O, int64_t n_opt, const float* __restrict__ G, PT* __restrict__ P,
                            const int64_t* __restrict__ chunks, AdamHyper hp, const float* __restrict__ sumsq) {
  const int64_t* c = chunks + blockIdx.x * 5;
  const int64_t a = c[0], o = c[1], n = c[2];
  const float wd = c[3] ? hp.wd : 0.f;
  float scale = hp.grad_scale;
  if (sumsq != nullptr && hp.max_norm > 0.f) {
    float norm = sqrtf(*sumsq) * hp.grad_scale;
    float clip = hp.max_norm / (norm + 1e-6f);
    if (clip < 1.f) scale *= clip;
  }
  float* mw = O + o;
  float* m1 = O + n_opt + o;
  float* m2 = O + 2 * n_opt + o;
  const float* g = G + a;
  const float step_size = hp.lr / hp.bc1;
  const float inv_bc2 = 1.f / hp.bc2;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    float gi = g[i] * scale;
    float e1 = hp.b1 * m1[i] + (1.f - hp.b1) * gi;
    float e2 = hp.b2 * m2[i] + (1.f - hp.b2) * gi * gi;
    float w = mw[i];
    w = w * (1.f - hp.lr * wd);
    w -= step_size * e1 / (sqrtf(e2 * inv_bc2) + hp.eps);
    m1[i] = e1;
    m2[i] = e2;
    mw[i] = w;
    store_param<PT>(P + a, i, w);
  }
}

void adam_segments(at::Tensor O, at::Tensor G, at::Tensor P, at::Tensor chunks, double lr, double b1,
                   double b2, double eps, double wd, int64_t step, double grad_scale, double max_norm,
                   c10::optional<at::Tensor> sumsq) {
  TORCH_CHECK(O.scalar_type() == at::kFloat && O.dim() == 2 && O.size(0) == 3 && O.is_contiguous());
  TORCH_CHECK(G.scalar_type() == at::kFloat && G.is_contiguous());
  TORCH_CHECK(chunks.scalar_type() == at::kLong && chunks.is_cuda() && chunks.size(1) == 5);
  const int64_t nch = chunks.size(0);
  if (nch == 0) return;
  AdamHyper hp;
  hp.lr = (float)lr;
  hp.b1 = (float)b1;
  hp.b2 = (float)b2;
  hp.eps = (float)eps;
  hp.wd = (float)wd;
  hp.bc1 = (float)(1.0 - std::pow(b1, (double)step));
  hp.bc2 = (float)(1.0 - std::pow(b2, (double)step));
  hp.grad_scale = (float)grad_scale;
  hp.max_norm = (float)max_norm;
  const float* sq = (sumsq.has_value() && sumsq->defined()) ? sumsq->data_ptr<float>() : nullptr;
  auto st = cur_stream();
  if (P.scalar_type() == at::kBFloat16) {
    adam_kernel<__nv_bfloat16><<<nch, 512, 0, st>>>(O.data_ptr<float>(), O.size(1), G.data_ptr<float>(),
                                                     (__nv_bfloat16*)P.data_ptr(), chunks.data_ptr<int64_t>(), hp, sq);
  } else {
    TORCH_CHECK(P.scalar_type() == at::kFloat);
    adam_kernel<float><<<nch, 512, 0, st>>>(O.data_ptr<float>(), O.size(1), G.data_ptr<float>(), P.data_ptr<float>(),
                                            chunks.data_ptr<int64_t>(), hp, sq);
  }
  EMB_LAUNCH_CHECK();
  count_launch();
}

// Per-chunk partial sums of squares of counted chunks, then a fixed-order sum (deterministic).
__global__ void sumsq_partial_kernel(const float* __restrict__ G, const int64_t* __restrict__ chunks,
                                     float* __restrict__ part) {
  __shared__ float sh[32];
  const int64_t* c = chunks + blockIdx.x * 5;
  float s = 0.f;
  if (c[4]) {
    const float* g = G + c[0];
    for (int64_t i = threadIdx.x; i < c[2]; i += blockDim.x) s += g[i] * g[i];
  }
  s = block_sum(s, sh);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

__global__ void sum_kernel(const float* __restrict__ part, int n, float* __restrict__ out) {
  __shared__ float sh[32];
  // fixed assignment of elements to threads -> deterministic
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += part[i];
  s = block_sum(s, sh);
  if (threadIdx.x == 0) out[0] = s;
}

at::Tensor seg_sumsq(at::Tensor G, at::Tensor chunks) {
  const int64_t nch = chunks.size(0);
  auto out = at::zeros({1}, G.options().dtype(at::kFloat));
  if (nch == 0) return out;
  auto part = at::empty({nch}, G.options().dtype(at::kFloat));
  auto st = cur_stream();
  sumsq_partial_kernel<<<nch, 512, 0, st>>>(G.data_ptr<float>(), chunks.data_ptr<int64_t>(), part.data_ptr<float>());
  sum_kernel<<<1, 1024, 0, st>>>(part.data_ptr<float>(), (int)nch, out.data_ptr<float>());
  EMB_LAUNCH_CHECK();
  count_launch(2);
  return out;
}

}  // namespace emb
