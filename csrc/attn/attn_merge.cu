// Merge of partial attention results by their log-sum-exp (context parallelism: one query chunk attends to
// several key blocks, one flash-attention call per block).
//
//   l_new = log(exp(l) + exp(l_b));   out = out * exp(l - l_new) + o_b * exp(l_b - l_new);   l = l_new
//
// out [rows, H, 128] fp32 (rows = sequence x batch, the attention output layout), lse [b, H, s] fp32 (natural log,
// the layout attn_fwd returns), o_b [rows, H * 128] bf16 and l_b [b, H, s] from attn_fwd of the block.  A row
// whose running lse is -inf (no block seen yet) takes the block's values without reading `out` (so `out` may
// start uninitialised); a block row at -inf (fully masked) leaves the row unchanged.  One warp per (row, head),
// four of the 128 features per lane.
#include "../include/common.cuh"

namespace emb {

namespace {

__global__ void attn_merge_kernel(float* __restrict__ out, float* __restrict__ lse, const __nv_bfloat16* __restrict__ ob,
                                  const float* __restrict__ lb, int s, int b, int H) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)s * b * H;
  if (warp >= total) return;
  const int h = (int)(warp % H);
  const int64_t row = warp / H;  // = i * b + bb
  const int bb = (int)(row % b), i = (int)(row / b);
  const int64_t li = ((int64_t)bb * H + h) * s + i;
  const float l0 = lse[li], l1 = lb[li];
  float w0, w1, ln;
  if (l1 == -INFINITY) {
    return;
  } else if (l0 == -INFINITY) {
    w0 = 0.f;
    w1 = 1.f;
    ln = l1;
  } else {
    const float m = fmaxf(l0, l1);
    const float e0 = expf(l0 - m), e1 = expf(l1 - m);
    ln = m + logf(e0 + e1);
    const float inv = 1.f / (e0 + e1);
    w0 = e0 * inv;
    w1 = e1 * inv;
  }
  float4* o = reinterpret_cast<float4*>(out + (size_t)warp * 128) + lane;
  const uint2 pb = reinterpret_cast<const uint2*>(ob + (size_t)warp * 128)[lane];
  float4 v = w0 == 0.f ? make_float4(0.f, 0.f, 0.f, 0.f) : *o;
  const float b0 = __uint_as_float(pb.x << 16), b1 = __uint_as_float(pb.x & 0xffff0000u);
  const float b2 = __uint_as_float(pb.y << 16), b3 = __uint_as_float(pb.y & 0xffff0000u);
  v.x = v.x * w0 + b0 * w1;
  v.y = v.y * w0 + b1 * w1;
  v.z = v.z * w0 + b2 * w1;
  v.w = v.w * w0 + b3 * w1;
  *o = v;
  if (lane == 0) lse[li] = ln;
}

}  // namespace

void attn_merge(at::Tensor out, at::Tensor lse, at::Tensor o_b, at::Tensor l_b) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous(), "out: contiguous fp32 CUDA");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.dim() == 3, "lse: contiguous fp32 [b, H, s]");
  TORCH_CHECK(o_b.scalar_type() == at::kBFloat16 && o_b.is_contiguous(), "o_b: contiguous bf16");
  TORCH_CHECK(l_b.scalar_type() == at::kFloat && l_b.is_contiguous() && l_b.sizes() == lse.sizes(), "l_b like lse");
  const int64_t b = lse.size(0), H = lse.size(1), s = lse.size(2);
  TORCH_CHECK(out.numel() == s * b * H * 128 && o_b.numel() == out.numel(), "out / o_b: [s, b, H, 128]");
  const int64_t warps = s * b * H;
  if (warps == 0) return;
  TORCH_CHECK(warps < ((int64_t)1 << 31) / 32, "attn_merge: too many rows");
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  attn_merge_kernel<<<(unsigned)blocks, threads, 0, cur_stream()>>>(
      out.data_ptr<float>(), lse.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(o_b.data_ptr()),
      l_b.data_ptr<float>(), (int)s, (int)b, (int)H);
  EMB_LAUNCH_CHECK();
  count_launch();
}

}  // namespace emb
