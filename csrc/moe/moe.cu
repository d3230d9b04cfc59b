// Mixture-of-experts token routing kernels (sm_100a): router softmax / top-k / load statistics, expert-grouped
// token layout with per-expert segments padded to the grouped GEMM's 128-row tile, and the weighted row
// scatter / gather that move tokens into and out of that layout.
//
// Layout.  Assignment r (= token * k + slot for the local dispatch, or a received row for expert parallelism)
// with group g[r] lands at row pos[r] = seg[g] + (stable rank of r among the rows of group g); seg[g] is the
// exclusive prefix sum of the group counts rounded up to 128.  tile_group[i] is the group of 128-row tile i
// (-1 past the last segment), which is what the grouped GEMM (csrc/gemm) reads.  Padding rows inside a segment
// are zero so that they contribute nothing to weight gradients.
//
// The router follows Mixtral / Megatron "softmax after top-k": probs = softmax(logits[top-k]); the auxiliary
// load-balancing statistics are the per-expert assignment counts and sum_t softmax(logits)[t, e] (returned as
// per-block partial sums so that their reduction order is fixed).
#include "../include/common.cuh"

namespace emb {
namespace {

constexpr int SEG_ALIGN = 128;
constexpr int MAX_E_PER_LANE = 8;  // E <= 256

// one warp per token
__global__ void router_fwd_kernel(const float* __restrict__ logits, int T, int E, int k, int* __restrict__ top_idx,
                                  float* __restrict__ probs, int* __restrict__ counts, float* __restrict__ score_part) {
  extern __shared__ float s_part[];  // [E] per block
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_part[e] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const float* row = logits + (size_t)t * E;
    float v[MAX_E_PER_LANE];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? row[e] : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) sum += (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      if (e < E) atomicAdd(&s_part[e], __expf(v[i] - mx) * inv);  // shared-memory partial of this block
    }
    // top-k by repeated arg-max (lowest index wins ties); softmax over the selected logits
    float sel[8];
    int sid[8];
    unsigned taken = 0;  // bit i: expert lane + 32 i already selected
    for (int j = 0; j < k; ++j) {
      float best = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < MAX_E_PER_LANE; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !((taken >> i) & 1u) && (v[i] > best || (v[i] == best && e < bi))) {
          best = v[i];
          bi = e;
        }
      }
      for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) {
          best = ob;
          bi = oi;
        }
      }
      sel[j] = best;
      sid[j] = bi;
      if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    }
    if (lane == 0) {
      const float m0 = sel[0];
      float z = 0.f;
      for (int j = 0; j < k; ++j) z += __expf(sel[j] - m0);
      for (int j = 0; j < k; ++j) {
        top_idx[(size_t)t * k + j] = sid[j];
        probs[(size_t)t * k + j] = __expf(sel[j] - m0) / z;
        atomicAdd(&counts[sid[j]], 1);
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) score_part[(size_t)blockIdx.x * E + e] = s_part[e];
}

// dlogits[t, e] = softmax-over-top-k backward (from dprobs) + full-softmax backward of the aux statistics with
// upstream gradient g_aux[e] for scores[t, e].
__global__ void router_bwd_kernel(const float* __restrict__ logits, const int* __restrict__ top_idx,
                                  const float* __restrict__ probs, const float* __restrict__ dprobs,
                                  const float* __restrict__ g_aux, int T, int E, int k, float* __restrict__ dlogits) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const float* row = logits + (size_t)t * E;
    float v[MAX_E_PER_LANE];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? row[e] : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) sum += (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
    // aux: scores s = softmax(v); d = s * (g - <s, g>)
    float sg = 0.f;
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      if (e < E) sg += __expf(v[i] - mx) * inv * g_aux[e];
    }
    sg = warp_sum(sg);
    // top-k softmax: dl_j = p_j * (dp_j - <p, dp>)
    float pdp = 0.f;
    for (int j = 0; j < k; ++j) pdp += probs[(size_t)t * k + j] * dprobs[(size_t)t * k + j];
#pragma unroll
    for (int i = 0; i < MAX_E_PER_LANE; ++i) {
      const int e = lane + 32 * i;
      if (e >= E) continue;
      const float s = __expf(v[i] - mx) * inv;
      float d = s * (g_aux[e] - sg);
      for (int j = 0; j < k; ++j) {
        if (top_idx[(size_t)t * k + j] == e) {
          const float pj = probs[(size_t)t * k + j];
          d += pj * (dprobs[(size_t)t * k + j] - pdp);
        }
      }
      dlogits[(size_t)t * E + e] = d;
    }
  }
}

// seg[g] (g = 0..G) and tile_group[i] from the group counts (segments rounded up to `align` rows); one block
__global__ void segments_kernel(const int* __restrict__ counts, int G, int align, int n_tiles, int* __restrict__ seg,
                                int* __restrict__ tile_group) {
  __shared__ int s_seg[1025];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int g = 0; g < G; ++g) {
      s_seg[g] = o;
      o += (counts[g] + align - 1) / align * align;
    }
    s_seg[G] = o;
  }
  __syncthreads();
  for (int g = threadIdx.x; g <= G; g += blockDim.x) seg[g] = s_seg[g];
  for (int i = threadIdx.x; i < n_tiles; i += blockDim.x) {
    const int row = i * SEG_ALIGN;
    int grp = -1;
    for (int g = 0; g < G; ++g)
      if (row >= s_seg[g] && row < s_seg[g + 1]) grp = g;
    tile_group[i] = grp;
  }
}

// Stable positions: block g walks the rows in order and gives every row of group g the next slot of its segment.
__global__ void positions_kernel(const int* __restrict__ gid, int R, const int* __restrict__ seg, int* __restrict__ pos) {
  const int g = blockIdx.x;
  __shared__ int s_warp[32];
  __shared__ int s_base;
  if (threadIdx.x == 0) s_base = seg[g];
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int r0 = 0; r0 < R; r0 += blockDim.x) {
    const int r = r0 + threadIdx.x;
    const int mine = (r < R && gid[r] == g) ? 1 : 0;
    const unsigned bal = __ballot_sync(0xffffffffu, mine);
    const int in_warp = __popc(bal & ((1u << lane) - 1));
    if (lane == 0) s_warp[w] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int i = 0; i < nw; ++i) {
      before += i < w ? s_warp[i] : 0;
      total += s_warp[i];
    }
    if (mine) pos[r] = s_base + before + in_warp;
    __syncthreads();
    if (threadIdx.x == 0) s_base += total;
    __syncthreads();
  }
}

// dst[pos[r]] = w[r] * src[src_row(r)]   (src_row(r) = r / k_div; w optional)
__global__ void scatter_rows_kernel(const __nv_bfloat16* __restrict__ src, int k_div, const int* __restrict__ pos,
                                    const float* __restrict__ w, int R, int H8, __nv_bfloat16* __restrict__ dst) {
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)(r / k_div) * H8 * 8);
    uint4* d = reinterpret_cast<uint4*>(dst + (size_t)pos[r] * H8 * 8);
    if (w == nullptr) {
      for (int i = threadIdx.x; i < H8; i += blockDim.x) d[i] = s[i];
    } else {
      const float wr = w[r];
      for (int i = threadIdx.x; i < H8; i += blockDim.x) {
        float f[8];
        unpack8(s[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] *= wr;
        d[i] = pack8(f);
      }
    }
  }
}

// zero rows [seg[g] + counts[g], seg[g + 1]) of every segment
__global__ void zero_padding_kernel(const int* __restrict__ seg, const int* __restrict__ counts, int G, int H8,
                                    __nv_bfloat16* __restrict__ dst) {
  for (int g = blockIdx.y; g < G; g += gridDim.y) {
    const int r0 = seg[g] + counts[g], r1 = seg[g + 1];
    for (int r = r0 + blockIdx.x; r < r1; r += gridDim.x) {
      uint4* d = reinterpret_cast<uint4*>(dst + (size_t)r * H8 * 8);
      for (int i = threadIdx.x; i < H8; i += blockDim.x) d[i] = make_uint4(0, 0, 0, 0);
    }
  }
}

// out[i] = sum_{j<k} w[i, j] * src[pos[i * k + j]]   (fp32 accumulation; w optional = 1)
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ pos,
                                   const float* __restrict__ w, int n_out, int k, int H8,
                                   __nv_bfloat16* __restrict__ out) {
  for (int i = blockIdx.x; i < n_out; i += gridDim.x) {
    for (int c = threadIdx.x; c < H8; c += blockDim.x) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int j = 0; j < k; ++j) {
        const float wj = w ? w[(size_t)i * k + j] : 1.f;
        float f[8];
        unpack8(reinterpret_cast<const uint4*>(src + (size_t)pos[(size_t)i * k + j] * H8 * 8)[c], f);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += wj * f[q];
      }
      reinterpret_cast<uint4*>(out + (size_t)i * H8 * 8)[c] = pack8(acc);
    }
  }
}

// d[r] = <a[r / k], b[pos[r]]>  (gradient of the combine weights); one warp per r
__global__ void row_dot_kernel(const __nv_bfloat16* __restrict__ a, int k, const __nv_bfloat16* __restrict__ b,
                               const int* __restrict__ pos, int R, int H8, float* __restrict__ d) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < R; r += gridDim.x * warps) {
    const uint4* x = reinterpret_cast<const uint4*>(a + (size_t)(r / k) * H8 * 8);
    const uint4* y = reinterpret_cast<const uint4*>(b + (size_t)pos[r] * H8 * 8);
    float acc = 0.f;
    for (int c = lane; c < H8; c += 32) {
      float f[8], g[8];
      unpack8(x[c], f);
      unpack8(y[c], g);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc += f[q] * g[q];
    }
    acc = warp_sum(acc);
    if (lane == 0) d[r] = acc;
  }
}

int grid_for(int64_t n, int per) { return (int)std::max<int64_t>(1, std::min<int64_t>((n + per - 1) / per, num_sms() * 16)); }

}  // namespace

std::vector<at::Tensor> moe_router_fwd(at::Tensor logits, int64_t k) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.is_contiguous());
  const int64_t T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E >= 1 && E <= 32 * MAX_E_PER_LANE && k >= 1 && k <= 8 && k <= E, "router: E <= 256, k <= 8");
  auto oi = logits.options().dtype(at::kInt);
  auto top = at::empty({T, k}, oi);
  auto probs = at::empty({T, k}, logits.options());
  auto counts = at::zeros({E}, oi);
  const int threads = 256, warps = threads / 32;
  const int grid = grid_for(std::max<int64_t>(T, 1), warps);
  auto part = at::empty({grid, E}, logits.options());
  router_fwd_kernel<<<grid, threads, E * sizeof(float), cur_stream()>>>(
      logits.data_ptr<float>(), (int)T, (int)E, (int)k, top.data_ptr<int>(), probs.data_ptr<float>(),
      counts.data_ptr<int>(), part.data_ptr<float>());
  EMB_LAUNCH_CHECK();
  count_launch();
  return {top, probs, counts, part};
}

at::Tensor moe_router_bwd(at::Tensor logits, at::Tensor top_idx, at::Tensor probs, at::Tensor dprobs, at::Tensor g_aux) {
  const int64_t T = logits.size(0), E = logits.size(1), k = top_idx.size(1);
  TORCH_CHECK(dprobs.is_contiguous() && dprobs.scalar_type() == at::kFloat && g_aux.numel() == E &&
              g_aux.scalar_type() == at::kFloat);
  auto d = at::empty_like(logits);
  const int threads = 256;
  router_bwd_kernel<<<grid_for(std::max<int64_t>(T, 1), threads / 32), threads, 0, cur_stream()>>>(
      logits.data_ptr<float>(), top_idx.data_ptr<int>(), probs.data_ptr<float>(), dprobs.data_ptr<float>(),
      g_aux.data_ptr<float>(), (int)T, (int)E, (int)k, d.data_ptr<float>());
  EMB_LAUNCH_CHECK();
  count_launch();
  return d;
}

// Group layout for R rows with group ids gid [R] (int32) and per-group counts [G]; segments are rounded up to
// `align` rows (128 for the grouped GEMM, 1 for a dense send buffer); rows_cap = allocated rows (>= the sum of
// rounded counts).  Returns {pos [R], seg [G + 1], tile_group [rows_cap / 128]} (tile_group empty unless
// align == 128).
std::vector<at::Tensor> moe_layout(at::Tensor gid, at::Tensor counts, int64_t rows_cap, int64_t align) {
  TORCH_CHECK(gid.is_cuda() && gid.scalar_type() == at::kInt && counts.scalar_type() == at::kInt);
  TORCH_CHECK(align == 1 || align == SEG_ALIGN, "moe_layout: align must be 1 or 128");
  TORCH_CHECK(align == 1 || rows_cap % SEG_ALIGN == 0);
  const int64_t R = gid.numel(), G = counts.numel();
  TORCH_CHECK(G >= 1 && G <= 1024);
  auto oi = gid.options();
  auto pos = at::empty({R}, oi);
  auto seg = at::empty({G + 1}, oi);
  const int64_t n_tiles = align == SEG_ALIGN ? rows_cap / SEG_ALIGN : 0;
  auto tg = at::empty({n_tiles}, oi);
  segments_kernel<<<1, 256, 0, cur_stream()>>>(counts.data_ptr<int>(), (int)G, (int)align, (int)n_tiles,
                                               seg.data_ptr<int>(), tg.data_ptr<int>());
  EMB_LAUNCH_CHECK();
  if (R > 0) {
    positions_kernel<<<(int)G, 1024, 0, cur_stream()>>>(gid.data_ptr<int>(), (int)R, seg.data_ptr<int>(),
                                                        pos.data_ptr<int>());
    EMB_LAUNCH_CHECK();
  }
  count_launch(2);
  return {pos, seg, tg};
}

// dst [rows_cap, H] = rows src[r / k_div] (times w[r]) placed at pos[r]; padding rows of each segment zeroed.
at::Tensor moe_scatter(at::Tensor src, int64_t k_div, at::Tensor pos, c10::optional<at::Tensor> w, at::Tensor seg,
                       at::Tensor counts, int64_t rows_cap) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.size(1) % 8 == 0);
  const int64_t H = src.size(1), R = pos.numel(), G = counts.numel();
  auto dst = at::empty({rows_cap, H}, src.options());
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == R);
    wp = w->data_ptr<float>();
  }
  if (R > 0) {
    scatter_rows_kernel<<<grid_for(R, 1), 128, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), (int)k_div, pos.data_ptr<int>(), wp, (int)R,
        (int)(H / 8), reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
    EMB_LAUNCH_CHECK();
  }
  zero_padding_kernel<<<dim3(16, (unsigned)std::min<int64_t>(G, 1024)), 128, 0, cur_stream()>>>(
      seg.data_ptr<int>(), counts.data_ptr<int>(), (int)G, (int)(H / 8), reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
  EMB_LAUNCH_CHECK();
  count_launch(2);
  return dst;
}

// out [n_out, H] = sum_{j<k} w[i, j] * src[pos[i * k + j]]
at::Tensor moe_gather(at::Tensor src, at::Tensor pos, c10::optional<at::Tensor> w, int64_t n_out, int64_t k) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.size(1) % 8 == 0);
  TORCH_CHECK(pos.numel() == n_out * k);
  const int64_t H = src.size(1);
  auto out = at::empty({n_out, H}, src.options());
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == n_out * k);
    wp = w->data_ptr<float>();
  }
  if (n_out > 0) {
    gather_rows_kernel<<<grid_for(n_out, 1), 128, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), pos.data_ptr<int>(), wp, (int)n_out, (int)k,
        (int)(H / 8), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
    EMB_LAUNCH_CHECK();
  }
  count_launch();
  return out;
}

// d[r] = <a[r / k], b[pos[r]]>
at::Tensor moe_row_dot(at::Tensor a, int64_t k, at::Tensor b, at::Tensor pos) {
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.size(1) == b.size(1));
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && a.size(1) % 8 == 0);
  const int64_t R = pos.numel(), H = a.size(1);
  auto d = at::empty({R}, a.options().dtype(at::kFloat));
  if (R > 0) {
    row_dot_kernel<<<grid_for(R, 8), 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(a.data_ptr()), (int)k, reinterpret_cast<const __nv_bfloat16*>(b.data_ptr()),
        pos.data_ptr<int>(), (int)R, (int)(H / 8), d.data_ptr<float>());
    EMB_LAUNCH_CHECK();
  }
  count_launch();
  return d;
}

}  // namespace emb
