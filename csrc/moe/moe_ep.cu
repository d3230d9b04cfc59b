// Expert-parallel token movement over NVLink peer memory (sm_100a): the MoE all-to-all dispatch and combine
// as direct stores into the other GPUs' buffers, replacing two NCCL all-to-alls and the local re-layout
// around each of them.
//
// Every rank of the expert-parallel group owns symmetric buffers (one cudaMalloc arena per rank, CUDA-IPC
// mapped by every peer): a landing area laid out exactly like the grouped GEMM's input (per local expert,
// segments padded to 128 rows) plus an origin array, and a return area of T * k rows.
//
//  * dispatch: assignment r (= token * k + slot) of this rank goes to expert e on rank d; its row is stored
//    straight into rank d's landing area at its final row (the host computed every rank's segment layout from
//    the exchanged counts; the kernel adds the row's rank inside its expert), optionally scaled by w[r], and
//    origin[row] = (this rank << 24) | r is stored beside it, so the combine can send each expert output home
//    without another exchange;
//  * combine: every valid landing row p sends its expert output back into the return area of rank
//    origin[p] >> 24 at row origin[p] & 0xffffff.
//
// Ordering between ranks is a stream-ordered peer-flag barrier after each move (csrc/comm/symmetric.cu); the
// kernels here never wait, so they cannot hang.
#include "../include/common.cuh"

namespace emb {
namespace {

struct PeerPtrs {
  void* p[8];
};

constexpr int MAX_R = 1 << 24;  // rows addressable through the 24-bit row field of an origin entry

// One warp per assignment row.  Assignment r of global expert g = gid[r]: owner rank g / e_loc, row base[g] + (pos[r] - seg[g]) there (pos /
// seg: the sender's stable expert-sorted order, so rows keep their order inside a segment)
__global__ void ep_push_kernel(const __nv_bfloat16* __restrict__ src, int k_div, const int* __restrict__ gid,
                               const int* __restrict__ pos, const int* __restrict__ seg, const int* __restrict__ base,
                               int e_loc, const float* __restrict__ w, int R, int H8, PeerPtrs bufs,
                               PeerPtrs origins, int me) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < R; r += gridDim.x * warps) {
    const int g = gid[r];
    const int d = g / e_loc, row = base[g] + (pos[r] - seg[g]);
    const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)(r / k_div) * H8 * 8);
    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(bufs.p[d]) + (size_t)row * H8 * 8);
    if (w == nullptr) {
      for (int c = lane; c < H8; c += 32) o[c] = s[c];
    } else {
      const float wr = w[r];
      for (int c = lane; c < H8; c += 32) {
        float f[8];
        unpack8(s[c], f);
#pragma unroll
        for (int q = 0; q < 8; ++q) f[q] *= wr;
        o[c] = pack8(f);
      }
    }
    if (origins.p[0] != nullptr && lane == 0) reinterpret_cast<int*>(origins.p[d])[row] = (me << 24) | r;
  }
}

// one warp per landing row; rows whose origin is negative (segment padding) are skipped
__global__ void ep_return_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ origin, int rows,
                                 int H8, PeerPtrs rets) {
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < rows; p += gridDim.x * warps) {
    const int og = origin[p];
    if (og < 0) continue;
    const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)p * H8 * 8);
    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(rets.p[og >> 24]) +
                                        (size_t)(og & 0xffffff) * H8 * 8);
    for (int c = lane; c < H8; c += 32) o[c] = s[c];
  }
}

// padding rows of every local segment: zero row, origin -1
__global__ void ep_pad_kernel(const int* __restrict__ seg, const int* __restrict__ counts, int G, int H8,
                              __nv_bfloat16* __restrict__ land, int* __restrict__ origin) {
  for (int g = blockIdx.y; g < G; g += gridDim.y) {
    const int r0 = seg[g] + counts[g], r1 = seg[g + 1];
    for (int r = r0 + blockIdx.x; r < r1; r += gridDim.x) {
      uint4* d = reinterpret_cast<uint4*>(land + (size_t)r * H8 * 8);
      for (int i = threadIdx.x; i < H8; i += blockDim.x) d[i] = make_uint4(0, 0, 0, 0);
      if (origin != nullptr && threadIdx.x == 0) origin[r] = -1;
    }
  }
}

PeerPtrs peers_of(const at::Tensor& ptrs) {
  TORCH_CHECK(!ptrs.is_cuda() && ptrs.scalar_type() == at::kLong && ptrs.numel() >= 1 && ptrs.numel() <= 8,
              "peer pointer table: int64 CPU tensor of 1..8 entries");
  PeerPtrs p{};
  auto c = ptrs.contiguous();
  for (int64_t i = 0; i < c.numel(); ++i) {
    p.p[i] = reinterpret_cast<void*>(c.data_ptr<int64_t>()[i]);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(p.p[i]) & 15) == 0, "peer buffer must be 16-byte aligned");
  }
  return p;
}

int grid_rows(int64_t n) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 7) / 8, (int64_t)num_sms() * 8));
}

}  // namespace

// Push rows src[r / k_div] (times w[r]) of assignments r with global experts gid[r] to the owners' landing
// buffers (see ep_push_kernel for the row); with `origin_ptrs` also record (me << 24 | r) in the owner's origin
// array.  gid / pos: int32 [R]; seg / base: int32 [E]; bufs / origin_ptrs: int64 CPU [ep].
void ep_push(at::Tensor src, int64_t k_div, at::Tensor gid, at::Tensor pos, at::Tensor seg, at::Tensor base,
             int64_t e_loc, c10::optional<at::Tensor> w, at::Tensor bufs, c10::optional<at::Tensor> origin_ptrs,
             int64_t me) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.size(1) % 8 == 0);
  for (const at::Tensor* t : {&gid, &pos, &seg, &base})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kInt && t->is_contiguous(), "ep_push: int32 CUDA index arrays");
  TORCH_CHECK(gid.numel() == pos.numel() && seg.numel() >= base.numel() && e_loc >= 1);
  const int64_t R = gid.numel();
  TORCH_CHECK(R < MAX_R && me < 128, "ep_push: too many rows for the origin encoding");
  const float* wp = nullptr;
  if (w.has_value() && w->defined()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == R);
    wp = w->data_ptr<float>();
  }
  PeerPtrs b = peers_of(bufs);
  TORCH_CHECK(base.numel() <= e_loc * bufs.numel(), "ep_push: experts beyond the group");
  PeerPtrs o{};
  if (origin_ptrs.has_value() && origin_ptrs->defined()) o = peers_of(*origin_ptrs);
  if (R == 0) return;
  ep_push_kernel<<<grid_rows(R), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), (int)k_div, gid.data_ptr<int>(), pos.data_ptr<int>(),
      seg.data_ptr<int>(), base.data_ptr<int>(), (int)e_loc, wp, (int)R, (int)(src.size(1) / 8), b, o, (int)me);
  EMB_LAUNCH_CHECK();
  count_launch();
}

// Send rows 0 .. rows-1 of `src` (landing layout) home: row p goes to rank origin[p] >> 24, return row
// origin[p] & 0xffffff; negative origins are skipped.  rets: int64 CPU [ep] of the ranks' return buffers.
void ep_return(at::Tensor src, at::Tensor origin, int64_t rows, at::Tensor rets) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kBFloat16 && src.is_contiguous() && src.size(1) % 8 == 0);
  TORCH_CHECK(origin.scalar_type() == at::kInt && origin.numel() >= rows && src.size(0) >= rows);
  PeerPtrs r = peers_of(rets);
  if (rows == 0) return;
  ep_return_kernel<<<grid_rows(rows), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), origin.data_ptr<int>(), (int)rows,
      (int)(src.size(1) / 8), r);
  EMB_LAUNCH_CHECK();
  count_launch();
}

// Zero the padding rows of every segment of `land` and mark them in `origin` (optional) with -1.
void ep_pad(at::Tensor land, at::Tensor seg, at::Tensor counts, c10::optional<at::Tensor> origin) {
  TORCH_CHECK(land.is_cuda() && land.scalar_type() == at::kBFloat16 && land.size(1) % 8 == 0);
  TORCH_CHECK(seg.scalar_type() == at::kInt && counts.scalar_type() == at::kInt && seg.numel() == counts.numel() + 1);
  const int64_t G = counts.numel();
  int* op = nullptr;
  if (origin.has_value() && origin->defined()) {
    TORCH_CHECK(origin->scalar_type() == at::kInt);
    op = origin->data_ptr<int>();
  }
  ep_pad_kernel<<<dim3(16, (unsigned)std::min<int64_t>(G, 1024)), 128, 0, cur_stream()>>>(
      seg.data_ptr<int>(), counts.data_ptr<int>(), (int)G, (int)(land.size(1) / 8),
      reinterpret_cast<__nv_bfloat16*>(land.data_ptr()), op);
  EMB_LAUNCH_CHECK();
  count_launch();
}

}  // namespace emb
