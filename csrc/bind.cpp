// Python bindings of the elasticmegatron_b200._C extension.
#include <torch/extension.h>

namespace emb {
int64_t launch_count();
void reset_launch_count();
torch::Tensor arena_alloc(int64_t nbytes, int64_t device);
torch::Tensor ipc_get_handle(torch::Tensor arena);
int64_t ipc_open(torch::Tensor handle);
void ipc_close_all();
bool ipc_close(torch::Tensor handle);
int64_t ipc_open_count();
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps);
std::vector<torch::Tensor> rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd,
                                       c10::optional<torch::Tensor> dw_accum, c10::optional<torch::Tensor> dres);
std::vector<torch::Tensor> layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, double eps);
std::vector<torch::Tensor> layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean,
                                         torch::Tensor rstd, c10::optional<torch::Tensor> dw_accum,
                                         c10::optional<torch::Tensor> db_accum);
std::vector<torch::Tensor> add_rmsnorm_fwd(torch::Tensor x, torch::Tensor o, torch::Tensor w, double eps);
torch::Tensor swiglu_fwd(torch::Tensor h);
torch::Tensor swiglu_bwd(torch::Tensor dy, torch::Tensor h);
torch::Tensor rope_fwd(torch::Tensor qkv, torch::Tensor cosv, torch::Tensor sinv, int64_t nrot, bool inverse);
torch::Tensor ce_local_max(torch::Tensor logits);
torch::Tensor ce_local_stats(torch::Tensor logits, torch::Tensor labels, torch::Tensor lmax, int64_t vstart);
torch::Tensor ce_bwd(torch::Tensor logits, torch::Tensor labels, torch::Tensor lmax, torch::Tensor sumexp,
                     torch::Tensor dloss, int64_t vstart);
torch::Tensor embedding_fwd(torch::Tensor ids, torch::Tensor w, int64_t vstart);
void embedding_bwd(torch::Tensor ids, torch::Tensor dy, torch::Tensor target, int64_t vstart);
void adam_segments(torch::Tensor O, torch::Tensor G, torch::Tensor P, torch::Tensor chunks, double lr, double b1,
                   double b2, double eps, double wd, int64_t step, double grad_scale, double max_norm,
                   c10::optional<torch::Tensor> sumsq);
torch::Tensor seg_sumsq(torch::Tensor G, torch::Tensor chunks);
void reshard_copy(torch::Tensor tasks, int64_t ntasks, int64_t grid);
int64_t copy_task_bytes();
torch::Tensor gemm(torch::Tensor a, torch::Tensor b, bool trans_a, bool trans_b, c10::optional<torch::Tensor> out,
                   bool accumulate);
torch::Tensor gemm_tc(torch::Tensor a, torch::Tensor b, bool trans_a, bool trans_b, c10::optional<torch::Tensor> out,
                      bool accumulate, int64_t variant);
bool gemm_tc_supported(torch::Tensor a, torch::Tensor b, bool trans_a, bool trans_b, c10::optional<torch::Tensor> out,
                       bool accumulate);
std::vector<torch::Tensor> attn_fwd(torch::Tensor qkv, int64_t hpg, bool causal);
bool attn_supported(torch::Tensor qkv);
int64_t attn_error_flag();
torch::Tensor attn_bwd(torch::Tensor dO, torch::Tensor qkv, torch::Tensor o, torch::Tensor lse, int64_t hpg,
                       bool causal);
int64_t attn_bwd_error_flag();
void attn_merge(torch::Tensor out, torch::Tensor lse, torch::Tensor o_b, torch::Tensor l_b);
int64_t gemm_error_flag();
int64_t gemm_fallback_count();
at::Tensor attn_exp2_emulated(at::Tensor x);
void dp_signal(at::Tensor flags, int64_t me, int64_t slot0, int64_t nslots, int64_t epoch);
void dp_rs_pull(at::Tensor peers, int64_t me, int64_t off, int64_t count, at::Tensor flags, int64_t slot,
                int64_t epoch, int64_t timeout_ms);
void dp_ag_pull(at::Tensor peers, int64_t me, int64_t off, int64_t shard_bytes, at::Tensor flags, int64_t slot,
                int64_t epoch, int64_t timeout_ms);
std::vector<int64_t> attn_debug_counters();
std::vector<int64_t> gemm_debug_counters();
void gemm_rs(torch::Tensor a, torch::Tensor b, bool trans_a, bool trans_b, torch::Tensor peers, int64_t my_slot,
             int64_t rows_per_rank);
torch::Tensor rs_reduce(torch::Tensor stage, int64_t tp, int64_t rows, int64_t n);
torch::Tensor gemm_ag(torch::Tensor local, torch::Tensor b, bool trans_b, torch::Tensor peers, int64_t my_slot,
                      int64_t rows_per_rank, torch::Tensor claim, torch::Tensor shard, torch::Tensor flags,
                      int64_t epoch, int64_t units_max);
torch::Tensor gemm_grouped(torch::Tensor a, torch::Tensor w, bool trans_b, torch::Tensor tile_group);
void gemm_grouped_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor seg, torch::Tensor out, bool accumulate);
std::vector<torch::Tensor> moe_router_fwd(torch::Tensor logits, int64_t k);
torch::Tensor moe_router_bwd(torch::Tensor logits, torch::Tensor top_idx, torch::Tensor probs, torch::Tensor dprobs,
                             torch::Tensor g_aux);
std::vector<torch::Tensor> moe_layout(torch::Tensor gid, torch::Tensor counts, int64_t rows_cap, int64_t align);
torch::Tensor moe_scatter(torch::Tensor src, int64_t k_div, torch::Tensor pos, c10::optional<torch::Tensor> w,
                          torch::Tensor seg, torch::Tensor counts, int64_t rows_cap);
torch::Tensor moe_gather(torch::Tensor src, torch::Tensor pos, c10::optional<torch::Tensor> w, int64_t n_out, int64_t k);
torch::Tensor moe_row_dot(torch::Tensor a, int64_t k, torch::Tensor b, torch::Tensor pos);
void ep_push(torch::Tensor src, int64_t k_div, torch::Tensor gid, torch::Tensor pos, torch::Tensor seg,
             torch::Tensor base, int64_t e_loc, c10::optional<torch::Tensor> w, torch::Tensor bufs,
             c10::optional<torch::Tensor> origin_ptrs, int64_t me);
void ep_return(torch::Tensor src, torch::Tensor origin, int64_t rows, torch::Tensor rets);
void ep_pad(torch::Tensor land, torch::Tensor seg, torch::Tensor counts, c10::optional<torch::Tensor> origin);
void sym_barrier(torch::Tensor sig_ptrs, int64_t me, int64_t epoch, int64_t timeout_ms);
void nvls_allreduce_f32(int64_t mc_slice, int64_t count);
void p2p_allreduce_f32(torch::Tensor bufs, int64_t off, int64_t count);
int64_t comm_error_flag();
void comm_clear_error();
}  // namespace emb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace emb;
  m.def("launch_count", &launch_count);
  m.def("reset_launch_count", &reset_launch_count);
  m.def("arena_alloc", &arena_alloc);
  m.def("ipc_get_handle", &ipc_get_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close_all", &ipc_close_all);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_open_count", &ipc_open_count);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("rstd"),
        py::arg("dw_accum") = py::none(), py::arg("dres") = py::none());
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("layernorm_fwd", &layernorm_fwd);
  m.def("layernorm_bwd", &layernorm_bwd, py::arg("dy"), py::arg("x"), py::arg("w"), py::arg("mean"), py::arg("rstd"),
        py::arg("dw_accum") = py::none(), py::arg("db_accum") = py::none());
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("rope_fwd", &rope_fwd);
  m.def("ce_local_max", &ce_local_max);
  m.def("ce_local_stats", &ce_local_stats);
  m.def("ce_bwd", &ce_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("adam_segments", &adam_segments, py::arg("O"), py::arg("G"), py::arg("P"), py::arg("chunks"), py::arg("lr"),
        py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("step"), py::arg("grad_scale"),
        py::arg("max_norm") = 0.0, py::arg("sumsq") = py::none());
  m.def("seg_sumsq", &seg_sumsq);
  m.def("reshard_copy", &reshard_copy, py::arg("tasks"), py::arg("ntasks"), py::arg("grid") = 0);
  m.def("copy_task_bytes", &copy_task_bytes);
  m.def("gemm", &gemm, py::arg("a"), py::arg("b"), py::arg("trans_a") = false, py::arg("trans_b") = false,
        py::arg("out") = py::none(), py::arg("accumulate") = false);
  m.def("gemm_tc", &gemm_tc, py::arg("a"), py::arg("b"), py::arg("trans_a") = false, py::arg("trans_b") = false,
        py::arg("out") = py::none(), py::arg("accumulate") = false, py::arg("variant") = 0);
  m.def("attn_fwd", &attn_fwd, py::arg("qkv"), py::arg("hpg"), py::arg("causal") = true);
  m.def("attn_supported", &attn_supported);
  m.def("attn_bwd", &attn_bwd, py::arg("dO"), py::arg("qkv"), py::arg("o"), py::arg("lse"), py::arg("hpg"),
        py::arg("causal") = true);
  m.def("attn_bwd_error_flag", &attn_bwd_error_flag);
  m.def("attn_merge", &attn_merge);
  m.def("attn_error_flag", &attn_error_flag);
  m.def("attn_exp2_emulated", &attn_exp2_emulated);
  m.def("dp_signal", &dp_signal);
  m.def("dp_rs_pull", &dp_rs_pull);
  m.def("dp_ag_pull", &dp_ag_pull);
  m.def("attn_debug_counters", &attn_debug_counters);
  m.def("gemm_fallback_count", &gemm_fallback_count);
  m.def("gemm_error_flag", &gemm_error_flag);
  m.def("gemm_debug_counters", &gemm_debug_counters);
  m.def("gemm_rs", &gemm_rs);
  m.def("rs_reduce", &rs_reduce);
  m.def("gemm_ag", &gemm_ag);
  m.def("nvls_allreduce_f32", &nvls_allreduce_f32);
  m.def("p2p_allreduce_f32", &p2p_allreduce_f32);
  m.def("sym_barrier", &sym_barrier, py::arg("sig_ptrs"), py::arg("me"), py::arg("epoch"),
        py::arg("timeout_ms") = 60000);
  m.def("comm_error_flag", &comm_error_flag);
  m.def("ep_push", &ep_push, py::arg("src"), py::arg("k_div"), py::arg("gid"), py::arg("pos"), py::arg("seg"),
        py::arg("base"), py::arg("e_loc"), py::arg("w"), py::arg("bufs"), py::arg("origin_ptrs"), py::arg("me"));
  m.def("ep_return", &ep_return);
  m.def("ep_pad", &ep_pad, py::arg("land"), py::arg("seg"), py::arg("counts"), py::arg("origin"));
  m.def("gemm_grouped", &gemm_grouped);
  m.def("gemm_grouped_wgrad", &gemm_grouped_wgrad);
  m.def("moe_router_fwd", &moe_router_fwd);
  m.def("moe_router_bwd", &moe_router_bwd);
  m.def("moe_layout", &moe_layout, py::arg("gid"), py::arg("counts"), py::arg("rows_cap"), py::arg("align") = 128);
  m.def("moe_scatter", &moe_scatter, py::arg("src"), py::arg("k_div"), py::arg("pos"), py::arg("w"), py::arg("seg"),
        py::arg("counts"), py::arg("rows_cap"));
  m.def("moe_gather", &moe_gather, py::arg("src"), py::arg("pos"), py::arg("w"), py::arg("n_out"), py::arg("k"));
  m.def("moe_row_dot", &moe_row_dot);
  m.def("comm_clear_error", &comm_clear_error);
  m.def("gemm_tc_supported", &gemm_tc_supported, py::arg("a"), py::arg("b"), py::arg("trans_a") = false,
        py::arg("trans_b") = false, py::arg("out") = py::none(), py::arg("accumulate") = false);
}
