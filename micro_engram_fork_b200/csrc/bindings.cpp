// Python bindings of the sm_100a extension (micro_engram_fork_b200._C).
#include <torch/extension.h>

// engram.cu
torch::Tensor engram_hash(torch::Tensor ids, c10::optional<torch::Tensor> pos, torch::Tensor canon,
                          torch::Tensor mults, torch::Tensor orders, torch::Tensor rows, int64_t pad_id);
torch::Tensor engram_hash_prev(torch::Tensor ids, torch::Tensor canon, torch::Tensor mults, torch::Tensor orders,
                               torch::Tensor rows, int64_t pad_id);
torch::Tensor engram_gather(torch::Tensor idx, torch::Tensor ptrs, torch::Tensor per, int64_t world, int64_t dim,
                            int64_t src_dtype, torch::ScalarType out_dtype, c10::optional<torch::Tensor> status);
void engram_scatter_grad(torch::Tensor g, torch::Tensor idx, torch::Tensor acc_ptrs, torch::Tensor pos_ptrs,
                         torch::Tensor list_ptrs, torch::Tensor cnt_ptrs, torch::Tensor per, torch::Tensor caps,
                         int64_t world, double scale, c10::optional<torch::Tensor> status, int64_t my_rank);
void engram_push_grads(torch::Tensor g, torch::Tensor idx, torch::Tensor acc_ptrs, torch::Tensor pos_ptrs,
                       torch::Tensor list_ptrs, torch::Tensor cnt_ptrs, torch::Tensor per, torch::Tensor caps,
                       torch::Tensor xbases, int64_t me, double scale, int64_t cap_e, int64_t region_bytes,
                       int64_t rows_off, int64_t call, double timeout_s, torch::Tensor status);
void engram_accumulate_grads(torch::Tensor acc_ptrs, torch::Tensor pos_ptrs, torch::Tensor list_ptrs,
                             torch::Tensor cnt_ptrs, torch::Tensor per, torch::Tensor caps, torch::Tensor xbases,
                             int64_t n_tables, int64_t dim, int64_t me, double scale, int64_t cap_e,
                             int64_t region_bytes, int64_t rows_off, int64_t call, double timeout_s,
                             torch::Tensor status);
void engram_fetch_serve(torch::Tensor fbases, torch::Tensor wptrs, torch::Tensor per, int64_t me, int64_t n_tables,
                        int64_t row_bytes, int64_t ntok, int64_t cap_tok, int64_t recv_off, int64_t call,
                        double timeout_s, torch::Tensor status);
void engram_fetch_collect(torch::Tensor fbases, torch::Tensor wptrs, torch::Tensor per, int64_t me, int64_t n_tables,
                          int64_t row_bytes, int64_t ntok, int64_t cap_tok, int64_t recv_off, int64_t call,
                          double timeout_s, torch::Tensor status, torch::Tensor out);
void engram_touched_sqnorm(torch::Tensor acc_ptrs, torch::Tensor cnt_ptrs, torch::Tensor caps, int64_t dim,
                           torch::Tensor sq);
void engram_clip_coef(torch::Tensor sq, double max_norm, torch::Tensor coef, torch::Tensor norm);
void engram_adam_touched(torch::Tensor p, torch::Tensor m, torch::Tensor v, torch::Tensor acc, torch::Tensor pos,
                         torch::Tensor list, torch::Tensor cnt, c10::optional<torch::Tensor> coef, double lr,
                         double beta1, double beta2, double eps, double wd, double bc1, double bc2, bool sr,
                         int64_t seed, int64_t step, int64_t table_id);
void engram_adam_rows(std::vector<torch::Tensor> p, std::vector<torch::Tensor> m, std::vector<torch::Tensor> v,
                      std::vector<torch::Tensor> acc, std::vector<torch::Tensor> pos, std::vector<torch::Tensor> list,
                      std::vector<torch::Tensor> cnt, std::vector<int64_t> table_ids, std::vector<double> bc1,
                      std::vector<double> bc2, std::vector<int64_t> steps, c10::optional<torch::Tensor> coef,
                      double lr, double beta1, double beta2, double eps, double wd, bool sr, int64_t seed);
void adam_dense(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, double lr, double beta1,
                double beta2, double eps, double wd, double bc1, double bc2, double gscale, bool sr, int64_t seed,
                int64_t step);
std::vector<torch::Tensor> engram_gate_fwd(torch::Tensor h, torch::Tensor k, torch::Tensor v,
                                           c10::optional<torch::Tensor> qs, c10::optional<torch::Tensor> ks,
                                           c10::optional<torch::Tensor> keep, bool sqrt_gate,
                                           c10::optional<torch::Tensor> gate_acc);
std::vector<torch::Tensor> engram_gate_bwd(torch::Tensor g, torch::Tensor h, torch::Tensor k, torch::Tensor v,
                                           c10::optional<torch::Tensor> qs, c10::optional<torch::Tensor> ks,
                                           c10::optional<torch::Tensor> keep, torch::Tensor stats, bool sqrt_gate);
void engram_fill_ids(torch::Tensor out, torch::Tensor input_ids, torch::Tensor positions, torch::Tensor idx_mapping,
                     torch::Tensor qsl, torch::Tensor all_ids, int64_t num_reqs, int64_t num_tokens,
                     int64_t num_padded);
// norm.cu
std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, c10::optional<torch::Tensor> w, double eps);
torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, c10::optional<torch::Tensor> w, torch::Tensor rstd,
                          c10::optional<torch::Tensor> dx_add);
std::vector<torch::Tensor> post_norm_add(torch::Tensor r, torch::Tensor a, torch::Tensor w_post,
                                         c10::optional<torch::Tensor> ls, c10::optional<torch::Tensor> w_next,
                                         double eps);
std::vector<torch::Tensor> post_norm_add_bwd(c10::optional<torch::Tensor> dxo, c10::optional<torch::Tensor> dh,
                                             torch::Tensor a, torch::Tensor x, torch::Tensor w_post,
                                             c10::optional<torch::Tensor> ls, c10::optional<torch::Tensor> w_next,
                                             torch::Tensor rstd_a, c10::optional<torch::Tensor> rstd_x);
std::vector<torch::Tensor> qkv_norm_rope(torch::Tensor qkv, torch::Tensor qw, torch::Tensor kw,
                                         torch::Tensor inv_freq, torch::Tensor pos, int64_t Hq, int64_t Hk, int64_t D,
                                         bool kv_shared, double eps);
torch::Tensor qkv_norm_rope_bwd(torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor qkv,
                                torch::Tensor qw, torch::Tensor kw, torch::Tensor inv_freq, torch::Tensor pos,
                                torch::Tensor rstd, int64_t Hq, int64_t Hk, int64_t D, bool kv_shared);
torch::Tensor geglu_fwd(torch::Tensor gu);
torch::Tensor geglu_bwd(torch::Tensor dm, torch::Tensor gu);
// ce.cu
std::vector<torch::Tensor> ce_fwd(torch::Tensor z, torch::Tensor labels, int64_t start, double softcap);
void ce_bwd_inplace(torch::Tensor z, torch::Tensor labels, int64_t start, double softcap, torch::Tensor lse,
                    torch::Tensor w_row);
// attention.cu
std::vector<torch::Tensor> attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor doc_start,
                                    int64_t window, double scale);
std::vector<torch::Tensor> attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                    torch::Tensor o, torch::Tensor lse, torch::Tensor doc_start, int64_t window,
                                    double scale);
// attention_tc.cu
std::vector<torch::Tensor> attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor doc_start,
                                       int64_t window, double scale);
torch::Tensor attn_tc_status(int64_t device);
std::vector<torch::Tensor> attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                       torch::Tensor o, torch::Tensor lse, torch::Tensor doc_start, int64_t window,
                                       double scale);
void p2p_allreduce_mean(torch::Tensor bases, int64_t rank, int64_t stage_off, int64_t n, int64_t call, double scale,
                        double timeout_s, torch::Tensor out, torch::Tensor status);
std::vector<torch::Tensor> attn_bwd_mat(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                        torch::Tensor o, torch::Tensor lse, torch::Tensor doc_start, int64_t window,
                                        double scale, int64_t tile_budget_bytes);
// gemm.cu
torch::Tensor gemm(torch::Tensor A, torch::Tensor W, bool b_kmajor, c10::optional<torch::Tensor> out);
std::vector<torch::Tensor> gemm_geglu(torch::Tensor A, torch::Tensor Wgu, bool save_gu);
torch::Tensor gemm_dgeglu(torch::Tensor dY, torch::Tensor Wdown, torch::Tensor gu);
torch::Tensor gemm_f32(torch::Tensor A, torch::Tensor W);
torch::Tensor gemm_tn_f32(torch::Tensor At, torch::Tensor Bt);
void gemm_carry_copy(int64_t device, int64_t segs, int64_t nsegs, int64_t begin16, int64_t end16);
void layer_gather(torch::Tensor segs, int64_t begin16, int64_t end16);
void gemm_f32_scatter(torch::Tensor A, torch::Tensor W, torch::Tensor recv_ptrs, int64_t rows_per_rank,
                      int64_t slot, int64_t slot_elems, bool b_kmajor);
void p2p_gather(torch::Tensor bases, int64_t rank, int64_t call, int64_t stage_off, int64_t half_bytes, int64_t n16,
                torch::Tensor out, double timeout_s, torch::Tensor status, bool poison);
void p2p_sum_slots(torch::Tensor bases, int64_t rank, int64_t call, int64_t recv_off, int64_t slot_elems,
                   torch::Tensor out, double timeout_s, torch::Tensor status);
std::vector<torch::Tensor> gemm_ce(torch::Tensor H, torch::Tensor E, torch::Tensor labels, int64_t lab_start,
                                   double cap, bool keep_logits, int64_t n_valid);
torch::Tensor gemm_status(int64_t device);
// gemm_nf4.cu
torch::Tensor gemm_nf4(torch::Tensor A, torch::Tensor codes, torch::Tensor absmax, int64_t rows, int64_t cols,
                       bool b_kmajor, c10::optional<torch::Tensor> out);
std::vector<torch::Tensor> gemm_geglu_nf4(torch::Tensor A, torch::Tensor codes, torch::Tensor absmax, int64_t rows,
                                          int64_t cols, bool save_gu);
torch::Tensor gemm_dgeglu_nf4(torch::Tensor dY, torch::Tensor codes, torch::Tensor absmax, int64_t rows,
                              int64_t cols, torch::Tensor gu);
// nf4.cu
std::vector<torch::Tensor> nf4_quantize(torch::Tensor w);
void nf4_dequant(torch::Tensor codes, torch::Tensor absmax, torch::Tensor out);
// symm.cpp
int64_t symm_alloc(int64_t nbytes, int64_t device);
void symm_free(int64_t ptr, int64_t device);
py::bytes symm_export(int64_t ptr, int64_t device);
int64_t symm_import(py::bytes handle, int64_t device);
void symm_close(int64_t ptr, int64_t device);
torch::Tensor symm_view(int64_t ptr, std::vector<int64_t> shape, torch::ScalarType dtype, int64_t device);
bool can_access_peer(int64_t dev, int64_t peer);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "micro_engram_fork_b200 sm_100a kernels";
  m.def("engram_hash", &engram_hash);
  m.def("engram_hash_prev", &engram_hash_prev);
  m.def("engram_gather", &engram_gather);
  m.def("engram_scatter_grad", &engram_scatter_grad);
  m.def("engram_push_grads", &engram_push_grads);
  m.def("engram_accumulate_grads", &engram_accumulate_grads);
  m.def("engram_adam_rows", &engram_adam_rows);
  m.def("engram_fetch_serve", &engram_fetch_serve);
  m.def("engram_fetch_collect", &engram_fetch_collect);
  m.def("engram_touched_sqnorm", &engram_touched_sqnorm);
  m.def("engram_clip_coef", &engram_clip_coef);
  m.def("engram_adam_touched", &engram_adam_touched);
  m.def("adam_dense", &adam_dense);
  m.def("engram_gate_fwd", &engram_gate_fwd);
  m.def("engram_gate_bwd", &engram_gate_bwd);
  m.def("engram_fill_ids", &engram_fill_ids);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("post_norm_add", &post_norm_add);
  m.def("post_norm_add_bwd", &post_norm_add_bwd);
  m.def("qkv_norm_rope", &qkv_norm_rope);
  m.def("qkv_norm_rope_bwd", &qkv_norm_rope_bwd);
  m.def("geglu_fwd", &geglu_fwd);
  m.def("geglu_bwd", &geglu_bwd);
  m.def("ce_fwd", &ce_fwd);
  m.def("ce_bwd_inplace", &ce_bwd_inplace);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd);
  m.def("attn_fwd_tc", &attn_fwd_tc);
  m.def("attn_tc_status", &attn_tc_status);
  m.def("attn_bwd_tc", &attn_bwd_tc);
  m.def("attn_bwd_mat", &attn_bwd_mat);
  m.def("p2p_allreduce_mean", &p2p_allreduce_mean);
  m.def("gemm", &gemm, py::arg("A"), py::arg("W"), py::arg("b_kmajor") = true, py::arg("out") = py::none());
  m.def("gemm_geglu", &gemm_geglu);
  m.def("gemm_dgeglu", &gemm_dgeglu);
  m.def("gemm_f32", &gemm_f32);
  m.def("gemm_tn_f32", &gemm_tn_f32);
  m.def("gemm_carry_copy", &gemm_carry_copy);
  m.def("layer_gather", &layer_gather);
  m.def("gemm_f32_scatter", &gemm_f32_scatter, py::arg("A"), py::arg("W"), py::arg("recv_ptrs"),
        py::arg("rows_per_rank"), py::arg("slot"), py::arg("slot_elems"), py::arg("b_kmajor") = false);
  m.def("p2p_gather", &p2p_gather, py::arg("bases"), py::arg("rank"), py::arg("call"), py::arg("stage_off"),
        py::arg("half_bytes"), py::arg("n16"), py::arg("out"), py::arg("timeout_s"), py::arg("status"),
        py::arg("poison") = false);
  m.def("p2p_sum_slots", &p2p_sum_slots);
  m.def("gemm_ce", &gemm_ce);
  m.def("gemm_status", &gemm_status);
  m.def("gemm_nf4", &gemm_nf4);
  m.def("gemm_geglu_nf4", &gemm_geglu_nf4);
  m.def("gemm_dgeglu_nf4", &gemm_dgeglu_nf4);
  m.def("nf4_quantize", &nf4_quantize);
  m.def("nf4_dequant", &nf4_dequant);
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_free", &symm_free);
  m.def("symm_export", &symm_export);
  m.def("symm_import", &symm_import);
  m.def("symm_close", &symm_close);
  m.def("symm_view", &symm_view);
  m.def("can_access_peer", &can_access_peer);
}
