// Python bindings of the sm_100a kernels (module nanovllm_b200._C).
#include <torch/extension.h>

void rms_norm_cuda(torch::Tensor out, torch::Tensor x, c10::optional<torch::Tensor> residual,
                   c10::optional<torch::Tensor> weight, double eps, int64_t mode, c10::optional<torch::Tensor> xpart);
void layer_norm_cuda(torch::Tensor out, torch::Tensor x, c10::optional<torch::Tensor> residual, torch::Tensor weight,
                     torch::Tensor bias, double eps);
void qk_norm_rope_store_cuda(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin,
                             c10::optional<torch::Tensor> q_w, c10::optional<torch::Tensor> k_w, int64_t norm_mode,
                             bool v_norm, double eps, torch::Tensor q_out, c10::optional<torch::Tensor> k_cache,
                             c10::optional<torch::Tensor> v_cache, c10::optional<torch::Tensor> slots, int64_t nq,
                             int64_t nkv, int64_t head_dim, bool apply_rope, c10::optional<torch::Tensor> qkv_part);
void paged_decode_cuda(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                       torch::Tensor ctx_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_lse,
                       double scale, double softcap, int64_t window, int64_t part_tiles, int64_t nsplit,
                       c10::optional<torch::Tensor> err, c10::optional<torch::Tensor> combine_counters);
void prefill_attention_cuda(torch::Tensor q, torch::Tensor out, torch::Tensor cu_q, torch::Tensor cu_k,
                            int64_t max_q, c10::optional<torch::Tensor> k_cache, c10::optional<torch::Tensor> v_cache,
                            c10::optional<torch::Tensor> block_tables, c10::optional<torch::Tensor> kv_src,
                            int64_t nq, int64_t nkv, int64_t hd, double scale, double softcap, int64_t window,
                            bool causal, c10::optional<torch::Tensor> err);
int64_t gemm_cuda(torch::Tensor x, torch::Tensor w, torch::Tensor out, int64_t act, c10::optional<torch::Tensor> workspace,
                  int64_t force_splits, c10::optional<torch::Tensor> err, bool partial_out);
int64_t gemm_splits_for(int64_t M, int64_t N, int64_t K, int64_t act);
std::vector<int64_t> gemm_sp_cuda(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> out, int64_t act,
                                  c10::optional<torch::Tensor> workspace, c10::optional<torch::Tensor> err,
                                  bool partial_out, std::vector<int64_t> sp_plan, double eps);
void splitk_sum_cuda(torch::Tensor parts, torch::Tensor out);
int64_t qgemm_splits_cuda(int64_t M, int64_t N, int64_t K, int64_t type);
int64_t qgemm_row_step_bytes(int64_t type);
void qgemm_set_trace(c10::optional<torch::Tensor> t);
int64_t qgemm_cuda(torch::Tensor x, torch::Tensor w, int64_t type, int64_t N, int64_t K, torch::Tensor out,
                   c10::optional<torch::Tensor> parts, c10::optional<torch::Tensor> err, bool partial_out);
void qdequant_cuda(torch::Tensor w, int64_t type, int64_t N, int64_t K, torch::Tensor out);
void embedding_cuda(torch::Tensor out, torch::Tensor table, torch::Tensor ids, double scale, int64_t vstart,
                    int64_t vend);
void act_mul_cuda(torch::Tensor out, torch::Tensor x, int64_t act, bool interleaved);
void bias_act_cuda(torch::Tensor x, c10::optional<torch::Tensor> bias, int64_t act);
void gather_rows_cuda(torch::Tensor out, torch::Tensor src, torch::Tensor idx);
void mean_pool_l2_cuda(torch::Tensor out, torch::Tensor x, torch::Tensor cu);
void shortconv_cuda(torch::Tensor proj, torch::Tensor weight, torch::Tensor cu, torch::Tensor rows, torch::Tensor fresh,
                    torch::Tensor state, int64_t state_off, torch::Tensor out);
void sample_cuda(torch::Tensor logits, torch::Tensor temps, torch::Tensor topk, torch::Tensor topp, torch::Tensor seeds,
                 torch::Tensor seq_ids, torch::Tensor steps, double softcap, torch::Tensor out,
                 c10::optional<torch::Tensor> ids);
void rms_norm_post_add_cuda(torch::Tensor x, torch::Tensor residual, c10::optional<torch::Tensor> weight, double eps,
                            int64_t mode, double post_scale);
void ple_combine_cuda(torch::Tensor out, torch::Tensor proj, torch::Tensor tok, torch::Tensor weight, double eps,
                      double proj_scale, double out_scale);
void gate_act_mul_cuda(torch::Tensor out, torch::Tensor gate, torch::Tensor other);
void srq_cuda(torch::Tensor x, double scale);
std::vector<torch::Tensor> symm_alloc_cuda(int64_t nbytes);
int64_t ipc_open_cuda(torch::Tensor handle);
void ipc_close_cuda(int64_t ptr);
void tp_allreduce_norm_cuda(std::vector<int64_t> in, std::vector<int64_t> res, std::vector<int64_t> out,
                            std::vector<int64_t> sig, int64_t rank, int64_t T, int64_t H,
                            c10::optional<torch::Tensor> weight, double eps, int64_t mode, torch::Tensor counters,
                            c10::optional<torch::Tensor> err, int64_t max_blocks, int64_t oneshot,
                            int64_t wait_ns);

void sp_begin_cuda(int64_t epoch_ptr);
int64_t sp_embed_rs_cuda(torch::Tensor table, torch::Tensor ids, double scale, int64_t vstart, int64_t vend,
                         std::vector<int64_t> plan);
int64_t sp_rs_push_cuda(torch::Tensor x, std::vector<int64_t> plan);
void sp_ag_norm_cuda(std::vector<int64_t> plan, double eps, c10::optional<torch::Tensor> err);
void sp_argmax_cuda(torch::Tensor logits, int64_t ncols, int64_t col0, double softcap, torch::Tensor out,
                    int64_t rank, std::vector<int64_t> exch, std::vector<int64_t> flags, int64_t epoch,
                    int64_t wait_ns, c10::optional<torch::Tensor> err);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nanovllm_b200 sm_100a kernels";
  m.def("rms_norm", &rms_norm_cuda);
  m.def("layer_norm", &layer_norm_cuda);
  m.def("qk_norm_rope_store", &qk_norm_rope_store_cuda);
  m.def("paged_decode", &paged_decode_cuda);
  m.def("prefill_attention", &prefill_attention_cuda);
  m.def("gemm", &gemm_cuda);
  m.def("gemm_splits_for", &gemm_splits_for);
  m.def("gemm_sp", &gemm_sp_cuda);
  m.def("sp_begin", &sp_begin_cuda);
  m.def("sp_embed_rs", &sp_embed_rs_cuda);
  m.def("sp_rs_push", &sp_rs_push_cuda);
  m.def("sp_ag_norm", &sp_ag_norm_cuda);
  m.def("sp_argmax", &sp_argmax_cuda);
  m.def("splitk_sum", &splitk_sum_cuda);
  m.def("qgemm_splits", &qgemm_splits_cuda);
  m.def("qgemm_row_step_bytes", &qgemm_row_step_bytes);
  m.def("qgemm_set_trace", &qgemm_set_trace);
  m.def("qgemm", &qgemm_cuda);
  m.def("qdequant", &qdequant_cuda);
  m.def("embedding", &embedding_cuda);
  m.def("act_mul", &act_mul_cuda);
  m.def("bias_act", &bias_act_cuda);
  m.def("gather_rows", &gather_rows_cuda);
  m.def("mean_pool_l2", &mean_pool_l2_cuda);
  m.def("sample", &sample_cuda);
  m.def("shortconv", &shortconv_cuda);
  m.def("rms_norm_post_add", &rms_norm_post_add_cuda);
  m.def("ple_combine", &ple_combine_cuda);
  m.def("gate_act_mul", &gate_act_mul_cuda);
  m.def("srq", &srq_cuda);
  m.def("symm_alloc", &symm_alloc_cuda);
  m.def("ipc_open", &ipc_open_cuda);
  m.def("ipc_close", &ipc_close_cuda);
  m.def("tp_allreduce_norm", &tp_allreduce_norm_cuda, py::arg("in_ptrs"), py::arg("res_ptrs"), py::arg("out_ptrs"),
        py::arg("sig_ptrs"), py::arg("rank"), py::arg("T"), py::arg("H"), py::arg("weight"), py::arg("eps"),
        py::arg("mode"), py::arg("counters"), py::arg("err"), py::arg("max_blocks"), py::arg("oneshot"),
        py::arg("wait_ns") = 0);
}
