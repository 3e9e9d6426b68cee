// Python bindings of llm_research_b200._C
#include <torch/extension.h>

#include <tuple>
#include <vector>

namespace lrb {
// norm.cu
std::tuple<at::Tensor, at::Tensor, c10::optional<at::Tensor>> rmsnorm_fwd(const at::Tensor&, const at::Tensor&, double,
                                                                          const c10::optional<at::Tensor>&,
                                                                          at::ScalarType);
std::tuple<at::Tensor, at::Tensor> rmsnorm_bwd(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                               const at::Tensor&, const c10::optional<at::Tensor>&);
// elementwise.cu
at::Tensor swiglu_fwd(const at::Tensor&);
at::Tensor swiglu_bwd(const at::Tensor&, const at::Tensor&);
at::Tensor exp2_fma_eval(const at::Tensor&);
std::tuple<at::Tensor, at::Tensor, at::Tensor> rope_qkv_fwd(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                                            int64_t, int64_t, int64_t, int64_t);
at::Tensor rope_qkv_bwd(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                        int64_t, int64_t, int64_t, int64_t);
// loss.cu
std::tuple<at::Tensor, at::Tensor, at::Tensor> ce_fwd(const at::Tensor&, const at::Tensor&, int64_t);
at::Tensor ce_bwd(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t);
at::Tensor ce_bwd_vocab_shard(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t);
// routing.cu
std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> route_slots(const at::Tensor&, int64_t, int64_t, int64_t);
std::tuple<at::Tensor, at::Tensor, at::Tensor> softmax_topk_fwd(const at::Tensor&, int64_t);
at::Tensor chunk_mean_pool_fwd(const at::Tensor&, int64_t);
std::tuple<at::Tensor, at::Tensor> compact_chunks(const at::Tensor&);
// optim.cu
at::Tensor muon_prologue(std::vector<at::Tensor>, std::vector<at::Tensor>, std::vector<at::Tensor>,
                         std::vector<at::Tensor>, double, double, double);
void muon_epilogue(std::vector<at::Tensor>, std::vector<at::Tensor>, at::Tensor, double);
void axpy_list(std::vector<at::Tensor>, std::vector<at::Tensor>, double);
void adamw_step(std::vector<at::Tensor>, std::vector<at::Tensor>, std::vector<at::Tensor>, std::vector<at::Tensor>,
                std::vector<double>, std::vector<double>, double, double, double, double, double);
// ns.cu
at::Tensor newton_schulz(const at::Tensor&, int64_t, double, double, double);
void gemm_batched(const at::Tensor&, const at::Tensor&, bool, const at::Tensor&, const c10::optional<at::Tensor>&, double,
                  double);
int64_t gemm_batched_error(int64_t);
// quant.cu
std::tuple<at::Tensor, at::Tensor> int4_quantize(const at::Tensor&, int64_t);
at::Tensor int4_dequantize(const at::Tensor&, const at::Tensor&, int64_t);
std::tuple<at::Tensor, at::Tensor, at::Tensor> nvfp4_quantize(const at::Tensor&, bool, int64_t);
std::vector<at::Tensor> nvfp4_quantize_dual(const at::Tensor&, const c10::optional<at::Tensor>&, bool, bool, bool,
                                            int64_t);
at::Tensor nvfp4_dequantize(const at::Tensor&, const at::Tensor&, const at::Tensor&, at::ScalarType);
// attention.cu
std::tuple<at::Tensor, at::Tensor> attn_fwd(const at::Tensor&, const at::Tensor&, const at::Tensor&, bool, double);
std::tuple<at::Tensor, at::Tensor, at::Tensor> attn_bwd(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                                        const at::Tensor&, const at::Tensor&, const at::Tensor&, bool,
                                                        double, bool);
// gemm_sm100.cu
at::Tensor gemm_tn(const at::Tensor&, const at::Tensor&, at::ScalarType, double);
void gemm_tn_accumulate(const at::Tensor&, const at::Tensor&, at::Tensor&, double);
int64_t sm100_error(int64_t);
// gemm_pair_sm100.cu
void gemm_pair(const at::Tensor&, const at::Tensor&, bool, bool, at::Tensor&, bool, double);
int64_t gemm_pair_error(int64_t);
void gemm_pair_axpby(const at::Tensor&, const at::Tensor&, bool, at::Tensor&, const at::Tensor&, double, double);
void gemm_pair_swiglu_bwd(const at::Tensor&, const at::Tensor&, const at::Tensor&, at::Tensor&);
void gemm_pair_set_trace(const c10::optional<at::Tensor>&);
void gemm_pair_swiglu(const at::Tensor&, const at::Tensor&, const at::Tensor&, at::Tensor&, at::Tensor&);
void gemm_pair_rope(const at::Tensor&, const at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                    int64_t, int64_t);
// attention_sm100.cu
bool attn_sm100_supported(const at::Tensor&, const at::Tensor&, const at::Tensor&);
std::tuple<at::Tensor, at::Tensor> attn_fwd_sm100(const at::Tensor&, const at::Tensor&, const at::Tensor&, bool, double);
int64_t attn_sm100_error(int64_t);
// attention_bwd_sm100.cu
int64_t attn_bwd_sm100_error(int64_t);
void attn_bwd_set_trace(const c10::optional<at::Tensor>&);
// memory.cu
std::tuple<at::Tensor, at::Tensor, at::Tensor> topk_softmax_gather(const at::Tensor&, const at::Tensor&, int64_t);
std::tuple<at::Tensor, at::Tensor> memory_topk_candidates(const at::Tensor&, const at::Tensor&, int64_t);
int64_t memory_topk_error(int64_t);
std::tuple<at::Tensor, at::Tensor> topk_gather_fwd(const at::Tensor&, const at::Tensor&, const at::Tensor&);
at::Tensor topk_gather_bwd(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                           const at::Tensor&);
// gemm_nvfp4_sm100.cu
at::Tensor gemm_nvfp4(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                      const at::Tensor&);
int64_t gemm_nvfp4_error(int64_t);
// comm/symm.cu
std::tuple<int64_t, at::Tensor> symm_alloc(int64_t, int64_t);
int64_t symm_open(const at::Tensor&, int64_t);
void symm_close(int64_t, int64_t);
void symm_free(int64_t, int64_t);
at::Tensor symm_view(int64_t, int64_t, at::IntArrayRef, at::ScalarType, int64_t);
void p2p_rs_push(at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                 at::Tensor&, at::Tensor&);
void p2p_rs_reduce(const at::Tensor&, at::Tensor&, int64_t, double, bool, const at::Tensor&, at::Tensor&, int64_t,
                   c10::optional<at::Tensor>, at::Tensor&, at::Tensor&);
void p2p_ag_publish(const at::Tensor&, at::Tensor&, at::Tensor&, int64_t, at::Tensor&);
void p2p_rows_rs_push(const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                      at::Tensor&, at::Tensor&);
void p2p_rows_rs_reduce(const at::Tensor&, const c10::optional<at::Tensor>&, at::Tensor&, int64_t, const at::Tensor&,
                        at::Tensor&, int64_t, at::Tensor&, at::Tensor&);
void p2p_pull(at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, at::Tensor&);
void p2p_a2av_pull(at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, at::Tensor&);
void diloco_push(const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, int64_t,
                 int64_t, at::Tensor&, at::Tensor&);
void diloco_reduce_nesterov(const at::Tensor&, at::Tensor&, at::Tensor&, at::Tensor&, int64_t, double, double,
                            const at::Tensor&, at::Tensor&, at::Tensor&, int64_t, at::Tensor&, at::Tensor&);
// comm/nvls.cu
void nvls_all_reduce(at::Tensor&, int64_t, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, double, at::Tensor&,
                     at::Tensor&);
void nvls_rs_stage(at::Tensor&, at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t,
                   at::Tensor&, at::Tensor&);
void nvls_rs_reduce(int64_t, at::Tensor&, double, bool, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t,
                    int64_t, c10::optional<at::Tensor>, at::Tensor&, at::Tensor&);
void nvls_ag_publish(const at::Tensor&, int64_t, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t,
                     int64_t, int64_t, at::Tensor&, at::Tensor&);
void nvls_wait(const at::Tensor&, int64_t, int64_t, at::Tensor&);
void nvls_diloco_outer(at::Tensor&, int64_t, const at::Tensor&, int64_t, const at::Tensor&, at::Tensor&, int64_t, int64_t,
                       int64_t, double, double, bool, at::Tensor&, at::Tensor&);
// comm/ep.cu
void ep_push(const at::Tensor&, const c10::optional<at::Tensor>&, bool, const at::Tensor&, int64_t, int64_t, int64_t,
             int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, const at::Tensor&, const at::Tensor&,
             const at::Tensor&, at::Tensor&, at::Tensor&);
void ep_pull(at::Tensor&, const c10::optional<at::Tensor>&, const c10::optional<at::Tensor>&, const at::Tensor&,
             int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, const at::Tensor&,
             const at::Tensor&, const at::Tensor&, at::Tensor&, at::Tensor&);
void ep_flag_wait(const at::Tensor&, int64_t, int64_t, at::Tensor&);
void ep_flag_set(at::Tensor&, int64_t);
// comm/gemm_comm.cu
void gemm_rs(const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t, int64_t,
             int64_t, at::Tensor&, at::Tensor&);
void tp_reduce(const at::Tensor&, const c10::optional<at::Tensor>&, at::Tensor&, int64_t, const at::Tensor&,
               at::Tensor&, int64_t, at::Tensor&, at::Tensor&);
void shard_publish(const at::Tensor&, at::Tensor&, at::Tensor&, int64_t, at::Tensor&);
at::Tensor ag_gemm(const at::Tensor&, at::Tensor&, at::Tensor&, const at::Tensor&, int64_t, int64_t, int64_t, int64_t,
                   int64_t, int64_t, at::Tensor&);
}  // namespace lrb

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of the llm_research_b200 framework";
  m.def("rmsnorm_fwd", &lrb::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &lrb::rmsnorm_bwd);
  m.def("swiglu_fwd", &lrb::swiglu_fwd);
  m.def("swiglu_bwd", &lrb::swiglu_bwd);
  m.def("exp2_fma_eval", &lrb::exp2_fma_eval, "2^x by the FMA-pipe polynomial of the attention softmax");
  m.def("rope_qkv_fwd", &lrb::rope_qkv_fwd);
  m.def("rope_qkv_bwd", &lrb::rope_qkv_bwd);
  m.def("ce_fwd", &lrb::ce_fwd);
  m.def("ce_bwd", &lrb::ce_bwd);
  m.def("ce_bwd_vocab_shard", &lrb::ce_bwd_vocab_shard);
  m.def("route_slots", &lrb::route_slots, "capacity slots, owner ranks and per-expert counts of routed assignments");
  m.def("softmax_topk_fwd", &lrb::softmax_topk_fwd);
  m.def("chunk_mean_pool_fwd", &lrb::chunk_mean_pool_fwd);
  m.def("compact_chunks", &lrb::compact_chunks);
  m.def("muon_prologue", &lrb::muon_prologue);
  m.def("muon_epilogue", &lrb::muon_epilogue);
  m.def("adamw_step", &lrb::adamw_step);
  m.def("axpy_list", &lrb::axpy_list);
  m.def("newton_schulz", &lrb::newton_schulz);
  m.def("gemm_batched", &lrb::gemm_batched, "C = alpha A op(B) + beta D, batched tcgen05 (bf16); C written in place");
  m.def("gemm_batched_error", &lrb::gemm_batched_error);
  m.def("int4_quantize", &lrb::int4_quantize);
  m.def("int4_dequantize", &lrb::int4_dequantize);
  m.def("nvfp4_quantize", &lrb::nvfp4_quantize);
  m.def("nvfp4_quantize_dual", &lrb::nvfp4_quantize_dual, "x (M,K) -> row-wise and/or transposed NVFP4 with atom-layout scales",
        py::arg("x"), py::arg("amax") = py::none(), py::arg("rowwise") = true, py::arg("colwise") = true,
        py::arg("stochastic") = false, py::arg("seed") = 0);
  m.def("nvfp4_dequantize", &lrb::nvfp4_dequantize);
  m.def("attn_fwd", &lrb::attn_fwd);
  m.def("attn_bwd", &lrb::attn_bwd);
  m.def("gemm_tn", &lrb::gemm_tn);
  m.def("gemm_tn_accumulate", &lrb::gemm_tn_accumulate);
  m.def("sm100_error", &lrb::sm100_error);
  m.def("gemm_pair", &lrb::gemm_pair,
        "C (=|+=) alpha op(A) op(B)^T on CTA pairs (tcgen05 cta_group::2); a_mn/b_mn: operand stored (K, M)/(K, N)");
  m.def("gemm_pair_error", &lrb::gemm_pair_error);
  m.def("gemm_pair_rope", &lrb::gemm_pair_rope, "QKV projection with RoPE on the query/key heads in the epilogue");
  m.def("gemm_pair_axpby", &lrb::gemm_pair_axpby, "C = alpha A op(B)^T + beta D on the CTA-pair kernel (2-D or batched)");
  m.def("gemm_pair_swiglu_bwd", &lrb::gemm_pair_swiglu_bwd, "dgu = swiglu_bwd(dY W2, gu) in one CTA-pair launch");
  m.def("gemm_pair_set_trace", &lrb::gemm_pair_set_trace, "pipeline trace of the pair GEMM (None switches it off)");
  m.def("gemm_pair_swiglu", &lrb::gemm_pair_swiglu, "gu = [x W1^T | x Wg^T], h = silu(x Wg^T) * x W1^T in one launch");
  m.def("attn_sm100_supported", &lrb::attn_sm100_supported);
  m.def("attn_fwd_sm100", &lrb::attn_fwd_sm100);
  m.def("attn_sm100_error", &lrb::attn_sm100_error);
  m.def("attn_bwd_sm100_error", &lrb::attn_bwd_sm100_error);
  m.def("attn_bwd_set_trace", &lrb::attn_bwd_set_trace, "stage timestamps of CTA (0,0) of the next backward launches");
  m.def("topk_softmax_gather", &lrb::topk_softmax_gather);
  m.def("memory_topk_candidates", &lrb::memory_topk_candidates,
        "tcgen05 similarity + streaming top-32 per query over bank slices");
  m.def("memory_topk_error", &lrb::memory_topk_error);
  m.def("topk_gather_fwd", &lrb::topk_gather_fwd);
  m.def("topk_gather_bwd", &lrb::topk_gather_bwd);
  m.def("gemm_nvfp4", &lrb::gemm_nvfp4);
  m.def("gemm_nvfp4_error", &lrb::gemm_nvfp4_error);
  m.def("ep_push", &lrb::ep_push);
  m.def("ep_pull", &lrb::ep_pull);
  m.def("ep_flag_wait", &lrb::ep_flag_wait);
  m.def("ep_flag_set", &lrb::ep_flag_set);
  m.def("gemm_rs", &lrb::gemm_rs);
  m.def("tp_reduce", &lrb::tp_reduce);
  m.def("shard_publish", &lrb::shard_publish);
  m.def("ag_gemm", &lrb::ag_gemm);
  m.def("symm_alloc", &lrb::symm_alloc);
  m.def("symm_open", &lrb::symm_open);
  m.def("symm_close", &lrb::symm_close);
  m.def("symm_free", &lrb::symm_free);
  m.def("symm_view", &lrb::symm_view);
  m.def("p2p_rs_push", &lrb::p2p_rs_push);
  m.def("p2p_rs_reduce", &lrb::p2p_rs_reduce);
  m.def("p2p_ag_publish", &lrb::p2p_ag_publish);
  m.def("p2p_rows_rs_push", &lrb::p2p_rows_rs_push);
  m.def("p2p_rows_rs_reduce", &lrb::p2p_rows_rs_reduce);
  m.def("p2p_pull", &lrb::p2p_pull);
  m.def("p2p_a2av_pull", &lrb::p2p_a2av_pull, "all-to-all-v by P2P loads from the peers' symmetric heaps");
  m.def("diloco_push", &lrb::diloco_push);
  m.def("diloco_reduce_nesterov", &lrb::diloco_reduce_nesterov);
  m.def("nvls_all_reduce", &lrb::nvls_all_reduce, "in-place all-reduce through NVSwitch multicast (multimem)");
  m.def("nvls_rs_stage", &lrb::nvls_rs_stage);
  m.def("nvls_rs_reduce", &lrb::nvls_rs_reduce);
  m.def("nvls_ag_publish", &lrb::nvls_ag_publish);
  m.def("nvls_wait", &lrb::nvls_wait);
  m.def("nvls_diloco_outer", &lrb::nvls_diloco_outer);
}
