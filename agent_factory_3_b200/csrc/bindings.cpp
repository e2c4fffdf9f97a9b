// Python bindings of the sm_100a extension (module agent_factory_3_b200._C).
#include <torch/extension.h>

#include "common.h"

namespace af3 {
void gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor out,
          int64_t epi, int64_t sched, int64_t M, int64_t N, int64_t K,
          c10::optional<torch::Tensor> group_offsets, int64_t num_groups,
          c10::optional<torch::Tensor> bias, int64_t bias_group_stride,
          c10::optional<torch::Tensor> row_scale, c10::optional<torch::Tensor> aux,
          c10::optional<torch::Tensor> out2, double alpha, double beta, double act_alpha,
          double act_limit, c10::optional<torch::Tensor> labels, int64_t vocab_offset,
          c10::optional<torch::Tensor> lse_part, c10::optional<torch::Tensor> label_logit,
          c10::optional<torch::Tensor> row_stats, int64_t n_tiles_total, int64_t bn,
          int64_t band, int64_t out_group_stride, int64_t max_ctas,
          c10::optional<torch::Tensor> a2, c10::optional<torch::Tensor> b2, int64_t K2,
          c10::optional<torch::Tensor> acc_add);
void mxfp4_dequant(torch::Tensor blocks, torch::Tensor scales, torch::Tensor out);
void mxfp4_dequant_gather(torch::Tensor block_ptrs, torch::Tensor scale_ptrs,
                          int64_t experts_per_rank, torch::Tensor out);
void peer_cast_copy(int64_t dst_ptr, int64_t dst_numel, std::vector<torch::Tensor> srcs,
                    std::vector<int64_t> offsets);
std::tuple<torch::Tensor, pybind11::bytes> symm_alloc(int64_t nbytes, int64_t device);
int64_t ipc_open(pybind11::bytes handle);
void ipc_close(int64_t ptr);
void copy_from_address(int64_t src, torch::Tensor dst);
void copy_to_address(torch::Tensor src, int64_t dst);
void mxfp4_to_e4m3(torch::Tensor blocks, torch::Tensor scales, torch::Tensor out,
                   torch::Tensor expert_scale);
void transpose_u8(torch::Tensor in, torch::Tensor out);
void quant_rows_e4m3(torch::Tensor x, torch::Tensor out, torch::Tensor scale);
void gemm_f8(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t epi, int64_t sched,
             int64_t M, int64_t N, int64_t K, c10::optional<torch::Tensor> group_offsets,
             int64_t num_groups, torch::Tensor a_scale, torch::Tensor b_scale,
             c10::optional<torch::Tensor> bias, int64_t bias_group_stride,
             c10::optional<torch::Tensor> row_scale, c10::optional<torch::Tensor> aux,
             c10::optional<torch::Tensor> out2, c10::optional<torch::Tensor> acc_add,
             double alpha, double act_alpha, double act_limit, int64_t bn, int64_t band,
             int64_t max_ctas);
void grad_signal(std::vector<int64_t> flag_ptrs, int64_t rank, int64_t epoch);
void grad_reduce(int64_t inbox_ptr, int64_t flags_ptr, int64_t world, int64_t epoch,
                 torch::Tensor out, torch::Tensor sumsq, double timeout_s);
void enable_peer_access(int64_t peer);
void tp_allreduce_norm(std::vector<int64_t> bufs, std::vector<int64_t> flags, int64_t rank,
                       int64_t epoch, int64_t ld_buf, c10::optional<torch::Tensor> residual,
                       c10::optional<torch::Tensor> w, double eps, torch::Tensor out_x,
                       c10::optional<torch::Tensor> out_n, int64_t T, int64_t H,
                       double timeout_s);
void moe_mxfp4_gemm(torch::Tensor x, torch::Tensor blocks, torch::Tensor scales,
                    c10::optional<torch::Tensor> bias, torch::Tensor offsets, torch::Tensor counts,
                    int64_t epi, c10::optional<torch::Tensor> row_scale, torch::Tensor out,
                    double act_alpha, double act_limit, int64_t bn,
                    c10::optional<torch::Tensor> lora_b, c10::optional<torch::Tensor> xa, int64_t int_cvt);
void moe_route(torch::Tensor logits, torch::Tensor ids, torch::Tensor gates, bool replay);
void moe_group(torch::Tensor ids, torch::Tensor gates, int64_t E, torch::Tensor offsets,
               torch::Tensor expert_counts, torch::Tensor dest, torch::Tensor row_src,
               torch::Tensor row_gate, torch::Tensor scratch);
void gather_rows(torch::Tensor x, torch::Tensor src, c10::optional<torch::Tensor> scale,
                 torch::Tensor out, bool zero_pad);
void combine_rows(torch::Tensor y, torch::Tensor dest, int64_t K,
                  c10::optional<torch::Tensor> residual, torch::Tensor out);
void rmsnorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y,
                 c10::optional<torch::Tensor> rstd, double eps);
void rmsnorm_bwd(torch::Tensor x, torch::Tensor w, torch::Tensor dy, torch::Tensor rstd,
                 c10::optional<torch::Tensor> dres, torch::Tensor dx,
                 c10::optional<torch::Tensor> dw);
void rope_apply(torch::Tensor qkv, int64_t n_rot_heads, int64_t head_dim, torch::Tensor pos,
                torch::Tensor cos_t, torch::Tensor sin_t, bool inverse);
void lse_merge(torch::Tensor parts, torch::Tensor label_logit, torch::Tensor logprob,
               torch::Tensor entropy, torch::Tensor logz);
void swiglu_fwd(torch::Tensor gu, torch::Tensor out, double alpha, double limit);
void swiglu_bwd(torch::Tensor gu, torch::Tensor dout, torch::Tensor dgu, double alpha,
                double limit);
void attn_fwd(torch::Tensor qkv, torch::Tensor sinks, torch::Tensor tiles, torch::Tensor cu,
              torch::Tensor out, torch::Tensor lse, int64_t hq, int64_t hkv, int64_t d,
              int64_t window, double scale);
void attn_bwd(torch::Tensor qkv, torch::Tensor sinks, torch::Tensor kv_tiles, torch::Tensor cu,
              torch::Tensor out, torch::Tensor dout, torch::Tensor lse, torch::Tensor dqkv,
              torch::Tensor dsinks, int64_t hq, int64_t hkv, int64_t d, int64_t window,
              double scale);
void decode_attention(torch::Tensor q, torch::Tensor k_pages, torch::Tensor v_pages,
                      torch::Tensor page_table, torch::Tensor seq_lens, torch::Tensor sinks,
                      torch::Tensor out, c10::optional<torch::Tensor> lse, int64_t hq, int64_t hkv,
                      int64_t window, double scale, int64_t max_seq_len);
void kv_store(torch::Tensor qkv, int64_t k_off, int64_t v_off, torch::Tensor slots,
              torch::Tensor k_pages, torch::Tensor v_pages);
void kv_gather(torch::Tensor qkv, int64_t k_off, int64_t v_off, torch::Tensor slots,
               torch::Tensor k_pages, torch::Tensor v_pages);
void sample_tokens(torch::Tensor logits, torch::Tensor temperature, c10::optional<torch::Tensor> min_p,
                   torch::Tensor seeds, int64_t step, torch::Tensor tokens, torch::Tensor logprobs,
                   torch::Tensor entropy);
}  // namespace af3

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  namespace py = pybind11;
  m.doc() = "agent_factory_3_b200 sm_100a kernels";
  m.def("gemm", &af3::gemm, py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"),
        py::arg("out"), py::arg("epi"), py::arg("sched"), py::arg("M"), py::arg("N"),
        py::arg("K"), py::arg("group_offsets"), py::arg("num_groups"), py::arg("bias"),
        py::arg("bias_group_stride"), py::arg("row_scale"), py::arg("aux"), py::arg("out2"),
        py::arg("alpha"), py::arg("beta"), py::arg("act_alpha"), py::arg("act_limit"),
        py::arg("labels"), py::arg("vocab_offset"), py::arg("lse_part"),
        py::arg("label_logit"), py::arg("row_stats"), py::arg("n_tiles_total"), py::arg("bn"),
        py::arg("band"), py::arg("out_group_stride"), py::arg("max_ctas"),
        py::arg("a2") = py::none(), py::arg("b2") = py::none(), py::arg("K2") = 0,
        py::arg("acc_add") = py::none());
  m.def("mxfp4_dequant", &af3::mxfp4_dequant);
  m.def("mxfp4_dequant_gather", &af3::mxfp4_dequant_gather,
        "MXFP4 -> bf16 of an expert stack sharded over peer-mapped per-rank buffers");
  m.def("peer_cast_copy", &af3::peer_cast_copy,
        "cast fp32/bf16 tensors to bf16 and store them into a (peer) staging buffer");
  m.def("symm_alloc", &af3::symm_alloc, "zeroed cudaMalloc buffer + its CUDA IPC handle");
  m.def("ipc_open", &af3::ipc_open, "map another process's IPC buffer; returns a device pointer");
  m.def("ipc_close", &af3::ipc_close);
  m.def("mxfp4_to_e4m3", &af3::mxfp4_to_e4m3,
        "MXFP4 experts -> e4m3 bytes [E, N, K] + one fp32 scale per expert");
  m.def("transpose_u8", &af3::transpose_u8, "[G, R, C] -> [G, C, R] bytes");
  m.def("quant_rows_e4m3", &af3::quant_rows_e4m3, "bf16 rows -> e4m3 + per-row fp32 scale");
  m.def("gemm_f8", &af3::gemm_f8, "tcgen05 kind::f8f6f4 GEMM (e4m3, K-major) with scaled epilogues");
  m.def("copy_to_address", &af3::copy_to_address,
        "copy a contiguous tensor to a device address (own or peer-mapped) on the current stream");
  m.def("grad_signal", &af3::grad_signal, "publish this rank's gradient pushes of a step");
  m.def("grad_reduce", &af3::grad_reduce,
        "sum the inbox slots of all ranks into the local gradient shard (+ sum of squares)");
  m.def("copy_from_address", &af3::copy_from_address,
        "copy dst.nbytes() bytes from a device address (own or peer-mapped) into dst");
  m.def("enable_peer_access", &af3::enable_peer_access,
        "allow kernels on the current device to access device `peer` (same process)");
  m.def("tp_allreduce_norm", &af3::tp_allreduce_norm,
        "one-shot NVLink all-reduce of per-rank partials + residual add + RMSNorm");
  m.def("moe_mxfp4_gemm", &af3::moe_mxfp4_gemm, "MXFP4 expert GEMM (swap-AB, few tokens/expert)",
        py::arg("x"), py::arg("blocks"), py::arg("scales"), py::arg("bias"), py::arg("offsets"),
        py::arg("counts"), py::arg("epi"), py::arg("row_scale"), py::arg("out"),
        py::arg("act_alpha") = 1.702, py::arg("act_limit") = 7.0, py::arg("bn") = 32,
        py::arg("lora_b") = py::none(), py::arg("xa") = py::none(), py::arg("int_cvt") = 0);
  m.def("moe_route", &af3::moe_route);
  m.def("moe_group", &af3::moe_group);
  m.def("gather_rows", &af3::gather_rows, py::arg("x"), py::arg("src"), py::arg("scale"),
        py::arg("out"), py::arg("zero_pad") = true);
  m.def("combine_rows", &af3::combine_rows);
  m.def("rmsnorm_fwd", &af3::rmsnorm_fwd);
  m.def("rmsnorm_bwd", &af3::rmsnorm_bwd);
  m.def("rope_apply", &af3::rope_apply);
  m.def("lse_merge", &af3::lse_merge);
  m.def("swiglu_fwd", &af3::swiglu_fwd);
  m.def("swiglu_bwd", &af3::swiglu_bwd);
  m.def("attn_fwd", &af3::attn_fwd);
  m.def("attn_bwd", &af3::attn_bwd);
  m.def("decode_attention", &af3::decode_attention);
  m.def("kv_store", &af3::kv_store);
  m.def("kv_gather", &af3::kv_gather);
  m.def("sample_tokens", &af3::sample_tokens);
  m.def("device_error", &af3::device_error_take,
        "Read and clear the current device's kernel error word (0 = no error).");
}
