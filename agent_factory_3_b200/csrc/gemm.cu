// Torch-facing entry point of the tcgen05 GEMM (see gemm_sm100.cuh for the kernel).
#include "common.h"
#include "gemm_dispatch.h"
#include "gemm_launch.cuh"

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
          c10::optional<torch::Tensor> acc_add) {
  check_cuda_bf16(a, "a");
  check_cuda_bf16(b, "b");
  AF3_CHECK(a.dim() == 2 && a.stride(1) == 1, "a must be 2-D with unit inner stride");
  AF3_CHECK((b.dim() == 2 || b.dim() == 3) && b.stride(-1) == 1,
            "b must be 2-D or 3-D with unit inner stride");
  AF3_CHECK(M >= 0 && N > 0 && K > 0, "bad GEMM shape");
  AF3_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "GEMM dims must fit int32");
  const c10::cuda::CUDAGuard guard(a.device());
  if (M == 0) return;  // nothing to compute (and TMA descriptors cannot describe empty tensors)
  GemmOperands o;
  o.a = a.data_ptr();
  o.a_mn = a_mn;
  o.lda = a.stride(0);
  o.a_rows = a.size(0);
  o.a_cols = a.size(1);
  o.b = b.data_ptr();
  o.b_mn = b_mn;
  o.b_3d = b.dim() == 3;
  o.ldb = b.stride(-2);
  o.b_rows = b.size(-2);
  o.b_cols = b.size(-1);
  o.b_groups = o.b_3d ? b.size(0) : 1;
  o.b_gstride = o.b_3d ? b.stride(0) : 0;

  const bool dual = a2.has_value() && b2.has_value() && K2 > 0;
  if (dual) {
    check_cuda_bf16(*a2, "a2");
    check_cuda_bf16(*b2, "b2");
    AF3_CHECK(a2->dim() == 2 && a2->stride(1) == 1, "a2 must be 2-D, unit inner stride");
    AF3_CHECK(b2->dim() == b.dim() && b2->stride(-1) == 1, "b2 must match b's rank");
    o.a2 = a2->data_ptr();
    o.lda2 = a2->stride(0);
    o.a2_rows = a2->size(0);
    o.a2_cols = a2->size(1);
    o.b2 = b2->data_ptr();
    o.ldb2 = b2->stride(-2);
    o.b2_rows = b2->size(-2);
    o.b2_cols = b2->size(-1);
    o.b2_gstride = b2->dim() == 3 ? b2->stride(0) : 0;
  }
  GemmArgs args{};
  args.K2 = dual ? (int)K2 : 0;
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.num_groups = (int)num_groups;
  args.group_offsets = group_offsets.has_value() ? group_offsets->data_ptr<int>() : nullptr;
  args.band = (int)std::max<int64_t>(band, 1);
  args.out = out.data_ptr();
  args.ldo = out.stride(-2 + (out.dim() == 1 ? 1 : 0));
  if (out.dim() >= 2) args.ldo = out.stride(out.dim() - 2);
  args.out_group_stride = out_group_stride;
  args.bias = bias.has_value() ? bias->data_ptr<float>() : nullptr;
  args.bias_group_stride = bias_group_stride;
  args.row_scale = row_scale.has_value() ? row_scale->data_ptr<float>() : nullptr;
  args.aux = aux.has_value() ? reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr()) : nullptr;
  args.ld_aux = aux.has_value() ? aux->stride(0) : 0;
  args.out2 = out2.has_value() ? out2->data_ptr() : nullptr;
  args.ldo2 = out2.has_value() ? out2->stride(0) : 0;
  args.alpha = (float)alpha;
  args.beta = (float)beta;
  args.act_alpha = (float)act_alpha;
  args.act_limit = (float)act_limit;
  args.labels = labels.has_value() ? labels->data_ptr<int>() : nullptr;
  args.vocab_offset = (int)vocab_offset;
  args.lse_part = lse_part.has_value() ? lse_part->data_ptr<float>() : nullptr;
  args.label_logit = label_logit.has_value() ? label_logit->data_ptr<float>() : nullptr;
  args.row_stats = row_stats.has_value() ? row_stats->data_ptr<float>() : nullptr;
  args.n_tiles_total = (int)n_tiles_total;
  args.err = device_error_ptr();
  if (acc_add.has_value()) {
    check_cuda_bf16(*acc_add, "acc_add");
    AF3_CHECK(acc_add->dim() == 2 && acc_add->stride(1) == 1 && acc_add->size(0) >= M &&
                  acc_add->size(1) >= N && acc_add->stride(0) % 8 == 0,
              "acc_add must be bf16 [M, N] with unit inner stride and 16-byte rows");
    args.acc_add = reinterpret_cast<const __nv_bfloat16*>(acc_add->data_ptr());
    args.ld_acc_add = acc_add->stride(0);
  }

  if (sched != kSchedPlain) {
    AF3_CHECK(group_offsets.has_value(), "grouped GEMM needs group_offsets");
    AF3_CHECK(num_groups >= 1 && num_groups <= kMaxGroups, "num_groups out of range");
  }
  int ctas = max_ctas > 0 ? (int)max_ctas : num_sms();
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const GemmKey key{(int)bn, a_mn, b_mn, o.b_3d, (int)sched, (int)epi, dual};
  bool ok = false;
  if (sched == kSchedPlain) {
    ok = b_mn ? gemm_dispatch_dense_bwd(key, o, args, ctas, stream)
              : gemm_dispatch_dense_fwd(key, o, args, ctas, stream);
  } else {
    ok = (b_mn || sched == kSchedGroupedK) ? gemm_dispatch_grouped_bwd(key, o, args, ctas, stream)
                                           : gemm_dispatch_grouped_fwd(key, o, args, ctas, stream);
  }
  AF3_CHECK(ok, "no GEMM variant for bn=" + std::to_string(bn) + " a_mn=" +
                    std::to_string(a_mn) + " b_mn=" + std::to_string(b_mn) + " b_3d=" +
                    std::to_string(o.b_3d) + " sched=" + std::to_string(sched) +
                    " epi=" + std::to_string(epi) + " dual=" + std::to_string(dual));
}

}  // namespace af3
