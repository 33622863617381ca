// Python module `fw_radix_cuda`: drop-in for the reference's pybind11 module
// of the same name (src/cuda/binding.cpp:1-13), built on the C ABI of
// libfwloss_b200.so (include/fwloss_b200.h).
//
// The four reference functions keep their names, arguments, output tuples,
// dtypes (H/losses/mean fp32, kappa int32, selected bool, candidates
// fp32/int32) and the hard-coded "mean" scaling of the gradient (1/N).
// Differences, all in the direction of stricter checking:
//   * launches go to the current torch stream of the logits' device (under a
//     device guard) instead of the legacy default stream;
//   * targets are checked (1-D int64, N entries, same device); logits may be
//     non-contiguous along rows (row stride is passed through);
//   * `mean` is a fixed-order fp64 reduction (deterministic);
//   * candidate_buffer/indices rows hold exactly the support (kappa entries),
//     so fw_backward needs no zero-initialised [N,K] buffer.
// Extra functions used by the autograd layer (fwloss_b200 package):
//   fused_fwd_bwd, forward_rows, scale_grad, loss_reduce, loss_allreduce and its exchange
//   buffers (peer_buffer_*), shard_scan, shard_solve, and the
//   LM-head pieces shard_scan_into, label_logits, lmhead_fused_scan, chunks_solve,
//   sparse_grad_hidden, sparse_grad_weight.
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "../../include/fwloss_b200.h"

namespace {

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == FWB_OK, what, " failed: ", fw_error_string(rc));
}

void check_logits(const torch::Tensor& logits, bool any_float = false) {
  TORCH_CHECK(logits.is_cuda(), "logits must be a CUDA tensor");
  TORCH_CHECK(logits.dim() == 2, "logits must have shape [N, K]");
  if (any_float) {
    TORCH_CHECK(logits.scalar_type() == torch::kFloat32 || logits.scalar_type() == torch::kBFloat16 ||
                    logits.scalar_type() == torch::kHalf || logits.scalar_type() == torch::kFloat64,
                "logits must be float32, bfloat16, float16 or float64");
  } else {
    TORCH_CHECK(logits.scalar_type() == torch::kFloat32, "logits must be float32");
  }
  TORCH_CHECK(logits.size(1) >= 1, "logits must have K >= 1 columns");
}

int dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kBFloat16: return FWB_DTYPE_BF16;
    case torch::kHalf: return FWB_DTYPE_F16;
    default: return FWB_DTYPE_F32;
  }
}

void check_targets(const torch::Tensor& targets, int64_t N, const torch::Tensor& like) {
  TORCH_CHECK(targets.is_cuda() && targets.device() == like.device(),
              "targets must be a CUDA tensor on the logits' device");
  TORCH_CHECK(targets.dim() == 1 && targets.size(0) == N, "targets must have shape [N]");
  TORCH_CHECK(targets.scalar_type() == torch::kLong, "targets must be int64");
}

// Row-major view with unit column stride; returns the row stride.
torch::Tensor rows_view(const torch::Tensor& logits, int64_t* ld) {
  torch::Tensor z = logits;
  if (z.stride(1) != 1 || z.stride(0) < z.size(1)) z = z.contiguous();
  *ld = z.size(0) > 1 ? z.stride(0) : z.size(1);
  if (*ld < z.size(1)) *ld = z.size(1);
  return z;
}

void* cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

torch::Tensor mean_of(const torch::Tensor& losses) {
  auto out = torch::empty({}, losses.options());
  const int64_t n = losses.size(0);
  check_rc(fw_loss_reduce(losses.data_ptr<float>(), n, n > 0 ? 1.0 / (double)n : NAN,
                          out.data_ptr<float>(), cur_stream()),
           "fw_loss_reduce");
  return out;
}

torch::TensorOptions i32(const torch::Tensor& like) {
  return torch::TensorOptions().dtype(torch::kInt32).device(like.device());
}

}  // namespace

// reference: fw_radix_forward_small (src/cuda/fw_radix_argmax.cu:1381-1414)
std::vector<torch::Tensor> fw_forward_small(torch::Tensor logits, torch::Tensor targets) {
  check_logits(logits);
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), K = logits.size(1);
  check_targets(targets, N, logits);
  int64_t ld = K;
  auto z = rows_view(logits, &ld);
  auto y = targets.contiguous();
  auto selected = torch::empty({N, K}, logits.options().dtype(torch::kBool));
  auto H = torch::empty({N}, logits.options());
  auto losses = torch::empty({N}, logits.options());
  auto kappa = torch::empty({N}, i32(logits));
  check_rc(fw_forward_mask(z.data_ptr<float>(), y.data_ptr<int64_t>(), N, K, ld,
                           H.data_ptr<float>(), losses.data_ptr<float>(), kappa.data_ptr<int32_t>(),
                           reinterpret_cast<uint8_t*>(selected.data_ptr<bool>()), nullptr,
                           cur_stream()),
           "fw_forward_mask");
  return {H, losses, mean_of(losses), kappa, selected};
}

// reference: fw_radix_backward_small (src/cuda/fw_radix_argmax.cu:1591-1608)
torch::Tensor fw_backward_small(torch::Tensor targets, torch::Tensor selected_logits,
                                torch::Tensor kappas) {
  TORCH_CHECK(selected_logits.is_cuda() && selected_logits.dim() == 2 &&
                  selected_logits.scalar_type() == torch::kBool,
              "selected_logits must be a 2-D CUDA bool tensor");
  const c10::cuda::CUDAGuard guard(selected_logits.device());
  const int64_t N = selected_logits.size(0), K = selected_logits.size(1);
  check_targets(targets, N, selected_logits);
  TORCH_CHECK(kappas.is_cuda() && kappas.numel() == N && kappas.scalar_type() == torch::kInt32,
              "kappas must be an int32 CUDA tensor with N entries");
  auto sel = selected_logits.contiguous();
  auto y = targets.contiguous();
  auto kap = kappas.contiguous();
  auto grad = torch::empty({N, K}, selected_logits.options().dtype(torch::kFloat32));
  check_rc(fw_backward_mask(y.data_ptr<int64_t>(), reinterpret_cast<const uint8_t*>(sel.data_ptr<bool>()),
                            kap.data_ptr<int32_t>(), N, K, N > 0 ? 1.0f / (float)N : 0.0f,
                            grad.data_ptr<float>(), nullptr, cur_stream()),
           "fw_backward_mask");
  return grad;
}

// reference: fw_radix_forward (src/cuda/fw_radix_argmax.cu:1417-1496)
std::vector<torch::Tensor> fw_forward(torch::Tensor logits, torch::Tensor targets) {
  check_logits(logits);
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), K = logits.size(1);
  check_targets(targets, N, logits);
  int64_t ld = K;
  auto z = rows_view(logits, &ld);
  auto y = targets.contiguous();
  auto cand_val = torch::empty({N, K}, logits.options());
  auto cand_idx = torch::empty({N, K}, i32(logits));
  auto cand_cnt = torch::empty({N}, i32(logits));
  auto H = torch::empty({N}, logits.options());
  auto losses = torch::empty({N}, logits.options());
  auto kappa = torch::empty({N}, i32(logits));
  check_rc(fw_forward_candidates(z.data_ptr<float>(), y.data_ptr<int64_t>(), N, K, ld,
                                 H.data_ptr<float>(), losses.data_ptr<float>(),
                                 kappa.data_ptr<int32_t>(), cand_val.data_ptr<float>(),
                                 cand_idx.data_ptr<int32_t>(), cand_cnt.data_ptr<int32_t>(), nullptr,
                                 cur_stream()),
           "fw_forward_candidates");
  return {H, losses, mean_of(losses), kappa, cand_val, cand_idx, cand_cnt};
}

// reference: fw_radix_backward (src/cuda/fw_radix_argmax.cu:1536-1559)
torch::Tensor fw_backward(torch::Tensor logits, torch::Tensor targets, torch::Tensor H,
                          torch::Tensor kappas, torch::Tensor candidate_buffer,
                          torch::Tensor candidate_indices, torch::Tensor candidate_counts) {
  check_logits(logits);
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), K = logits.size(1);
  check_targets(targets, N, logits);
  TORCH_CHECK(H.is_cuda() && H.numel() == N && H.scalar_type() == torch::kFloat32, "H must be float32 [N]");
  TORCH_CHECK(kappas.is_cuda() && kappas.numel() == N && kappas.scalar_type() == torch::kInt32,
              "kappas must be int32 [N]");
  TORCH_CHECK(candidate_buffer.is_cuda() && candidate_buffer.numel() == N * K &&
                  candidate_buffer.scalar_type() == torch::kFloat32,
              "candidate_buffer must be float32 [N, K]");
  TORCH_CHECK(candidate_indices.is_cuda() && candidate_indices.numel() == N * K &&
                  candidate_indices.scalar_type() == torch::kInt32,
              "candidate_indices must be int32 [N, K]");
  TORCH_CHECK(candidate_counts.is_cuda() && candidate_counts.numel() == N &&
                  candidate_counts.scalar_type() == torch::kInt32,
              "candidate_counts must be int32 [N]");
  auto y = targets.contiguous();
  auto cv = candidate_buffer.contiguous();
  auto ci = candidate_indices.contiguous();
  auto cc = candidate_counts.contiguous();
  auto h = H.contiguous();
  auto kap = kappas.contiguous();
  auto grad = torch::empty({N, K}, logits.options());
  check_rc(fw_backward_candidates(cv.data_ptr<float>(), ci.data_ptr<int32_t>(), cc.data_ptr<int32_t>(),
                                  h.data_ptr<float>(), kap.data_ptr<int32_t>(), y.data_ptr<int64_t>(),
                                  N, K, N > 0 ? 1.0f / (float)N : 0.0f, grad.data_ptr<float>(),
                                  nullptr, cur_stream()),
           "fw_backward_candidates");
  return grad;
}

// Fused forward + backward (new): (grad, H, losses, kappa), grad scaled by
// grad_scale and of the logits' dtype (float32, bfloat16, float16 or
// float64); H and losses float32 (float64 for float64 logits); `status` is an
// optional int32 [1] device word.
std::vector<torch::Tensor> fused_fwd_bwd(torch::Tensor logits, torch::Tensor targets,
                                         double grad_scale, c10::optional<torch::Tensor> status) {
  check_logits(logits, true);
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), K = logits.size(1);
  check_targets(targets, N, logits);
  int64_t ld = K;
  auto z = rows_view(logits, &ld);
  auto y = targets.contiguous();
  auto grad = (ld == K) ? torch::empty({N, K}, logits.options())
                        : torch::empty_strided({N, K}, {ld, 1}, logits.options());
  const bool f64 = z.scalar_type() == torch::kFloat64;
  const auto out_t = f64 ? torch::kFloat64 : torch::kFloat32;
  auto H = torch::empty({N}, logits.options().dtype(out_t));
  auto losses = torch::empty({N}, logits.options().dtype(out_t));
  auto kappa = torch::empty({N}, i32(logits));
  int32_t* st = nullptr;
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->scalar_type() == torch::kInt32 && status->numel() >= 1,
                "status must be an int32 CUDA tensor");
    st = status->data_ptr<int32_t>();
  }
  if (f64) {
    check_rc(fw_fused_fwd_bwd_f64(z.data_ptr<double>(), y.data_ptr<int64_t>(), N, K, ld, grad_scale,
                                  grad.data_ptr<double>(), H.data_ptr<double>(), losses.data_ptr<double>(),
                                  kappa.data_ptr<int32_t>(), st, cur_stream()),
             "fw_fused_fwd_bwd_f64");
    return {grad, H, losses, kappa};
  }
  check_rc(fw_fused_fwd_bwd_typed(dtype_code(z), z.data_ptr(), y.data_ptr<int64_t>(), N, K, ld,
                                  (float)grad_scale, grad.data_ptr(), H.data_ptr<float>(),
                                  losses.data_ptr<float>(), kappa.data_ptr<int32_t>(), st, cur_stream()),
           "fw_fused_fwd_bwd");
  return {grad, H, losses, kappa};
}

// Forward only (new): (H, losses, kappa) without a gradient -- the logits are
// read once and nothing of their size is written.  H and losses float32
// (float64 for float64 logits).
std::vector<torch::Tensor> forward_rows(torch::Tensor logits, torch::Tensor targets,
                                        c10::optional<torch::Tensor> status) {
  check_logits(logits, true);
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), K = logits.size(1);
  check_targets(targets, N, logits);
  int64_t ld = K;
  auto z = rows_view(logits, &ld);
  auto y = targets.contiguous();
  const bool f64 = z.scalar_type() == torch::kFloat64;
  const auto out_t = f64 ? torch::kFloat64 : torch::kFloat32;
  auto H = torch::empty({N}, logits.options().dtype(out_t));
  auto losses = torch::empty({N}, logits.options().dtype(out_t));
  auto kappa = torch::empty({N}, i32(logits));
  int32_t* st = nullptr;
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->scalar_type() == torch::kInt32 && status->numel() >= 1,
                "status must be an int32 CUDA tensor");
    st = status->data_ptr<int32_t>();
  }
  if (f64) {
    check_rc(fw_forward_rows_f64(z.data_ptr<double>(), y.data_ptr<int64_t>(), N, K, ld, H.data_ptr<double>(),
                                 losses.data_ptr<double>(), kappa.data_ptr<int32_t>(), st, cur_stream()),
             "fw_forward_rows_f64");
    return {H, losses, kappa};
  }
  check_rc(fw_forward_rows(dtype_code(z), z.data_ptr(), y.data_ptr<int64_t>(), N, K, ld, H.data_ptr<float>(),
                           losses.data_ptr<float>(), kappa.data_ptr<int32_t>(), st, cur_stream()),
           "fw_forward_rows");
  return {H, losses, kappa};
}

// grad (in place) *= grad_output[per_row ? r : 0] / assumed_scale.
void scale_grad(torch::Tensor grad, torch::Tensor grad_output, bool per_row, double assumed_scale) {
  TORCH_CHECK(grad.is_cuda() && grad.dim() == 2 && grad.stride(1) == 1 &&
                  (grad.scalar_type() == torch::kFloat32 || grad.scalar_type() == torch::kBFloat16 ||
                   grad.scalar_type() == torch::kHalf || grad.scalar_type() == torch::kFloat64),
              "grad must be a row-major float32/bfloat16/float16/float64 CUDA matrix");
  const c10::cuda::CUDAGuard guard(grad.device());
  const int64_t ld = grad.size(0) > 1 ? grad.stride(0) : grad.size(1);
  if (grad.scalar_type() == torch::kFloat64) {
    auto go = grad_output.to(grad.device(), torch::kFloat64).contiguous();
    TORCH_CHECK(go.numel() >= (per_row ? grad.size(0) : 1), "grad_output too small");
    check_rc(fw_scale_grad_f64(grad.data_ptr<double>(), go.data_ptr<double>(), per_row ? 1 : 0,
                               assumed_scale, grad.size(0), grad.size(1), ld, cur_stream()),
             "fw_scale_grad_f64");
    return;
  }
  auto go = grad_output.to(grad.device(), torch::kFloat32).contiguous();
  TORCH_CHECK(go.numel() >= (per_row ? grad.size(0) : 1), "grad_output too small");
  check_rc(fw_scale_grad_typed(dtype_code(grad), grad.data_ptr(), go.data_ptr<float>(), per_row ? 1 : 0,
                               (float)assumed_scale, grad.size(0), grad.size(1), ld, cur_stream()),
           "fw_scale_grad");
}

// fused_fwd_bwd (float32/bfloat16/float16 logits) that also lists every row's
// support columns: (grad, H, losses, kappa, sup_cols [N, sup_k] int32).
std::vector<torch::Tensor> fused_fwd_bwd_cols(torch::Tensor logits, torch::Tensor targets, double grad_scale,
                                              int64_t sup_k, c10::optional<torch::Tensor> status) {
  check_logits(logits, true);
  TORCH_CHECK(logits.scalar_type() != torch::kFloat64, "fused_fwd_bwd_cols takes 32- and 16-bit logits");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t N = logits.size(0), K = logits.size(1);
  check_targets(targets, N, logits);
  int64_t ld = K;
  auto z = rows_view(logits, &ld);
  auto y = targets.contiguous();
  auto grad = (ld == K) ? torch::empty({N, K}, logits.options())
                        : torch::empty_strided({N, K}, {ld, 1}, logits.options());
  auto H = torch::empty({N}, logits.options().dtype(torch::kFloat32));
  auto losses = torch::empty({N}, logits.options().dtype(torch::kFloat32));
  auto kappa = torch::empty({N}, i32(logits));
  auto cols = torch::empty({N, sup_k}, i32(logits));
  int32_t* st = nullptr;
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->scalar_type() == torch::kInt32 && status->numel() >= 1,
                "status must be an int32 CUDA tensor");
    st = status->data_ptr<int32_t>();
  }
  check_rc(fw_fused_fwd_bwd_cols(dtype_code(z), z.data_ptr(), y.data_ptr<int64_t>(), N, K, ld, (float)grad_scale,
                                 grad.data_ptr(), H.data_ptr<float>(), losses.data_ptr<float>(),
                                 kappa.data_ptr<int32_t>(), cols.data_ptr<int32_t>(), (int)sup_k, st, cur_stream()),
           "fw_fused_fwd_bwd_cols");
  return {grad, H, losses, kappa, cols};
}

// scale_grad for a gradient from fused_fwd_bwd_cols: rows with a listed
// support rewrite kappa + 1 entries only.
void scale_grad_cols(torch::Tensor grad, torch::Tensor sup_cols, torch::Tensor kappa, torch::Tensor targets,
                     torch::Tensor grad_output, bool per_row, double assumed_scale) {
  TORCH_CHECK(grad.is_cuda() && grad.dim() == 2 && grad.stride(1) == 1 &&
                  (grad.scalar_type() == torch::kFloat32 || grad.scalar_type() == torch::kBFloat16 ||
                   grad.scalar_type() == torch::kHalf),
              "grad must be a row-major float32/bfloat16/float16 CUDA matrix");
  TORCH_CHECK(sup_cols.scalar_type() == torch::kInt32 && sup_cols.is_contiguous() && sup_cols.dim() == 2 &&
                  sup_cols.size(0) == grad.size(0),
              "sup_cols must be contiguous int32 [N, sup_k]");
  const c10::cuda::CUDAGuard guard(grad.device());
  const int64_t ld = grad.size(0) > 1 ? grad.stride(0) : grad.size(1);
  auto go = grad_output.to(grad.device(), torch::kFloat32).contiguous();
  TORCH_CHECK(go.numel() >= (per_row ? grad.size(0) : 1), "grad_output too small");
  auto y = targets.contiguous();
  check_rc(fw_scale_grad_cols(dtype_code(grad), grad.data_ptr(), ld, sup_cols.data_ptr<int32_t>(),
                              (int)sup_cols.size(1), kappa.data_ptr<int32_t>(), y.data_ptr<int64_t>(),
                              go.data_ptr<float>(), per_row ? 1 : 0, (float)assumed_scale, grad.size(0),
                              grad.size(1), cur_stream()),
           "fw_scale_grad_cols");
}

// scale * sum(losses), fixed-order fp64 reduction; 0-d, of the losses' dtype
// (float32 or float64).
torch::Tensor loss_reduce(torch::Tensor losses, double scale) {
  TORCH_CHECK(losses.is_cuda() && losses.dim() == 1 &&
                  (losses.scalar_type() == torch::kFloat32 || losses.scalar_type() == torch::kFloat64),
              "losses must be a float32 or float64 CUDA vector");
  const c10::cuda::CUDAGuard guard(losses.device());
  auto l = losses.contiguous();
  auto out = torch::empty({}, l.options());
  if (l.scalar_type() == torch::kFloat64) {
    check_rc(fw_loss_reduce_f64(l.data_ptr<double>(), l.size(0), scale, out.data_ptr<double>(), cur_stream()),
             "fw_loss_reduce_f64");
    return out;
  }
  check_rc(fw_loss_reduce(l.data_ptr<float>(), l.size(0), scale, out.data_ptr<float>(), cur_stream()),
           "fw_loss_reduce");
  return out;
}

// Cross-GPU loss sum over peer memory (one process per GPU): 0-d
// scale * (sum of every rank's losses), the same value on every rank.  bufs:
// the world exchange buffers in rank order as mapped in this process (this
// rank's own at index `rank`), from peer_buffer_create / peer_buffer_open.
torch::Tensor loss_allreduce(torch::Tensor losses, double scale, std::vector<int64_t> bufs, int64_t rank,
                             c10::optional<torch::Tensor> status, double timeout_s) {
  TORCH_CHECK(losses.is_cuda() && losses.dim() == 1 &&
                  (losses.scalar_type() == torch::kFloat32 || losses.scalar_type() == torch::kFloat64),
              "losses must be a float32 or float64 CUDA vector");
  const c10::cuda::CUDAGuard guard(losses.device());
  auto l = losses.contiguous();
  auto out = torch::empty({}, l.options());
  std::vector<void*> ptrs;
  for (int64_t b : bufs) ptrs.push_back(reinterpret_cast<void*>(b));
  int32_t* st = nullptr;
  if (status.has_value()) {
    TORCH_CHECK(status->is_cuda() && status->scalar_type() == torch::kInt32 && status->numel() >= 1,
                "status must be an int32 CUDA tensor");
    st = status->data_ptr<int32_t>();
  }
  if (l.scalar_type() == torch::kFloat64) {
    check_rc(fw_loss_allreduce_f64(l.data_ptr<double>(), l.size(0), scale, ptrs.data(), (int)ptrs.size(), (int)rank,
                                   out.data_ptr<double>(), st, timeout_s, cur_stream()),
             "fw_loss_allreduce_f64");
    return out;
  }
  check_rc(fw_loss_allreduce(l.data_ptr<float>(), l.size(0), scale, ptrs.data(), (int)ptrs.size(), (int)rank,
                             out.data_ptr<float>(), st, timeout_s, cur_stream()),
           "fw_loss_allreduce");
  return out;
}

// Exchange-buffer set-up (host calls, once per rank): create on the current
// device -> (address, IPC handle bytes); open a peer's handle -> address.
py::tuple peer_buffer_create() {
  void* buf = nullptr;
  char handle[FWB_PEER_HANDLE_BYTES];
  check_rc(fw_peer_buffer_create(&buf, handle), "fw_peer_buffer_create");
  return py::make_tuple(reinterpret_cast<int64_t>(buf), py::bytes(handle, FWB_PEER_HANDLE_BYTES));
}

int64_t peer_buffer_open(py::bytes handle) {
  const std::string h = handle;
  TORCH_CHECK(h.size() == FWB_PEER_HANDLE_BYTES, "an exchange-buffer handle has ", FWB_PEER_HANDLE_BYTES, " bytes");
  void* p = nullptr;
  check_rc(fw_peer_buffer_open(h.data(), &p), "fw_peer_buffer_open");
  return reinterpret_cast<int64_t>(p);
}

// Class-sharded step 1: (grad shard zero-filled, summary [B, 4+K], local_idx [B, K]).
std::vector<torch::Tensor> shard_scan(torch::Tensor z_local, int64_t K) {
  check_logits(z_local);
  const c10::cuda::CUDAGuard guard(z_local.device());
  const int64_t N = z_local.size(0), C = z_local.size(1);
  int64_t ld = C;
  auto z = rows_view(z_local, &ld);
  auto grad = (ld == C) ? torch::empty({N, C}, z.options()) : torch::empty_strided({N, C}, {ld, 1}, z.options());
  auto summary = torch::empty({N, 4 + K}, i32(z));
  auto local_idx = torch::empty({N, K}, i32(z));
  check_rc(fw_shard_scan(z.data_ptr<float>(), N, C, ld, (int)K, grad.data_ptr<float>(),
                         summary.data_ptr<int32_t>(), local_idx.data_ptr<int32_t>(), cur_stream()),
           "fw_shard_scan");
  return {grad, summary, local_idx};
}

// Class-sharded step 3: (H, kappa, loss_part, fb_rows, fb_count); patches grad in place.
std::vector<torch::Tensor> shard_solve(torch::Tensor gathered, int64_t rank, std::vector<int64_t> col_start,
                                       torch::Tensor z_local, torch::Tensor targets, double grad_scale,
                                       torch::Tensor grad, torch::Tensor local_idx,
                                       c10::optional<torch::Tensor> status) {
  check_logits(z_local);
  const c10::cuda::CUDAGuard guard(z_local.device());
  const int64_t N = z_local.size(0);
  check_targets(targets, N, z_local);
  const int64_t nranks = (int64_t)col_start.size() - 1;
  TORCH_CHECK(gathered.is_cuda() && gathered.scalar_type() == torch::kInt32 && gathered.dim() == 3 &&
                  gathered.size(0) == nranks && gathered.size(1) == N,
              "gathered must be int32 [nranks, B, 4 + K]");
  const int64_t K = gathered.size(2) - 4;
  TORCH_CHECK(local_idx.is_cuda() && local_idx.scalar_type() == torch::kInt32 && local_idx.numel() == N * K,
              "local_idx must be int32 [B, K]");
  TORCH_CHECK(grad.is_cuda() && grad.scalar_type() == torch::kFloat32 && grad.stride(1) == 1 &&
                  grad.size(0) == N && grad.size(1) == z_local.size(1),
              "grad must be the float32 gradient shard");
  int64_t ld = z_local.size(1);
  auto z = rows_view(z_local, &ld);
  const int64_t gld = N > 1 ? grad.stride(0) : grad.size(1);
  TORCH_CHECK(gld == ld, "grad and logits shards must share the row stride");
  auto g = gathered.contiguous();
  auto li = local_idx.contiguous();
  auto y = targets.contiguous();
  auto H = torch::empty({N}, z.options());
  auto kappa = torch::empty({N}, i32(z));
  auto loss_part = torch::empty({N}, z.options());
  auto fb_rows = torch::empty({N > 0 ? N : 1}, i32(z));
  auto fb_count = torch::empty({1}, i32(z));
  int32_t* st = nullptr;
  if (status.has_value()) st = status->data_ptr<int32_t>();
  check_rc(fw_shard_solve(g.data_ptr<int32_t>(), (int)nranks, (int)rank, col_start.data(), N, (int)K,
                          z.data_ptr<float>(), ld, y.data_ptr<int64_t>(), (float)grad_scale,
                          grad.data_ptr<float>(), li.data_ptr<int32_t>(), H.data_ptr<float>(),
                          kappa.data_ptr<int32_t>(), loss_part.data_ptr<float>(), fb_rows.data_ptr<int32_t>(),
                          fb_count.data_ptr<int32_t>(), st, cur_stream()),
           "fw_shard_solve");
  return {H, kappa, loss_part, fb_rows, fb_count};
}

// Summaries of one logit chunk written into given buffers (no gradient shard).
void shard_scan_into(torch::Tensor z_chunk, int64_t K, torch::Tensor summary, torch::Tensor local_idx) {
  check_logits(z_chunk);
  const c10::cuda::CUDAGuard guard(z_chunk.device());
  const int64_t N = z_chunk.size(0), C = z_chunk.size(1);
  int64_t ld = C;
  auto z = rows_view(z_chunk, &ld);
  TORCH_CHECK(summary.is_contiguous() && summary.scalar_type() == torch::kInt32 && summary.numel() == N * (4 + K),
              "summary must be contiguous int32 [B, 4 + K]");
  TORCH_CHECK(local_idx.is_contiguous() && local_idx.scalar_type() == torch::kInt32 && local_idx.numel() == N * K,
              "local_idx must be contiguous int32 [B, K]");
  check_rc(fw_shard_scan(z.data_ptr<float>(), N, C, ld, (int)K, nullptr, summary.data_ptr<int32_t>(),
                         local_idx.data_ptr<int32_t>(), cur_stream()),
           "fw_shard_scan");
}

void label_logits(torch::Tensor z_chunk, torch::Tensor targets, int64_t c0, torch::Tensor zy) {
  check_logits(z_chunk);
  const c10::cuda::CUDAGuard guard(z_chunk.device());
  const int64_t N = z_chunk.size(0), C = z_chunk.size(1);
  check_targets(targets, N, z_chunk);
  TORCH_CHECK(zy.is_cuda() && zy.scalar_type() == torch::kFloat32 && zy.numel() == N && zy.is_contiguous(),
              "zy must be a contiguous float32 [B] tensor");
  int64_t ld = C;
  auto z = rows_view(z_chunk, &ld);
  auto y = targets.contiguous();
  check_rc(fw_label_logits(z.data_ptr<float>(), N, C, ld, y.data_ptr<int64_t>(), c0, zy.data_ptr<float>(),
                           cur_stream()),
           "fw_label_logits");
}

// LM head, fused form: the chunk summaries and label logits of
// logits = hidden @ weight^T straight from the tensor-core GEMM (bf16 inputs),
// into the given buffers; no logits are formed.
void lmhead_fused_scan(torch::Tensor hidden, torch::Tensor weight, torch::Tensor targets,
                       std::vector<int64_t> col_start, torch::Tensor summaries, torch::Tensor local_idx,
                       torch::Tensor zy, c10::optional<torch::Tensor> status) {
  TORCH_CHECK(hidden.is_cuda() && weight.is_cuda() && hidden.device() == weight.device(),
              "hidden and weight must be CUDA tensors on one device");
  TORCH_CHECK(hidden.scalar_type() == torch::kBFloat16 && weight.scalar_type() == torch::kBFloat16,
              "the fused LM-head scan takes bfloat16 hidden and weight");
  TORCH_CHECK(hidden.dim() == 2 && weight.dim() == 2 && hidden.size(1) == weight.size(1) &&
                  hidden.is_contiguous() && weight.is_contiguous(),
              "hidden [B, D] and weight [C, D] must be contiguous");
  const c10::cuda::CUDAGuard guard(hidden.device());
  const int64_t B = hidden.size(0), D = hidden.size(1), C = weight.size(0);
  const int64_t n = (int64_t)col_start.size() - 1;
  TORCH_CHECK(summaries.is_contiguous() && summaries.scalar_type() == torch::kInt32 && summaries.dim() == 3 &&
                  summaries.size(0) == n && summaries.size(1) == B,
              "summaries must be contiguous int32 [nchunks, B, 4 + K]");
  const int64_t K = summaries.size(2) - 4;
  TORCH_CHECK(local_idx.is_contiguous() && local_idx.scalar_type() == torch::kInt32 && local_idx.numel() == n * B * K,
              "local_idx must be contiguous int32 [nchunks, B, K]");
  TORCH_CHECK(zy.is_cuda() && zy.scalar_type() == torch::kFloat32 && zy.numel() == B && zy.is_contiguous(),
              "zy must be a contiguous float32 [B] tensor");
  check_targets(targets, B, hidden);
  auto y = targets.contiguous();
  int32_t* st = nullptr;
  if (status.has_value()) st = status->data_ptr<int32_t>();
  check_rc(fw_lmhead_fused_scan(FWB_DTYPE_BF16, hidden.data_ptr(), B, D, weight.data_ptr(), C, (int)n,
                                col_start.data(), (int)K, y.data_ptr<int64_t>(), zy.data_ptr<float>(),
                                summaries.data_ptr<int32_t>(), local_idx.data_ptr<int32_t>(), st, cur_stream()),
           "fw_lmhead_fused_scan");
}

// (H, kappa, loss, sup_cols, fb_rows, fb_count) from the chunk summaries.
std::vector<torch::Tensor> chunks_solve(torch::Tensor summaries, torch::Tensor local_idx,
                                        std::vector<int64_t> col_start, torch::Tensor zy, torch::Tensor targets,
                                        c10::optional<torch::Tensor> status) {
  TORCH_CHECK(summaries.is_cuda() && summaries.scalar_type() == torch::kInt32 && summaries.dim() == 3 &&
                  summaries.is_contiguous(),
              "summaries must be contiguous int32 [nchunks, B, 4 + K]");
  const c10::cuda::CUDAGuard guard(summaries.device());
  const int64_t n = summaries.size(0), B = summaries.size(1), K = summaries.size(2) - 4;
  TORCH_CHECK((int64_t)col_start.size() == n + 1, "col_start must have nchunks + 1 entries");
  TORCH_CHECK(local_idx.is_contiguous() && local_idx.numel() == n * B * K, "local_idx must be [nchunks, B, K]");
  check_targets(targets, B, summaries);
  auto y = targets.contiguous();
  auto opt = summaries.options();
  auto H = torch::empty({B}, opt.dtype(torch::kFloat32));
  auto kappa = torch::empty({B}, opt);
  auto loss = torch::empty({B}, opt.dtype(torch::kFloat32));
  auto sup = torch::empty({B, n * K}, opt);
  auto fb_rows = torch::empty({B > 0 ? B : 1}, opt);
  auto fb_count = torch::empty({1}, opt);
  int32_t* st = nullptr;
  if (status.has_value()) st = status->data_ptr<int32_t>();
  check_rc(fw_chunks_solve(summaries.data_ptr<int32_t>(), local_idx.data_ptr<int32_t>(), (int)n, col_start.data(), B,
                           (int)K, zy.data_ptr<float>(), y.data_ptr<int64_t>(), H.data_ptr<float>(),
                           kappa.data_ptr<int32_t>(), loss.data_ptr<float>(), sup.data_ptr<int32_t>(),
                           fb_rows.data_ptr<int32_t>(), fb_count.data_ptr<int32_t>(), st, cur_stream()),
           "fw_chunks_solve");
  return {H, kappa, loss, sup, fb_rows, fb_count};
}

int lm_dtype(const torch::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == torch::kFloat32 || t.scalar_type() == torch::kBFloat16,
              "LM-head tensors must be float32 or bfloat16");
  return t.scalar_type() == torch::kBFloat16 ? FWB_DTYPE_BF16 : FWB_DTYPE_F32;
}

torch::Tensor sparse_grad_hidden(torch::Tensor weight, torch::Tensor sup_cols, torch::Tensor kappa,
                                 torch::Tensor targets, double scale, torch::Tensor grad_output, bool per_row) {
  TORCH_CHECK(weight.is_cuda() && weight.dim() == 2 && weight.is_contiguous(), "weight must be contiguous [C, D]");
  const c10::cuda::CUDAGuard guard(weight.device());
  const int64_t B = kappa.numel();
  auto dH = torch::empty({B, weight.size(1)}, weight.options());
  auto go = grad_output.to(weight.device(), torch::kFloat32).contiguous();
  check_rc(fw_sparse_grad_hidden(lm_dtype(weight), weight.data_ptr(), weight.size(0), weight.size(1),
                                 sup_cols.data_ptr<int32_t>(), (int)sup_cols.size(1), kappa.data_ptr<int32_t>(),
                                 targets.data_ptr<int64_t>(), B, (float)scale, go.data_ptr<float>(), per_row ? 1 : 0,
                                 dH.data_ptr(), cur_stream()),
           "fw_sparse_grad_hidden");
  return dH;
}

void sparse_grad_weight(torch::Tensor hidden, torch::Tensor sup_cols, torch::Tensor kappa, torch::Tensor targets,
                        double scale, torch::Tensor grad_output, bool per_row, torch::Tensor dweight) {
  TORCH_CHECK(hidden.is_cuda() && hidden.dim() == 2 && hidden.is_contiguous(), "hidden must be contiguous [B, D]");
  TORCH_CHECK(dweight.scalar_type() == torch::kFloat32 && dweight.is_contiguous() && dweight.size(1) == hidden.size(1),
              "dweight must be a contiguous float32 [C, D] accumulator");
  const c10::cuda::CUDAGuard guard(hidden.device());
  auto go = grad_output.to(hidden.device(), torch::kFloat32).contiguous();
  check_rc(fw_sparse_grad_weight(lm_dtype(hidden), hidden.data_ptr(), hidden.size(0), hidden.size(1),
                                 sup_cols.data_ptr<int32_t>(), (int)sup_cols.size(1), kappa.data_ptr<int32_t>(),
                                 targets.data_ptr<int64_t>(), dweight.size(0), (float)scale, go.data_ptr<float>(),
                                 per_row ? 1 : 0, dweight.data_ptr<float>(), cur_stream()),
           "fw_sparse_grad_weight");
}

torch::Tensor weight_grad_keys(torch::Tensor sup_cols, torch::Tensor kappa, torch::Tensor targets, int64_t C) {
  TORCH_CHECK(sup_cols.is_cuda() && sup_cols.scalar_type() == torch::kInt32 && sup_cols.dim() == 2 &&
                  sup_cols.is_contiguous(),
              "sup_cols must be contiguous int32 [B, S]");
  const c10::cuda::CUDAGuard guard(sup_cols.device());
  const int64_t B = sup_cols.size(0), S = sup_cols.size(1);
  auto keys = torch::empty({B * (S + 1)}, sup_cols.options().dtype(torch::kLong));
  check_rc(fw_weight_grad_keys(sup_cols.data_ptr<int32_t>(), (int)S, kappa.data_ptr<int32_t>(),
                               targets.data_ptr<int64_t>(), B, C, keys.data_ptr<int64_t>(), cur_stream()),
           "fw_weight_grad_keys");
  return keys;
}

// Vocabulary-parallel rank: fp32 partial dhidden [B, D] from the local weight
// shard (classes [c0, c0 + C_shard)).
torch::Tensor sparse_grad_hidden_shard(torch::Tensor weight_shard, int64_t c0, torch::Tensor sup_cols,
                                       torch::Tensor kappa, torch::Tensor targets, double scale,
                                       torch::Tensor grad_output, bool per_row) {
  TORCH_CHECK(weight_shard.is_cuda() && weight_shard.dim() == 2 && weight_shard.is_contiguous(),
              "weight_shard must be contiguous [C_shard, D]");
  TORCH_CHECK(sup_cols.scalar_type() == torch::kInt32 && sup_cols.is_contiguous() && sup_cols.dim() == 2,
              "sup_cols must be contiguous int32 [B, S]");
  const c10::cuda::CUDAGuard guard(weight_shard.device());
  const int64_t B = kappa.numel();
  auto dH = torch::empty({B, weight_shard.size(1)}, weight_shard.options().dtype(torch::kFloat32));
  auto go = grad_output.to(weight_shard.device(), torch::kFloat32).contiguous();
  check_rc(fw_sparse_grad_hidden_shard(lm_dtype(weight_shard), weight_shard.data_ptr(), c0, weight_shard.size(0),
                                       weight_shard.size(1), sup_cols.data_ptr<int32_t>(), (int)sup_cols.size(1),
                                       kappa.data_ptr<int32_t>(), targets.data_ptr<int64_t>(), B, (float)scale,
                                       go.data_ptr<float>(), per_row ? 1 : 0, dH.data_ptr<float>(), cur_stream()),
           "fw_sparse_grad_hidden_shard");
  return dH;
}

torch::Tensor weight_grad_keys_shard(torch::Tensor sup_cols, torch::Tensor kappa, torch::Tensor targets, int64_t c0,
                                     int64_t C_shard) {
  TORCH_CHECK(sup_cols.is_cuda() && sup_cols.scalar_type() == torch::kInt32 && sup_cols.dim() == 2 &&
                  sup_cols.is_contiguous(),
              "sup_cols must be contiguous int32 [B, S]");
  const c10::cuda::CUDAGuard guard(sup_cols.device());
  const int64_t B = sup_cols.size(0), S = sup_cols.size(1);
  auto keys = torch::empty({B * (S + 1)}, sup_cols.options().dtype(torch::kLong));
  check_rc(fw_weight_grad_keys_shard(sup_cols.data_ptr<int32_t>(), (int)S, kappa.data_ptr<int32_t>(),
                                     targets.data_ptr<int64_t>(), B, c0, C_shard, keys.data_ptr<int64_t>(),
                                     cur_stream()),
           "fw_weight_grad_keys_shard");
  return keys;
}

void segment_grad_weight(torch::Tensor hidden, torch::Tensor sorted_keys, torch::Tensor kappa, double scale,
                         torch::Tensor grad_output, bool per_row, torch::Tensor dweight) {
  TORCH_CHECK(hidden.is_cuda() && hidden.dim() == 2 && hidden.is_contiguous(), "hidden must be contiguous [B, D]");
  TORCH_CHECK(dweight.scalar_type() == hidden.scalar_type() && dweight.is_contiguous() &&
                  dweight.size(1) == hidden.size(1),
              "dweight must be contiguous [C, D] of hidden's dtype");
  TORCH_CHECK(sorted_keys.scalar_type() == torch::kLong && sorted_keys.is_contiguous(), "int64 sorted keys");
  const c10::cuda::CUDAGuard guard(hidden.device());
  auto go = grad_output.to(hidden.device(), torch::kFloat32).contiguous();
  check_rc(fw_segment_grad_weight(lm_dtype(hidden), hidden.data_ptr(), hidden.size(0), hidden.size(1),
                                  sorted_keys.data_ptr<int64_t>(), sorted_keys.numel(), kappa.data_ptr<int32_t>(),
                                  (float)scale, go.data_ptr<float>(), per_row ? 1 : 0, dweight.data_ptr(),
                                  cur_stream()),
           "fw_segment_grad_weight");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) Familywise loss: drop-in for the fw_radix_cuda module";
  m.def("fw_forward", &fw_forward, "FW forward (support as candidate lists)");
  m.def("fw_backward", &fw_backward, "FW backward from candidate lists (mean scaling)");
  m.def("fw_forward_small", &fw_forward_small, "FW forward (support as bool mask)");
  m.def("fw_backward_small", &fw_backward_small, "FW backward from the bool mask (mean scaling)");
  m.def("fused_fwd_bwd", &fused_fwd_bwd, "fused forward+backward: (grad, H, losses, kappa)",
        py::arg("logits"), py::arg("targets"), py::arg("grad_scale"), py::arg("status") = py::none());
  m.def("forward_rows", &forward_rows, "forward only, no gradient: (H, losses, kappa)", py::arg("logits"),
        py::arg("targets"), py::arg("status") = py::none());
  m.def("scale_grad", &scale_grad, "in-place grad scaling by a device-side grad_output");
  m.def("fused_fwd_bwd_cols", &fused_fwd_bwd_cols,
        "fused forward+backward listing the support columns: (grad, H, losses, kappa, sup_cols)",
        py::arg("logits"), py::arg("targets"), py::arg("grad_scale"), py::arg("sup_k"),
        py::arg("status") = py::none());
  m.def("scale_grad_cols", &scale_grad_cols, "in-place grad scaling touching only the listed support");
  m.def("loss_reduce", &loss_reduce, "deterministic scale * sum(losses)");
  m.def("loss_allreduce", &loss_allreduce, "scale * sum of every rank's losses, over peer memory",
        py::arg("losses"), py::arg("scale"), py::arg("bufs"), py::arg("rank"), py::arg("status") = py::none(),
        py::arg("timeout_s") = 10.0);
  m.def("peer_buffer_create", &peer_buffer_create, "this rank's exchange buffer: (address, IPC handle)");
  m.def("peer_buffer_open", &peer_buffer_open, "maps another rank's exchange buffer from its handle");
  m.def("peer_buffer_close", [](int64_t p) { check_rc(fw_peer_buffer_close(reinterpret_cast<void*>(p)), "fw_peer_buffer_close"); });
  m.def("peer_buffer_destroy", [](int64_t p) { check_rc(fw_peer_buffer_destroy(reinterpret_cast<void*>(p)), "fw_peer_buffer_destroy"); });
  m.def("shard_scan", &shard_scan, "class-sharded step 1: local solve, zero gradient shard, summaries");
  m.def("shard_scan_into", &shard_scan_into, "summaries of one logit chunk into given buffers");
  m.def("label_logits", &label_logits, "zy[r] = chunk[r, y[r] - c0] for labels inside the chunk");
  m.def("lmhead_fused_scan", &lmhead_fused_scan, "LM head: chunk summaries from the tensor-core GEMM",
        py::arg("hidden"), py::arg("weight"), py::arg("targets"), py::arg("col_start"), py::arg("summaries"),
        py::arg("local_idx"), py::arg("zy"), py::arg("status") = py::none());
  m.def("chunks_solve", &chunks_solve, "LM head: combine chunk summaries",
        py::arg("summaries"), py::arg("local_idx"), py::arg("col_start"), py::arg("zy"), py::arg("targets"),
        py::arg("status") = py::none());
  m.def("sparse_grad_hidden", &sparse_grad_hidden, "LM head backward: dhidden from the sparse logit gradient");
  m.def("sparse_grad_weight", &sparse_grad_weight, "LM head backward: dweight += (fp32 accumulator)");
  m.def("weight_grad_keys", &weight_grad_keys, "LM head backward: contribution keys [B * (S + 1)]");
  m.def("sparse_grad_hidden_shard", &sparse_grad_hidden_shard,
        "vocabulary-parallel LM head backward: this rank's fp32 part of dhidden");
  m.def("weight_grad_keys_shard", &weight_grad_keys_shard,
        "vocabulary-parallel LM head backward: contribution keys of the local classes");
  m.def("segment_grad_weight", &segment_grad_weight, "LM head backward: deterministic dweight rows from sorted keys");
  m.def("shard_solve", &shard_solve, "class-sharded step 3: global solve from gathered summaries",
        py::arg("gathered"), py::arg("rank"), py::arg("col_start"), py::arg("z_local"), py::arg("targets"),
        py::arg("grad_scale"), py::arg("grad"), py::arg("local_idx"), py::arg("status") = py::none());
  m.def("version", []() { return std::string(fw_version()); });
}
