// C ABI of libfwloss_b200.so: argument checks and launches.
// Declarations and semantics: include/fwloss_b200.h.  The fused row kernels
// (tier selection by class count) are launched through run_rows, whose
// instances live in the fw_rows_*.cu translation units (fw_rows.cuh).
#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <cstdint>

#include "../../include/fwloss_b200.h"
#include "fw_aux.cuh"
#include "fw_device.cuh"
#include "fw_f64.cuh"
#include "fw_lmhead.cuh"
#include "fw_lmhead_tc.cuh"
#include "fw_host.cuh"
#include "fw_shard.cuh"

namespace fwb200 {
namespace {

// The loss reduction: one CTA, or one cluster of kReduceCluster CTAs above
// kReduceClusterMinRows rows, launched as a programmatic dependent of the
// previous kernel on the stream.
template <class T>
cudaError_t launch_loss_reduce(const T* loss, int64_t B, double scale, T* out, cudaStream_t st) {
  const bool cl = B > kReduceClusterMinRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cl ? kReduceCluster : 1);
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kReduceCluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cl ? 2 : 1;
  const int vec = aligned16(loss) ? 1 : 0;
  return cl ? cudaLaunchKernelEx(&cfg, fw_loss_reduce_kernel<T, kReduceCluster>, loss, B, scale, out, vec)
            : cudaLaunchKernelEx(&cfg, fw_loss_reduce_kernel<T, 1>, loss, B, scale, out, vec);
}

int check_shape(int64_t B, int64_t C, int64_t ld) {
  if (B < 0 || C < 1 || ld < C) return FWB_E_SHAPE;
  if (C > (int64_t)INT_MAX - 64) return FWB_E_SHAPE;         // int32 column indices
  if (B > (int64_t)INT_MAX / 8) return FWB_E_SHAPE;          // grid of B * CS CTAs
  if (B > 0 && ld > ((int64_t)1 << 62) / B) return FWB_E_SHAPE;
  return FWB_OK;
}

RowArgs base_args(const void* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                  float* H, float* loss, int32_t* kappa, int32_t* status) {
  RowArgs a = {};
  a.z = z;
  a.y = y;
  a.B = B;
  a.C = C;
  a.ld = ld;
  a.scale = 1.0f;
  a.H = H;
  a.loss = loss;
  a.kappa = kappa;
  a.status = status;
  return a;
}

// fp64 rows: a warp per row up to kF64WarpRowMaxC columns, a CTA per row
// beyond; grid capped at the resident CTAs (rows are looped over).
template <int TW, bool VEC, bool GRAD>
cudaError_t launch_f64(const F64Args& a, cudaStream_t st) {
  auto k = fw_f64_rows_kernel<TW, VEC, GRAD>;
  static std::atomic<int> occ_cache{0};
  int occ = occ_cache.load(std::memory_order_relaxed);
  if (occ == 0) {
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, k, kF64Threads, 0) != cudaSuccess || r < 1) r = 1;
    occ = r;
    occ_cache.store(occ, std::memory_order_relaxed);
  }
  constexpr int64_t rows_per_block = kF64Warps / TW;
  const int64_t need = (a.B + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)sm_count() * occ;
  return launch(k, dim3((unsigned)(need < cap ? need : cap)), dim3(kF64Threads), 1, st, a);
}

// fp64 rows of any length; a.grad may be null (forward only).
int run_f64(const F64Args& a, cudaStream_t st) {
  const bool vec = aligned16(a.z) && (a.grad == nullptr || aligned16(a.grad)) && (a.ld % 2 == 0);
  cudaError_t e;
  if (a.grad) {
    if (a.C <= kF64WarpRowMaxC)
      e = vec ? launch_f64<1, true, true>(a, st) : launch_f64<1, false, true>(a, st);
    else
      e = vec ? launch_f64<kF64Warps, true, true>(a, st) : launch_f64<kF64Warps, false, true>(a, st);
  } else {
    if (a.C <= kF64WarpRowMaxC)
      e = vec ? launch_f64<1, true, false>(a, st) : launch_f64<1, false, false>(a, st);
    else
      e = vec ? launch_f64<kF64Warps, true, false>(a, st) : launch_f64<kF64Warps, false, false>(a, st);
  }
  return launch_status(e);
}

// cuTensorMapEncodeTiled, looked up through the runtime so that the library
// does not link the driver library itself.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Row-major bf16 matrix [rows, cols] as 64-column x box_rows tiles with the
// 128-byte swizzle (out-of-range elements read as zero).
bool make_tile_map_bf16(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kTcBK, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int aux_grid(int64_t rows, int per_block) {
  const int64_t need = (rows + per_block - 1) / per_block;
  const int64_t cap = (int64_t)sm_count() * 8;
  const int64_t g = need < cap ? need : cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace fwb200

using namespace fwb200;

extern "C" {

const char* fw_version(void) { return "0.1.0"; }

const char* fw_error_string(int code) {
  switch (code) {
    case FWB_OK: return "ok";
    case FWB_E_SHAPE: return "invalid shape (need B >= 0, 1 <= C < 2^31 - 64, ld >= C)";
    case FWB_E_POINTER: return "a required pointer is NULL";
    case FWB_E_LAUNCH: return "CUDA kernel launch failed";
    case FWB_E_CAPACITY: return "size exceeds the stated maximum";
    case FWB_E_DTYPE: return "unsupported element type code";
    case FWB_E_CUDA: return "a CUDA runtime call failed (allocation, IPC mapping or synchronisation)";
    default: return "unknown error";
  }
}

int fw_fused_fwd_bwd(const float* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                     float grad_scale, float* grad, float* H, float* loss, int32_t* kappa,
                     int32_t* status, void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B > 0 && (!z || !y || !grad)) return FWB_E_POINTER;
  RowArgs a = base_args(z, y, B, C, ld, H, loss, kappa, status);
  a.scale = grad_scale;
  a.grad = grad;
  const bool vec = aligned16(z) && aligned16(grad) && (ld % 4 == 0);
  return run_rows<float, kOutGrad>(a, static_cast<cudaStream_t>(stream), vec);
}

int fw_fused_fwd_bwd_typed(int dtype, const void* z, const int64_t* y, int64_t B, int64_t C,
                           int64_t ld, float grad_scale, void* grad, float* H, float* loss,
                           int32_t* kappa, int32_t* status, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16 && dtype != FWB_DTYPE_F16) return FWB_E_DTYPE;
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B > 0 && (!z || !y || !grad)) return FWB_E_POINTER;
  RowArgs a = base_args(z, y, B, C, ld, H, loss, kappa, status);
  a.scale = grad_scale;
  a.grad = grad;
  const int64_t eps = dtype == FWB_DTYPE_F32 ? 4 : 8;
  const bool vec = aligned16(z) && aligned16(grad) && (ld % eps == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FWB_DTYPE_BF16) return run_rows<__nv_bfloat16, kOutGrad>(a, st, vec);
  if (dtype == FWB_DTYPE_F16) return run_rows<__half, kOutGrad>(a, st, vec);
  return run_rows<float, kOutGrad>(a, st, vec);
}

int fw_fused_fwd_bwd_cols(int dtype, const void* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                          float grad_scale, void* grad, float* H, float* loss, int32_t* kappa,
                          int32_t* sup_cols, int sup_k, int32_t* status, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16 && dtype != FWB_DTYPE_F16) return FWB_E_DTYPE;
  if (int rc = check_shape(B, C, ld)) return rc;
  if (sup_k < 1 || sup_k > 1024) return FWB_E_CAPACITY;
  if (B > 0 && (!z || !y || !grad || !kappa || !sup_cols)) return FWB_E_POINTER;
  RowArgs a = base_args(z, y, B, C, ld, H, loss, kappa, status);
  a.scale = grad_scale;
  a.grad = grad;
  a.sup_cols = sup_cols;
  a.sup_k = sup_k;
  const int64_t eps = dtype == FWB_DTYPE_F32 ? 4 : 8;
  const bool vec = aligned16(z) && aligned16(grad) && (ld % eps == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FWB_DTYPE_BF16) return run_rows<__nv_bfloat16, kOutGradCols>(a, st, vec);
  if (dtype == FWB_DTYPE_F16) return run_rows<__half, kOutGradCols>(a, st, vec);
  return run_rows<float, kOutGradCols>(a, st, vec);
}

int fw_scale_grad_cols(int dtype, void* grad, int64_t ld, const int32_t* sup_cols, int sup_k,
                       const int32_t* kappa, const int64_t* y, const float* grad_output, int per_row,
                       float assumed_scale, int64_t B, int64_t C, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16 && dtype != FWB_DTYPE_F16) return FWB_E_DTYPE;
  if (int rc = check_shape(B, C, ld)) return rc;
  if (sup_k < 1 || sup_k > 1024) return FWB_E_CAPACITY;
  if (B == 0) return FWB_OK;
  if (!grad || !sup_cols || !kappa || !y || !grad_output) return FWB_E_POINTER;
  const int64_t blocks = (B + kAuxThreads / 32 - 1) / (kAuxThreads / 32);
  const dim3 grid((unsigned)(blocks < 65535 ? blocks : 65535)), block(kAuxThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == FWB_DTYPE_BF16)
    e = launch(fw_scale_grad_cols_kernel<__nv_bfloat16>, grid, block, 1, st, static_cast<__nv_bfloat16*>(grad), ld,
               sup_cols, sup_k, kappa, y, grad_output, per_row, assumed_scale, B, C);
  else if (dtype == FWB_DTYPE_F16)
    e = launch(fw_scale_grad_cols_kernel<__half>, grid, block, 1, st, static_cast<__half*>(grad), ld, sup_cols,
               sup_k, kappa, y, grad_output, per_row, assumed_scale, B, C);
  else
    e = launch(fw_scale_grad_cols_kernel<float>, grid, block, 1, st, static_cast<float*>(grad), ld, sup_cols,
               sup_k, kappa, y, grad_output, per_row, assumed_scale, B, C);
  return launch_status(e);
}

int fw_forward_mask(const float* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                    float* H, float* loss, int32_t* kappa, uint8_t* mask, int32_t* status,
                    void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B > 0 && (!z || !y || !mask)) return FWB_E_POINTER;
  RowArgs a = base_args(z, y, B, C, ld, H, loss, kappa, status);
  a.mask = mask;
  a.mask_vec = (C % 4 == 0) && ((reinterpret_cast<uintptr_t>(mask) & 3u) == 0);
  const bool vec = aligned16(z) && (ld % 4 == 0);
  return run_rows<float, kOutMask>(a, static_cast<cudaStream_t>(stream), vec);
}

int fw_backward_mask(const int64_t* y, const uint8_t* mask, const int32_t* kappa, int64_t B,
                     int64_t C, float grad_scale, float* grad, int32_t* status, void* stream) {
  if (int rc = check_shape(B, C, C)) return rc;
  if (B == 0) return FWB_OK;
  if (!y || !mask || !kappa || !grad) return FWB_E_POINTER;
  const int vec = (C % 4 == 0) && aligned16(grad) && ((reinterpret_cast<uintptr_t>(mask) & 3u) == 0);
  const int warps_per_block = kAuxThreads / 32;
  return launch_status(launch(fw_backward_mask_kernel, dim3(aux_grid(B, warps_per_block)),
                              dim3(kAuxThreads), 1, static_cast<cudaStream_t>(stream), y, mask,
                              kappa, B, C, grad_scale, grad, status, vec));
}

int fw_forward_candidates(const float* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                          float* H, float* loss, int32_t* kappa, float* cand_val,
                          int32_t* cand_idx, int32_t* cand_count, int32_t* status,
                          void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B > 0 && (!z || !y || !cand_val || !cand_idx)) return FWB_E_POINTER;
  RowArgs a = base_args(z, y, B, C, ld, H, loss, kappa, status);
  a.cand_val = cand_val;
  a.cand_idx = cand_idx;
  a.cand_count = cand_count;
  const bool vec = aligned16(z) && (ld % 4 == 0);
  return run_rows<float, kOutCand>(a, static_cast<cudaStream_t>(stream), vec);
}

int fw_backward_candidates(const float* cand_val, const int32_t* cand_idx,
                           const int32_t* cand_count, const float* H, const int32_t* kappa,
                           const int64_t* y, int64_t B, int64_t C, float grad_scale,
                           float* grad, int32_t* status, void* stream) {
  if (int rc = check_shape(B, C, C)) return rc;
  if (B == 0) return FWB_OK;
  if (!cand_val || !cand_idx || !cand_count || !H || !kappa || !y || !grad) return FWB_E_POINTER;
  const int vec = (C % 4 == 0) && aligned16(grad);
  return launch_status(launch(fw_backward_cand_kernel, dim3(aux_grid(B, 1)), dim3(kAuxThreads), 1,
                              static_cast<cudaStream_t>(stream), cand_val, cand_idx, cand_count,
                              H, kappa, y, B, C, grad_scale, grad, status, vec));
}

int fw_scale_grad(float* grad, const float* grad_output, int per_row, float assumed_scale,
                  int64_t B, int64_t C, int64_t ld, void* stream) {
  return fw_scale_grad_typed(FWB_DTYPE_F32, grad, grad_output, per_row, assumed_scale, B, C, ld,
                             stream);
}

int fw_scale_grad_typed(int dtype, void* grad, const float* grad_output, int per_row,
                        float assumed_scale, int64_t B, int64_t C, int64_t ld, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16 && dtype != FWB_DTYPE_F16) return FWB_E_DTYPE;
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B == 0) return FWB_OK;
  if (!grad || !grad_output) return FWB_E_POINTER;
  const int64_t eps = dtype == FWB_DTYPE_F32 ? 4 : 8;
  const int vec = aligned16(grad) && (ld % eps == 0);
  const dim3 grid(aux_grid(B, 1)), block(kAuxThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (dtype == FWB_DTYPE_BF16)
    e = launch(fw_scale_grad_kernel<__nv_bfloat16>, grid, block, 1, st,
               static_cast<__nv_bfloat16*>(grad), grad_output, per_row, assumed_scale, B, C, ld, vec);
  else if (dtype == FWB_DTYPE_F16)
    e = launch(fw_scale_grad_kernel<__half>, grid, block, 1, st, static_cast<__half*>(grad),
               grad_output, per_row, assumed_scale, B, C, ld, vec);
  else
    e = launch(fw_scale_grad_kernel<float>, grid, block, 1, st, static_cast<float*>(grad),
               grad_output, per_row, assumed_scale, B, C, ld, vec);
  return launch_status(e);
}

int fw_shard_scan(const float* z, int64_t B, int64_t C_local, int64_t ld, int K, float* grad,
                  int32_t* summary, int32_t* local_idx, void* stream) {
  if (int rc = check_shape(B, C_local, ld)) return rc;
  if (K < 1 || K > kShardMaxK) return FWB_E_CAPACITY;
  if (B > 0 && (!z || !summary || !local_idx)) return FWB_E_POINTER;  // grad optional
  RowArgs a = base_args(z, nullptr, B, C_local, ld, nullptr, nullptr, nullptr, nullptr);
  a.grad = grad;
  a.shard_sum = summary;
  a.shard_idx = local_idx;
  a.shard_k = K;
  const bool vec = aligned16(z) && (grad == nullptr || aligned16(grad)) && (ld % 4 == 0);
  return run_rows<float, kOutShard>(a, static_cast<cudaStream_t>(stream), vec);
}

int fw_shard_solve(const int32_t* gathered, int nranks, int rank, const int64_t* col_start,
                   int64_t B, int K, const float* z, int64_t ld, const int64_t* y,
                   float grad_scale, float* grad, const int32_t* local_idx, float* H,
                   int32_t* kappa, float* loss_part, int32_t* fb_rows, int32_t* fb_count,
                   int32_t* status, void* stream) {
  if (nranks < 1 || nranks > kMaxShards || rank < 0 || rank >= nranks || !col_start) return FWB_E_SHAPE;
  if (K < 1 || K > kShardMaxK || nranks * K > kShardListCap) return FWB_E_CAPACITY;
  if (col_start[0] != 0) return FWB_E_SHAPE;
  for (int q = 0; q < nranks; ++q)
    if (col_start[q + 1] <= col_start[q]) return FWB_E_SHAPE;
  const int64_t C_local = col_start[rank + 1] - col_start[rank];
  if (int rc = check_shape(B, C_local, ld)) return rc;
  if (!fb_count) return FWB_E_POINTER;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fb_count, 0, sizeof(int32_t), st) != cudaSuccess) return FWB_E_LAUNCH;
  if (B == 0) return FWB_OK;
  if (!gathered || !z || !y || !grad || !local_idx || !fb_rows) return FWB_E_POINTER;
  ShardSolveArgs a = {};
  a.gathered = gathered;
  a.nranks = nranks;
  a.rank = rank;
  a.K = K;
  a.B = B;
  for (int q = 0; q <= nranks; ++q) a.col_start[q] = col_start[q];
  a.z = z;
  a.ld = ld;
  a.y = y;
  a.scale = grad_scale;
  a.grad = grad;
  a.local_idx = local_idx;
  a.H = H;
  a.kappa = kappa;
  a.loss_part = loss_part;
  a.fb_rows = fb_rows;
  a.fb_count = fb_count;
  a.status = status;
  const int warps = kShardSolveThreads / 32;
  return launch_status(launch(fw_shard_solve_kernel, dim3(aux_grid(B, warps)), dim3(kShardSolveThreads), 1,
                              st, a));
}

int fw_label_logits(const float* z, int64_t B, int64_t C, int64_t ld, const int64_t* y, int64_t c0,
                    float* zy, void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B == 0) return FWB_OK;
  if (!z || !y || !zy) return FWB_E_POINTER;
  const int threads = 256;
  const int64_t blocks = (B + threads - 1) / threads;
  return launch_status(launch(fw_label_logit_kernel, dim3((unsigned)(blocks < 4096 ? blocks : 4096)),
                              dim3(threads), 1, static_cast<cudaStream_t>(stream), z, B, C, ld, y, c0, zy));
}

int fw_chunks_solve(const int32_t* summaries, const int32_t* local_idx, int nchunks,
                    const int64_t* col_start, int64_t B, int K, const float* zy, const int64_t* y,
                    float* H, int32_t* kappa, float* loss, int32_t* sup_cols, int32_t* fb_rows,
                    int32_t* fb_count, int32_t* status, void* stream) {
  if (nchunks < 1 || nchunks > kMaxShards || !col_start || B < 0) return FWB_E_SHAPE;
  if (K < 1 || K > kShardMaxK || nchunks * K > kShardListCap) return FWB_E_CAPACITY;
  if (col_start[0] != 0) return FWB_E_SHAPE;
  for (int q = 0; q < nchunks; ++q)
    if (col_start[q + 1] <= col_start[q]) return FWB_E_SHAPE;
  if (!fb_count) return FWB_E_POINTER;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(fb_count, 0, sizeof(int32_t), st) != cudaSuccess) return FWB_E_LAUNCH;
  if (B == 0) return FWB_OK;
  if (!summaries || !local_idx || !zy || !y || !kappa || !sup_cols || !fb_rows) return FWB_E_POINTER;
  ChunkSolveArgs a = {};
  a.summaries = summaries;
  a.local_idx = local_idx;
  a.nchunks = nchunks;
  a.K = K;
  a.B = B;
  for (int q = 0; q <= nchunks; ++q) a.col_start[q] = col_start[q];
  a.zy = zy;
  a.y = y;
  a.H = H;
  a.kappa = kappa;
  a.loss = loss;
  a.sup_cols = sup_cols;
  a.fb_rows = fb_rows;
  a.fb_count = fb_count;
  a.status = status;
  const int warps = kShardSolveThreads / 32;
  return launch_status(launch(fw_chunks_solve_kernel, dim3(aux_grid(B, warps)), dim3(kShardSolveThreads), 1,
                              st, a));
}

int fw_sparse_grad_hidden(int dtype, const void* weight, int64_t C, int64_t D, const int32_t* sup_cols,
                          int S, const int32_t* kappa, const int64_t* y, int64_t B, float scale,
                          const float* grad_output, int per_row, void* dhidden, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16) return FWB_E_DTYPE;
  if (B < 0 || C < 1 || D < 1 || S < 1) return FWB_E_SHAPE;
  if (B == 0) return FWB_OK;
  if (!weight || !sup_cols || !kappa || !y || !grad_output || !dhidden) return FWB_E_POINTER;
  SparseGradArgs a = {weight, dhidden, B, C, D, sup_cols, S, kappa, y, scale, grad_output, per_row};
  const dim3 grid(aux_grid(B, 1)), block(kSparseThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_status(dtype == FWB_DTYPE_BF16
                           ? launch(fw_sparse_dhidden_kernel<__nv_bfloat16>, grid, block, 1, st, a)
                           : launch(fw_sparse_dhidden_kernel<float>, grid, block, 1, st, a));
}

int fw_sparse_grad_weight(int dtype, const void* hidden, int64_t B, int64_t D, const int32_t* sup_cols,
                          int S, const int32_t* kappa, const int64_t* y, int64_t C, float scale,
                          const float* grad_output, int per_row, float* dweight, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16) return FWB_E_DTYPE;
  if (B < 0 || C < 1 || D < 1 || S < 1) return FWB_E_SHAPE;
  if (B == 0) return FWB_OK;
  if (!hidden || !sup_cols || !kappa || !y || !grad_output || !dweight) return FWB_E_POINTER;
  SparseGradArgs a = {hidden, dweight, B, C, D, sup_cols, S, kappa, y, scale, grad_output, per_row};
  const dim3 grid(aux_grid(B, 1)), block(kSparseThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_status(dtype == FWB_DTYPE_BF16
                           ? launch(fw_sparse_dweight_kernel<__nv_bfloat16>, grid, block, 1, st, a)
                           : launch(fw_sparse_dweight_kernel<float>, grid, block, 1, st, a));
}

int fw_weight_grad_keys(const int32_t* sup_cols, int S, const int32_t* kappa, const int64_t* y, int64_t B,
                        int64_t C, int64_t* keys, void* stream) {
  if (B < 0 || S < 1 || C < 1) return FWB_E_SHAPE;
  if (B == 0) return FWB_OK;
  if (!sup_cols || !kappa || !y || !keys) return FWB_E_POINTER;
  const int64_t n = B * (int64_t)(S + 1);
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  return launch_status(launch(fw_weight_keys_kernel, dim3((unsigned)(blocks < 65535 ? blocks : 65535)),
                              dim3(threads), 1, static_cast<cudaStream_t>(stream), sup_cols, S, kappa, y, B, C,
                              keys, (int64_t)0));
}

int fw_weight_grad_keys_shard(const int32_t* sup_cols, int S, const int32_t* kappa, const int64_t* y, int64_t B,
                              int64_t c0, int64_t C_shard, int64_t* keys, void* stream) {
  if (B < 0 || S < 1 || C_shard < 1 || c0 < 0) return FWB_E_SHAPE;
  if (B == 0) return FWB_OK;
  if (!sup_cols || !kappa || !y || !keys) return FWB_E_POINTER;
  const int64_t n = B * (int64_t)(S + 1);
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  return launch_status(launch(fw_weight_keys_kernel, dim3((unsigned)(blocks < 65535 ? blocks : 65535)),
                              dim3(threads), 1, static_cast<cudaStream_t>(stream), sup_cols, S, kappa, y, B, C_shard,
                              keys, c0));
}

int fw_sparse_grad_hidden_shard(int dtype, const void* weight_shard, int64_t c0, int64_t C_shard, int64_t D,
                                const int32_t* sup_cols, int S, const int32_t* kappa, const int64_t* y, int64_t B,
                                float scale, const float* grad_output, int per_row, float* dhidden_part,
                                void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16) return FWB_E_DTYPE;
  if (B < 0 || C_shard < 1 || D < 1 || S < 1 || c0 < 0) return FWB_E_SHAPE;
  if (B == 0) return FWB_OK;
  if (!weight_shard || !sup_cols || !kappa || !y || !grad_output || !dhidden_part) return FWB_E_POINTER;
  SparseGradArgs a = {weight_shard, dhidden_part, B, C_shard, D, sup_cols, S, kappa, y, scale, grad_output, per_row,
                      c0};
  const dim3 grid(aux_grid(B, 1)), block(kSparseThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_status(dtype == FWB_DTYPE_BF16
                           ? launch(fw_sparse_dhidden_kernel<__nv_bfloat16, float>, grid, block, 1, st, a)
                           : launch(fw_sparse_dhidden_kernel<float, float>, grid, block, 1, st, a));
}

int fw_segment_grad_weight(int dtype, const void* hidden, int64_t B, int64_t D, const int64_t* keys, int64_t nkeys,
                           const int32_t* kappa, float scale, const float* grad_output, int per_row, void* dweight,
                           void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16) return FWB_E_DTYPE;
  if (B < 0 || D < 1 || nkeys < 0) return FWB_E_SHAPE;
  if (nkeys == 0) return FWB_OK;
  if (!hidden || !keys || !kappa || !grad_output || !dweight) return FWB_E_POINTER;
  SegmentGradArgs a = {hidden, dweight, B, D, keys, nkeys, kappa, scale, grad_output, per_row};
  const int64_t windows = (nkeys + kSegmentWindow - 1) / kSegmentWindow;
  const dim3 grid(aux_grid(windows, 1)), block(kSparseThreads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return launch_status(dtype == FWB_DTYPE_BF16
                           ? launch(fw_segment_dweight_kernel<__nv_bfloat16>, grid, block, 1, st, a)
                           : launch(fw_segment_dweight_kernel<float>, grid, block, 1, st, a));
}

int fw_loss_reduce(const float* loss, int64_t B, double scale, float* out, void* stream) {
  if (B < 0) return FWB_E_SHAPE;
  if (!out || (B > 0 && !loss)) return FWB_E_POINTER;
  return launch_status(launch_loss_reduce<float>(loss, B, scale, out, static_cast<cudaStream_t>(stream)));
}

int fw_lmhead_fused_scan(int dtype, const void* hidden, int64_t B, int64_t D, const void* weight, int64_t C,
                         int nchunks, const int64_t* col_start, int K, const int64_t* y, float* zy,
                         int32_t* summaries, int32_t* local_idx, int32_t* status, void* stream) {
  if (dtype != FWB_DTYPE_BF16) return FWB_E_DTYPE;
  if (B < 0 || C < 1 || D < 8 || D % 8 != 0 || B > (int64_t)INT_MAX - kTcBM || C > (int64_t)INT_MAX - kTcBN ||
      D > (int64_t)INT_MAX - kTcBK)
    return FWB_E_SHAPE;
  if (nchunks < 1 || nchunks > kMaxShards || K < 1 || K > kShardMaxK) return FWB_E_CAPACITY;
  if (!col_start) return FWB_E_POINTER;
  if (col_start[0] != 0 || col_start[nchunks] != C) return FWB_E_SHAPE;
  for (int q = 0; q < nchunks; ++q)
    if (col_start[q + 1] <= col_start[q] || col_start[q] % kTcBN != 0) return FWB_E_SHAPE;
  if (B == 0) return FWB_OK;
  if (!hidden || !weight || !y || !zy || !summaries || !local_idx) return FWB_E_POINTER;
  if (!aligned16(hidden) || !aligned16(weight)) return FWB_E_SHAPE;
  TcArgs a = {};
  a.B = B;
  a.C = C;
  a.D = D;
  a.nchunks = nchunks;
  a.K = K;
  a.n_mblocks = (int)((B + kTcBM - 1) / kTcBM);
  for (int q = 0; q <= nchunks; ++q) a.col_start[q] = col_start[q];
  a.y = y;
  a.zy = zy;
  a.summaries = summaries;
  a.local_idx = local_idx;
  a.status = status;
  CUtensorMap tm_h, tm_w;
  if (!make_tile_map_bf16(&tm_h, hidden, B, D, kTcBM) || !make_tile_map_bf16(&tm_w, weight, C, D, kTcBN))
    return FWB_E_LAUNCH;
  static std::atomic<bool> attr_set[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return FWB_E_LAUNCH;
  if (dev >= kMaxDevices || !attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(fw_lmhead_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kTcSmemBytes) != cudaSuccess)
      return FWB_E_LAUNCH;
    if (dev < kMaxDevices) attr_set[dev].store(true, std::memory_order_release);
  }
  const int64_t nwork = (int64_t)a.n_mblocks * nchunks;
  const int64_t sms = sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nwork < sms ? nwork : sms));
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  return launch_status(cudaLaunchKernelEx(&cfg, fw_lmhead_tc_kernel, tm_h, tm_w, a));
}

int fw_loss_reduce_f64(const double* loss, int64_t B, double scale, double* out, void* stream) {
  if (B < 0) return FWB_E_SHAPE;
  if (!out || (B > 0 && !loss)) return FWB_E_POINTER;
  return launch_status(launch_loss_reduce<double>(loss, B, scale, out, static_cast<cudaStream_t>(stream)));
}

int fw_fused_fwd_bwd_f64(const double* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                         double grad_scale, double* grad, double* H, double* loss, int32_t* kappa,
                         int32_t* status, void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B == 0) return FWB_OK;
  if (!z || !y || !grad) return FWB_E_POINTER;
  const F64Args a = {z, y, B, C, ld, grad_scale, grad, H, loss, kappa, status};
  return run_f64(a, static_cast<cudaStream_t>(stream));
}

int fw_forward_rows(int dtype, const void* z, const int64_t* y, int64_t B, int64_t C, int64_t ld,
                    float* H, float* loss, int32_t* kappa, int32_t* status, void* stream) {
  if (dtype != FWB_DTYPE_F32 && dtype != FWB_DTYPE_BF16 && dtype != FWB_DTYPE_F16) return FWB_E_DTYPE;
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B > 0 && (!z || !y)) return FWB_E_POINTER;
  const RowArgs a = base_args(z, y, B, C, ld, H, loss, kappa, status);
  const int64_t eps = dtype == FWB_DTYPE_F32 ? 4 : 8;
  const bool vec = aligned16(z) && (ld % eps == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FWB_DTYPE_BF16) return run_rows<__nv_bfloat16, kOutNone>(a, st, vec);
  if (dtype == FWB_DTYPE_F16) return run_rows<__half, kOutNone>(a, st, vec);
  return run_rows<float, kOutNone>(a, st, vec);
}

int fw_forward_rows_f64(const double* z, const int64_t* y, int64_t B, int64_t C, int64_t ld, double* H,
                        double* loss, int32_t* kappa, int32_t* status, void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B == 0) return FWB_OK;
  if (!z || !y) return FWB_E_POINTER;
  const F64Args a = {z, y, B, C, ld, 1.0, nullptr, H, loss, kappa, status};
  return run_f64(a, static_cast<cudaStream_t>(stream));
}

int fw_scale_grad_f64(double* grad, const double* grad_output, int per_row, double assumed_scale,
                      int64_t B, int64_t C, int64_t ld, void* stream) {
  if (int rc = check_shape(B, C, ld)) return rc;
  if (B == 0) return FWB_OK;
  if (!grad || !grad_output) return FWB_E_POINTER;
  return launch_status(launch(fw_scale_grad_f64_kernel, dim3(aux_grid(B, 1)), dim3(256), 1,
                              static_cast<cudaStream_t>(stream), grad, grad_output, per_row,
                              assumed_scale, B, C, ld));
}

}  // extern "C"
