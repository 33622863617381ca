/*
 * fwloss_b200.h -- C ABI of the B200 (sm_100a) Familywise-loss library.
 *
 * The Familywise (FW) loss of one row z[0..C) with label y is
 *     L(z, y) = 1 - z_y + h*,   h* = max_k (S_k - 1) / k,
 * S_k being the sum of the k largest logits.  h* is also the root of
 * sum_j max(z_j - h, 0) = 1, and the gradient is
 *     dL/dz = (1/kappa) 1[z > h*] - e_y,   kappa = |{j : z_j > h*}|.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*, NULL = legacy default stream), launches asynchronously on
 * that stream and returns an int status (FWB_OK or one of the FWB_E* codes
 * below).  Nothing here allocates device memory, synchronises the stream or
 * reads device data on the host, except the set-up calls of the cross-GPU
 * exchange buffer (fw_peer_buffer_create / _open / _close / _destroy).  Logits are fp32 row-major with row stride
 * `ld` (elements, ld >= C); labels are int64.  Data-dependent problems that
 * only the device can see (a label outside [0, C), a non-finite row maximum)
 * are reported through the optional device word `status` (bit-or of
 * FWB_STATUS_* flags; the caller zeroes it) and by a NaN loss for that row.
 *
 * Outputs per row r (all optional pointers may be NULL):
 *   H[r]      fp32 threshold, rounded toward -inf from the exact h*, so that
 *             for every fp32 x:  x > H[r]  <=>  x > h*.
 *   loss[r]   fp32 1 - z_y + h*.
 *   kappa[r]  int32 support size.
 * Thresholds and kappa are computed by the same procedure in every entry
 * point, so the mask-, candidate- and gradient-producing paths agree.
 */
#ifndef FWLOSS_B200_H
#define FWLOSS_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define FWB_API __attribute__((visibility("default")))
#else
#define FWB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FWB_OK 0
#define FWB_E_SHAPE 1      /* B < 0, C < 1, ld < C, or a size overflows      */
#define FWB_E_POINTER 2    /* a required pointer is NULL                       */
#define FWB_E_LAUNCH 3     /* the CUDA launch failed (cudaGetLastError)        */
#define FWB_E_CAPACITY 4   /* a size exceeds a stated maximum                  */
#define FWB_E_DTYPE 5      /* unknown element type code                        */
#define FWB_E_CUDA 6       /* a CUDA runtime call of a set-up function failed  */

/* Element types of logits / gradient for the *_typed entry points (the
 * arithmetic is fp32/fp64 for all of them; 16-bit values are passed as their
 * bit patterns). */
#define FWB_DTYPE_F32 0
#define FWB_DTYPE_BF16 1
#define FWB_DTYPE_F16 2

#define FWB_STATUS_LABEL_RANGE 1   /* some label y[r] is outside [0, C)          */
#define FWB_STATUS_NONFINITE 2     /* some row maximum is NaN or +-inf           */
#define FWB_STATUS_TIMEOUT 4       /* a bounded wait gave up (fused LM-head kernel, staged streaming tiles, cross-GPU loss sum) */

/* Library version, "major.minor.patch". */
FWB_API const char* fw_version(void);

/* Human-readable text for an FWB_* return code. */
FWB_API const char* fw_error_string(int code);

/*
 * Fused forward + backward: per-row threshold search, loss and the dense
 * gradient, in one pass that reads z once and writes grad once.
 *   grad[r, j] = grad_scale * ((1/kappa_r) 1[z_rj > h*_r] - 1[j == y_r])
 * grad has the same row stride `ld` as z (columns C..ld-1 are not written).
 * grad_scale is 1/B for reduction "mean", 1 for "sum" and "none".
 * Replaces the pair fw_radix_forward_small + fw_radix_backward_small and the
 * pair fw_radix_forward + fw_radix_backward of the reference
 * (src/cuda/fw_radix_argmax.cu:1381-1414, :1417-1496, :1536-1559, :1591-1608,
 * bound in src/cuda/binding.cpp:3-6), and the forward of the CPU autograd
 * function (src/cpu/fw_cpu.cpp:722-733).
 */
FWB_API int fw_fused_fwd_bwd(const float* z, const int64_t* y, int64_t B, int64_t C,
                     int64_t ld, float grad_scale, float* grad, float* H,
                     float* loss, int32_t* kappa, int32_t* status,
                     void* stream);

/*
 * fw_fused_fwd_bwd for logits of element type `dtype` (FWB_DTYPE_*); the
 * gradient has the same element type and the logits' row stride, H and loss
 * stay fp32.  16-bit logits halve the bytes per row; the threshold, kappa
 * and the loss are computed exactly from the 16-bit values.  Extends the
 * reference's fp32-only entry points (src/cuda/fw_radix_argmax.cu:1387,1422
 * reject other dtypes); the CPU kernel's dtype dispatch
 * (src/cpu/fw_cpu.cpp:698-704) covers fp32/fp64.
 */
FWB_API int fw_fused_fwd_bwd_typed(int dtype, const void* z, const int64_t* y, int64_t B,
                                   int64_t C, int64_t ld, float grad_scale, void* grad,
                                   float* H, float* loss, int32_t* kappa, int32_t* status,
                                   void* stream);

/*
 * fw_fused_fwd_bwd_typed that also lists each row's support columns:
 * sup_cols[r * sup_k + p] for p < min(kappa[r], sup_k) (order unspecified);
 * rows whose support is not listed (dense rows solved by the radix passes)
 * get -1 in their first slot.  kappa is required.  1 <= sup_k <= 1024.  With
 * fw_scale_grad_cols this gives the per-row ("none") reduction a backward
 * that touches kappa + 1 entries per row instead of the whole row.
 * Extends the forward of the CPU autograd function (src/cpu/fw_cpu.cpp:
 * 722-733), which keeps the dense gradient for its backward.
 */
FWB_API int fw_fused_fwd_bwd_cols(int dtype, const void* z, const int64_t* y, int64_t B, int64_t C,
                                  int64_t ld, float grad_scale, void* grad, float* H, float* loss,
                                  int32_t* kappa, int32_t* sup_cols, int sup_k, int32_t* status,
                                  void* stream);

/*
 * fw_scale_grad_typed for a gradient written by fw_fused_fwd_bwd_cols: row r
 * is multiplied by grad_output[per_row ? r : 0] / assumed_scale; a row with a
 * finite factor != 1 and a listed support of kappa <= sup_k entries rewrites
 * only those entries and its label entry, other rows are handled as by
 * fw_scale_grad_typed.  Replaces the scaling of the CPU autograd backward
 * (src/cpu/fw_cpu.cpp:734-740).
 */
FWB_API int fw_scale_grad_cols(int dtype, void* grad, int64_t ld, const int32_t* sup_cols, int sup_k,
                               const int32_t* kappa, const int64_t* y, const float* grad_output,
                               int per_row, float assumed_scale, int64_t B, int64_t C, void* stream);

/*
 * Forward producing the boolean support mask (uint8, [B, C] contiguous):
 * mask[r, j] = 1[z_rj > h*_r].  Replaces fw_radix_forward_small
 * (src/cuda/fw_radix_argmax.cu:1381-1414; binding.cpp:5,11); the reference
 * returns the same mask as `selected_logits`.
 */
FWB_API int fw_forward_mask(const float* z, const int64_t* y, int64_t B, int64_t C,
                    int64_t ld, float* H, float* loss, int32_t* kappa,
                    uint8_t* mask, int32_t* status, void* stream);

/*
 * Dense gradient from a support mask: grad[r, j] = grad_scale *
 * (mask[r, j] / kappa[r] - 1[j == y[r]]), grad row stride C.
 * Replaces fw_radix_backward_small (src/cuda/fw_radix_argmax.cu:1591-1608,
 * kernel :1561-1589; binding.cpp:6,12).
 */
FWB_API int fw_backward_mask(const int64_t* y, const uint8_t* mask,
                     const int32_t* kappa, int64_t B, int64_t C,
                     float grad_scale, float* grad, int32_t* status,
                     void* stream);

/*
 * Forward producing the support as a candidate list: for row r,
 * cand_val[r*C + p] / cand_idx[r*C + p] for p < cand_count[r] hold the value
 * and column of every z_rj > h*_r (cand_count[r] == kappa[r]; order
 * unspecified).  Replaces fw_radix_forward (src/cuda/fw_radix_argmax.cu:
 * 1417-1496; binding.cpp:3,9), whose candidate_buffer / candidate_indices /
 * candidate_counts outputs have this meaning and layout.
 */
FWB_API int fw_forward_candidates(const float* z, const int64_t* y, int64_t B,
                          int64_t C, int64_t ld, float* H, float* loss,
                          int32_t* kappa, float* cand_val, int32_t* cand_idx,
                          int32_t* cand_count, int32_t* status, void* stream);

/*
 * Dense gradient from a candidate list: grad = 0, then for every candidate
 * p < cand_count[r] with cand_val > H[r]: grad[r, cand_idx] =
 * grad_scale / kappa[r]; finally grad[r, y[r]] -= grad_scale.  grad row
 * stride C.  Replaces fw_radix_backward (src/cuda/fw_radix_argmax.cu:
 * 1536-1559, kernel :1498-1534; binding.cpp:4,10).
 */
FWB_API int fw_backward_candidates(const float* cand_val, const int32_t* cand_idx,
                           const int32_t* cand_count, const float* H,
                           const int32_t* kappa, const int64_t* y, int64_t B,
                           int64_t C, float grad_scale, float* grad,
                           int32_t* status, void* stream);

/*
 * Backward scaling by the upstream gradient, read on the device (no host
 * sync).  Row r of grad (row stride ld, C columns) is multiplied by
 * grad_output[per_row ? r : 0] / assumed_scale; rows whose factor is exactly
 * 1 are not touched, and inside a touched row only the non-zero entries are
 * rewritten.  Replaces the host-synchronising scaling of the CPU autograd
 * backward (src/cpu/fw_cpu.cpp:734-740).
 */
FWB_API int fw_scale_grad(float* grad, const float* grad_output, int per_row,
                  float assumed_scale, int64_t B, int64_t C, int64_t ld,
                  void* stream);

/*
 * Forward only: H, loss and kappa per row, no gradient (z is read once and
 * nothing of size C is written: half the HBM bytes of fw_fused_fwd_bwd).
 * Same threshold search, so H, loss and kappa equal those of
 * fw_fused_fwd_bwd bit for bit.  `dtype` is FWB_DTYPE_F32, _BF16 or _F16.
 * Replaces the forward of FWLoss when no gradient is wanted (evaluation,
 * torch.no_grad; reference_impl.py:11-35) and the forward of the reference
 * CUDA path without its [N, K] mask or candidate buffers
 * (src/cuda/fw_radix_argmax.cu:1381-1414, :1417-1496).
 */
FWB_API int fw_forward_rows(int dtype, const void* z, const int64_t* y, int64_t B, int64_t C,
                            int64_t ld, float* H, float* loss, int32_t* kappa, int32_t* status,
                            void* stream);

/* fw_forward_rows for float64 logits (fp64 H and loss), the forward of the
 * reference CPU kernel's float64 branch (src/cpu/fw_cpu.cpp:698-704). */
FWB_API int fw_forward_rows_f64(const double* z, const int64_t* y, int64_t B, int64_t C,
                                int64_t ld, double* H, double* loss, int32_t* kappa,
                                int32_t* status, void* stream);

/* fw_scale_grad for a gradient of element type `dtype` (FWB_DTYPE_*). */
FWB_API int fw_scale_grad_typed(int dtype, void* grad, const float* grad_output, int per_row,
                                float assumed_scale, int64_t B, int64_t C, int64_t ld,
                                void* stream);

/*
 * Class-sharded rows (tensor-parallel LM heads): rank q of nranks holds
 * columns [col_start[q], col_start[q+1]) of every row.  No counterpart in the
 * reference (its rows are always whole); the math is
 * the reference's (reference_impl.py:11-26).
 *
 * Step 1, on every rank: fw_shard_scan solves each row of the local shard
 * [B, C_local] on its own, zero-fills the local gradient shard `grad`
 * (row stride ld; NULL: no gradient shard) and writes a summary record per row into
 * summary[B, 4 + K] (int32 words: local max as float bits, local support size
 * kappa_q, flags, first maximal column; then up to K support values as float
 * bits) and the support's local columns into local_idx[B, K].  1 <= K <= 64.
 *
 * Step 2 (caller): all-gather the summaries of all ranks into
 * gathered[nranks, B, 4 + K], rank-major.
 *
 * Step 3, on every rank: fw_shard_solve combines the summaries: the global
 * threshold is >= every shard's own threshold, so the union of the shard
 * supports contains the global support.  It writes H and kappa (identical on
 * all ranks), patches this rank's gradient shard (support entries, and the
 * label entry when y[r] falls in this rank's columns), and writes
 * loss_part[r] = the row's loss if this rank owns the label, else 0 (sum over
 * ranks = the per-row losses).  Rows where some shard's support exceeds K
 * entries are not solved: their indices go to fb_rows[0 .. *fb_count)
 * (device; *fb_count is reset by this call) for the caller to solve from the
 * full rows.  col_start is a HOST array of nranks + 1 increasing offsets
 * starting at 0; nranks <= 16 and nranks * K <= 256.
 */
FWB_API int fw_shard_scan(const float* z, int64_t B, int64_t C_local, int64_t ld, int K,
                          float* grad, int32_t* summary, int32_t* local_idx, void* stream);

FWB_API int fw_shard_solve(const int32_t* gathered, int nranks, int rank,
                           const int64_t* col_start, int64_t B, int K, const float* z,
                           int64_t ld, const int64_t* y, float grad_scale, float* grad,
                           const int32_t* local_idx, float* H, int32_t* kappa,
                           float* loss_part, int32_t* fb_rows, int32_t* fb_count,
                           int32_t* status, void* stream);

/*
 * LM head, logits = hidden [B, D] x weight [C, D]^T, without a resident
 * [B, C] logit matrix.  No counterpart in the reference (it takes logits as
 * input); the math is the reference's (reference_impl.py:11-26).
 *
 * The caller produces the logits one column chunk [col_start[q],
 * col_start[q+1]) at a time (any GEMM) and, per chunk, calls
 * fw_shard_scan(chunk, ..., grad = NULL, summary_q, local_idx_q) (summaries
 * only) and fw_label_logits(chunk, ..., c0 = col_start[q], zy) (keeps the
 * logit at the label).  fw_chunks_solve then combines the nchunks summaries
 * (summaries [nchunks, B, 4 + K], local_idx [nchunks, B, K]; nchunks <= 16,
 * nchunks * K <= 256) into H, kappa, loss and the support's columns
 * sup_cols[B, nchunks * K] (first kappa entries of each row).  Rows whose chunk
 * supports exceed K get kappa = 0 and are listed in fb_rows[0 .. *fb_count)
 * for the caller's exact path.
 *
 * The logit gradient then has kappa + 1 non-zeros per row, so the LM-head
 * backward is two sparse kernels instead of two dense GEMMs:
 *   fw_sparse_grad_hidden:  dhidden[r] = g_r (sum_{j in supp} W[j] / kappa_r - W[y_r])
 *   fw_sparse_grad_weight:  dweight[j] += g_r (hidden[r] / kappa_r, j in supp(r);
 *                                          -hidden[r], j = y_r)   (fp32, atomics)
 * with g_r = scale * grad_output[per_row ? r : 0]; rows with kappa 0 are
 * skipped (dhidden row set to 0).  dtype: FWB_DTYPE_F32 or FWB_DTYPE_BF16 for
 * weight / hidden / dhidden.
 */
FWB_API int fw_label_logits(const float* z, int64_t B, int64_t C, int64_t ld, const int64_t* y,
                            int64_t c0, float* zy, void* stream);

/*
 * LM-head chunk summaries straight from the GEMM (sm_100a tensor cores):
 * logits = hidden [B, D] x weight [C, D]^T (bf16, row-major, D % 8 == 0,
 * 16-byte aligned bases) are accumulated in tensor memory and reduced to the
 * chunk summary records that fw_shard_scan writes from stored logits
 * (summaries [nchunks, B, 4 + K], local_idx [nchunks, B, K]), plus the label
 * logit zy[r] = logits[r, y[r]]; no logit is written to memory.  col_start
 * (host, nchunks + 1 entries) starts every chunk at a multiple of 256 columns
 * and ends at C.  A chunk whose candidates overflow the on-chip list is
 * recorded with kappa = K + 1 (the row then takes the exact full-row path in
 * fw_chunks_solve).  Status bit FWB_STATUS_TIMEOUT reports a bounded on-chip
 * wait that gave up.  No counterpart in the reference: the fused form of
 * logits = hidden @ W^T followed by FWLoss (reference_impl.py:11-26).
 */
FWB_API int fw_lmhead_fused_scan(int dtype, const void* hidden, int64_t B, int64_t D, const void* weight,
                                 int64_t C, int nchunks, const int64_t* col_start, int K,
                                 const int64_t* y, float* zy, int32_t* summaries, int32_t* local_idx,
                                 int32_t* status, void* stream);

FWB_API int fw_chunks_solve(const int32_t* summaries, const int32_t* local_idx, int nchunks,
                            const int64_t* col_start, int64_t B, int K, const float* zy,
                            const int64_t* y, float* H, int32_t* kappa, float* loss,
                            int32_t* sup_cols, int32_t* fb_rows, int32_t* fb_count,
                            int32_t* status, void* stream);

FWB_API int fw_sparse_grad_hidden(int dtype, const void* weight, int64_t C, int64_t D,
                                  const int32_t* sup_cols, int S, const int32_t* kappa,
                                  const int64_t* y, int64_t B, float scale,
                                  const float* grad_output, int per_row, void* dhidden,
                                  void* stream);

FWB_API int fw_sparse_grad_weight(int dtype, const void* hidden, int64_t B, int64_t D,
                                  const int32_t* sup_cols, int S, const int32_t* kappa,
                                  const int64_t* y, int64_t C, float scale,
                                  const float* grad_output, int per_row, float* dweight,
                                  void* stream);

/*
 * Deterministic dweight for the LM head, without data-dependent shapes:
 * fw_weight_grad_keys writes keys[B * (S + 1)], one per non-zero of the logit
 * gradient, key = (j << 32) | (r << 1) | is_label (unused slots:
 * 0x7fffffffffffffff); the caller sorts them ascending; then
 * fw_segment_grad_weight writes, for every column j present,
 * dweight[j] = sum over its entries, in key order, of g_r / kappa_r * hidden[r]
 * (support) or -g_r * hidden[r] (label), in the weight's element type.  Rows
 * of dweight with no entry are not written (caller zeroes them).
 */
FWB_API int fw_weight_grad_keys(const int32_t* sup_cols, int S, const int32_t* kappa, const int64_t* y,
                                int64_t B, int64_t C, int64_t* keys, void* stream);

FWB_API int fw_segment_grad_weight(int dtype, const void* hidden, int64_t B, int64_t D,
                                   const int64_t* keys, int64_t nkeys, const int32_t* kappa,
                                   float scale, const float* grad_output, int per_row,
                                   void* dweight, void* stream);

/*
 * Vocabulary-parallel LM head: rank q holds the weight rows of classes
 * [c0, c0 + C_shard) and all ranks hold the same hidden, labels and (after
 * an all-gather of the chunk summaries and fw_chunks_solve) the same support
 * columns sup_cols (global class ids) and kappa.  No counterpart in the
 * reference (its logits are whole); the math is the reference's
 * (reference_impl.py:11-26).
 *   fw_sparse_grad_hidden_shard: this rank's part of dhidden, in fp32 for the
 *     all-reduce:  dhidden_part[r] = g_r (sum_{j in supp, j local} W[j - c0] /
 *     kappa_r - [y_r local] W[y_r - c0]); rows with kappa 0 are written as 0.
 *   fw_weight_grad_keys_shard: the keys of fw_weight_grad_keys restricted to
 *     the local classes, with class ids relative to c0, for
 *     fw_segment_grad_weight on the local weight gradient.
 */
FWB_API int fw_sparse_grad_hidden_shard(int dtype, const void* weight_shard, int64_t c0, int64_t C_shard,
                                        int64_t D, const int32_t* sup_cols, int S, const int32_t* kappa,
                                        const int64_t* y, int64_t B, float scale, const float* grad_output,
                                        int per_row, float* dhidden_part, void* stream);

FWB_API int fw_weight_grad_keys_shard(const int32_t* sup_cols, int S, const int32_t* kappa, const int64_t* y,
                                      int64_t B, int64_t c0, int64_t C_shard, int64_t* keys, void* stream);

/*
 * Deterministic (fixed-order, fp64) reduction out[0] = scale * sum_r loss[r].
 * Gives the "mean" (scale 1/B) and "sum" (scale 1) values of the reference
 * (reference_impl.py:28-31, src/cuda/fw_radix_argmax.cu:1411,1493,
 * src/cpu/fw_cpu.cpp:729-732).
 */
FWB_API int fw_loss_reduce(const float* loss, int64_t B, double scale, float* out,
                   void* stream);

/*
 * float64 logits: fw_fused_fwd_bwd with fp64 logits, gradient, H and loss
 * (grad: [B, ld] fp64, same row stride as z).  Replaces the float64 branch of
 * the reference CPU kernel (src/cpu/fw_cpu.cpp:698-704, fw_row<double> at
 * :419-470); the reference CUDA kernels are fp32-only.  Support:
 * {x > t0 and fl(x - M) > tau} with t0 = M - 1 rounded down, which is the
 * exact support whenever the row max M >= 2 and otherwise agrees with it up
 * to fp64 rounding; H = fl(M + tau).
 */
FWB_API int fw_fused_fwd_bwd_f64(const double* z, const int64_t* y, int64_t B, int64_t C,
                                 int64_t ld, double grad_scale, double* grad, double* H,
                                 double* loss, int32_t* kappa, int32_t* status, void* stream);

/* fw_scale_grad for an fp64 gradient with fp64 grad_output (FWFunction::backward,
 * src/cpu/fw_cpu.cpp:734-740, for float64 logits). */
FWB_API int fw_scale_grad_f64(double* grad, const double* grad_output, int per_row,
                              double assumed_scale, int64_t B, int64_t C, int64_t ld,
                              void* stream);

/* fw_loss_reduce for fp64 losses and an fp64 result (the float64 total of
 * src/cpu/fw_cpu.cpp:729-732). */
FWB_API int fw_loss_reduce_f64(const double* loss, int64_t B, double scale, double* out,
                               void* stream);

/*
 * Cross-GPU loss sum for row-sharded data parallelism (one process per GPU,
 * GPUs that reach each other's memory over NVLink / NVSwitch).  The
 * reference has no multi-GPU code; this replaces the pair "fw_loss_reduce,
 * then an all-reduce of its scalar" that sharding its row-wise loss needs,
 * by one kernel: each rank sums its rows' losses in fp64, stores the partial
 * into every rank's exchange buffer through peer memory, waits (bounded) for
 * the other ranks' partials in its own buffer and writes
 *     out[0] = scale * (partial_0 + partial_1 + ... + partial_{world-1})
 * (fp64, rank order: every rank gets the same value).
 *
 * Set-up, once per rank (these allocate and synchronise):
 *   fw_peer_buffer_create  allocates this rank's FWB_PEER_BUFFER_BYTES
 *                          exchange buffer on the current device, zeroes it
 *                          and returns it with its CUDA IPC handle
 *                          (FWB_PEER_HANDLE_BYTES bytes); the host sends the
 *                          handles to every rank (e.g. an all-gather);
 *   fw_peer_buffer_open    maps another rank's buffer from its handle;
 *   fw_peer_buffer_close / fw_peer_buffer_destroy  undo the two.
 * fw_loss_allreduce(_f64) takes the world buffers in rank order (this rank's
 * own buffer at index `rank`, the opened ones elsewhere).  Every rank must
 * make the same sequence of calls on its buffers, each on one stream at a
 * time (calls that overlap on one rank race).  A rank whose peers do not
 * publish within timeout_s seconds sets FWB_STATUS_TIMEOUT in *status (if
 * given) and writes NaN; the buffers cannot be used after that.  Returns
 * FWB_E_CAPACITY for world > FWB_PEER_MAX.
 */
#define FWB_PEER_MAX 8
#define FWB_PEER_HANDLE_BYTES 64
#define FWB_PEER_BUFFER_BYTES 512
FWB_API int fw_peer_buffer_create(void** buf, void* handle);
FWB_API int fw_peer_buffer_open(const void* handle, void** peer);
FWB_API int fw_peer_buffer_close(void* peer);
FWB_API int fw_peer_buffer_destroy(void* buf);
FWB_API int fw_loss_allreduce(const float* loss, int64_t B, double scale, void* const* bufs, int world,
                              int rank, float* out, int32_t* status, double timeout_s, void* stream);
FWB_API int fw_loss_allreduce_f64(const double* loss, int64_t B, double scale, void* const* bufs,
                                  int world, int rank, double* out, int32_t* status, double timeout_s,
                                  void* stream);

/*
 * LM-head forward in one call that allocates nothing: fw_lmhead_fused_scan
 * followed by fw_chunks_solve (same arguments, outputs and limits as those
 * two), with their workspace -- the chunk summaries, the support's local
 * columns and the label logits -- kept in a fixed array inside the library
 * instead of buffers from the caller.  For callers that cannot call
 * cudaMalloc: plugins whose host framework owns all device memory, servers
 * that forbid allocation after start-up, FFI hosts that only hold the buffers
 * handed to them.  The workspace needs
 *     round_up(nchunks * B * (4 + K), 64) + round_up(nchunks * B * K, 64) + B
 * 4-byte words, at most FWB_NOALLOC_SCRATCH_BYTES / 4, and nchunks * K <= 256
 * (fw_chunks_solve's limit); other problems return FWB_E_CAPACITY before any
 * kernel runs (e.g. B = 8192, nchunks = 8, K = 16 fits).  The array is
 * FWB_NOALLOC_SCRATCH_BYTES on every GPU that loads the library, held until
 * exit.  The first call in a CUDA context looks up the array's address with
 * that context current and caches it under the context's unique id (a device
 * reset makes a new context, whose first call looks it up again); make the
 * first call on each device before any stream capture.  All calls share the
 * array: calls that overlap on the GPU race.  No counterpart in the reference.
 */
#define FWB_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)

FWB_API int fw_lmhead_fused_loss_noalloc(int dtype, const void* hidden, int64_t B, int64_t D,
                                         const void* weight, int64_t C, int nchunks,
                                         const int64_t* col_start, int K, const int64_t* y,
                                         float* H, int32_t* kappa, float* loss, int32_t* sup_cols,
                                         int32_t* fb_rows, int32_t* fb_count, int32_t* status,
                                         void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FWLOSS_B200_H */
