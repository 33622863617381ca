// Tier selection and launches of the fused row kernels (run_rows).  Included
// by the fw_rows_*.cu translation units, each of which instantiates run_rows
// for some (element type, output form) pairs, so that the kernel instances
// compile in parallel.
//
// Tier selection by class count C (the tile shape scales with C):
//   C <= 2048          a group of 8/16/32 lanes per row, row in registers
//                      (fw_warp_tier.cuh).
//   C  > 2048          CTA per row (CS = 1) or a cluster of CS = 2/4/8 CTAs per
//                      row when there are too few rows to fill the GPU
//                      (fw_stream_tier.cuh; launch plan: dispatch_stream).
// 128-bit loads/stores are used when every row starts on a 16-byte boundary
// (base pointers 16-byte aligned and ld % 4 == 0); otherwise the same kernels
// run with coalesced 32-bit accesses.
#pragma once

#include "fw_host.cuh"
#include "fw_stream_tier.cuh"
#include "fw_warp_tier.cuh"

namespace fwb200 {
namespace {

constexpr int64_t kWarpTierMaxC = 2048;

// ------------------------------------------------------------- warp tier
template <class T, int G, int NS, bool VEC, int OUT>
cudaError_t launch_warp_tier(const RowArgs& a, cudaStream_t st) {
  // FULLV: every 16-byte slot fully inside or outside the row (one predicate
  // per slot); only meaningful for 16-byte accesses
  const bool fullv = VEC && (a.C % Elem<T>::kEPS == 0);
  auto k = fullv ? fw_warp_rows_kernel<T, G, NS, VEC, OUT, VEC>
                 : fw_warp_rows_kernel<T, G, NS, VEC, OUT, false>;
  constexpr int threads = warp_tier_threads<NS * Elem<T>::kEPS>();
  static std::atomic<int> occ[2] = {};  // resident CTAs per SM of the two instances
  int o = occ[fullv ? 1 : 0].load(std::memory_order_relaxed);
  if (o == 0) {
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, k, threads, 0) != cudaSuccess || r < 1)
      r = 1;
    o = r;
    occ[fullv ? 1 : 0].store(o, std::memory_order_relaxed);
  }
  const int64_t rows_per_block = (int64_t)(threads / 32) * (32 / G);
  const int64_t need = (a.B + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)sm_count() * o;
  const int grid = (int)(need < cap ? need : cap);
  return launch(k, dim3(grid), dim3(threads), 1, st, a);
}

// Lanes per row G and register values per lane NV by class count:
//   C <= 64: 8 x 8,  <= 128: 8 x 16,  <= 256: 16 x 16,  <= 512: 32 x 16,
//   <= 1024: 32 x 32,  <= 2048: 32 x 64  (NS = NV / EPS 16-byte slots).
template <class T, bool VEC, int OUT>
cudaError_t dispatch_warp(const RowArgs& a, cudaStream_t st) {
  constexpr int E = Elem<T>::kEPS;
  if (a.C <= 64) return launch_warp_tier<T, 8, 8 / E, VEC, OUT>(a, st);
  if (a.C <= 128) return launch_warp_tier<T, 8, 16 / E, VEC, OUT>(a, st);
  if (a.C <= 256) return launch_warp_tier<T, 16, 16 / E, VEC, OUT>(a, st);
  if (a.C <= 512) return launch_warp_tier<T, 32, 16 / E, VEC, OUT>(a, st);
  if (a.C <= 1024) return launch_warp_tier<T, 32, 32 / E, VEC, OUT>(a, st);
  return launch_warp_tier<T, 32, 64 / E, VEC, OUT>(a, st);
}

// ----------------------------------------------------------- stream tier
// after_prior: launched as a programmatic dependent of the previous kernel on
// the stream (its CTAs may start while that kernel's last CTAs run) and
// waiting for that kernel before exiting (RowArgs::wait_prior).
template <class T, int CS, bool VEC, int OUT, int SHAPE>
cudaError_t prepare_stream_instance() {
  if constexpr (is_staged<SHAPE>() && VEC) {
    // the ring of stages is dynamic shared memory above the 48 KB default:
    // raise the instance's limit once per device
    static std::atomic<bool> attr_set[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return cudaErrorInvalidDevice;
    if (dev >= kMaxDevices || !attr_set[dev].load(std::memory_order_acquire)) {
      cudaError_t e = cudaFuncSetAttribute(fw_stream_rows_kernel<T, CS, VEC, OUT, SHAPE>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)staged_smem_bytes<SHAPE>());
      // the whole unified L1 / shared array as shared memory: the narrow
      // shape's 8 CTAs per SM need 227 KB of it (a preference, not a limit)
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fw_stream_rows_kernel<T, CS, VEC, OUT, SHAPE>,
                                 cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
      if (dev < kMaxDevices) attr_set[dev].store(true, std::memory_order_release);
    }
  }
  return cudaSuccess;
}

template <class T, int CS, bool VEC, int OUT, int SHAPE = kShapeWide>
cudaError_t launch_stream_tier(const RowArgs& a, cudaStream_t st, bool after_prior = false) {
  auto kernel = fw_stream_rows_kernel<T, CS, VEC, OUT, SHAPE>;
  constexpr bool kStaged = (is_staged<SHAPE>() && VEC);
  {
    const cudaError_t e = prepare_stream_instance<T, CS, VEC, OUT, SHAPE>();
    if (e != cudaSuccess) return e;
  }
  RowArgs b = a;
  b.wait_prior = after_prior ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.B * CS));
  cfg.blockDim = dim3(stream_threads<SHAPE>());
  cfg.dynamicSmemBytes = kStaged ? staged_smem_bytes<SHAPE>() : 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (CS > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = CS;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (after_prior) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, b);
}

// The arguments for rows [r0, r0 + n) of a (every per-row pointer advanced).
template <class T>
RowArgs rows_from(const RowArgs& a, int64_t r0, int64_t n) {
  RowArgs b = a;
  b.B = n;
  b.z = static_cast<const T*>(a.z) + r0 * a.ld;
  if (a.y) b.y = a.y + r0;
  if (a.grad) b.grad = static_cast<T*>(a.grad) + r0 * a.ld;
  if (a.mask) b.mask = a.mask + r0 * a.C;
  if (a.cand_val) b.cand_val = a.cand_val + r0 * a.C;
  if (a.cand_idx) b.cand_idx = a.cand_idx + r0 * a.C;
  if (a.cand_count) b.cand_count = a.cand_count + r0;
  if (a.H) b.H = a.H + r0;
  if (a.loss) b.loss = a.loss + r0;
  if (a.kappa) b.kappa = a.kappa + r0;
  if (a.shard_sum) b.shard_sum = a.shard_sum + r0 * (int64_t)(kShardHeader + a.shard_k);
  if (a.shard_idx) b.shard_idx = a.shard_idx + r0 * (int64_t)a.shard_k;
  if (a.sup_cols) b.sup_cols = a.sup_cols + r0 * (int64_t)a.sup_k;
  return b;
}

// Cluster size for few rows: the largest CS in {1, 2, 4, 8} whose CTAs
// (rows x CS) fit in `slots`, every CTA keeping >= 4096 columns.
inline int fit_cluster(int64_t rows, int64_t C, int64_t slots) {
  int cs = 1;
  while (cs < 8 && rows * cs * 2 <= slots && C / (cs * 2) >= 4096) cs *= 2;
  return cs;
}

// Few rows (at most two CTAs per SM): 16-byte-aligned rows take the staged
// shape (bulk-copied tiles), the others the deep one.
template <class T, bool VEC, int OUT>
cudaError_t launch_deep(const RowArgs& a, cudaStream_t st, int cs, bool after_prior) {
  constexpr int SH = VEC ? kShapeStaged : kShapeDeep;
  switch (cs) {
    case 8: return launch_stream_tier<T, 8, VEC, OUT, SH>(a, st, after_prior);
    case 4: return launch_stream_tier<T, 4, VEC, OUT, SH>(a, st, after_prior);
    case 2: return launch_stream_tier<T, 2, VEC, OUT, SH>(a, st, after_prior);
    default: return launch_stream_tier<T, 1, VEC, OUT, SH>(a, st, after_prior);
  }
}

// Long fp32 rows that write a gradient (or a gradient shard) stream through
// the staged shape from this many columns on (B200, fraction of the HBM
// roofline, wide / staged, fwd+bwd: C = 32000, 4096 rows 0.935 / 0.877;
// C = 48000, 4096 rows 0.947 / 0.974; C = 65536, 1024 / 4096 rows 0.855 /
// 0.890, 0.947 / 0.997; C = 128256, 8192 rows 0.959 / 1.005.  Forward only,
// the wide shape stays ahead at every length: 0.984 / 0.711 at 65536 x 4096).
constexpr int64_t kStagedMinCols = 40960;
// ... and through the 4-CTAs-per-SM staged shape (8 KB tiles) from this many
// columns on, when the batch is more than one wave of the wide shape (B200,
// C = 32000, wide / staged4: 1024 rows 0.788 / 0.827, 2048 rows 0.890 /
// 0.916, 4096 rows 0.943 / 0.970; one wave or less the wide shape is ahead,
// 512 rows 0.900 / 0.820; so are short rows, C = 8192 x 8192 0.854 / 0.762).
constexpr int64_t kStaged4MinCols = 24576;
// 16-bit rows writing a gradient take the staged4 shape from this many
// columns on (B200, bf16, staged4 / narrow / wide: 65536 x 4096 0.959 /
// 0.923 / 0.890; 128256 x 8192 1.003 / 0.979 / 0.931; 128256 x 1024 0.835 /
// 0.748 / 0.713) ...
constexpr int64_t kStaged4MinCols16 = 49152;
// ... and shorter 16-bit rows, or fp32 rows of fewer than kNarrowMaxCols
// columns, the narrow shape (1184 resident CTAs) once the batch holds this
// many elements (B200, narrow / wide / staged4: bf16 32000 x 4096 0.876 /
// 0.835 / 0.799, 32000 x 8192 0.950 / 0.883 / 0.839, 16000 x 8192 0.802 /
// 0.756 / 0.649, 8192 x 16384 0.674 / 0.631 / 0.480; fp32 8192 x 8192 0.953 /
// 0.908 / 0.765, 8192 x 16384 1.009 / 0.945 / 0.793; below it the wide shape
// is ahead or level: bf16 32000 x 1024 0.698 / 0.703, 16000 x 2048 0.624 /
// 0.674, fp32 8192 x 4096 0.858 / 0.853; longer fp32 rows stay with wide and
// staged4: 16000 x 8192 0.966 / 0.969 / 0.980, 32000 x 4096 0.938 / 0.949 /
// 0.976).
constexpr int64_t kNarrowMinElems = int64_t(64) << 20;
constexpr int64_t kNarrowMaxCols = 12288;

// Launch plan for B rows (one CTA per row; resident slots per SM: wide 5,
// deep and staged 2, staged4 4, narrow 8):
//  * B <= deep slots: the staged shape (the deep one for rows not 16-byte
//    aligned), with clusters of CS CTAs per row when rows x CS still fits
//    one such wave (e.g. 32 rows x 1e6 columns: CS 8);
//  * 16-byte-aligned rows that write a gradient: the staged, staged4 or
//    narrow shape by element size, row length and batch size (the
//    constants above);
//  * otherwise one CTA per row in the wide shape; when that is one full wave
//    and a last wave of at most (deep slots) rows, those rows go to a second
//    launch in the deep shape (clustered as above), started as a
//    programmatic dependent so that it runs under the first launch's last
//    CTAs: a short last wave of the wide shape is latency-bound (B200,
//    C = 32000 fp32: 768 rows took 44.0 us against 22.6 us for 512 rows).
//    Over more waves the CTAs have drifted apart and the second launch costs
//    more than it saves (fp32 8192 x 8192: 95.9 us split, 90.3 us one launch).
template <class T, bool VEC, int OUT>
cudaError_t dispatch_stream(const RowArgs& a, cudaStream_t st) {
  const int64_t sms = sm_count();
  const int64_t deep = sms * stream_min_blocks<kShapeDeep>();
  const int64_t wide = sms * stream_min_blocks<kShapeWide>();
  if (a.B <= deep) return launch_deep<T, VEC, OUT>(a, st, fit_cluster(a.B, a.C, deep), false);
  if constexpr (VEC && (OUT == kOutGrad || OUT == kOutShard)) {
    const bool many = a.B * a.C >= kNarrowMinElems;
    if constexpr (sizeof(T) == 4) {
      // long fp32 rows: one staged CTA per row (2 per SM); mid-length ones
      // over more than one wide wave: 4 per SM; short ones in large batches:
      // 8 narrow CTAs per SM
      if (a.C >= kStagedMinCols) return launch_stream_tier<T, 1, VEC, OUT, kShapeStaged>(a, st);
      if (a.C >= kStaged4MinCols && a.B > wide) return launch_stream_tier<T, 1, VEC, OUT, kShapeStaged4>(a, st);
      if (a.C < kNarrowMaxCols && many) return launch_stream_tier<T, 1, VEC, OUT, kShapeNarrow>(a, st);
    } else {
      if (a.C >= kStaged4MinCols16 && a.B > wide) return launch_stream_tier<T, 1, VEC, OUT, kShapeStaged4>(a, st);
      if (a.C < kStaged4MinCols16 && many) return launch_stream_tier<T, 1, VEC, OUT, kShapeNarrow>(a, st);
    }
  }
  const int64_t tail = a.B % wide;
  if (a.B <= wide || a.B > 2 * wide || tail == 0 || tail > deep) return launch_stream_tier<T, 1, VEC, OUT>(a, st);
  const int64_t head = a.B - tail;
  const cudaError_t e = launch_stream_tier<T, 1, VEC, OUT>(rows_from<T>(a, 0, head), st);
  if (e != cudaSuccess) return e;
  return launch_deep<T, VEC, OUT>(rows_from<T>(a, head, tail), st, fit_cluster(tail, a.C, deep), true);
}

}  // namespace

template <class T, int OUT>
int run_rows(const RowArgs& a, cudaStream_t st, bool vec) {
  if (a.B == 0) return FWB_OK;
  // the streaming tier lists the support columns under a runtime check
  constexpr int OUT_STREAM = (OUT == kOutGradCols) ? kOutGrad : OUT;
  cudaError_t e;
  if (a.C <= kWarpTierMaxC)
    e = vec ? dispatch_warp<T, true, OUT>(a, st) : dispatch_warp<T, false, OUT>(a, st);
  else
    e = vec ? dispatch_stream<T, true, OUT_STREAM>(a, st) : dispatch_stream<T, false, OUT_STREAM>(a, st);
  return launch_status(e);
}

}  // namespace fwb200
