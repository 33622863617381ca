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
//                      (fw_stream_tier.cuh).
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
  static std::atomic<int> occ[2] = {};  // resident CTAs per SM of the two instances
  int o = occ[fullv ? 1 : 0].load(std::memory_order_relaxed);
  if (o == 0) {
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, k, kWarpTierThreads, 0) != cudaSuccess || r < 1)
      r = 1;
    o = r;
    occ[fullv ? 1 : 0].store(o, std::memory_order_relaxed);
  }
  const int64_t rows_per_block = (int64_t)kWarpTierWarps * (32 / G);
  const int64_t need = (a.B + rows_per_block - 1) / rows_per_block;
  const int64_t cap = (int64_t)sm_count() * o;
  const int grid = (int)(need < cap ? need : cap);
  return launch(k, dim3(grid), dim3(kWarpTierThreads), 1, st, a);
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
template <class T, int CS, bool VEC, int OUT, bool DEEP = false>
cudaError_t launch_stream_tier(const RowArgs& a, cudaStream_t st) {
  auto k = fw_stream_rows_kernel<T, CS, VEC, OUT, DEEP>;
  const int64_t grid = a.B * CS;
  return launch(k, dim3((unsigned)grid), dim3(kST), CS, st, a);
}

// Cluster size: the smallest CS in {1, 2, 4, 8} giving at least 4 CTAs per SM,
// while every CTA keeps a segment of at least 4096 columns.
inline int choose_cluster(int64_t B, int64_t C) {
  const int64_t want = (int64_t)sm_count() * 4;
  int cs = 1;
  while (cs < 8 && B * cs < want && C / (cs * 2) >= 4096) cs *= 2;
  return cs;
}

template <class T, bool VEC, int OUT>
cudaError_t dispatch_stream(const RowArgs& a, cudaStream_t st) {
  switch (choose_cluster(a.B, a.C)) {
    case 8:  // at most two CTAs per SM: the instance with deeper load pipelining
      return (a.B * 8 <= 2 * (int64_t)sm_count()) ? launch_stream_tier<T, 8, VEC, OUT, true>(a, st)
                                                  : launch_stream_tier<T, 8, VEC, OUT>(a, st);
    case 4: return launch_stream_tier<T, 4, VEC, OUT>(a, st);
    case 2: return launch_stream_tier<T, 2, VEC, OUT>(a, st);
    default: return launch_stream_tier<T, 1, VEC, OUT>(a, st);
  }
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
