// Host-side helpers shared by the translation units of libfwloss_b200.so:
// device properties, alignment tests and the launch wrapper.  Every
// translation unit gets its own copy (anonymous namespace), including its
// own per-process caches.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <utility>

#include "../../include/fwloss_b200.h"
#include "fw_device.cuh"

namespace fwb200 {
namespace {

constexpr int kMaxDevices = 64;

// Per-process caches below are filled on first use; concurrent callers may
// both compute the same value, so they are atomics (relaxed: the values
// never change once set).
inline int sm_count() {
  static std::atomic<int> cache[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return 148;
  if (dev < kMaxDevices) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (dev < kMaxDevices) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status(cudaError_t e) { return e == cudaSuccess ? FWB_OK : FWB_E_LAUNCH; }

template <class... KArgs, class... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, int cluster,
                   cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (cluster > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace

// Fused forward(+backward) over rows of element type T with output form OUT
// (fw_rows.cuh; one explicit instantiation per (T, OUT) in the fw_rows_*.cu
// translation units).  vec: rows are 16-byte aligned (16-byte accesses).
template <class T, int OUT>
int run_rows(const RowArgs& a, cudaStream_t st, bool vec);

}  // namespace fwb200
