// Sizes and the per-thread loop of the deterministic loss reduction, shared
// by fw_loss_reduce_kernel (fw_aux.cuh) and the cross-GPU loss sum
// (fw_peer.cu): header-only, no kernels, so both translation units can hold it.
#pragma once

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kReduceCluster = 8;
constexpr int64_t kReduceClusterMinRows = 16384;  // B above which CL = kReduceCluster
constexpr int kReduceThreads = 512;
constexpr int kReduceBatch = 4;  // 16-byte loads in flight per thread

// Sixteen bytes of T (four floats or two doubles) per load.
template <class T>
struct Vec16;
template <>
struct Vec16<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, double (&v)[4]) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  }
};
template <>
struct Vec16<double> {
  static constexpr int N = 2;
  __device__ static void load(const double* p, double (&v)[2]) {
    const double2 x = *reinterpret_cast<const double2*>(p);
    v[0] = x.x; v[1] = x.y;
  }
};

// This thread's fp64 sum of loss over the 16-byte groups [g_lo, g_hi) of
// Vec16<T>::N entries (kReduceThreads threads, kReduceBatch groups in flight
// per thread; a fixed order, so the result is deterministic).
template <class T>
__device__ __forceinline__ double thread_loss_sum(const T* __restrict__ loss, int64_t B, int64_t g_lo,
                                                  int64_t g_hi, int vec) {
  constexpr int N = Vec16<T>::N;
  double s = 0.0;
  for (int64_t g0 = g_lo + threadIdx.x; g0 < g_hi; g0 += (int64_t)kReduceThreads * kReduceBatch) {
    double v[kReduceBatch][N];
#pragma unroll
    for (int k = 0; k < kReduceBatch; ++k) {
      const int64_t g = g0 + (int64_t)k * kReduceThreads;
      const int64_t i0 = g * N;
      if (vec && g < g_hi && i0 + N <= B) {
        Vec16<T>::load(loss + i0, v[k]);
      } else {
#pragma unroll
        for (int j = 0; j < N; ++j) v[k][j] = (g < g_hi && i0 + j < B) ? (double)loss[i0 + j] : 0.0;
      }
    }
#pragma unroll
    for (int k = 0; k < kReduceBatch; ++k)
#pragma unroll
      for (int j = 0; j < N; ++j) s += v[k][j];
  }
  return s;
}

}  // namespace fwb200
