// Kernels around the fused search: the two legacy backward forms, the
// device-side scaling by the upstream gradient and the deterministic loss
// reduction.  All are HBM-streaming kernels (no tensor-core work).
#pragma once

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kAuxThreads = 256;

// grad[r, j] = scale * (mask[r, j] / kappa[r] - [j == y[r]]); one warp per
// row, 4 columns per lane per step (uchar4 in, float4 out when C % 4 == 0).
// Same result as fw_backward_mask_kernel (src/cuda/fw_radix_argmax.cu:
// 1561-1589), which reads one bool and writes one float per thread-step.
__global__ void __launch_bounds__(kAuxThreads)
    fw_backward_mask_kernel(const int64_t* __restrict__ y,
                            const uint8_t* __restrict__ mask,
                            const int32_t* __restrict__ kappa, int64_t B,
                            int64_t C, float scale, float* __restrict__ grad,
                            int32_t* status, int vec) {
  const int lane = threadIdx.x & 31;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < B;
       r += nw) {
    const int64_t yl = y[r];
    const bool yok = (yl >= 0 && yl < C);
    const float inv = (float)((double)scale / (double)kappa[r]);
    const uint8_t* mr = mask + r * C;
    float* gr = grad + r * C;
    if (vec) {
      for (int64_t q = lane; q < C / 4; q += 32) {
        const uchar4 b = *reinterpret_cast<const uchar4*>(mr + 4 * q);
        float4 g = make_float4(b.x ? inv : 0.f, b.y ? inv : 0.f, b.z ? inv : 0.f,
                               b.w ? inv : 0.f);
        const int64_t c0 = 4 * q;
        if (yl >= c0 && yl < c0 + 4) {
          if (yl == c0) g.x -= scale;
          if (yl == c0 + 1) g.y -= scale;
          if (yl == c0 + 2) g.z -= scale;
          if (yl == c0 + 3) g.w -= scale;
        }
        *reinterpret_cast<float4*>(gr + c0) = g;
      }
    } else {
      for (int64_t c = lane; c < C; c += 32) {
        float g = mr[c] ? inv : 0.f;
        if (c == yl) g -= scale;
        gr[c] = g;
      }
    }
    if (!yok && lane == 0) raise_status(status, 1);
  }
}

// grad = 0; grad[r, idx] = scale / kappa[r] for candidates with value > H[r];
// grad[r, y[r]] -= scale.  One CTA per row.  Same result as
// torch::zeros_like + fw_backward_candidate_kernel
// (src/cuda/fw_radix_argmax.cu:1498-1559), in one launch.  Candidate
// columns outside [0, C) are skipped and flagged instead of written.
__global__ void __launch_bounds__(kAuxThreads)
    fw_backward_cand_kernel(const float* __restrict__ cand_val,
                            const int32_t* __restrict__ cand_idx,
                            const int32_t* __restrict__ cand_count,
                            const float* __restrict__ H,
                            const int32_t* __restrict__ kappa,
                            const int64_t* __restrict__ y, int64_t B, int64_t C,
                            float scale, float* __restrict__ grad,
                            int32_t* status, int vec) {
  for (int64_t r = blockIdx.x; r < B; r += gridDim.x) {
    float* gr = grad + r * C;
    if (vec) {
      for (int64_t q = threadIdx.x; q < C / 4; q += blockDim.x)
        *reinterpret_cast<float4*>(gr + 4 * q) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int64_t c = threadIdx.x; c < C; c += blockDim.x) gr[c] = 0.f;
    }
    __syncthreads();
    const float h = H[r];
    const float inv = (float)((double)scale / (double)kappa[r]);
    int n = cand_count[r];
    n = n < 0 ? 0 : (n > C ? (int)C : n);
    bool bad = false;
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
      const float v = cand_val[r * C + p];
      const int j = cand_idx[r * C + p];
      if (v > h) {
        if (j >= 0 && j < C)
          gr[j] = inv;
        else
          bad = true;
      }
    }
    if (bad) raise_status(status, 1);
    __syncthreads();
    if (threadIdx.x == 0) {
      const int64_t yl = y[r];
      if (yl >= 0 && yl < C)
        gr[yl] -= scale;
      else
        raise_status(status, 1);
    }
    __syncthreads();
  }
}

// Row r of grad *= grad_output[per_row ? r : 0] / assumed.  Rows whose factor
// is exactly 1 are skipped; for finite factors only non-zero entries are
// rewritten (the gradient has kappa + 1 of them), for non-finite factors the
// whole row is (0 * inf = NaN, as in a dense multiply).  T is the gradient's
// element type; 16-byte slots when vec.
template <class T>
__global__ void __launch_bounds__(kAuxThreads)
    fw_scale_grad_kernel(T* __restrict__ grad, const float* __restrict__ grad_output, int per_row,
                         float assumed, int64_t B, int64_t C, int64_t ld, int vec) {
  constexpr int EPS = Elem<T>::kEPS;
  for (int64_t r = blockIdx.x; r < B; r += gridDim.x) {
    const float f = grad_output[per_row ? r : 0] / assumed;
    if (f == 1.0f) continue;
    const bool dense = !isfinite(f);
    T* gr = grad + r * ld;
    int64_t done = 0;
    if (vec) {
      for (int64_t q = threadIdx.x; q < C / EPS; q += blockDim.x) {
        const uint4 u = *reinterpret_cast<const uint4*>(gr + EPS * q);
        if (dense || (u.x | u.y | u.z | u.w) != 0u) {
          float g[EPS];
          unpack16<T>(u, g);
#pragma unroll
          for (int j = 0; j < EPS; ++j) g[j] *= f;
          *reinterpret_cast<uint4*>(gr + EPS * q) = pack16<T>(g);
        }
      }
      done = EPS * (C / EPS);
    }
    for (int64_t c = done + threadIdx.x; c < C; c += blockDim.x) {
      const float g = ld_elem(gr + c);
      if (dense || g != 0.f) st_elem(gr + c, g * f);
    }
  }
}

// out[0] = scale * sum(loss[0..B)), fp64 accumulation in a fixed order (one
// CTA; thread t sums t, t + 1024, ...; then a fixed tree).  T: fp32 or fp64
// losses and result.
constexpr int kReduceThreads = 1024;
template <class T>
__global__ void __launch_bounds__(kReduceThreads)
    fw_loss_reduce_kernel(const T* __restrict__ loss, int64_t B,
                          double scale, T* __restrict__ out) {
  __shared__ double part[kReduceThreads / 32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < B; i += kReduceThreads) s += (double)loss[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = part[threadIdx.x];
    t = warp_sum(t);
    if (threadIdx.x == 0) out[0] = (T)(t * scale);
  }
}

}  // namespace fwb200
