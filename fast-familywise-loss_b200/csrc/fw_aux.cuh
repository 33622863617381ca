// Kernels around the fused search: the two legacy backward forms, the
// device-side scaling by the upstream gradient and the deterministic loss
// reduction.  All are HBM-streaming kernels (no tensor-core work).
#pragma once

#include <cooperative_groups.h>

#include "fw_device.cuh"
#include "fw_reduce.cuh"

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

// fw_scale_grad_kernel for a gradient whose support columns were listed by
// the forward (sup_cols [B, sup_k], first slot -1 when not listed): a row
// with a finite factor != 1, kappa <= sup_k and a list rewrites only its
// kappa support entries and its label entry (kappa + 1 elements instead of
// reading the row); other rows scale the whole row as fw_scale_grad_kernel
// does.  One warp per row.
template <class T>
__global__ void __launch_bounds__(kAuxThreads)
    fw_scale_grad_cols_kernel(T* __restrict__ grad, int64_t ld, const int32_t* __restrict__ sup_cols, int sup_k,
                              const int32_t* __restrict__ kappa, const int64_t* __restrict__ y,
                              const float* __restrict__ grad_output, int per_row, float assumed, int64_t B,
                              int64_t C) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kAuxThreads / 32);
  for (int64_t r = (int64_t)blockIdx.x * (kAuxThreads / 32) + (threadIdx.x >> 5); r < B; r += warps) {
    const float f = grad_output[per_row ? r : 0] / assumed;
    if (f == 1.0f) continue;
    T* gr = grad + r * ld;
    const int kap = kappa[r];
    const int32_t* sc = sup_cols + r * (int64_t)sup_k;
    const bool listed = isfinite(f) && kap >= 1 && kap <= sup_k && sc[0] >= 0;
    if (listed) {
      const int64_t yl = y[r];
      bool yin = false;
      for (int k = lane; k < kap; k += 32) {
        const int col = sc[k];
        yin |= (col == yl);
        st_elem(gr + col, ld_elem(gr + col) * f);
      }
      yin = __any_sync(kFull, yin);
      if (lane == 0 && !yin && yl >= 0 && yl < C) st_elem(gr + yl, ld_elem(gr + yl) * f);
    } else {
      const bool dense = !isfinite(f);
      for (int64_t c = lane; c < C; c += 32) {
        const float g = ld_elem(gr + c);
        if (dense || g != 0.f) st_elem(gr + c, g * f);
      }
    }
  }
}

// out[0] = scale * sum(loss[0..B)) with fp64 accumulation in a fixed order,
// by CL CTAs (one thread-block cluster when CL > 1): CTA r owns the r-th of
// CL equal slices of the 16-byte groups of `loss`; thread t of a CTA sums
// the groups t, t + T, t + 2T, ... of its slice (values in index order inside
// a group, kReduceBatch groups loaded before they are added, so that each
// thread keeps several loads in flight), then a fixed butterfly and a fixed
// tree over the warps give the CTA's partial; CTA 0 adds the partials in rank
// order through distributed shared memory.  Large batches use CL = 8 (eight
// SMs keep eight times the loads of one in flight; the losses are read from
// L2), small ones CL = 1 (a cluster launch costs about a microsecond more).
// The choice and the partition depend only on B, so the result is
// deterministic.  `vec`: loss is 16-byte aligned; otherwise scalar loads in
// the same order.
//
// The kernel is launched as a programmatic dependent of the kernel before it
// on the stream (usually the one that wrote the losses): it may be scheduled
// while that kernel drains, and griddepcontrol.wait holds every thread until
// that kernel has completed and its writes are visible.  T: fp32 or fp64.
template <class T, int CL>
__global__ void __launch_bounds__(kReduceThreads)
    fw_loss_reduce_kernel(const T* __restrict__ loss, int64_t B,
                          double scale, T* __restrict__ out, int vec) {
  constexpr int N = Vec16<T>::N;
  __shared__ double part[kReduceThreads / 32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int rank = 0;
  if constexpr (CL > 1) rank = (int)cooperative_groups::this_cluster().block_rank();
  const int64_t ngroups = (B + N - 1) / N;
  const int64_t g_lo = ngroups * rank / CL;
  const int64_t g_hi = ngroups * (rank + 1) / CL;
  double s = thread_loss_sum<T>(loss, B, g_lo, g_hi, vec);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = (threadIdx.x < kReduceThreads / 32) ? part[threadIdx.x] : 0.0;
    t = warp_sum(t);
    if (threadIdx.x == 0) {
      if constexpr (CL == 1) out[0] = (T)(t * scale);
      part[0] = t;
    }
  }
  if constexpr (CL > 1) {
    auto cluster = cooperative_groups::this_cluster();
    cluster.sync();  // every CTA's partial is in its part[0]
    if (rank == 0 && threadIdx.x == 0) {
      double t = 0.0;
      for (int r = 0; r < CL; ++r) t += *cluster.map_shared_rank(&part[0], r);
      out[0] = (T)(t * scale);
    }
    cluster.sync();  // the partials stay readable until CTA 0 has read them
  }
}

}  // namespace fwb200
