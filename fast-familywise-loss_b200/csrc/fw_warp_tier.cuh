// Warp-per-row tier (C <= 32 * 4 * VW): the whole row sits in registers of
// one warp, so the row is read from HBM once and its output is written once,
// with no shared-memory traffic except the short candidate list.
//
// Per row:
//   1. load (128-bit when rows are 16-byte aligned), M = NaN-propagating max
//      by shuffles;
//   2. candidates z > t0 are compacted into a per-warp list by an exclusive
//      shuffle scan (the common case: a handful of elements);
//   3. exact threshold: Michelot's fixed point on the list
//      (michelot_list), or on the registers when the list would overflow
//      (near-constant rows where most of the row is within 1 of the max);
//   4. output written straight from the registers: the gradient
//      grad_scale * ((1/kappa) [z > h*] - e_y), the support mask, or the
//      support list.
//
// Reference counterpart: fw_radix_shared_kernel<8,32,100> / <8,128,5000>
// (src/cuda/fw_radix_argmax.cu:1192-1356) followed by fw_backward_mask_kernel
// (:1561-1589).  The reference finds h* by up to four 8-bit digit passes
// with four shared-memory atomics per element and then needs a second kernel
// for the gradient; here the threshold comes from the candidate list and the
// gradient is written by the same warp.
#pragma once

#include <climits>

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kWarpTierThreads = 256;
constexpr int kWarpTierWarps = kWarpTierThreads / 32;
constexpr int kWarpListCap = 128;

// Column of register slot (i, j) of `lane`.  Aligned rows use 128-bit loads
// (lane owns 4 consecutive columns per slot group); unaligned rows use
// lane-contiguous scalar loads so that every load instruction is coalesced.
template <bool VEC>
__device__ __forceinline__ int warp_slot_col(int i, int j, int lane) {
  return VEC ? ((i * 32 + lane) * 4 + j) : ((i * 4 + j) * 32 + lane);
}

template <int VW, bool VEC, int OUT>
__global__ void __launch_bounds__(kWarpTierThreads)
    fw_warp_rows_kernel(RowArgs a) {
  constexpr int NS = VW * 4;
  __shared__ float s_list[kWarpTierWarps][kWarpListCap];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int C = (int)a.C;
  const int64_t nwarps = (int64_t)gridDim.x * kWarpTierWarps;

  for (int64_t row = (int64_t)blockIdx.x * kWarpTierWarps + wib; row < a.B;
       row += nwarps) {
    const float* zr = a.z + row * a.ld;
    const int64_t ylab = a.y[row];
    float v[NS];
#pragma unroll
    for (int i = 0; i < VW; ++i) {
      if (VEC) {
        const int c0 = (i * 32 + lane) * 4;
        if (c0 + 3 < C) {
          const float4 q = ld_stream4(zr + c0);
          v[4 * i + 0] = q.x;
          v[4 * i + 1] = q.y;
          v[4 * i + 2] = q.z;
          v[4 * i + 3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            v[4 * i + j] = (c0 + j < C) ? ld_stream1(zr + c0 + j) : -CUDART_INF_F;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = warp_slot_col<false>(i, j, lane);
          v[4 * i + j] = (c < C) ? ld_stream1(zr + c) : -CUDART_INF_F;
        }
      }
    }

    float m = -CUDART_INF_F;
#pragma unroll
    for (int s = 0; s < NS; ++s) m = max_nan(m, v[s]);
    m = warp_max_nan(m);

    const bool yok = (ylab >= 0 && ylab < a.C);
    const int yc = yok ? (int)ylab : -1;
    const bool nonfinite = !isfinite(m);  // warp-uniform
    const double Md = (double)m;
    const float t0 = __fsub_rd(m, 1.0f);
    double tau = 0.0;
    int kap = 1;
    int jstar = -1;

    if (!nonfinite) {
      int c = 0;
#pragma unroll
      for (int s = 0; s < NS; ++s) c += (v[s] > t0) ? 1 : 0;
      const int tot = warp_sum(c);
      if (tot <= kWarpListCap) {
        int off = warp_excl_scan(c, lane);
        float* L = s_list[wib];
#pragma unroll
        for (int s = 0; s < NS; ++s)
          if (v[s] > t0) L[off++] = v[s];
        __syncwarp();
        michelot_list(L, tot, Md, lane, tau, kap);
        __syncwarp();
      } else {
        // Same fixed point, evaluated on the registers (dense rows).
        double t = -CUDART_INF;
        int prev = -1;
        for (int it = 0; it <= C; ++it) {
          double sum = 0.0;
          int cnt = 0;
#pragma unroll
          for (int s = 0; s < NS; ++s) {
            const double d = (double)v[s] - Md;
            if (v[s] > t0 && d > t) { sum += d; ++cnt; }
          }
          cnt = warp_sum(cnt);
          sum = warp_sum(sum);
          if (cnt == prev) break;
          prev = cnt;
          t = (sum - 1.0) / (double)cnt;
        }
        tau = t;
        kap = prev;
      }
    } else {
      // Non-finite maximum: kappa = 1 at the first column holding the
      // maximum (the first NaN for NaN rows), H = M.
      const bool isn = (m != m);
      int best = INT_MAX;
#pragma unroll
      for (int i = 0; i < VW; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = warp_slot_col<VEC>(i, j, lane);
          const float x = v[4 * i + j];
          if (c < C && (isn ? (x != x) : (x == m))) best = min(best, c);
        }
      jstar = (int)__reduce_min_sync(kFull, (unsigned)best);
    }

    const float zy = yok ? __ldg(zr + yc) : CUDART_NAN_F;

    auto selected = [&](int s, int c) -> bool {
      if (nonfinite) return c == jstar;
      return v[s] > t0 && ((double)v[s] - Md) > tau;
    };

    if (OUT == kOutGrad) {
      const float inv = nonfinite ? a.scale : (float)((double)a.scale / (double)kap);
      float* gr = a.grad + row * a.ld;
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        float g[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = warp_slot_col<VEC>(i, j, lane);
          g[j] = selected(4 * i + j, c) ? inv : 0.0f;
          if (c == yc) g[j] -= a.scale;
        }
        if (VEC) {
          const int c0 = (i * 32 + lane) * 4;
          if (c0 + 3 < C) {
            *reinterpret_cast<float4*>(gr + c0) = make_float4(g[0], g[1], g[2], g[3]);
          } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              if (c0 + j < C) gr[c0 + j] = g[j];
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = warp_slot_col<false>(i, j, lane);
            if (c < C) gr[c] = g[j];
          }
        }
      }
    } else if (OUT == kOutMask) {
      uint8_t* mr = a.mask + row * a.C;
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        uint8_t b[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          b[j] = selected(4 * i + j, warp_slot_col<VEC>(i, j, lane)) ? 1 : 0;
        if (VEC && a.mask_vec && (i * 32 + lane) * 4 + 3 < C) {
          const int c0 = (i * 32 + lane) * 4;
          *reinterpret_cast<uchar4*>(mr + c0) = make_uchar4(b[0], b[1], b[2], b[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = warp_slot_col<VEC>(i, j, lane);
            if (c < C) mr[c] = b[j];
          }
        }
      }
    } else {  // kOutCand
      int cnt = 0;
#pragma unroll
      for (int i = 0; i < VW; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          cnt += selected(4 * i + j, warp_slot_col<VEC>(i, j, lane)) ? 1 : 0;
      int off = warp_excl_scan(cnt, lane);
      float* cv = a.cand_val + row * a.C;
      int32_t* ci = a.cand_idx + row * a.C;
#pragma unroll
      for (int i = 0; i < VW; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = warp_slot_col<VEC>(i, j, lane);
          if (selected(4 * i + j, c)) {
            cv[off] = v[4 * i + j];
            ci[off] = c;
            ++off;
          }
        }
      if (lane == 0 && a.cand_count) a.cand_count[row] = kap;
    }

    if (lane == 0) {
      float Hf, lf;
      if (!nonfinite) {
        Hf = threshold_fp32(m, tau);
        lf = yok ? row_loss(m, tau, zy) : CUDART_NAN_F;
      } else {
        Hf = m;
        lf = yok ? (1.0f - zy + m) : CUDART_NAN_F;
      }
      if (a.H) a.H[row] = Hf;
      if (a.loss) a.loss[row] = lf;
      if (a.kappa) a.kappa[row] = kap;
      if (!yok) raise_status(a.status, 1);
      if (nonfinite) raise_status(a.status, 2);
    }
  }
}

}  // namespace fwb200
