// Register tier (C <= 2048): a group of G lanes (G = 8, 16 or 32; 32/G rows
// per warp) holds one row in registers, so the row is read from HBM once and
// its output written once, with no shared-memory traffic except the short
// candidate list.  Element type T = float, bf16 or fp16 (arithmetic in
// fp32/fp64); a lane owns NS 16-byte slots of EPS elements.
//
// Per row:
//   1. load (16-byte loads when rows are 16-byte aligned), M = NaN-propagating
//      max by xor shuffles inside the group;
//   2. n = |{z > t0}|; a unique maximum (n == 1) is solved on the spot
//      (kappa = 1, h* = M - 1), and so are more than G candidates that all
//      equal M (kappa = n, h* = M - 1/n; rows of up to 16 values per lane);
//      otherwise the candidates are
//      compacted into a per-group list by an exclusive shuffle scan;
//   3. exact threshold: Michelot's fixed point with one candidate per lane
//      when there are at most G of them (michelot_lane: counts are a
//      ballot), on the list otherwise (michelot_list), or on the registers
//      when the list would overflow (near-constant rows where most of the
//      row is within 1 of the max); every form reduces the kept count first
//      and the fp64 sum only while the kept set changes;
//   4. output straight from the registers with the fp32 predicate z > H:
//      the gradient grad_scale * ((1/kappa) [z > h*] - e_y), the support mask,
//      or the support list.
//
// Reference counterpart: fw_radix_shared_kernel<8,32,100> / <8,128,5000>
// (src/cuda/fw_radix_argmax.cu:1192-1356) followed by fw_backward_mask_kernel
// (:1561-1589).  The reference finds h* by up to four 8-bit digit passes with
// four shared-memory atomics per element, writes a bool mask, and needs a
// second kernel to turn it into the gradient; here the threshold comes from
// the candidate list and the gradient is written by the same lanes.
#pragma once

#include <climits>

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kWarpListCap = 128;  // list entries per warp, split between its groups

// Column of register value (i, j) (slot i, element j) of lane `li` of a G-lane
// group.  Aligned rows use 16-byte loads (a lane owns EPS consecutive columns
// per slot); unaligned rows use lane-contiguous scalar loads so every load
// instruction coalesces.
template <int G, int EPS, bool VEC>
__device__ __forceinline__ int group_slot_col(int i, int j, int li) {
  return VEC ? ((i * G + li) * EPS + j) : ((i * EPS + j) * G + li);
}

// Stores the EPS values of slot i.  FULLV: C % EPS == 0 (a slot is entirely
// inside or outside the row).
template <class T, int G, bool VEC, bool FULLV>
__device__ __forceinline__ void warp_tier_store_slot(T* gr, int i, int li, int C, const float* g) {
  constexpr int EPS = Elem<T>::kEPS;
  if (VEC) {
    const int c0 = (i * G + li) * EPS;
    if (FULLV || c0 + EPS - 1 < C) {
      if (FULLV && c0 >= C) return;
      *reinterpret_cast<uint4*>(gr + c0) = pack16<T>(g);
    } else {
#pragma unroll
      for (int j = 0; j < EPS; ++j)
        if (c0 + j < C) st_elem(gr + c0 + j, g[j]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < EPS; ++j) {
      const int c = group_slot_col<G, EPS, false>(i, j, li);
      if (c < C) st_elem(gr + c, g[j]);
    }
  }
}

template <int G, bool VEC, bool FULLV>
__device__ __forceinline__ void warp_tier_store_mask(uint8_t* mr, int i, int li, int C, int mask_vec,
                                                     const uint8_t (&b)[4]) {
  const int c0 = (i * G + li) * 4;
  if (VEC && mask_vec && (FULLV || c0 + 3 < C)) {
    if (FULLV && c0 >= C) return;
    *reinterpret_cast<uchar4*>(mr + c0) = make_uchar4(b[0], b[1], b[2], b[3]);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = group_slot_col<G, 4, VEC>(i, j, li);
      if (c < C) mr[c] = b[j];
    }
  }
}

// Row whose maximum is NaN or +-inf: kappa = 1 at the first column holding
// the maximum (the first NaN for NaN rows), H = M, loss = 1 - z_y + M (fp32).
template <class T, int G, int NS, bool VEC, int OUT>
__device__ __forceinline__ void warp_tier_nonfinite(const RowArgs& a, int64_t row,
                                                    const float (&v)[NS * Elem<T>::kEPS], float m,
                                                    int li, unsigned gmask, int yc, float zy) {
  constexpr int EPS = Elem<T>::kEPS;
  const int C = (int)a.C;
  const bool isn = (m != m);
  unsigned best = 0xffffffffu;
#pragma unroll
  for (int i = 0; i < NS; ++i)
#pragma unroll
    for (int j = 0; j < EPS; ++j) {
      const int c = group_slot_col<G, EPS, VEC>(i, j, li);
      const float x = v[EPS * i + j];
      if (c < C && (isn ? (x != x) : (x == m))) best = min(best, (unsigned)c);
    }
  const int jstar = (int)group_min<G>(best, gmask);
  if (OUT == kOutGrad || OUT == kOutGradCols) {
    T* gr = static_cast<T*>(a.grad) + row * a.ld;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      float g[EPS];
#pragma unroll
      for (int j = 0; j < EPS; ++j)
        g[j] = (group_slot_col<G, EPS, VEC>(i, j, li) == jstar) ? a.scale : 0.0f;
      warp_tier_store_slot<T, G, VEC, false>(gr, i, li, C, g);
    }
    if (yc >= 0) {
      __syncwarp(gmask);
      if (li == 0) st_elem(gr + yc, ((yc == jstar) ? a.scale : 0.0f) - a.scale);
    }
    if (OUT == kOutGradCols && li == 0) a.sup_cols[row * (int64_t)a.sup_k] = jstar;
  } else if (OUT == kOutMask) {
    uint8_t* mr = a.mask + row * a.C;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      uint8_t b[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = (group_slot_col<G, 4, VEC>(i, j, li) == jstar) ? 1 : 0;
      warp_tier_store_mask<G, VEC, false>(mr, i, li, C, a.mask_vec, b);
    }
  } else if (OUT == kOutCand) {
    if (li == 0) {
      a.cand_val[row * a.C] = ld_elem(static_cast<const T*>(a.z) + row * a.ld + jstar);
      a.cand_idx[row * a.C] = jstar;
      if (a.cand_count) a.cand_count[row] = 1;
    }
  } else if (OUT == kOutNone) {
    // forward only: no per-element output
  } else {  // kOutShard: zero gradient shard (if any), summary of a non-finite row
    if (a.grad) {
      T* gr = static_cast<T*>(a.grad) + row * a.ld;
      const float zero[Elem<T>::kEPS] = {};
#pragma unroll
      for (int i = 0; i < NS; ++i) warp_tier_store_slot<T, G, VEC, false>(gr, i, li, C, zero);
    }
    if (li == 0) {
      int32_t* rec = a.shard_sum + row * (int64_t)(kShardHeader + a.shard_k);
      rec[0] = __float_as_int(m);
      rec[1] = 1;
      rec[2] = kShardNonFinite;
      rec[3] = jstar;
      if (a.shard_k > 0) {
        rec[kShardHeader] = __float_as_int(m);
        a.shard_idx[row * (int64_t)a.shard_k] = jstar;
      }
    }
    return;
  }
  if (li == 0) {
    if (a.H) a.H[row] = m;
    if (a.loss) a.loss[row] = (yc >= 0) ? (1.0f - zy + m) : CUDART_NAN_F;
    if (a.kappa) a.kappa[row] = 1;
    if (yc < 0) raise_status(a.status, 1);
    raise_status(a.status, 2);
  }
}

// Threads per CTA and resident CTAs per SM the register budget is sized
// for, by register values per lane NV.  Short rows are latency- and
// issue-bound (a serial chain per row: load, max, solve, write), so the
// budgets keep every row of a few-thousand-row batch resident at once:
//   NV <= 16   256 threads x 4 CTAs (64 registers);
//   NV == 32   128 threads x 7 CTAs (73 registers): 4144 resident
//              warps on 148 SMs, one per row of a 4096-row batch;
//   NV == 64   256 threads x 1 CTA.
template <int NV>
__host__ __device__ constexpr int warp_tier_threads() {
  return NV == 32 ? 128 : 256;
}

template <int NV>
__host__ __device__ constexpr int warp_tier_min_blocks() {
  return NV <= 16 ? 4 : (NV == 32 ? 7 : 1);
}

template <class T, int G, int NS, bool VEC, int OUT, bool FULLV>
__global__ void __launch_bounds__(warp_tier_threads<NS * Elem<T>::kEPS>(),
                                  warp_tier_min_blocks<NS * Elem<T>::kEPS>())
    fw_warp_rows_kernel(RowArgs a) {
  allow_dependent_launch();
  constexpr int EPS = Elem<T>::kEPS;
  constexpr int NV = NS * EPS;          // register values per lane
  constexpr int WW = warp_tier_threads<NV>() / 32;  // warps per CTA
  constexpr int RPW = 32 / G;           // rows per warp
  constexpr int CAPG = kWarpListCap / RPW;
  static_assert(OUT == kOutGrad || OUT == kOutGradCols || OUT == kOutNone || sizeof(T) == 4,
                "mask/candidate/shard outputs are fp32-only");
  __shared__ float s_list[WW][kWarpListCap];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int gi = lane / G;              // group in warp
  const int li = lane % G;              // lane in group
  const unsigned gmask = (G == 32) ? kFull : (((1u << G) - 1u) << (gi * G));
  float* L = &s_list[wib][gi * CAPG];
  const int C = (int)a.C;
  const int64_t ngroups = (int64_t)gridDim.x * WW * RPW;
  const T* zbase = static_cast<const T*>(a.z);

  for (int64_t row = ((int64_t)blockIdx.x * WW + wib) * RPW + gi; row < a.B;
       row += ngroups) {
    const T* zr = zbase + row * a.ld;
    const int64_t ylab = a.y ? a.y[row] : -1;  // no labels in kOutShard
    float v[NV];
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      if (VEC) {
        const int c0 = (i * G + li) * EPS;
        if (FULLV || c0 + EPS - 1 < C) {
          uint4 u = make_uint4(0u, 0u, 0u, 0u);
          const bool in = !FULLV || c0 < C;
          if (in) u = ld_stream16(zr + c0);
          unpack16<T>(u, &v[EPS * i]);
          if (!in) {
#pragma unroll
            for (int j = 0; j < EPS; ++j) v[EPS * i + j] = -CUDART_INF_F;
          }
        } else {
#pragma unroll
          for (int j = 0; j < EPS; ++j)
            v[EPS * i + j] = (c0 + j < C) ? ld_elem(zr + c0 + j) : -CUDART_INF_F;
        }
      } else {
#pragma unroll
        for (int j = 0; j < EPS; ++j) {
          const int c = group_slot_col<G, EPS, false>(i, j, li);
          v[EPS * i + j] = (c < C) ? ld_elem(zr + c) : -CUDART_INF_F;
        }
      }
    }

    // the label logit: its load is issued now, under the row's loads
    const bool yok = (ylab >= 0 && ylab < a.C);
    const int yc = yok ? (int)ylab : -1;
    const float zy = yok ? ld_elem(zr + yc) : CUDART_NAN_F;

    float m = -CUDART_INF_F;
#pragma unroll
    for (int s = 0; s < NV; ++s) m = max_nan(m, v[s]);
    m = group_max_nan<G>(m, gmask);

    if (!isfinite(m)) {  // group-uniform; rare
      warp_tier_nonfinite<T, G, NS, VEC, OUT>(a, row, v, m, li, gmask, yc, zy);
      continue;
    }

    const float t0 = __fsub_rd(m, 1.0f);
    int c = 0;
#pragma unroll
    for (int s = 0; s < NV; ++s) c += (v[s] > t0) ? 1 : 0;
    const int n = group_sum<G>(c, gmask);
    double tau;
    int kap;
    // More candidates than lanes: are they all equal to the maximum (ties of
    // quantized logits)?  Then the fixed point ends at its first step,
    // kappa = n and h* = M - 1/n (sum of z - M over the set is 0; bit-equal
    // to what the list form computes), without the list.  Checked with at
    // most 16 values per lane (the 32-value instance has no registers left
    // for it under its 7-CTAs-per-SM budget).
    bool ties = false;
    if (NV <= 16 && n > G) {
      int e = 0;
#pragma unroll
      for (int s = 0; s < NV; ++s) e += (v[s] == m) ? 1 : 0;
      ties = group_sum<G>(e, gmask) == n;
    }
    if (n == 1) {
      // a unique maximum and nothing else above M - 1: h* = M - 1, kappa = 1
      tau = -1.0;
      kap = 1;
    } else if (ties) {
      tau = (0.0 - 1.0) / (double)n;
      kap = n;
    } else if (n <= CAPG) {
      int off = group_excl_scan<G>(c, li, gmask);
      if (c > 0) {
#pragma unroll
        for (int s = 0; s < NV; ++s)
          if (v[s] > t0) L[off++] = v[s];
      }
      __syncwarp(gmask);
      if (n <= G)  // one candidate per lane
        michelot_lane<G>(li < n ? L[li] : -CUDART_INF_F, n, m, gmask, tau, kap);
      else
        michelot_list<G, CAPG>(L, n, m, li, gmask, tau, kap);
      __syncwarp(gmask);
    } else {
      // more candidates than the list holds (near-constant rows): the same
      // fixed point on the registers
      michelot_regs<G, NV>(v, m, t0, gmask, tau, kap);
    }
    const float Hf = threshold_fp32(m, tau);  // x > Hf <=> x in the support

    if (OUT == kOutGrad || OUT == kOutGradCols) {
      // Support entries first; the label entry is rewritten by lane 0 after a
      // group barrier (which orders the two stores to that address).
      // correctly rounded in fp32, equal to the fp64 quotient rounded to fp32
      const float inv = __fdiv_rn(a.scale, (float)kap);
      T* gr = static_cast<T*>(a.grad) + row * a.ld;
#pragma unroll
      for (int i = 0; i < NS; ++i) {
        float g[EPS];
#pragma unroll
        for (int j = 0; j < EPS; ++j) g[j] = (v[EPS * i + j] > Hf) ? inv : 0.0f;
        warp_tier_store_slot<T, G, VEC, FULLV>(gr, i, li, C, g);
      }
      if (yok) {
        __syncwarp(gmask);
        if (li == 0) st_elem(gr + yc, ((zy > Hf) ? inv : 0.0f) - a.scale);
      }
      if constexpr (OUT == kOutGradCols) {  // the support's columns, in lane order (first sup_k)
        int cnt = 0;
#pragma unroll
        for (int s = 0; s < NV; ++s) cnt += (v[s] > Hf) ? 1 : 0;
        int off = group_excl_scan<G>(cnt, li, gmask);
        int32_t* sc = a.sup_cols + row * (int64_t)a.sup_k;
        if (cnt > 0 && off < a.sup_k) {
#pragma unroll
          for (int i = 0; i < NS; ++i)
#pragma unroll
            for (int j = 0; j < EPS; ++j)
              if (v[EPS * i + j] > Hf) {
                if (off < a.sup_k) sc[off] = group_slot_col<G, EPS, VEC>(i, j, li);
                ++off;
              }
        }
      }
    } else if (OUT == kOutMask) {
      uint8_t* mr = a.mask + row * a.C;
#pragma unroll
      for (int i = 0; i < NS; ++i) {
        uint8_t b[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = (v[4 * i + j] > Hf) ? 1 : 0;
        warp_tier_store_mask<G, VEC, FULLV>(mr, i, li, C, a.mask_vec, b);
      }
    } else if (OUT == kOutShard) {
      // zero gradient shard (if any); the support goes to the summary record
      if (a.grad) {
        T* gr = static_cast<T*>(a.grad) + row * a.ld;
        const float zero[EPS] = {};
#pragma unroll
        for (int i = 0; i < NS; ++i) warp_tier_store_slot<T, G, VEC, FULLV>(gr, i, li, C, zero);
      }
      int cnt = 0;
#pragma unroll
      for (int s = 0; s < NV; ++s) cnt += (v[s] > Hf) ? 1 : 0;
      int off = group_excl_scan<G>(cnt, li, gmask);
      const int K = a.shard_k;
      int32_t* rec = a.shard_sum + row * (int64_t)(kShardHeader + K);
      int32_t* ridx = a.shard_idx + row * (int64_t)K;
      if (cnt > 0 && off < K) {
#pragma unroll
        for (int i = 0; i < NS; ++i)
#pragma unroll
          for (int j = 0; j < EPS; ++j)
            if (v[EPS * i + j] > Hf) {
              if (off < K) {
                rec[kShardHeader + off] = __float_as_int(v[EPS * i + j]);
                ridx[off] = group_slot_col<G, EPS, VEC>(i, j, li);
              }
              ++off;
            }
      }
      if (li == 0) {
        rec[0] = __float_as_int(m);
        rec[1] = kap;
        rec[2] = 0;
        rec[3] = -1;
      }
      continue;
    } else if (OUT == kOutNone) {
      // forward only: H, loss and kappa below
    } else {  // kOutCand
      int cnt = 0;
#pragma unroll
      for (int s = 0; s < NV; ++s) cnt += (v[s] > Hf) ? 1 : 0;
      int off = group_excl_scan<G>(cnt, li, gmask);
      float* cv = a.cand_val + row * a.C;
      int32_t* ci = a.cand_idx + row * a.C;
      if (cnt > 0) {
#pragma unroll
        for (int i = 0; i < NS; ++i)
#pragma unroll
          for (int j = 0; j < EPS; ++j)
            if (v[EPS * i + j] > Hf) {
              cv[off] = v[EPS * i + j];
              ci[off] = group_slot_col<G, EPS, VEC>(i, j, li);
              ++off;
            }
      }
      if (li == 0 && a.cand_count) a.cand_count[row] = kap;
    }

    if (li == 0) {
      if (a.H) a.H[row] = Hf;
      if (a.loss) a.loss[row] = yok ? row_loss(m, tau, zy) : CUDART_NAN_F;
      if (a.kappa) a.kappa[row] = kap;
      if (!yok) raise_status(a.status, 1);
    }
  }
}

}  // namespace fwb200
