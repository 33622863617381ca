// fp64 logits.  The reference's CPU kernel dispatches float64 rows
// (src/cpu/fw_cpu.cpp:698-704, fw_row<double> at :419-470: fp64 loss and
// gradient); its CUDA kernels are fp32-only (src/cuda/fw_radix_argmax.cu:1387,
// 1422).
//
// One team of TW warps per row: TW = 1 for C <= kF64WarpRowMaxC (eight rows
// per CTA), TW = 8 for longer rows (one row per CTA).  The structure is the
// one of the fp32 streaming tier:
//
//   stream   one pass over the row with 16-byte loads: zero gradient, a
//            NaN-propagating running max per warp, and a per-warp list of the
//            elements above (running max - 1), re-filtered when it fills up;
//   solve    the row max M and t0 = M - 1 rounded down; the listed
//            candidates above t0 (a superset of the support) are gathered in
//            a fixed order and Michelot's fixed point runs on them;
//   patch    the support entries and the label entry are written over the
//            zeros (after a team barrier, so they win).
//
// Selection predicate.  No wider type holds z - M exactly, so the support is
// {x : x > t0 and fl(x - M) > tau}, fl being the round-to-nearest fp64
// subtraction.  fl(x - M) is non-decreasing in x, so this is the set of the
// kappa largest elements, and kappa, the gradient and the loss all use this
// one predicate.  When M >= 2 every candidate satisfies M/2 <= x <= M, so
// x - M is exact (Sterbenz) and the predicate is exact; otherwise results
// agree with exact arithmetic up to fp64 rounding.  H is reported as
// fl(M + tau).
//
// Dense rows (some warp list overflows even after re-filtering: more than
// kF64ListCap of the warp's elements within 1 of its max) run Michelot's
// iteration over the row itself: each step is one pass summing fl(x - M)
// over the elements above the current threshold.  The threshold never
// decreases, so the sets are nested and the loop ends after at most
// (candidates + 1) passes; near-constant rows need two or three.
#pragma once

#include <climits>

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kF64Threads = 256;
constexpr int kF64Warps = kF64Threads / 32;
constexpr int kF64ListCap = 128;          // candidates per warp list
constexpr int kF64SolveCap = 1024;        // gathered candidates per row (TW = 8)
constexpr int64_t kF64WarpRowMaxC = 1024;  // longest row given to one warp

struct F64Args {
  const double* z;   // [B, ld]
  const int64_t* y;  // [B]
  int64_t B;
  int64_t C;
  int64_t ld;
  double scale;      // gradient scale (1/B for "mean")
  double* grad;      // [B, ld]; null: forward only (H, loss, kappa), the GRAD = false instance
  double* H;         // [B] or null
  double* loss;      // [B] or null
  int32_t* kappa;    // [B] or null
  int32_t* status;   // device word or null
};

// max() that returns NaN when either input is NaN.
__device__ __forceinline__ double max_nan64(double a, double b) { return (a > b || a != a) ? a : b; }

__device__ __forceinline__ double warp_max_nan64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max_nan64(v, __shfl_xor_sync(kFull, v, o));
  return __shfl_sync(kFull, v, 0);  // one value for every lane (+-0 ties)
}

__device__ __forceinline__ double ld_stream_f64(const double* p) {
  double r;
  asm volatile("ld.global.nc.L1::no_allocate.f64 %0, [%1];" : "=d"(r) : "l"(p));
  return r;
}

// Keeps the entries > t of a warp list, in order.  Warp-collective.
__device__ __forceinline__ int f64_list_compact(double* lz, int* li, int cnt, double t, int lane) {
  constexpr int PER = kF64ListCap / 32;
  __syncwarp();
  double vv[PER];
  int ii[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = k * 32 + lane;
    vv[k] = (e < cnt) ? lz[e] : -CUDART_INF;
    ii[k] = (e < cnt) ? li[e] : 0;
  }
  __syncwarp();
  int n = 0;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const bool keep = vv[k] > t;
    const unsigned b = __ballot_sync(kFull, keep);
    if (keep) {
      const int pos = n + __popc(b & lanemask_lt(lane));
      lz[pos] = vv[k];
      li[pos] = ii[k];
    }
    n += __popc(b);
  }
  __syncwarp();
  return n;
}

// Appends (val, col) for lanes with pred.  Warp-collective; cnt and ovf are
// warp-uniform.
__device__ __forceinline__ void f64_list_append(double* lz, int* li, int& cnt, bool& ovf, double val,
                                                int col, bool pred, double t, int lane) {
  const unsigned b = __ballot_sync(kFull, pred);
  if (b == 0u || ovf) return;
  const int k = __popc(b);
  if (cnt + k > kF64ListCap) {
    cnt = f64_list_compact(lz, li, cnt, t, lane);
    if (cnt + k > kF64ListCap) {
      ovf = true;
      return;
    }
  }
  if (pred) {
    const int pos = cnt + __popc(b & lanemask_lt(lane));
    lz[pos] = val;
    li[pos] = col;
  }
  cnt += k;
}

// Michelot's fixed point on n >= 1 fp64 candidates (all > t0, the row max
// among them): T <- {x : fl(x - M) > tau}, tau = (sum_T fl(x - M) - 1)/|T|,
// tau never decreasing, until |T| repeats.  Fixed-order fp64 sums (lane
// strided, then a butterfly).  Warp-collective; every lane returns the same.
__device__ __forceinline__ void michelot_list64(const double* L, int n, double M, int lane, double& tau,
                                                int& kappa) {
  double t = -CUDART_INF;
  int prev = -1;
  for (int it = 0; it <= n; ++it) {
    double s = 0.0;
    int c = 0;
    for (int i = lane; i < n; i += 32) {
      const double d = L[i] - M;
      if (d > t) {
        s += d;
        ++c;
      }
    }
    c = warp_sum(c);
    s = warp_sum(s);
    if (c == prev) break;
    prev = c;
    t = fmax(t, (s - 1.0) / (double)c);
  }
  tau = t;
  kappa = prev;
}

template <int TW>
__device__ __forceinline__ void f64_team_sync() {
  if constexpr (TW == 1) {
    __syncwarp();
  } else {
    __syncthreads();
  }
}

// GRAD: write the gradient (a.grad); without it, forward only.
template <int TW, bool VEC, bool GRAD>
__global__ void __launch_bounds__(kF64Threads) fw_f64_rows_kernel(F64Args a) {
  allow_dependent_launch();
  constexpr int NT = 32 * TW;          // threads per row
  constexpr int RPB = kF64Warps / TW;  // rows per CTA
  constexpr int W = VEC ? 2 : 1;       // doubles per item
  constexpr int IPT = VEC ? 4 : 8;     // items per thread per streaming step
  constexpr int SOLVE = TW > 1 ? kF64SolveCap : 1;
  __shared__ double s_lz[kF64Warps][kF64ListCap];
  __shared__ int s_li[kF64Warps][kF64ListCap];
  __shared__ double s_sz[SOLVE];
  __shared__ int s_si[SOLVE];
  __shared__ double s_wmax[kF64Warps];
  __shared__ double s_rs[kF64Warps];
  __shared__ int s_rc[kF64Warps];
  __shared__ int s_wovf[kF64Warps];
  __shared__ int s_first[RPB];
  __shared__ int s_n;
  __shared__ int s_dense;

  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int team = w / TW;
  const int tw = w % TW;
  const int tt = tw * 32 + lane;
  const int64_t C = a.C;
  const int64_t nitems = VEC ? C / 2 : C;
  double* lz = s_lz[w];
  int* li = s_li[w];

  for (int64_t row0 = (int64_t)blockIdx.x * RPB; row0 < a.B; row0 += (int64_t)gridDim.x * RPB) {
    const int64_t row = row0 + team;
    if (row < a.B) {  // team-uniform (TW = 8: RPB = 1, block-uniform)
      const double* zr = a.z + row * a.ld;
      double* gr = GRAD ? a.grad + row * a.ld : nullptr;
      if (tt == 0) s_first[team] = INT_MAX;

      // ------------------------------------------------------------ stream
      double run = -CUDART_INF;
      int cnt = 0;
      bool ovf = false;
      for (int64_t base = 0; base < nitems; base += (int64_t)NT * IPT) {
        double v[IPT * W];
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
          const int64_t it = base + (int64_t)u * NT + tt;
          if (VEC) {
            if (it < nitems) {
              const uint4 q = ld_stream16(zr + 2 * it);
              v[2 * u] = __hiloint2double((int)q.y, (int)q.x);
              v[2 * u + 1] = __hiloint2double((int)q.w, (int)q.z);
            } else {
              v[2 * u] = -CUDART_INF;
              v[2 * u + 1] = -CUDART_INF;
            }
          } else {
            v[u] = (it < nitems) ? ld_stream_f64(zr + it) : -CUDART_INF;
          }
        }
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
          const int64_t it = base + (int64_t)u * NT + tt;
          if (GRAD && it < nitems) {
            if (VEC)
              *reinterpret_cast<uint4*>(gr + 2 * it) = make_uint4(0u, 0u, 0u, 0u);
            else
              gr[it] = 0.0;
          }
        }
        double m = -CUDART_INF;
#pragma unroll
        for (int k = 0; k < IPT * W; ++k) m = max_nan64(m, v[k]);
        run = max_nan64(run, warp_max_nan64(m));
        const double t = __dsub_rd(run, 1.0);
        bool anyc = false;
#pragma unroll
        for (int k = 0; k < IPT * W; ++k) anyc |= (v[k] > t);
        if (__any_sync(kFull, anyc)) {
#pragma unroll
          for (int u = 0; u < IPT; ++u) {
            const int64_t it = base + (int64_t)u * NT + tt;
#pragma unroll
            for (int j = 0; j < W; ++j)
              f64_list_append(lz, li, cnt, ovf, v[u * W + j], (int)(it * W + j), v[u * W + j] > t, t, lane);
          }
        }
      }
      if (VEC && (C & 1) && tw == 0) {  // odd C: the last column
        const int64_t c = C - 1;
        const double x = (lane == 0) ? zr[c] : -CUDART_INF;
        if (GRAD && lane == 0) gr[c] = 0.0;
        run = max_nan64(run, warp_max_nan64(x));
        const double t = __dsub_rd(run, 1.0);
        f64_list_append(lz, li, cnt, ovf, x, (int)c, x > t, t, lane);
      }

      // --------------------------------------------------------- row max
      double M;
      bool dense;
      if constexpr (TW == 1) {
        M = run;
        dense = ovf;
        __syncwarp();
      } else {
        if (lane == 0) {
          s_wmax[w] = run;
          s_wovf[w] = ovf ? 1 : 0;
        }
        __syncthreads();
        M = -CUDART_INF;
        int o = 0;
#pragma unroll
        for (int k = 0; k < TW; ++k) {
          M = max_nan64(M, s_wmax[k]);
          o |= s_wovf[k];
        }
        dense = o != 0;
      }
      const double t0 = __dsub_rd(M, 1.0);
      const int64_t ylab = a.y[row];
      const bool yok = ylab >= 0 && ylab < C;
      const int64_t yc = yok ? ylab : -1;

      if (!isfinite(M)) {
        // ---------------------------------------------- non-finite rows
        // kappa = 1 at the first column holding the maximum (first NaN)
        const bool isn = (M != M);
        int best = INT_MAX;
        for (int64_t c = tt; c < C; c += NT) {
          const double x = zr[c];
          if (isn ? (x != x) : (x == M)) {
            best = (int)c;
            break;
          }
        }
        best = (int)__reduce_min_sync(kFull, (unsigned)best);
        if (lane == 0) atomicMin(&s_first[team], best);
        f64_team_sync<TW>();
        // some element equals M (the padding is -inf and only raises nothing)
        const int j = min(s_first[team], (int)(C - 1));
        if (tt == 0) {
          const double zy = yok ? zr[yc] : CUDART_NAN;
          if (GRAD) gr[j] = a.scale - ((j == yc) ? a.scale : 0.0);
          if (GRAD && yok && j != yc) gr[yc] = -a.scale;
          if (a.H) a.H[row] = M;
          if (a.loss) a.loss[row] = yok ? (1.0 - zy + M) : CUDART_NAN;
          if (a.kappa) a.kappa[row] = 1;
          raise_status(a.status, 2 | (yok ? 0 : 1));
        }
      } else {
        // ------------------------------------------------ sparse rows
        int n = 0;
        const double* L = lz;
        const int* LI = li;
        if (!dense) {
          if constexpr (TW == 1) {
            n = f64_list_compact(lz, li, cnt, t0, lane);
          } else {
            if (lane == 0) s_rc[w] = cnt;
            __syncthreads();
            if (w == 0) {
              bool full = false;
              for (int ww = 0; ww < TW && !full; ++ww) {
                const int cw = s_rc[ww];
                for (int k0 = 0; k0 < cw; k0 += 32) {
                  const int k = k0 + lane;
                  const double val = (k < cw) ? s_lz[ww][k] : -CUDART_INF;
                  const int col = (k < cw) ? s_li[ww][k] : 0;
                  const bool keep = val > t0;
                  const unsigned b = __ballot_sync(kFull, keep);
                  if (n + __popc(b) > kF64SolveCap) {
                    full = true;
                    break;
                  }
                  if (keep) {
                    const int pos = n + __popc(b & lanemask_lt(lane));
                    s_sz[pos] = val;
                    s_si[pos] = col;
                  }
                  n += __popc(b);
                }
              }
              if (lane == 0) {
                s_n = n;
                s_dense = full ? 1 : 0;
              }
            }
            __syncthreads();
            n = s_n;
            dense = s_dense != 0;
            L = s_sz;
            LI = s_si;
          }
        }
        if (!dense) {
          if (w == team * TW) {  // the team's first warp solves and patches
            double tau;
            int kap;
            michelot_list64(L, n, M, lane, tau, kap);
            const double inv = a.scale / (double)kap;
            bool ysel = false;
            for (int k = lane; k < n; k += 32) {
              if (L[k] - M > tau) {
                const int col = LI[k];
                double gv = inv;
                if (col == yc) {
                  gv -= a.scale;
                  ysel = true;
                }
                if (GRAD) gr[col] = gv;
              }
            }
            ysel = __any_sync(kFull, ysel);
            if (lane == 0) {
              if (GRAD && yok && !ysel) gr[yc] = -a.scale;
              const double zy = yok ? zr[yc] : CUDART_NAN;
              if (a.H) a.H[row] = M + tau;
              if (a.loss) a.loss[row] = yok ? (1.0 + (M - zy)) + tau : CUDART_NAN;
              if (a.kappa) a.kappa[row] = kap;
              if (!yok) raise_status(a.status, 1);
            }
          }
        } else {
          // -------------------------------------------------- dense rows
          double t = -CUDART_INF;
          int prev = -1;
          for (int64_t it = 0; it <= C; ++it) {
            double sl = 0.0;
            int cl = 0;
            for (int64_t c = tt; c < C; c += NT) {
              const double x = zr[c];
              if (x > t0) {
                const double d = x - M;
                if (d > t) {
                  sl += d;
                  ++cl;
                }
              }
            }
            sl = warp_sum(sl);
            cl = warp_sum(cl);
            if constexpr (TW > 1) {
              if (lane == 0) {
                s_rs[w] = sl;
                s_rc[w] = cl;
              }
              __syncthreads();
              sl = 0.0;
              cl = 0;
#pragma unroll
              for (int k = 0; k < TW; ++k) {
                sl += s_rs[k];
                cl += s_rc[k];
              }
              __syncthreads();
            }
            if (cl == prev) break;
            prev = cl;
            t = fmax(t, (sl - 1.0) / (double)cl);
          }
          const double tau = t;
          const int kap = prev;
          const double inv = a.scale / (double)kap;
          for (int64_t c = tt; GRAD && c < C; c += NT) {
            const double x = zr[c];
            if (x > t0 && x - M > tau) gr[c] = inv;
          }
          f64_team_sync<TW>();
          if (tt == 0) {
            const double zy = yok ? zr[yc] : CUDART_NAN;
            if (GRAD && yok) gr[yc] = ((zy > t0 && zy - M > tau) ? inv : 0.0) - a.scale;
            if (a.H) a.H[row] = M + tau;
            if (a.loss) a.loss[row] = yok ? (1.0 + (M - zy)) + tau : CUDART_NAN;
            if (a.kappa) a.kappa[row] = kap;
            if (!yok) raise_status(a.status, 1);
          }
        }
      }
    }
    f64_team_sync<TW>();  // shared memory is reused by the next row
  }
}

// Row r of grad *= grad_output[per_row ? r : 0] / assumed (fp64); rows whose
// factor is exactly 1 are skipped, and for finite factors only the non-zero
// entries are rewritten.
__global__ void __launch_bounds__(256)
    fw_scale_grad_f64_kernel(double* __restrict__ grad, const double* __restrict__ grad_output,
                             int per_row, double assumed, int64_t B, int64_t C, int64_t ld) {
  for (int64_t r = blockIdx.x; r < B; r += gridDim.x) {
    const double f = grad_output[per_row ? r : 0] / assumed;
    if (f == 1.0) continue;
    const bool dense = !isfinite(f);
    double* gr = grad + r * ld;
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
      const double g = gr[c];
      if (dense || g != 0.0) gr[c] = g * f;
    }
  }
}

}  // namespace fwb200
