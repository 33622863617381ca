// FW loss on top of an LM head, logits = hidden [B, D] x weight[C, D]^T,
// without a resident [B, C] logit matrix and with a sparse backward.
//
// Forward (host side: fwloss_b200/lm_head.py): the logits are produced one
// column chunk at a time by the GEMM; each chunk is summarised by the fused
// kernel in kOutShard mode (per row: chunk max, the chunk's own support,
// up to K values and their columns) and fw_label_logit_kernel keeps z_y.
// fw_chunks_solve_kernel then combines the chunk summaries of a row exactly
// as for class-sharded rows (the global threshold is >= each chunk's own
// threshold, so the union of the chunk supports contains the row's support),
// and writes H, kappa, the loss and the support's columns.
//
// Backward: the logit gradient of row r is scale * (1/kappa on the support,
// -1 at the label), i.e. kappa + 1 non-zeros.  So
//   dhidden[r] = go * scale * (sum_{j in supp(r)} W[j] / kappa_r - W[y_r])
//   dweight[j] += go * scale * (H[r] / kappa_r  for r with j in supp(r),
//                               -H[r]           for r with y_r = j)
// are row gathers and scatter-adds of kappa + 1 rows per sample, instead of
// two dense [B, C] x [C, D] GEMMs.
#pragma once

#include "fw_device.cuh"
#include "fw_shard.cuh"

namespace fwb200 {

// zy[r] = z[r, y[r] - c0] when y[r] lies in [c0, c0 + C); untouched otherwise.
__global__ void fw_label_logit_kernel(const float* __restrict__ z, int64_t B, int64_t C, int64_t ld,
                                      const int64_t* __restrict__ y, int64_t c0, float* __restrict__ zy) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < B; r += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = y[r] - c0;
    if (j >= 0 && j < C) zy[r] = z[r * ld + j];
  }
}

struct ChunkSolveArgs {
  const int32_t* summaries;  // [nchunks, B, kShardHeader + K]
  const int32_t* local_idx;  // [nchunks, B, K]
  int nchunks;
  int K;
  int64_t B;
  int64_t col_start[kMaxShards + 1];
  const float* zy;           // [B] logit at the label
  const int64_t* y;          // [B]
  float* H;
  int32_t* kappa;            // 0 for rows left to the exact path
  float* loss;
  int32_t* sup_cols;         // [B, nchunks * K] support columns (first kappa entries)
  int32_t* fb_rows;
  int32_t* fb_count;
  int32_t* status;
};

__global__ void __launch_bounds__(kShardSolveThreads)
    fw_chunks_solve_kernel(ChunkSolveArgs a) {
  __shared__ float s_val[kShardSolveThreads / 32][kShardListCap];
  __shared__ int s_col[kShardSolveThreads / 32][kShardListCap];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  float* L = s_val[wib];
  int* LC = s_col[wib];
  const int S = kShardHeader + a.K;
  const int SC = a.nchunks * a.K;
  const int64_t nwarps = (int64_t)gridDim.x * (kShardSolveThreads / 32);
  const int64_t C = a.col_start[a.nchunks];

  for (int64_t row = (int64_t)blockIdx.x * (kShardSolveThreads / 32) + wib; row < a.B; row += nwarps) {
    float Mq = -CUDART_INF_F;
    int kq = 0, fq = 0, iq = -1;
    if (lane < a.nchunks) {
      const int32_t* rec = a.summaries + ((int64_t)lane * a.B + row) * S;
      Mq = __int_as_float(rec[0]);
      kq = rec[1];
      fq = rec[2];
      iq = rec[3];
    }
    const float M = warp_max_nan(Mq);
    const int64_t ylab = a.y[row];
    const bool yok = ylab >= 0 && ylab < C;
    const float zy = yok ? a.zy[row] : CUDART_NAN_F;
    int32_t* cols = a.sup_cols + row * (int64_t)SC;

    if (!isfinite(M)) {
      const bool isn = (M != M);
      const bool match = lane < a.nchunks && (fq & kShardNonFinite) && (isn ? (Mq != Mq) : (Mq == M));
      const unsigned b = __ballot_sync(kFull, match);
      const int owner = b ? __ffs(b) - 1 : 0;
      const int jloc = __shfl_sync(kFull, iq, owner);
      if (lane == 0) {
        cols[0] = (int32_t)(a.col_start[owner] + jloc);
        a.kappa[row] = 1;
        if (a.H) a.H[row] = M;
        if (a.loss) a.loss[row] = yok ? (1.0f - zy + M) : CUDART_NAN_F;
        raise_status(a.status, 2 | (yok ? 0 : 1));
      }
      continue;
    }
    if (__any_sync(kFull, lane < a.nchunks && kq > a.K)) {
      if (lane == 0) {
        a.fb_rows[atomicAdd(a.fb_count, 1)] = (int32_t)row;
        a.kappa[row] = 0;
        if (a.loss) a.loss[row] = 0.0f;
        if (a.H) a.H[row] = CUDART_NAN_F;
      }
      continue;
    }

    // union of the chunk supports above t0 (values and global columns)
    const float t0 = __fsub_rd(M, 1.0f);
    int n = 0;
    for (int q = 0; q < a.nchunks; ++q) {
      const int cnt = __shfl_sync(kFull, kq, q);
      const int32_t* vals = a.summaries + ((int64_t)q * a.B + row) * S + kShardHeader;
      const int32_t* idx = a.local_idx + ((int64_t)q * a.B + row) * a.K;
      for (int k0 = 0; k0 < cnt; k0 += 32) {
        const int k = k0 + lane;
        const float x = (k < cnt) ? __int_as_float(vals[k]) : -CUDART_INF_F;
        const bool keep = x > t0;
        const unsigned b = __ballot_sync(kFull, keep);
        const int pos = n + __popc(b & lanemask_lt(lane));
        if (keep && pos < kShardListCap) {
          L[pos] = x;
          LC[pos] = (int)(a.col_start[q] + idx[k]);
        }
        n += __popc(b);
      }
    }
    n = min(n, kShardListCap);
    __syncwarp();
    double tau;
    int kap;
    michelot_list<32>(L, n, M, lane, kFull, tau, kap);
    const float Hf = threshold_fp32(M, tau);
    int pos0 = 0;
    for (int k0 = 0; k0 < n; k0 += 32) {
      const int k = k0 + lane;
      const bool sel = k < n && L[k] > Hf;
      const unsigned b = __ballot_sync(kFull, sel);
      if (sel) cols[pos0 + __popc(b & lanemask_lt(lane))] = LC[k];
      pos0 += __popc(b);
    }
    __syncwarp();
    if (lane == 0) {
      a.kappa[row] = kap;
      if (a.H) a.H[row] = Hf;
      if (a.loss) a.loss[row] = yok ? row_loss(M, tau, zy) : CUDART_NAN_F;
      if (!yok) raise_status(a.status, 1);
    }
  }
}

struct SparseGradArgs {
  const void* src;       // dhidden: weight [C, D]; dweight: hidden [B, D] (element type T)
  void* dst;             // dhidden: [B, D] (T); dweight: [C, D] fp32, accumulated
  int64_t B, C, D;
  const int32_t* sup_cols;
  int S;                 // row stride of sup_cols
  const int32_t* kappa;  // 0: row handled elsewhere (skipped; dhidden row written as 0)
  const int64_t* y;
  float scale;
  const float* go;       // upstream gradient (device)
  int per_row;
  int64_t c0;            // sup_cols and y are global class ids; src/dst rows of the
                         // weight cover classes [c0, c0 + C) (0 for a whole weight)
};

constexpr int kSparseThreads = 256;
constexpr int kSparseCols = 8;  // D columns per thread per pass

// dhidden[r] = go * scale * (sum_j W[j] / kappa - W[y]); one CTA per row.
// Only the classes j in [c0, c0 + C) held by W contribute (all of them for a
// whole weight); a vocabulary-parallel rank writes its partial sum in fp32
// (TO = float) for the all-reduce.
template <class T, class TO = T>
__global__ void __launch_bounds__(kSparseThreads) fw_sparse_dhidden_kernel(SparseGradArgs a) {
  const T* W = static_cast<const T*>(a.src);
  TO* dH = static_cast<TO*>(a.dst);
  for (int64_t r = blockIdx.x; r < a.B; r += gridDim.x) {
    const int kap = a.kappa[r];
    const int64_t yl = a.y[r] - a.c0;
    const bool yok = yl >= 0 && yl < a.C;
    const float g = a.go[a.per_row ? r : 0] * a.scale;
    const float inv = kap > 0 ? (float)((double)g / (double)kap) : 0.0f;
    const int32_t* cols = a.sup_cols + r * (int64_t)a.S;
    for (int64_t d0 = 0; d0 < a.D; d0 += (int64_t)kSparseThreads * kSparseCols) {
      float acc[kSparseCols];
#pragma unroll
      for (int i = 0; i < kSparseCols; ++i) acc[i] = 0.0f;
      for (int k = 0; k < kap; ++k) {
        const int64_t j = (int64_t)cols[k] - a.c0;
        if (j < 0 || j >= a.C) continue;  // a class held by another rank
        const T* wr = W + j * a.D;
#pragma unroll
        for (int i = 0; i < kSparseCols; ++i) {
          const int64_t d = d0 + (int64_t)i * kSparseThreads + threadIdx.x;
          if (d < a.D) acc[i] += inv * ld_elem(wr + d);
        }
      }
      if (kap > 0 && yok) {
        const T* wr = W + yl * a.D;
#pragma unroll
        for (int i = 0; i < kSparseCols; ++i) {
          const int64_t d = d0 + (int64_t)i * kSparseThreads + threadIdx.x;
          if (d < a.D) acc[i] -= g * ld_elem(wr + d);
        }
      }
#pragma unroll
      for (int i = 0; i < kSparseCols; ++i) {
        const int64_t d = d0 + (int64_t)i * kSparseThreads + threadIdx.x;
        if (d < a.D) st_elem(dH + r * a.D + d, acc[i]);
      }
    }
  }
}

// dweight[j] += go * scale * (hidden[r] / kappa for j in supp(r), -hidden[r]
// for j = y_r); fp32 accumulation with atomics (order of the additions is not
// fixed).  One CTA per row.
template <class T>
__global__ void __launch_bounds__(kSparseThreads) fw_sparse_dweight_kernel(SparseGradArgs a) {
  const T* Hd = static_cast<const T*>(a.src);
  float* dW = static_cast<float*>(a.dst);
  for (int64_t r = blockIdx.x; r < a.B; r += gridDim.x) {
    const int kap = a.kappa[r];
    if (kap <= 0) continue;
    const int64_t yl = a.y[r];
    const bool yok = yl >= 0 && yl < a.C;
    const float g = a.go[a.per_row ? r : 0] * a.scale;
    const float inv = (float)((double)g / (double)kap);
    const int32_t* cols = a.sup_cols + r * (int64_t)a.S;
    for (int64_t d = threadIdx.x; d < a.D; d += kSparseThreads) {
      const float h = ld_elem(Hd + r * a.D + d);
      for (int k = 0; k < kap; ++k) atomicAdd(dW + (int64_t)cols[k] * a.D + d, inv * h);
      if (yok) atomicAdd(dW + yl * a.D + d, -g * h);
    }
  }
}

// Deterministic dweight.  Contribution keys (j << 32) | (r << 1) | is_label,
// one per non-zero of the logit gradient, are built at fixed shape
// [B, S + 1] (unused slots get kNoKey, which sorts last), sorted, and each run
// of equal column j is summed in key order by the CTA that owns the run's
// first entry (no segment table, no data-dependent shapes):
//   dweight[j] = sum g_r / kappa_r * hidden[r]  (support entries)
//              + sum -g_r * hidden[r]           (label entries)
// Columns without contributions are left to the caller (zero).
constexpr int64_t kNoKey = 0x7fffffffffffffffLL;

// Keys of the classes in [c0, c0 + C) only, with class ids relative to c0
// (c0 = 0 and C = all classes for a whole weight).
__global__ void fw_weight_keys_kernel(const int32_t* __restrict__ sup_cols, int S, const int32_t* __restrict__ kappa,
                                      const int64_t* __restrict__ y, int64_t B, int64_t C, int64_t* __restrict__ keys,
                                      int64_t c0) {
  const int64_t n = B * (int64_t)(S + 1);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / (S + 1);
    const int k = (int)(e - r * (S + 1));
    const int kap = kappa[r];
    int64_t key = kNoKey;
    if (kap > 0) {
      if (k < kap) {
        const int64_t j = (int64_t)sup_cols[r * S + k] - c0;
        if (j >= 0 && j < C) key = (j << 32) | (r << 1);
      } else if (k == S) {
        const int64_t yl = y[r] - c0;
        if (yl >= 0 && yl < C) key = (yl << 32) | (r << 1) | 1;
      }
    }
    keys[e] = key;
  }
}

struct SegmentGradArgs {
  const void* hidden;        // [B, D] (T)
  void* dweight;             // [C, D] (T)
  int64_t B, D;
  const int64_t* keys;       // sorted, kNoKey entries last
  int64_t nkeys;
  const int32_t* kappa;
  float scale;
  const float* go;
  int per_row;
};

constexpr int kSegmentWindow = 32;  // sorted entries scanned for run starts per CTA step

template <class T>
__global__ void __launch_bounds__(kSparseThreads) fw_segment_dweight_kernel(SegmentGradArgs a) {
  const T* Hd = static_cast<const T*>(a.hidden);
  T* dW = static_cast<T*>(a.dweight);
  for (int64_t w0 = (int64_t)blockIdx.x * kSegmentWindow; w0 < a.nkeys; w0 += (int64_t)gridDim.x * kSegmentWindow) {
    const int64_t wend = min(w0 + kSegmentWindow, a.nkeys);
    for (int64_t e0 = w0; e0 < wend; ++e0) {
      const int64_t k0 = a.keys[e0];
      if (k0 == kNoKey) return;  // the rest of the array is unused slots
      const int64_t j = k0 >> 32;
      if (e0 > 0 && (a.keys[e0 - 1] >> 32) == j) continue;  // not the first entry of its run
      int64_t e1 = e0 + 1;
      while (e1 < a.nkeys && a.keys[e1] != kNoKey && (a.keys[e1] >> 32) == j) ++e1;
      for (int64_t d0 = 0; d0 < a.D; d0 += (int64_t)kSparseThreads * kSparseCols) {
        float acc[kSparseCols];
#pragma unroll
        for (int i = 0; i < kSparseCols; ++i) acc[i] = 0.0f;
        for (int64_t e = e0; e < e1; ++e) {
          const int64_t key = a.keys[e];
          const int64_t r = (key >> 1) & 0x7fffffffLL;
          const float g = a.go[a.per_row ? r : 0] * a.scale;
          const float coef = (key & 1) ? -g : (float)((double)g / (double)a.kappa[r]);
          const T* hr = Hd + r * a.D;
#pragma unroll
          for (int i = 0; i < kSparseCols; ++i) {
            const int64_t d = d0 + (int64_t)i * kSparseThreads + threadIdx.x;
            if (d < a.D) acc[i] += coef * ld_elem(hr + d);
          }
        }
#pragma unroll
        for (int i = 0; i < kSparseCols; ++i) {
          const int64_t d = d0 + (int64_t)i * kSparseThreads + threadIdx.x;
          if (d < a.D) st_elem(dW + j * a.D + d, acc[i]);
        }
      }
    }
  }
}

}  // namespace fwb200
