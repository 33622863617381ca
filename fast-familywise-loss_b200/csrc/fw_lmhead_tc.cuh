// LM-head logits and their chunk summaries in one kernel (sm_100a tcgen05):
// logits = hidden [B, D] x weight[C, D]^T are accumulated in tensor memory
// and reduced by the epilogue to the per-(row, chunk) summary records of the
// class-sharded protocol (fw_shard.cuh), so no logit reaches HBM.
// fw_chunks_solve_kernel (fw_lmhead.cuh) then combines the summaries.
//
// Layout: one CTA per SM (persistent), 6 warps:
//   warp 0       TMA producer: 128 x 64 hidden tile + 256 x 64 weight tile
//                per stage (bf16, 128-byte swizzle), kTcStages stages;
//   warp 1       TMEM allocation and the MMA issuer: four
//                tcgen05.mma.kind::f16 (M = 128, N = 256, K = 16) per stage
//                into one of two 256-column fp32 accumulators;
//   warps 2..5   epilogue: each thread owns one row of the 128-row tile
//                (TMEM lane quadrant = warp % 4), reads its 256 accumulator
//                columns with tcgen05.ld and keeps, across the tiles of the
//                chunk, a running maximum and a list of the values above
//                (running maximum - 1) -- a superset of the chunk's own
//                support.  At the chunk's end it solves the chunk's support
//                (Michelot's fixed point on the list, fp64) and writes the
//                summary record; it also captures the label logit.
// A work item is (128-row block, chunk); chunk boundaries are multiples of
// the 256-column tile.  The two accumulators let the epilogue of tile t run
// under the MMAs of tile t + 1.
//
// Exactness: the record is the chunk's own support computed from the fp32
// accumulators, as fw_shard_scan computes it from stored logits.  A chunk
// whose candidate list overflows (more than kTcListCap values within 1 of
// its running max) is recorded with kappa = K + 1, which sends the row to the
// exact full-row path; non-finite maxima are recorded with the first column
// holding them (first NaN), as the other summary producers do.
//
// Every mbarrier wait is bounded: on a timeout the kernel sets status bit
// FWB_STATUS_TIMEOUT and a CTA-wide abort flag, every role leaves its loop,
// the producer waits (bounded) for the TMA loads it issued to land, the MMA
// warp commits to a drain barrier and waits (bounded) for its issued MMAs,
// and only then is TMEM released and the CTA allowed to exit.
#pragma once

#include <cuda.h>

#include "fw_device.cuh"
#include "fw_shard.cuh"

namespace fwb200 {

constexpr int kTcBM = 128;
constexpr int kTcBN = 256;
constexpr int kTcBK = 64;
constexpr int kTcStages = 4;
constexpr int kTcThreads = 192;
constexpr int kTcListCap = 32;
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;
constexpr uint32_t kTcBBytes = kTcBN * kTcBK * 2;
constexpr uint32_t kTcTmemCols = 2 * kTcBN;
// instruction descriptor: fp32 accumulator, bf16 A and B, both K-major,
// N = 256, M = 128
constexpr uint32_t kTcIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTcBN >> 3) << 17) |
                              ((uint32_t)(kTcBM >> 4) << 24);
constexpr uint32_t kTcListBytes = (uint32_t)kTcListCap * kTcBM * 8;  // values + columns
constexpr uint32_t kTcSmemBytes =
    1024 + kTcStages * (kTcABytes + kTcBBytes) + kTcListBytes + 256;
constexpr int kTcStatusTimeout = 4;
constexpr uint64_t kTcWaitLimitNs = 2000000000ull;  // 2 s; a tile's MMAs take ~20 us
constexpr uint64_t kTcDrainLimitNs = 100000000ull;  // 100 ms per drain wait after an abort

struct TcArgs {
  int64_t B;
  int64_t C;
  int64_t D;
  int nchunks;
  int K;
  int n_mblocks;
  int64_t col_start[kMaxShards + 1];
  const int64_t* y;
  float* zy;
  int32_t* summaries;  // [nchunks, B, kShardHeader + K]
  int32_t* local_idx;  // [nchunks, B, K]
  int32_t* status;
};

// Bounded wait for the phase of the given parity, by a whole warp.  Returns
// false for every lane (after raising the abort flag and the status bit) on
// a timeout, or when another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  bool ok = mbar_try(bar, parity);
  if (!ok) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
      if (mbar_try(bar, parity)) {
        ok = true;
        break;
      }
      if (*abort_flag) break;
      if ((i & 255u) == 0 && global_ns() - t0 > kTcWaitLimitNs) break;
    }
  }
  ok = __all_sync(kFull, ok);
  if (!ok && (threadIdx.x & 31) == 0) {
    if (!*abort_flag) raise_status(status, kTcStatusTimeout);
    *abort_flag = 1;
  }
  return ok;
}

// Abort path, one thread: waits (at most kTcDrainLimitNs) for the phase of
// the given parity to complete, i.e. for the asynchronous operations that
// arrive on `bar` to finish writing.  Gives up silently at the limit.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try(bar, parity)) return;
    if ((i & 255u) == 255u && global_ns() - t0 > kTcDrainLimitNs) return;
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// UMMA shared-memory descriptor of a K-major tile in the 128-byte swizzle
// layout written by TMA: 8-row x 128-byte atoms, 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Per-row running state of the epilogue across the tiles of one chunk.
struct TcRowState {
  float run;     // NaN-propagating running maximum
  int n;         // list entries
  bool ovf;      // list overflowed: the row takes the exact path
  int nan_col;   // first NaN column (global), -1 if none
  int pinf_col;  // first +inf column (global), -1 if none
};

// Keeps the list entries > t (in order).  The list is column-major in shared
// memory (entry k of row r at k * kTcBM + r) so that a warp's 32 rows hit 32
// banks.
__device__ __forceinline__ int tc_list_compact(float* lv, int* lc, int r, int n, float t) {
  int m = 0;
  for (int k = 0; k < n; ++k) {
    const float x = lv[k * kTcBM + r];
    if (x > t) {
      lv[m * kTcBM + r] = x;
      lc[m * kTcBM + r] = lc[k * kTcBM + r];
      ++m;
    }
  }
  return m;
}

// Folds 32 accumulator values (global columns col0 .. col0 + 31, of which
// the first `valid` are inside the chunk) into the row state.  Every loop
// over v is unrolled so that v stays in registers.
__device__ __forceinline__ void tc_fold32(const float (&v)[32], int64_t col0, int valid, TcRowState& st,
                                          float* lv, int* lc, int r) {
  float m = -CUDART_INF_F;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < valid) m = max_nan(m, v[i]);
  if (!(fabsf(m) < CUDART_INF_F)) {  // NaN or +-inf inside: record first columns
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < valid && v[i] != v[i] && st.nan_col < 0) st.nan_col = (int)(col0 + i);
      if (i < valid && v[i] == CUDART_INF_F && st.pinf_col < 0) st.pinf_col = (int)(col0 + i);
    }
  }
  st.run = max_nan(st.run, m);
  const float t = __fsub_rd(st.run, 1.0f);
  if (m > t && !st.ovf) {
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) cnt += (i < valid && v[i] > t) ? 1 : 0;
    if (st.n + cnt > kTcListCap) {
      st.n = tc_list_compact(lv, lc, r, st.n, t);
      if (st.n + cnt > kTcListCap) {
        st.ovf = true;
        return;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (i < valid && v[i] > t) {
        lv[st.n * kTcBM + r] = v[i];
        lc[st.n * kTcBM + r] = (int)(col0 + i);
        ++st.n;
      }
    }
  }
}

// Writes the summary record of (row, chunk q) from the row state.
__device__ __forceinline__ void tc_finish_row(const TcArgs& a, int q, int64_t row, TcRowState& st, float* lv,
                                              int* lc, int r) {
  const int K = a.K;
  const int64_t c0 = a.col_start[q];
  int32_t* rec = a.summaries + ((int64_t)q * a.B + row) * (kShardHeader + K);
  int32_t* ridx = a.local_idx + ((int64_t)q * a.B + row) * K;
  const float M = st.run;
  if (!isfinite(M)) {
    // kappa = 1 at the first column holding the maximum (first NaN)
    const int64_t j = (M != M) ? st.nan_col : (M > 0.0f ? st.pinf_col : c0);
    rec[0] = __float_as_int(M);
    rec[1] = 1;
    rec[2] = kShardNonFinite;
    rec[3] = (int32_t)(j - c0);
    rec[kShardHeader] = __float_as_int(M);
    ridx[0] = (int32_t)(j - c0);
    return;
  }
  rec[0] = __float_as_int(M);
  rec[2] = 0;
  rec[3] = -1;
  if (st.ovf) {
    rec[1] = K + 1;  // the chunk support is not known: exact full-row path
    return;
  }
  const float t0 = __fsub_rd(M, 1.0f);
  const int n = tc_list_compact(lv, lc, r, st.n, t0);
  // Michelot's fixed point on the n >= 1 candidates (the maximum is one)
  const double Md = (double)M;
  double tau = -CUDART_INF;
  float Ht = -CUDART_INF_F;
  int prev = -1;
  for (int it = 0; it <= n; ++it) {
    double s = 0.0;
    int c = 0;
    for (int k = 0; k < n; ++k) {
      const float x = lv[k * kTcBM + r];
      if (x > Ht) {
        s += (double)x - Md;
        ++c;
      }
    }
    if (c == prev) break;
    prev = c;
    tau = (s - 1.0) / (double)c;
    Ht = threshold_fp32(M, tau);
  }
  rec[1] = prev;
  int p = 0;
  for (int k = 0; k < n && p < K; ++k) {
    const float x = lv[k * kTcBM + r];
    if (x > Ht) {
      rec[kShardHeader + p] = __float_as_int(x);
      ridx[p] = (int32_t)(lc[k * kTcBM + r] - c0);
      ++p;
    }
  }
}

__global__ void __launch_bounds__(kTcThreads, 1)
    fw_lmhead_tc_kernel(const __grid_constant__ CUtensorMap tm_hidden, const __grid_constant__ CUtensorMap tm_weight,
                        TcArgs a) {
  extern __shared__ uint8_t tc_smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* smA = base;
  uint8_t* smB = base + kTcStages * kTcABytes;
  float* lv = reinterpret_cast<float*>(smB + kTcStages * kTcBBytes);
  int* lc = reinterpret_cast<int*>(lv + kTcListCap * kTcBM);
  uint64_t* bars = reinterpret_cast<uint64_t*>(lc + kTcListCap * kTcBM);
  uint64_t* full = bars;                     // [kTcStages] TMA -> MMA
  uint64_t* empty = bars + kTcStages;        // [kTcStages] MMA -> TMA
  uint64_t* tfull = bars + 2 * kTcStages;    // [2] MMA -> epilogue
  uint64_t* tempty = tfull + 2;              // [2] epilogue -> MMA
  uint64_t* drain = tempty + 2;              // abort path: completion of every issued MMA
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4 * 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTcTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int64_t nwork = (int64_t)a.n_mblocks * a.nchunks;
  const int nk = (int)((a.D + kTcBK - 1) / kTcBK);
  // Work still in flight when a role aborts: bit s of `issued` is set once
  // stage s has had a TMA load issued, bit s of `issued_par` is the parity of
  // that stage's last load; `mma_any` is set once an MMA has been issued.
  uint32_t issued = 0u, issued_par = 0u;
  bool mma_any = false;

  if (warp == 0) {
    // ------------------------------------------- TMA producer (lane 0 issues)
    uint32_t s = 0, ph = 0;
    for (int64_t w = blockIdx.x; w < nwork; w += gridDim.x) {
      const int q = (int)(w / a.n_mblocks);
      const int m0 = (int)(w % a.n_mblocks) * kTcBM;
      for (int64_t n0 = a.col_start[q]; n0 < a.col_start[q + 1]; n0 += kTcBN) {
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.status)) goto done;
          if (lane == 0) {
            mbar_expect_tx(&full[s], kTcABytes + kTcBBytes);
            tma_load_2d(smA + s * kTcABytes, &tm_hidden, kb * kTcBK, m0, &full[s]);
            tma_load_2d(smB + s * kTcBBytes, &tm_weight, kb * kTcBK, (int)n0, &full[s]);
          }
          issued |= 1u << s;
          issued_par = (issued_par & ~(1u << s)) | (ph << s);
          __syncwarp();
          if (++s == kTcStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // --------------------------------------------- MMA issuer (lane 0 issues)
    uint32_t s = 0, ph = 0, acc = 0, aph = 0;
    for (int64_t w = blockIdx.x; w < nwork; w += gridDim.x) {
      const int q = (int)(w / a.n_mblocks);
      for (int64_t n0 = a.col_start[q]; n0 < a.col_start[q + 1]; n0 += kTcBN) {
        if (!mbar_wait(&tempty[acc], aph ^ 1u, abort_flag, a.status)) goto done;
        tc_fence_after();
        const uint32_t d = tmem + acc * kTcBN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_flag, a.status)) goto done;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t sa = smem_u32(smA + s * kTcABytes);
            const uint32_t sb = smem_u32(smB + s * kTcBBytes);
#pragma unroll
            for (int k = 0; k < kTcBK / 16; ++k)
              umma_bf16(d, umma_desc_sw128(sa + 32 * k), umma_desc_sw128(sb + 32 * k), kTcIdesc,
                        (kb | k) != 0 ? 1u : 0u);
            umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
          }
          mma_any = true;
          __syncwarp();
          if (++s == kTcStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (lane == 0) umma_commit(&tfull[acc]);  // accumulator complete
        __syncwarp();
        if (++acc == 2) {
          acc = 0;
          aph ^= 1u;
        }
      }
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int quad = warp & 3;  // TMEM lanes this warp may read
    const int r = quad * 32 + lane;
    uint32_t acc = 0, aph = 0;
    for (int64_t w = blockIdx.x; w < nwork; w += gridDim.x) {
      const int q = (int)(w / a.n_mblocks);
      const int64_t row = (int64_t)(w % a.n_mblocks) * kTcBM + r;
      const int64_t c1 = a.col_start[q + 1];
      const int64_t yr = row < a.B ? a.y[row] : -1;
      TcRowState st = {-CUDART_INF_F, 0, false, -1, -1};
      for (int64_t n0 = a.col_start[q]; n0 < c1; n0 += kTcBN) {
        if (!mbar_wait(&tfull[acc], aph, abort_flag, a.status)) goto done;
        tc_fence_after();
        for (int cc = 0; cc < kTcBN / 32; ++cc) {
          const int64_t col0 = n0 + 32 * cc;
          if (col0 >= c1) break;  // warp-uniform
          float v[32];
          tmem_ld32(tmem + (uint32_t)((quad * 32) << 16) + acc * kTcBN + 32 * cc, v);
          const int valid = (int)min((int64_t)32, c1 - col0);
          tc_fold32(v, col0, valid, st, lv, lc, r);
          if ((uint64_t)(yr - col0) < (uint64_t)valid) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i == yr && row < a.B) a.zy[row] = v[i];
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          aph ^= 1u;
        }
      }
      if (row < a.B) tc_finish_row(a, q, row, st, lv, lc, r);
    }
  }
done:
  __syncwarp();
  if (*abort_flag && lane == 0) {
    // Aborted: let the copies and MMAs already issued land before the CTA
    // frees its TMEM and shared memory (each wait bounded, kTcDrainLimitNs).
    if (warp == 0) {
      for (int st = 0; st < kTcStages; ++st)
        if (issued & (1u << st)) mbar_drain(&full[st], (issued_par >> st) & 1u);
    } else if (warp == 1 && mma_any) {
      umma_commit(drain);  // arrives once every MMA issued by this thread is complete
      mbar_drain(drain, 0u);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols));
  }
}

}  // namespace fwb200
