// Class-sharded rows (tensor-parallel LM heads): the C classes of a row are
// split into column shards, one per rank (rank q owns columns
// [col_start[q], col_start[q+1])).  No rank ever sees a whole row.
//
// Why a bounded exchange suffices: f(t) = sum_j max(z_j - t, 0) over the
// whole row is >= the same sum over one shard, so the root h* of f = 1 is >=
// each shard's own threshold h*_q, and the part of the global support that
// lies in shard q is contained in shard q's own support {z > h*_q}.  The
// union of the shards' supports is therefore a superset of the global
// support, which is all Michelot's fixed point needs.
//
// Protocol (host side: fwloss_b200/sharded.py):
//   1. every rank runs the fused kernel in kOutShard mode on its shard: the
//      gradient shard is zero-filled and a summary record is written per row
//      (local max, local support size kappa_q, up to K support values; their
//      local columns stay on the rank);
//   2. all-gather of the summaries ([N, B, 4 + K] int32);
//   3. fw_shard_solve_kernel (below), per row on every rank: global max,
//      union of the supports, Michelot -> h*, kappa; then each rank patches
//      its own gradient shard (support entries and, if it owns the label,
//      the label entry) and writes the loss if it owns the label;
//   4. one scalar all-reduce of the loss sum.
// A row where some shard's support has more than K entries cannot be solved
// from the summaries; it is listed in fb_rows and solved from the full row by
// the host (exact, slower).
#pragma once

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kMaxShards = 16;
constexpr int kShardMaxK = 64;
constexpr int kShardSolveThreads = 256;
constexpr int kShardListCap = kMaxShards * kShardMaxK / 4;  // 256 candidates per row

struct ShardSolveArgs {
  const int32_t* gathered;  // [nranks, B, kShardHeader + K]
  int nranks;
  int rank;
  int K;
  int64_t B;
  int64_t col_start[kMaxShards + 1];
  const float* z;           // this rank's shard [B, ld]
  int64_t ld;
  const int64_t* y;         // global labels [B]
  float scale;
  float* grad;              // this rank's gradient shard [B, ld], zero-filled
  const int32_t* local_idx; // [B, K] local columns of this rank's summary values
  float* H;
  int32_t* kappa;
  float* loss_part;         // loss where this rank owns the label, else 0
  int32_t* fb_rows;
  int32_t* fb_count;
  int32_t* status;
};

__global__ void __launch_bounds__(kShardSolveThreads)
    fw_shard_solve_kernel(ShardSolveArgs a) {
  __shared__ float s_list[kShardSolveThreads / 32][kShardListCap];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  float* L = s_list[wib];
  const int S = kShardHeader + a.K;
  const int64_t nwarps = (int64_t)gridDim.x * (kShardSolveThreads / 32);
  const int64_t C = a.col_start[a.nranks];
  const int64_t c_lo = a.col_start[a.rank], c_hi = a.col_start[a.rank + 1];

  for (int64_t row = (int64_t)blockIdx.x * (kShardSolveThreads / 32) + wib; row < a.B; row += nwarps) {
    // headers of all shards (lane q reads shard q)
    float Mq = -CUDART_INF_F;
    int kq = 0, fq = 0, iq = -1;
    if (lane < a.nranks) {
      const int32_t* rec = a.gathered + ((int64_t)lane * a.B + row) * S;
      Mq = __int_as_float(rec[0]);
      kq = rec[1];
      fq = rec[2];
      iq = rec[3];
    }
    const float M = warp_max_nan(Mq);
    const int64_t ylab = a.y[row];
    const bool yok = ylab >= 0 && ylab < C;
    const bool own_y = yok && ylab >= c_lo && ylab < c_hi;
    const int64_t yl = own_y ? ylab - c_lo : -1;
    const float zy = own_y ? a.z[row * a.ld + yl] : CUDART_NAN_F;
    float* gr = a.grad + row * a.ld;

    if (!isfinite(M)) {
      // policy as in the unsharded kernels: kappa = 1 at the first column
      // holding the maximum (first NaN), H = M
      const bool isn = (M != M);
      const bool match = lane < a.nranks && (fq & kShardNonFinite) && (isn ? (Mq != Mq) : (Mq == M));
      const unsigned b = __ballot_sync(kFull, match);
      const int owner = b ? __ffs(b) - 1 : 0;
      const int jloc = __shfl_sync(kFull, iq, owner);
      const int64_t jstar = a.col_start[owner] + jloc;
      if (lane == 0) {
        if (owner == a.rank && jstar != ylab) gr[jloc] = a.scale;
        if (own_y) gr[yl] = ((jstar == ylab) ? a.scale : 0.0f) - a.scale;
        if (a.H) a.H[row] = M;
        if (a.kappa) a.kappa[row] = 1;
        if (a.loss_part) a.loss_part[row] = own_y ? (1.0f - zy + M) : ((!yok && a.rank == 0) ? CUDART_NAN_F : 0.0f);
        raise_status(a.status, 2 | (yok ? 0 : 1));
      }
      continue;
    }

    const bool truncated = __any_sync(kFull, lane < a.nranks && kq > a.K);
    if (truncated) {
      // left for the exact full-row path; its loss share starts at 0
      if (lane == 0) {
        a.fb_rows[atomicAdd(a.fb_count, 1)] = (int32_t)row;
        if (a.loss_part) a.loss_part[row] = 0.0f;
        if (a.kappa) a.kappa[row] = 0;
        if (a.H) a.H[row] = CUDART_NAN_F;
      }
      continue;
    }

    // union of the shard supports above t0, in rank order
    const float t0 = __fsub_rd(M, 1.0f);
    int n = 0;
    for (int q = 0; q < a.nranks; ++q) {
      const int cnt = __shfl_sync(kFull, kq, q);
      const int32_t* vals = a.gathered + ((int64_t)q * a.B + row) * S + kShardHeader;
      for (int k0 = 0; k0 < cnt; k0 += 32) {
        const int k = k0 + lane;
        const float x = (k < cnt) ? __int_as_float(vals[k]) : -CUDART_INF_F;
        const bool keep = x > t0;
        const unsigned b = __ballot_sync(kFull, keep);
        if (keep && n + __popc(b & lanemask_lt(lane)) < kShardListCap)
          L[n + __popc(b & lanemask_lt(lane))] = x;
        n += __popc(b);
      }
    }
    n = min(n, kShardListCap);  // n <= nranks * K <= kShardListCap by the host checks
    __syncwarp();
    double tau;
    int kap;
    michelot_list<32>(L, n, M, lane, kFull, tau, kap);
    __syncwarp();
    const float Hf = threshold_fp32(M, tau);
    const float inv = (float)((double)a.scale / (double)kap);

    // patch this rank's gradient shard
    const int kme = __shfl_sync(kFull, kq, a.rank);
    const int32_t* myvals = a.gathered + ((int64_t)a.rank * a.B + row) * S + kShardHeader;
    const int32_t* myidx = a.local_idx + row * (int64_t)a.K;
    for (int k = lane; k < kme; k += 32) {
      const int j = myidx[k];
      if (__int_as_float(myvals[k]) > Hf && j != yl) gr[j] = inv;
    }
    __syncwarp();
    if (lane == 0) {
      if (own_y) gr[yl] = ((zy > Hf) ? inv : 0.0f) - a.scale;
      if (a.H) a.H[row] = Hf;
      if (a.kappa) a.kappa[row] = kap;
      if (a.loss_part)
        a.loss_part[row] = own_y ? row_loss(M, tau, zy) : ((!yok && a.rank == 0) ? CUDART_NAN_F : 0.0f);
      if (!yok) raise_status(a.status, 1);
    }
  }
}

}  // namespace fwb200
