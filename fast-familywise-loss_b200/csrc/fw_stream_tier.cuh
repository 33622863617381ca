// Streaming tier: one CTA (CS == 1) or one thread-block cluster of CS CTAs
// per row, for rows too long for registers (C > 2048, up to vocab scale).
//
// The gradient of a row is zero except on the support (kappa entries) and
// at the label, and the support lies inside {z > M - 1}.  So the row never
// has to be held on chip:
//
//   stream   every CTA streams its segment of the row once with 128-bit
//            loads, writes the zero gradient (or zero mask) for it in the
//            same loop, keeps a NaN-propagating running max per warp (shared
//            across the CTA's warps through one shared-memory atomicMax) and
//            appends elements above (running max - 1) to a per-warp
//            candidate list (ballot compaction; when a list fills up it is
//            re-filtered against the newer, higher threshold);
//   exchange the CTAs publish max and list sizes; after one cluster barrier
//            every CTA knows the row max M;
//   solve    CTA 0 gathers the candidates z > t0 of all CTAs through DSMEM
//            into one list, in a fixed order, and one warp runs Michelot's
//            fixed point on it (exact support, deterministic sums);
//   patch    CTA 0 writes the kappa support entries and the label entry over
//            the zeros.  The zero stores of every CTA happen before the
//            cluster barrier (release) and the patch after it (acquire), so
//            the patch wins.
//
// HBM traffic is the minimum: 4C bytes read + 4C bytes written per row
// (1 byte written for the mask; none for the candidate form).
//
// Dense rows (a candidate list overflowed: most of the row is within 1 of
// the max, e.g. logits with sigma 1e-3) switch to an exact radix select over
// order-preserving uint32 keys with 8-bit digits: per pass every CTA builds
// a 256-bin histogram (count, fp64 sum of shifted logits) of the elements
// above t0 inside the current key prefix, CTA 0 merges the CS histograms
// through DSMEM, walks the bins from the top (accept / refine / stop) and
// broadcasts the decision; at most four passes.  The row is then re-read and
// the output rewritten densely.
//
// Reference counterpart: fw_precompact_histogram_kernel,
// fw_precompact_reduce_kernel, fw_compact_multiblock_kernel,
// fw_radix_buffer_kernel and fw_backward_candidate_kernel
// (src/cuda/fw_radix_argmax.cu:303-429, :497-636, :638-760, :871-1035,
// :1498-1534): five launches, two full reads of the row, an [N,K] candidate
// buffer pair and a full memset.
#pragma once

#include <climits>
#include <cooperative_groups.h>

#include "fw_device.cuh"

namespace fwb200 {

constexpr int kST = 256;              // threads per CTA (all shapes but the narrow one)
constexpr int kStreamListCap = 128;   // candidates per warp list
constexpr int kStreamItems = 4;       // 16-byte loads per thread per streaming step (VEC)
constexpr int kStreamScalars = 16;    // scalar loads per thread per streaming step (!VEC)

// Launch shapes of the streaming kernel, 256 threads each (bytes in flight
// per CTA, resident CTAs per SM the register budget is sized for):
//   kShapeWide    four 16-byte register loads per thread (16 KB), 5 CTAs per
//                 SM (<= 51 registers; 16-bit rows stream in half the time of
//                 fp32 ones, so more CTAs are needed to cover each row's
//                 exchange/solve/patch phase: B200, cfg2 shape, bf16 99.1 ->
//                 97.0 us, fp32 unchanged, six CTAs slower);
//   kShapeDeep    eight 16-byte register loads per thread (32 KB), 2 CTAs per
//                 SM: grids of at most two CTAs per SM (very few rows, or the
//                 rows left over after whole waves), where few CTAs share an
//                 SM and each has to keep more bytes in flight (B200, B = 32 x
//                 C = 1e6 fp32 on clusters of 8: 93.2 -> 83.1 us);
//   kShapeStaged  16 KB tiles bulk-copied (cp.async.bulk, no multicast, this
//                 GPU's own memory) into a ring of kStages shared-memory
//                 stages (64 KB in flight, none of it in registers), 2 CTAs
//                 per SM; 16-byte-aligned rows only (others stream as deep);
//   kShapeStaged4 the same with 8 KB tiles (32 KB in flight), 4 CTAs per SM;
//   kShapeNarrow  128 threads, 4 KB tiles (16 KB in flight), 8 CTAs per SM:
//                 1184 resident CTAs, so that batches of up to that many rows
//                 run as one wave (one ramp and one solve phase per launch).
// Without 16-byte loads (unaligned rows) every shape issues 16 scalar loads
// per thread per step.
enum StreamShape : int { kShapeWide = 0, kShapeDeep = 2, kShapeStaged = 3, kShapeStaged4 = 4, kShapeNarrow = 5 };

constexpr int kStages = 4;                                    // staged shapes: tiles in flight per CTA
constexpr uint64_t kStageWaitLimitNs = 1000000000ull;         // 1 s; a tile lands in a few us
constexpr uint64_t kStageDrainLimitNs = 100000000ull;         // 100 ms per stage after an abort

template <int SHAPE>
__host__ __device__ constexpr int stream_threads() {
  return SHAPE == kShapeNarrow ? 128 : kST;
}

template <bool VEC, int SHAPE = kShapeWide>
__host__ __device__ constexpr int stream_ipt() {
  return VEC ? (SHAPE == kShapeDeep ? 2 * kStreamItems
                                    : ((SHAPE == kShapeStaged4 || SHAPE == kShapeNarrow) ? kStreamItems / 2
                                                                                         : kStreamItems))
             : kStreamScalars;
}

template <int SHAPE>
__host__ __device__ constexpr int stream_min_blocks() {
  return SHAPE == kShapeWide ? 5 : (SHAPE == kShapeStaged4 ? 4 : (SHAPE == kShapeNarrow ? 8 : 2));
}

template <int SHAPE>
__host__ __device__ constexpr bool is_staged() {
  return SHAPE == kShapeStaged || SHAPE == kShapeStaged4 || SHAPE == kShapeNarrow;
}

// Staged shapes: 16-byte items per tile (one streaming step of every thread)
// and the ring's dynamic shared memory.
template <int SHAPE>
__host__ __device__ constexpr int stage_items() {
  return stream_threads<SHAPE>() * stream_ipt<true, SHAPE>();
}

template <int SHAPE>
__host__ __device__ constexpr size_t staged_smem_bytes() {
  return (size_t)kStages * stage_items<SHAPE>() * 16;
}

// Waits until the grid launched before this one on the stream has completed
// and its writes are visible (griddepcontrol.wait); returns at once for a
// launch that is not a programmatic dependent.
__device__ __forceinline__ void wait_prior_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Shared state of one CTA with NW warps.
template <int NW>
struct __align__(16) StreamShared {
  static constexpr int kSolve = NW * kStreamListCap;  // gathered candidates per row
  float lz[NW][kStreamListCap];
  int li[NW][kStreamListCap];
  float sz[kSolve];
  int si[kSolve];
  double hs[256];
  int hc[256];
  float wmax[NW];
  int wcnt[NW];
  int gcnt[8 * NW];  // cluster gather: kept candidates per (rank, warp) list
  int goff[8 * NW];  // and their offsets in the solve list
  unsigned run_key;
  int flags;        // bit 0: a warp list overflowed
  float cta_max;
  int go_dense;     // written by CTA 0 after the gather
  int first_idx;
  float label_z;    // the label's logit, stored by the thread that streams it
  int cand_pos;
  float row_max;
  int row_flags;    // bit-or of every CTA's flags
  int nsolve;
  // staged shape: one mbarrier per stage, abort flag of a bounded wait
  uint64_t stage_full[kStages];
  int stage_abort;
  // dense-path decision, written by CTA 0 into every CTA of the cluster
  unsigned long long dec_cut;
  double dec_sum;
  uint32_t dec_prefix, dec_mask;
  int dec_cnt, dec_done;
};

template <int CS, class S>
__device__ __forceinline__ S* cta_smem(S* s, int rank) {
  if constexpr (CS > 1) {
    return cooperative_groups::this_cluster().map_shared_rank(s, rank);
  } else {
    (void)rank;
    return s;
  }
}

template <int CS>
__device__ __forceinline__ void row_barrier() {
  if constexpr (CS > 1) {
    cooperative_groups::this_cluster().sync();
  } else {
    __syncthreads();
  }
}

// Keeps the entries > t of a warp list, in order.  Warp-collective.
__device__ __forceinline__ int list_compact(float* lz, int* li, int cnt, float t,
                                            int lane) {
  constexpr int PER = kStreamListCap / 32;
  __syncwarp();
  float vv[PER];
  int ii[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int e = k * 32 + lane;
    vv[k] = (e < cnt) ? lz[e] : -CUDART_INF_F;
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

// Appends (val, col) for lanes with pred to the warp list.  Warp-collective;
// cnt and ovf are warp-uniform.
__device__ __forceinline__ void list_append(float* lz, int* li, int& cnt,
                                            bool& ovf, float val, int col,
                                            bool pred, float t, int lane) {
  const unsigned b = __ballot_sync(kFull, pred);
  if (b == 0u || ovf) return;
  const int k = __popc(b);
  if (cnt + k > kStreamListCap) {
    cnt = list_compact(lz, li, cnt, t, lane);
    if (cnt + k > kStreamListCap) {
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

// Segment of the row owned by one CTA: items [i0, i1) where an item is a
// 16-byte slot of EPS elements (VEC) or one element.  With VEC, the C % EPS
// tail columns belong to the last CTA and are handled by its warp 0.
struct Segment {
  int64_t i0, i1;
};

template <int CS, bool VEC, int EPS>
__device__ __forceinline__ Segment row_segment(int64_t C, int rank) {
  const int64_t n = VEC ? C / EPS : C;
  Segment g;
  g.i0 = n * rank / CS;
  g.i1 = n * (rank + 1) / CS;
  return g;
}

// Calls f(value, column) for every element of this thread's share of the
// segment, in the fixed order used by all passes (loads are issued kStreamU
// 16-byte items ahead).  f must be thread-local work only.
template <class T, int CS, bool VEC, int NT, class F>
__device__ __forceinline__ void for_each_element(const T* zr, int64_t C,
                                                 int rank, F&& f) {
  constexpr int EPS = Elem<T>::kEPS;
  const Segment g = row_segment<CS, VEC, EPS>(C, rank);
  constexpr int W = VEC ? EPS : 1;
  constexpr int IPT = stream_ipt<VEC>();
  for (int64_t base = g.i0; base < g.i1; base += (int64_t)NT * IPT) {
    float v[IPT * W];
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
      const int64_t it = base + (int64_t)u * NT + threadIdx.x;
      if (VEC) {
        if (it < g.i1) {
          unpack16<T>(ld_stream16(zr + W * it), &v[W * u]);
        } else {
#pragma unroll
          for (int j = 0; j < W; ++j) v[W * u + j] = -CUDART_INF_F;
        }
      } else {
        v[u] = (it < g.i1) ? ld_elem(zr + it) : -CUDART_INF_F;
      }
    }
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
      const int64_t it = base + (int64_t)u * NT + threadIdx.x;
      if (it < g.i1) {
#pragma unroll
        for (int j = 0; j < W; ++j) f(v[u * W + j], (int)(it * W + j));
      }
    }
  }
  if (VEC && rank == CS - 1 && threadIdx.x < 32) {
    const int64_t c = EPS * (C / EPS) + threadIdx.x;
    if (c < C) f(ld_elem(zr + c), (int)c);
  }
}

template <class T, int CS, bool VEC, int OUT, int SHAPE>
__device__ __forceinline__ void stream_rows_body(const RowArgs& a,
                                                 StreamShared<stream_threads<SHAPE>() / 32>& s) {
  constexpr int NT = stream_threads<SHAPE>();  // threads per CTA
  constexpr int NW = NT / 32;                  // warps per CTA
  using SS = StreamShared<NW>;
  static_assert(OUT == kOutGrad || OUT == kOutNone || sizeof(T) == 4,
                "mask/candidate/shard outputs are fp32-only");
  constexpr bool kZeroFill = (OUT == kOutGrad || OUT == kOutShard);
  constexpr int EPS = Elem<T>::kEPS;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int w = tid >> 5;
  const int64_t row = blockIdx.x / CS;
  int rank = 0;
  if constexpr (CS > 1) rank = (int)cooperative_groups::this_cluster().block_rank();
  const bool leader = (rank == 0);
  const int64_t C = a.C;
  const T* zr = static_cast<const T*>(a.z) + row * a.ld;

  if (tid == 0) {
    s.run_key = 0u;
    s.flags = 0;
    s.go_dense = 0;
    s.first_idx = INT_MAX;
    s.cand_pos = 0;
    if constexpr (is_staged<SHAPE>()) {
      for (int k = 0; k < kStages; ++k) mbar_init(&s.stage_full[k], 1);
      s.stage_abort = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
  }
  __syncthreads();

  // ---------------------------------------------------------------- stream
  constexpr int W = VEC ? EPS : 1;
  constexpr int IPT = stream_ipt<VEC, SHAPE>();
  const Segment g = row_segment<CS, VEC, EPS>(C, rank);
  float run = -CUDART_INF_F;
  int wcnt = 0;
  bool ovf = false;
  // The label and its item: the thread whose streaming step holds the label
  // column records its value in its CTA's shared memory (a cluster's leader
  // copies it from the owning CTA after the exchange barrier), so the solve
  // needs no dependent global load.
  const int64_t ylab = a.y ? a.y[row] : -1;  // no labels in kOutShard
  const bool yok = (ylab >= 0 && ylab < C);
  const int yc = yok ? (int)ylab : -1;
  const int y_item = (yok && yc < (VEC ? EPS * (C / EPS) : C)) ? yc / W : -1;  // items < 2^31
  float* lz = s.lz[w];
  int* li = s.li[w];
  // kOutShard without a gradient shard (a.grad == null) only writes summaries
  T* gr = (kZeroFill && a.grad) ? static_cast<T*>(a.grad) + row * a.ld : nullptr;
  uint8_t* mr = (OUT == kOutMask) ? a.mask + row * C : nullptr;

  // One streaming step: this thread's IPT items base + u * NT + tid (values
  // in v, -inf past the segment): zero output, running max, candidates.
  // Outputs of one item that need no values: the zero gradient (or mask).
  auto zero_item = [&](int64_t it) {
    if (it < g.i1) {
      if (kZeroFill && (OUT == kOutGrad || gr != nullptr)) {
        if (VEC)
          *reinterpret_cast<uint4*>(gr + W * it) = make_uint4(0u, 0u, 0u, 0u);
        else
          st_elem(gr + it, 0.0f);
      } else if (OUT == kOutMask) {
        if (VEC && a.mask_vec)
          *reinterpret_cast<uchar4*>(mr + 4 * it) = make_uchar4(0, 0, 0, 0);
        else
#pragma unroll
          for (int j = 0; j < W; ++j) mr[it * W + j] = 0;
      }
    }
  };
  // The step's warp maximum joins the running maximum (shared across the
  // CTA's warps); returns the step's candidate threshold.
  auto step_threshold = [&](float m) -> float {
    m = warp_max_nan(m);
    run = max_nan(run, m);
    if (lane == 0) atomicMax(&s.run_key, sort_key(run));
    const float shared_max = key_value(*reinterpret_cast<volatile unsigned*>(&s.run_key));
    return __fsub_rd(fmaxf(run, shared_max), 1.0f);
  };
  // Candidates of one step: one count per lane, one warp scan for the
  // offsets, then every lane stores its own in element order (the list holds
  // them lane-major; a fixed order, so the solve stays deterministic).
  auto candidates = [&](float (&v)[IPT * W], int64_t base, float t) {
    int c = 0;
#pragma unroll
    for (int k = 0; k < IPT * W; ++k) c += (v[k] > t) ? 1 : 0;
    const int total = __reduce_add_sync(kFull, c);
    if (total > 0 && !ovf) {
      if (wcnt + total > kStreamListCap) {
        wcnt = list_compact(lz, li, wcnt, t, lane);  // older entries at or below t
        if (wcnt + total > kStreamListCap) ovf = true;
      }
      if (!ovf) {
        int pos = wcnt + warp_excl_scan(c, lane);
        if (c > 0) {
#pragma unroll
          for (int u = 0; u < IPT; ++u) {
            const int col0 = (int)((base + (int64_t)u * NT + tid) * W);
#pragma unroll
            for (int j = 0; j < W; ++j)
              if (v[u * W + j] > t) {
                lz[pos] = v[u * W + j];
                li[pos] = col0 + j;
                ++pos;
              }
          }
        }
        wcnt += total;
      }
    }
  };
  // One streaming step over element values (rows without 16-byte loads):
  // label, zero output, running max, candidates.
  auto consume = [&](float (&v)[IPT * W], int64_t base) {
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
      const int64_t it = base + (int64_t)u * NT + tid;
      if ((int)it == y_item) {  // rare: this item holds the label column
        const int jy = yc - y_item * W;
#pragma unroll
        for (int j = 0; j < W; ++j)
          if (j == jy) s.label_z = v[u * W + j];
      }
      zero_item(it);
    }
    float m = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < IPT * W; ++k) m = max_nan(m, v[k]);
    candidates(v, base, step_threshold(m));
  };
  // One streaming step over 16-byte slots (q: this thread's IPT slots, -inf
  // past the segment): each slot is reduced to its maximum first (packed
  // pairs for 16-bit types), and the elements are unpacked and counted only
  // when some lane of the warp has a slot above the step's threshold --
  // rarely, since candidates lie within 1 of the row maximum.
  auto consume_slots = [&](const uint4 (&q)[IPT], int64_t base) {
    float im[IPT];
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
      const int64_t it = base + (int64_t)u * NT + tid;
      if ((int)it == y_item) {  // rare: this item holds the label column
        float e[W];
        unpack16<T>(q[u], e);
        const int jy = yc - y_item * W;
#pragma unroll
        for (int j = 0; j < W; ++j)
          if (j == jy) s.label_z = e[j];
      }
      zero_item(it);
      im[u] = slot_max_nan<T>(q[u]);
    }
    float m = im[0];
#pragma unroll
    for (int u = 1; u < IPT; ++u) m = max_nan(m, im[u]);
    const float t = step_threshold(m);
    bool hit = false;
#pragma unroll
    for (int u = 0; u < IPT; ++u) hit |= im[u] > t;
    if (__any_sync(kFull, hit)) {
      float v[IPT * W];
#pragma unroll
      for (int u = 0; u < IPT; ++u) unpack16<T>(q[u], &v[u * W]);
      candidates(v, base, t);
    }
  };

  if constexpr (is_staged<SHAPE>() && VEC) {
    constexpr int kStageItems = stage_items<SHAPE>();
    // Tiles of kStageItems 16-byte items, bulk-copied into a ring of kStages
    // shared-memory stages by thread 0 (one tile per stage in flight); all
    // threads wait for a tile's mbarrier (bounded), consume it, and after a
    // CTA barrier thread 0 refills the stage with the tile kStages ahead.
    extern __shared__ __align__(16) uint4 stream_ring[];
    const uint4* src = reinterpret_cast<const uint4*>(zr);
    const int ntiles = (int)((g.i1 - g.i0 + kStageItems - 1) / kStageItems);
    int issued = 0;  // thread 0: tiles issued so far
    auto issue = [&](int k) {
      const int st = k % kStages;
      const int64_t first = g.i0 + (int64_t)k * kStageItems;
      const int64_t n = (g.i1 - first < kStageItems) ? (g.i1 - first) : (int64_t)kStageItems;
      const uint32_t bytes = (uint32_t)n * 16u;
      mbar_expect_tx(&s.stage_full[st], bytes);
      bulk_load(stream_ring + (size_t)st * kStageItems, src + first, bytes, &s.stage_full[st]);
    };
    if (tid == 0)
      for (; issued < kStages && issued < ntiles; ++issued) issue(issued);
    bool aborted = false;
    for (int k = 0; k < ntiles; ++k) {
      const int st = k % kStages;
      const int64_t base = g.i0 + (int64_t)k * kStageItems;
      bool ok = false;
      if (!aborted) {
        ok = mbar_wait_for(&s.stage_full[st], (uint32_t)(k / kStages) & 1u, kStageWaitLimitNs);
        if (!ok) s.stage_abort = 1;
      }
      const uint4* tile = stream_ring + (size_t)st * kStageItems;
      uint4 q[IPT];
#pragma unroll
      for (int u = 0; u < IPT; ++u) {
        const int l = u * NT + tid;
        q[u] = (ok && base + l < g.i1) ? tile[l] : neg_inf_slot<T>();
      }
      consume_slots(q, base);
      __syncthreads();  // every thread is done with this stage
      aborted = s.stage_abort != 0;
      if (tid == 0 && !aborted && issued < ntiles) issue(issued++);
    }
    if (aborted && tid == 0) {
      // a copy did not land in time: flag it, then let the copies already
      // issued land (bounded) before this CTA's shared memory is released
      raise_status(a.status, kStatusTimeout);
      for (int st = 0; st < kStages; ++st) {
        int last = -1;
        for (int k = st; k < issued; k += kStages) last = k;
        if (last >= 0) mbar_wait_for(&s.stage_full[st], (uint32_t)(last / kStages) & 1u, kStageDrainLimitNs);
      }
    }
  } else if constexpr (VEC) {
    for (int64_t base = g.i0; base < g.i1; base += (int64_t)NT * IPT) {
      uint4 q[IPT];
#pragma unroll
      for (int u = 0; u < IPT; ++u) {
        const int64_t it = base + (int64_t)u * NT + tid;
        q[u] = (it < g.i1) ? ld_stream16(zr + W * it) : neg_inf_slot<T>();
      }
      consume_slots(q, base);
    }
  } else {
    for (int64_t base = g.i0; base < g.i1; base += (int64_t)NT * IPT) {
      float v[IPT * W];
#pragma unroll
      for (int u = 0; u < IPT; ++u) {
        const int64_t it = base + (int64_t)u * NT + tid;
        v[u] = (it < g.i1) ? ld_elem(zr + it) : -CUDART_INF_F;
      }
      consume(v, base);
    }
  }
  if (VEC && rank == CS - 1 && w == 0) {
    // C % EPS tail columns.
    const int64_t c = EPS * (C / EPS) + lane;
    const bool in = c < C;
    const float x = in ? ld_elem(zr + c) : -CUDART_INF_F;
    if (in) {
      if (kZeroFill && (OUT == kOutGrad || gr != nullptr)) st_elem(gr + c, 0.0f);
      if (OUT == kOutMask) mr[c] = 0;
    }
    run = max_nan(run, warp_max_nan(x));
    const float shared_max = key_value(*reinterpret_cast<volatile unsigned*>(&s.run_key));
    const float t = __fsub_rd(fmaxf(run, shared_max), 1.0f);
    list_append(lz, li, wcnt, ovf, x, (int)c, x > t, t, lane);
    if (in && c == yc) s.label_z = x;
  }

  // -------------------------------------------------------------- exchange
  if (lane == 0) {
    s.wmax[w] = run;
    s.wcnt[w] = wcnt;
    if (ovf) atomicOr(&s.flags, 1);
  }
  __syncthreads();
  float M;
  int row_flags;
  if constexpr (CS == 1) {
    // One CTA per row: every thread reads the warp maxima itself, so the
    // row needs no second and third barrier.
    M = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < NW; ++k) M = max_nan(M, s.wmax[k]);
    row_flags = s.flags;
  } else {
    if (tid == 0) {
      float cm = -CUDART_INF_F;
#pragma unroll
      for (int k = 0; k < NW; ++k) cm = max_nan(cm, s.wmax[k]);
      s.cta_max = cm;
    }
    row_barrier<CS>();
    if (w == 0) {  // one remote read per lane instead of CS serial ones
      float rm = -CUDART_INF_F;
      int flags = 0;
      if (lane < CS) {
        const SS* rs = cta_smem<CS>(&s, lane);
        rm = rs->cta_max;
        flags = rs->flags;
      }
      rm = warp_max_nan(rm);
      flags = (int)__reduce_or_sync(kFull, (unsigned)flags);
      if (lane == 0) {
        s.row_max = rm;
        s.row_flags = flags;
        if (leader && yok) {
          // the label's logit from the CTA whose segment holds its column
          // (the C % EPS tail columns belong to the last CTA)
          int owner = CS - 1;
          if (y_item >= 0) {
            const int64_t n_items = VEC ? C / EPS : C;
            while (owner > 0 && n_items * owner / CS > y_item) --owner;
          }
          s.label_z = cta_smem<CS>(&s, owner)->label_z;
        }
      }
    }
    __syncthreads();
    M = s.row_max;
    row_flags = s.row_flags;
  }
  const double Md = (double)M;
  const float t0 = __fsub_rd(M, 1.0f);

  // ------------------------------------------------------- non-finite rows
  if (!isfinite(M)) {
    const bool isn = (M != M);
    int best = INT_MAX;
    for_each_element<T, CS, VEC, NT>(zr, C, rank, [&](float x, int c) {
      if (isn ? (x != x) : (x == M)) best = min(best, c);
    });
    best = (int)__reduce_min_sync(kFull, (unsigned)best);
    if (lane == 0) atomicMin(&s.first_idx, best);
    row_barrier<CS>();
    if (leader && tid == 0) {
      int j = INT_MAX;
      for (int r = 0; r < CS; ++r) j = min(j, cta_smem<CS>(&s, r)->first_idx);
      s.nsolve = j;
    }
    row_barrier<CS>();
    if (!(leader && tid == 0)) return;
    const int j = s.nsolve;
    const float zy = yok ? s.label_z : CUDART_NAN_F;
    if (OUT == kOutGrad) {
      st_elem(gr + j, a.scale - ((j == yc) ? a.scale : 0.0f));
      if (yok && j != yc) st_elem(gr + yc, -a.scale);
      if (a.sup_cols) a.sup_cols[row * (int64_t)a.sup_k] = j;
    } else if (OUT == kOutMask) {
      mr[j] = 1;
    } else if (OUT == kOutCand) {
      a.cand_val[row * C] = ld_elem(zr + j);
      a.cand_idx[row * C] = j;
      if (a.cand_count) a.cand_count[row] = 1;
    } else if (OUT == kOutNone) {
      // forward only: no per-element output
    } else {  // kOutShard: the gradient shard stays zero
      int32_t* rec = a.shard_sum + row * (int64_t)(kShardHeader + a.shard_k);
      rec[0] = __float_as_int(M);
      rec[1] = 1;
      rec[2] = kShardNonFinite;
      rec[3] = j;
      if (a.shard_k > 0) {
        rec[kShardHeader] = __float_as_int(M);
        a.shard_idx[row * (int64_t)a.shard_k] = j;
      }
      return;
    }
    if (a.H) a.H[row] = M;
    if (a.loss) a.loss[row] = yok ? (1.0f - zy + M) : CUDART_NAN_F;
    if (a.kappa) a.kappa[row] = 1;
    if (!yok) raise_status(a.status, 1);
    raise_status(a.status, 2);
    return;
  }

  // ---------------------------------------------------------------- gather
  const bool lists_ok = !(row_flags & 1);  // no warp list overflowed
  if constexpr (CS == 1) {
    // One CTA: the warp lists hold at most NW * kStreamListCap = SS::kSolve
    // candidates, so the gathered list cannot overflow and warp 0 alone
    // finishes the row; the zero stores of the other warps precede the
    // barrier above, which orders them before warp 0's patch.
    static_assert(NW * kStreamListCap <= SS::kSolve, "one CTA's lists must fit the solve list");
    if (lists_ok) {
      // every warp counts its own list's candidates above t0, takes its
      // offset in the fixed order (warp, then list position) and copies
      // them; then warp 0 alone solves and patches
      int kept = 0;
      for (int k0 = 0; k0 < wcnt; k0 += 32) {
        const int k = k0 + lane;
        kept += __popc(__ballot_sync(kFull, (k < wcnt) && (lz[k] > t0)));
      }
      if (lane == 0) s.gcnt[w] = kept;
      __syncthreads();
      int pos0 = 0, tot = 0;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) {
        const int c = s.gcnt[ww];
        pos0 += (ww < w) ? c : 0;
        tot += c;
      }
      for (int k0 = 0; k0 < wcnt; k0 += 32) {
        const int k = k0 + lane;
        const float val = (k < wcnt) ? lz[k] : -CUDART_INF_F;
        const bool keep = val > t0;
        const unsigned b = __ballot_sync(kFull, keep);
        if (keep) {
          const int pos = pos0 + __popc(b & lanemask_lt(lane));
          s.sz[pos] = val;
          s.si[pos] = li[k];
        }
        pos0 += __popc(b);
      }
      if (w == 0 && lane == 0) s.nsolve = tot;
      __syncthreads();
      if (w != 0) return;
    }
  }
  if constexpr (CS > 1) {
    // The leader CTA's warps gather the CS * NW lists in parallel (their
    // entries sit in other CTAs' shared memory): kept counts per list, their
    // offsets in the fixed list order (rank-major, then warp), then the
    // copies.  Same list, in the same order, as one warp walking the lists.
    if (lists_ok && leader) {
      constexpr int NL = CS * NW;
      for (int L = w; L < NL; L += NW) {
        const SS* rs = cta_smem<CS>(&s, L / NW);
        const int ww = L % NW;
        const int cnt = rs->wcnt[ww];
        int kept = 0;
        for (int k0 = 0; k0 < cnt; k0 += 32) {
          const int k = k0 + lane;
          kept += __popc(__ballot_sync(kFull, (k < cnt) && (rs->lz[ww][k] > t0)));
        }
        if (lane == 0) s.gcnt[L] = kept;
      }
      __syncthreads();
      if (w == 0) {
        int tot = 0;
        for (int L0 = 0; L0 < NL; L0 += 32) {
          const int L = L0 + lane;
          const int c = (L < NL) ? s.gcnt[L] : 0;
          const int x = warp_excl_scan(c, lane);
          if (L < NL) s.goff[L] = tot + x;
          tot += __reduce_add_sync(kFull, c);
        }
        if (lane == 0) {
          const bool full = tot > SS::kSolve;
          s.nsolve = full ? 0 : tot;
          for (int r = 0; r < CS; ++r) cta_smem<CS>(&s, r)->go_dense = full ? 1 : 0;
        }
      }
      __syncthreads();
      if (!s.go_dense) {
        for (int L = w; L < NL; L += NW) {
          const SS* rs = cta_smem<CS>(&s, L / NW);
          const int ww = L % NW;
          const int cnt = rs->wcnt[ww];
          int pos0 = s.goff[L];
          for (int k0 = 0; k0 < cnt; k0 += 32) {
            const int k = k0 + lane;
            float val = -CUDART_INF_F;
            int col = 0;
            if (k < cnt) {
              val = rs->lz[ww][k];
              col = rs->li[ww][k];
            }
            const bool keep = val > t0;
            const unsigned b = __ballot_sync(kFull, keep);
            if (keep) {
              const int pos = pos0 + __popc(b & lanemask_lt(lane));
              s.sz[pos] = val;
              s.si[pos] = col;
            }
            pos0 += __popc(b);
          }
        }
      }
    }
  }
  if constexpr (CS > 1) row_barrier<CS>();
  const bool dense = (row_flags & 1) || s.go_dense;

  // ------------------------------------------------------ solve and patch
  if (!dense) {
    if (!(leader && w == 0)) return;
    const int n = s.nsolve;
    double tau;
    int kap;
    if (n <= 32)  // one candidate per lane
      michelot_lane<32>(lane < n ? s.sz[lane] : -CUDART_INF_F, n, M, kFull, tau, kap);
    else
      michelot_list<32>(s.sz, n, M, lane, kFull, tau, kap);
    const float Hf = threshold_fp32(M, tau);  // x > Hf <=> x in the support
    if (OUT == kOutGrad) {
      const float inv = __fdiv_rn(a.scale, (float)kap);
      bool ysel = false;
      for (int k = lane; k < n; k += 32) {
        const int col = s.si[k];
        if (s.sz[k] > Hf) {
          float gv = inv;
          if (col == yc) {
            gv -= a.scale;
            ysel = true;
          }
          st_elem(gr + col, gv);
        }
      }
      ysel = __any_sync(kFull, ysel);
      if (lane == 0 && yok && !ysel) st_elem(gr + yc, -a.scale);
      if (a.sup_cols) {  // the support's columns (first sup_k of them)
        int32_t* sc = a.sup_cols + row * (int64_t)a.sup_k;
        int pos0 = 0;
        for (int k0 = 0; k0 < n && pos0 < a.sup_k; k0 += 32) {
          const int k = k0 + lane;
          const bool sel = (k < n) && (s.sz[k] > Hf);
          const unsigned b = __ballot_sync(kFull, sel);
          const int pos = pos0 + __popc(b & lanemask_lt(lane));
          if (sel && pos < a.sup_k) sc[pos] = s.si[k];
          pos0 += __popc(b);
        }
      }
    } else if (OUT == kOutMask) {
      for (int k = lane; k < n; k += 32)
        if (s.sz[k] > Hf) mr[s.si[k]] = 1;
    } else if (OUT == kOutShard) {
      const int K = a.shard_k;
      int32_t* rec = a.shard_sum + row * (int64_t)(kShardHeader + K);
      int32_t* ridx = a.shard_idx + row * (int64_t)K;
      int pos0 = 0;
      for (int k0 = 0; k0 < n && pos0 < K; k0 += 32) {
        const int k = k0 + lane;
        const bool sel = (k < n) && (s.sz[k] > Hf);
        const unsigned b = __ballot_sync(kFull, sel);
        const int pos = pos0 + __popc(b & lanemask_lt(lane));
        if (sel && pos < K) {
          rec[kShardHeader + pos] = __float_as_int(s.sz[k]);
          ridx[pos] = s.si[k];
        }
        pos0 += __popc(b);
      }
      if (lane == 0) {
        rec[0] = __float_as_int(M);
        rec[1] = kap;
        rec[2] = 0;
        rec[3] = -1;
      }
      return;
    } else if (OUT == kOutNone) {
      // forward only: H, loss and kappa below
    } else {
      float* cv = a.cand_val + row * C;
      int32_t* ci = a.cand_idx + row * C;
      int pos0 = 0;
      for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        const bool sel = (k < n) && (s.sz[k] > Hf);
        const unsigned b = __ballot_sync(kFull, sel);
        if (sel) {
          const int pos = pos0 + __popc(b & lanemask_lt(lane));
          cv[pos] = s.sz[k];
          ci[pos] = s.si[k];
        }
        pos0 += __popc(b);
      }
      if (lane == 0 && a.cand_count) a.cand_count[row] = kap;
    }
    if (lane == 0) {
      const float zy = yok ? s.label_z : CUDART_NAN_F;
      if (a.H) a.H[row] = Hf;
      if (a.loss) a.loss[row] = yok ? row_loss(M, tau, zy) : CUDART_NAN_F;
      if (a.kappa) a.kappa[row] = kap;
      if (!yok) raise_status(a.status, 1);
    }
    return;
  }

  // ------------------------------------------------ dense rows: radix select
  uint32_t prefix = 0u, pmask = 0u;
  int cnt_a = 0;
  double sum_a = 0.0;
  unsigned long long cut = 1ull << 32;  // selected <=> key >= cut (and z > t0)
  const double t0d = (double)t0 - Md;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += NT) {
      s.hc[b] = 0;
      s.hs[b] = 0.0;
    }
    __syncthreads();
    for_each_element<T, CS, VEC, NT>(zr, C, rank, [&](float x, int) {
      if (x > t0) {
        const uint32_t k = sort_key(x);
        if ((k & pmask) == prefix) {
          const int bin = (int)((k >> shift) & 255u);
          atomicAdd(&s.hc[bin], 1);
          atomicAdd(&s.hs[bin], (double)x - Md);
        }
      }
    });
    row_barrier<CS>();
    if (leader) {
      if (CS > 1) {
        for (int b = tid; b < 256; b += NT) {
          int c = s.hc[b];
          double sm = s.hs[b];
          for (int r = 1; r < CS; ++r) {
            const SS* rs = cta_smem<CS>(&s, r);
            c += rs->hc[b];
            sm += rs->hs[b];
          }
          s.hc[b] = c;
          s.hs[b] = sm;
        }
        __syncthreads();
      }
      if (tid == 0) {
        bool refine = false, done = false;
        for (int b = 255; b >= 0; --b) {
          const int cb = s.hc[b];
          if (cb == 0) continue;
          const double sb = s.hs[b];
          const uint32_t lo_key = prefix | ((uint32_t)b << shift);
          const uint32_t hi_key = lo_key | ((1u << shift) - 1u);
          double lo = (double)key_value(lo_key) - Md;
          double hi = (double)key_value(hi_key) - Md;
          if (lo != lo) lo = -CUDART_INF;
          if (hi != hi) hi = CUDART_INF;
          const double lo_eff = fmax(lo, t0d);
          // f(t) = sum_{d > t} (d - t): every element of this bin and above
          // is >= lo_eff, so f(min of bin) <= f(lo_eff).
          if ((sum_a + sb) - (double)(cnt_a + cb) * lo_eff < 1.0) {
            cnt_a += cb;
            sum_a += sb;
            cut = lo_key;
            continue;
          }
          // Nothing in this bin exceeds hi, so f(max of bin) >= f(hi).
          if (cnt_a > 0 && sum_a - (double)cnt_a * hi >= 1.0) {
            done = true;
            break;
          }
          prefix = lo_key;
          pmask |= 0xffu << shift;
          refine = true;
          break;
        }
        if (!refine) done = true;
        for (int r = 0; r < CS; ++r) {
          SS* rs = cta_smem<CS>(&s, r);
          rs->dec_prefix = prefix;
          rs->dec_mask = pmask;
          rs->dec_cnt = cnt_a;
          rs->dec_sum = sum_a;
          rs->dec_cut = cut;
          rs->dec_done = done ? 1 : 0;
        }
      }
    }
    row_barrier<CS>();
    prefix = s.dec_prefix;
    pmask = s.dec_mask;
    cnt_a = s.dec_cnt;
    sum_a = s.dec_sum;
    cut = s.dec_cut;
    if (s.dec_done) break;
  }
  const int kap = cnt_a;
  const double tau = (sum_a - 1.0) / (double)kap;
  const float inv = (float)((double)a.scale / (double)kap);
  auto sel_of = [&](float x) -> bool {
    return x > t0 && (unsigned long long)sort_key(x) >= cut;
  };
  if (OUT == kOutGrad) {
    for_each_element<T, CS, VEC, NT>(zr, C, rank, [&](float x, int c) {
      float gv = sel_of(x) ? inv : 0.0f;
      if (c == yc) gv -= a.scale;
      st_elem(gr + c, gv);
    });
    // dense rows do not list their support (consumers fall back to the row)
    if (a.sup_cols && leader && tid == 0) a.sup_cols[row * (int64_t)a.sup_k] = -1;
  } else if (OUT == kOutMask) {
    for_each_element<T, CS, VEC, NT>(zr, C, rank, [&](float x, int c) { mr[c] = sel_of(x) ? 1 : 0; });
  } else if (OUT == kOutShard) {
    int* pos_ctr = &cta_smem<CS>(&s, 0)->cand_pos;
    const int K = a.shard_k;
    int32_t* rec = a.shard_sum + row * (int64_t)(kShardHeader + K);
    int32_t* ridx = a.shard_idx + row * (int64_t)K;
    for_each_element<T, CS, VEC, NT>(zr, C, rank, [&](float x, int c) {
      if (sel_of(x)) {
        const int p = atomicAdd(pos_ctr, 1);
        if (p < K) {
          rec[kShardHeader + p] = __float_as_int(x);
          ridx[p] = c;
        }
      }
    });
    row_barrier<CS>();
    if (leader && tid == 0) {
      rec[0] = __float_as_int(M);
      rec[1] = kap;
      rec[2] = 0;
      rec[3] = -1;
    }
    return;
  } else if (OUT == kOutNone) {
    // forward only: the decision is all that is needed, no second pass
  } else {
    int* pos_ctr = &cta_smem<CS>(&s, 0)->cand_pos;
    float* cv = a.cand_val + row * C;
    int32_t* ci = a.cand_idx + row * C;
    for_each_element<T, CS, VEC, NT>(zr, C, rank, [&](float x, int c) {
      if (sel_of(x)) {
        const int p = atomicAdd(pos_ctr, 1);
        cv[p] = x;
        ci[p] = c;
      }
    });
  }
  row_barrier<CS>();
  if (leader && tid == 0) {
    const float zy = yok ? s.label_z : CUDART_NAN_F;
    if (a.H) a.H[row] = threshold_fp32(M, tau);
    if (a.loss) a.loss[row] = yok ? row_loss(M, tau, zy) : CUDART_NAN_F;
    if (a.kappa) a.kappa[row] = kap;
    if (OUT == kOutCand && a.cand_count) a.cand_count[row] = kap;
    if (!yok) raise_status(a.status, 1);
  }
}

template <class T, int CS, bool VEC, int OUT, int SHAPE = kShapeWide>
__global__ void __launch_bounds__(stream_threads<SHAPE>(), stream_min_blocks<SHAPE>())
    fw_stream_rows_kernel(RowArgs a) {
  allow_dependent_launch();
  __shared__ StreamShared<stream_threads<SHAPE>() / 32> s;
  stream_rows_body<T, CS, VEC, OUT, SHAPE>(a, s);
  // A launch of the rows left over after the previous launch's whole waves
  // starts early, as that launch's programmatic dependent; it ends only after
  // that launch has completed, so the work queued after it sees every row.
  if (a.wait_prior) wait_prior_grid();
}

}  // namespace fwb200
