// Device helpers shared by every FW-loss kernel: order-preserving keys,
// NaN-propagating max, warp reductions and the exact threshold solver that
// runs on a short candidate list.
//
// Notation used throughout (one row z[0..C), label y):
//   M       row maximum (fp32, NaN if any element is NaN)
//   t0      __fsub_rd(M, 1): the largest fp32 <= M - 1.  Because
//           h* >= M - 1 (k = 1 in max_k (S_k - 1)/k), every support element
//           satisfies z > t0, so {z > t0} is a superset of the support.
//   d_j     (double)z_j - (double)M, the shifted logit (<= 0).  The search
//           runs in the shifted domain, tau = h* - M, which keeps the
//           arithmetic exact for magnitudes up to ~1e38 (z - M is exact for
//           every candidate when M >= 2, Sterbenz) where the unshifted
//           S_k - 1 would lose the 1 entirely.
#pragma once

#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math_constants.h>
#include <stdint.h>

namespace fwb200 {

constexpr unsigned kFull = 0xffffffffu;

// Output of the forward search: the gradient row, the support mask, or the
// support as a (value, column) list.
// kOutShard: one column shard of a class-sharded row (fw_shard.cuh): zero
// gradient shard, plus a summary record of the shard's own solve.
// kOutGradCols: kOutGrad that also lists the support columns (RowArgs::sup_cols);
// a separate instance in the register tier so that kOutGrad carries no extra
// code, a runtime check of sup_cols in the streaming tier.
// kOutNone: forward only -- H, loss and kappa, no per-element output (the
// logits are read once and nothing of size C is written).
enum OutMode : int { kOutGrad = 0, kOutMask = 1, kOutCand = 2, kOutShard = 3, kOutGradCols = 4, kOutNone = 5 };

// Summary record of one row of one class shard (int32 words):
//   [0] local maximum M_r (float bits)   [1] local support size kappa_r
//   [2] flags (bit 0: M_r is NaN or +-inf)
//   [3] local column of the first maximal element when bit 0 is set
//   [4 .. 4+K) the values (float bits) of the first min(kappa_r, K) local
//   support elements; their local columns go to a separate [B, K] array.
constexpr int kShardHeader = 4;
constexpr int kShardNonFinite = 1;

// Element types of logits and gradient.  Arithmetic is fp32/fp64 for all of
// them; a 16-byte slot holds kEPS elements.
template <class T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kEPS = 4;
  __device__ static float to_f(float x) { return x; }
  __device__ static float from_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kEPS = 8;
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  __device__ static float bits_to_f(uint32_t b) { return __uint_as_float(b << 16); }
  __device__ static uint32_t f_to_bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
};
template <> struct Elem<__half> {
  static constexpr int kEPS = 8;
  __device__ static float to_f(__half x) { return __half2float(x); }
  __device__ static __half from_f(float x) { return __float2half_rn(x); }
  __device__ static float bits_to_f(uint32_t b) { return __half2float(__ushort_as_half((unsigned short)b)); }
  __device__ static uint32_t f_to_bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
};

// 16-byte slot <-> kEPS floats.
template <class T>
__device__ __forceinline__ void unpack16(const uint4& u, float* out) {
  if constexpr (sizeof(T) == 4) {
    out[0] = __uint_as_float(u.x);
    out[1] = __uint_as_float(u.y);
    out[2] = __uint_as_float(u.z);
    out[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[2 * k] = Elem<T>::bits_to_f(w[k] & 0xffffu);
      out[2 * k + 1] = Elem<T>::bits_to_f(w[k] >> 16);
    }
  }
}

template <class T>
__device__ __forceinline__ uint4 pack16(const float* in) {
  if constexpr (sizeof(T) == 4) {
    return make_uint4(__float_as_uint(in[0]), __float_as_uint(in[1]), __float_as_uint(in[2]),
                      __float_as_uint(in[3]));
  } else {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[k] = Elem<T>::f_to_bits(in[2 * k]) | (Elem<T>::f_to_bits(in[2 * k + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// A 16-byte slot of -inf elements (padding past the end of a segment).
template <class T>
__device__ __forceinline__ uint4 neg_inf_slot() {
  constexpr uint32_t w = sizeof(T) == 4 ? 0xff800000u
                                        : (std::is_same<T, __nv_bfloat16>::value ? 0xff80ff80u : 0xfc00fc00u);
  return make_uint4(w, w, w, w);
}

// Streaming 16-byte load that does not pollute L1.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <class T>
__device__ __forceinline__ float ld_elem(const T* p) {
  return Elem<T>::to_f(*p);
}

template <class T>
__device__ __forceinline__ void st_elem(T* p, float v) {
  *p = Elem<T>::from_f(v);
}

struct RowArgs {
  const void* z;         // [B, ld] of the element type
  const int64_t* y;      // [B]
  int64_t B;
  int64_t C;
  int64_t ld;
  float scale;           // gradient scale (1/B for "mean")
  void* grad;            // kOutGrad: [B, ld] of the element type
  uint8_t* mask;         // kOutMask: [B, C]
  float* cand_val;       // kOutCand: [B, C]
  int32_t* cand_idx;     // kOutCand: [B, C]
  int32_t* cand_count;   // kOutCand: [B]
  float* H;              // [B] or null
  float* loss;           // [B] or null
  int32_t* kappa;        // [B] or null
  int32_t* status;       // device word or null
  int mask_vec;          // mask rows are 4-byte aligned (C % 4 == 0)
  int32_t* shard_sum;    // kOutShard: [B, kShardHeader + shard_k]
  int32_t* shard_idx;    // kOutShard: [B, shard_k]
  int shard_k;           // kOutShard: support entries kept per row
  int32_t* sup_cols;     // kOutGrad, optional: [B, sup_k] support columns (the first
                         // min(kappa, sup_k)); -1 in the first slot when not listed
  int sup_k;
  int wait_prior;        // streaming tier: wait for the previous grid before exiting
};

// max() that returns NaN when either input is NaN (fmaxf would drop it).
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Largest element of a 16-byte slot as fp32, NaN when any element is NaN:
// three max.NaN for fp32; for 16-bit types three packed max.NaN on element
// pairs, then the larger of the two halves (an exact selection, so the same
// value as the fp32 max over the unpacked elements up to the sign of a zero).
template <class T>
__device__ __forceinline__ float slot_max_nan(const uint4& u) {
  if constexpr (sizeof(T) == 4) {
    return max_nan(max_nan(__uint_as_float(u.x), __uint_as_float(u.y)),
                   max_nan(__uint_as_float(u.z), __uint_as_float(u.w)));
  } else {
    uint32_t a, b, c;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(a) : "r"(u.x), "r"(u.y));
      asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(b) : "r"(u.z), "r"(u.w));
      asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(c) : "r"(a), "r"(b));
    } else {
      asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(a) : "r"(u.x), "r"(u.y));
      asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(b) : "r"(u.z), "r"(u.w));
      asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(c) : "r"(a), "r"(b));
    }
    return max_nan(Elem<T>::bits_to_f(c & 0xffffu), Elem<T>::bits_to_f(c >> 16));
  }
}


// Order-preserving fp32 -> uint32 key.  -0.0 is folded onto +0.0 first, so
// that keys order exactly like the float comparison used for selection
// (the reference keys -0.0 below +0.0, src/cuda/fw_radix_argmax.cu:60-69).
__device__ __forceinline__ uint32_t sort_key(float z) {
  uint32_t b = __float_as_uint(z);
  b = (b == 0x80000000u) ? 0u : b;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Inverse of sort_key (maps the +0.0 key back to +0.0).
__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(b);
}

__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max_nan(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Butterfly sum: every lane ends with the bit-identical total (each step adds
// a pair in both orders, which IEEE addition makes equal), and the order is
// fixed, so the result is deterministic.
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum(int v) { return __reduce_add_sync(kFull, v); }

__device__ __forceinline__ int warp_excl_scan(int v, int lane) {
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(kFull, x, o);
    if (lane >= o) x += t;
  }
  return x - v;
}

__device__ __forceinline__ unsigned lanemask_lt(int lane) { return (1u << lane) - 1u; }

// Lane-group helpers: a "group" is G consecutive lanes of a warp (G = 4, 8,
// 16 or 32) with member mask gmask; xor offsets below G never leave the group.
template <int G>
__device__ __forceinline__ float group_max_nan(float v, unsigned gmask) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v = max_nan(v, __shfl_xor_sync(gmask, v, o));
  return v;
}

template <int G>
__device__ __forceinline__ double group_sum(double v, unsigned gmask) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(gmask, v, o);
  return v;
}

// One redux.sync for a whole warp; xor shuffles inside smaller groups
// (redux.sync over partial member masks, one per group of a warp, was
// measured slower on B200: cfg3, 8-lane groups, 15.5 -> 17.2 us).
template <int G>
__device__ __forceinline__ int group_sum(int v, unsigned gmask) {
  if constexpr (G == 32) {
    return __reduce_add_sync(gmask, v);
  } else {
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(gmask, v, o);
    return v;
  }
}

template <int G>
__device__ __forceinline__ unsigned group_min(unsigned v, unsigned gmask) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(gmask, v, o));
  return v;
}

template <int G>
__device__ __forceinline__ int group_excl_scan(int v, int li, unsigned gmask) {
  int x = v;
#pragma unroll
  for (int o = 1; o < G; o <<= 1) {
    const int t = __shfl_up_sync(gmask, x, o, G);
    if (li >= o) x += t;
  }
  return x - v;
}

// fp32 threshold of a shifted threshold t: H(t) = M + t rounded toward -inf
// in two directed steps, so that for every fp32 x:  x > H(t) <=> x > M + t
// (exact real).  Selection always uses this predicate, which makes the
// support, kappa and the emitted H consistent by construction.
__device__ __forceinline__ float threshold_fp32(float M, double tau) {
  return __double2float_rd(__dadd_rd((double)M, tau));
}

// Exact threshold on a candidate list (Michelot's fixed-point iteration,
// i.e. Newton's method from below on f(t) = sum_j max(z_j - M - t, 0) - 1).
// `L` holds n >= 1 candidate logits (a superset of the support; it always
// contains the row maximum).  Iterates T <- {x in T : x > H(t_T)},
// t_T = (sum_T (x - M) - 1)/|T| until |T| stops changing.  The sets are
// nested and each step removes at least one element, so at most n + 1
// passes run.  At the fixed point every x in T exceeds M + t and every
// removed x does not, hence T is exactly the support and t = h* - M.  Sums
// are fp64 in a fixed order (lane-strided, then a butterfly), so the result
// is deterministic.  All G lanes of the group must call it with the same
// arguments; all return the same (tau, kappa).
// CAP > 0 bounds n (n <= CAP) and turns the per-lane loop into CAP/G
// predicated steps; CAP == 0 means any n.  The kept count is reduced first
// (one redux.sync); the fp64 sum only when the set changed, so the final,
// confirming pass costs no fp64 reduction.
template <int G, int CAP = 0>
__device__ __forceinline__ void michelot_list(const float* L, int n, float M, int li,
                                              unsigned gmask, double& tau, int& kappa) {
  const double Md = (double)M;
  double t = -CUDART_INF;
  float Ht = -CUDART_INF_F;
  int prev = -1;
  for (int it = 0; it <= n; ++it) {
    double s = 0.0;
    int c = 0;
    if constexpr (CAP > 0) {
#pragma unroll
      for (int k = 0; k < CAP / G; ++k) {
        const int i = li + k * G;
        const float x = (i < n) ? L[i] : -CUDART_INF_F;
        if (x > Ht) { s += (double)x - Md; ++c; }
      }
    } else {
      for (int i = li; i < n; i += G) {
        const float x = L[i];
        if (x > Ht) { s += (double)x - Md; ++c; }
      }
    }
    c = group_sum<G>(c, gmask);
    if (c == prev) break;
    s = group_sum<G>(s, gmask);
    prev = c;
    t = (s - 1.0) / (double)c;
    Ht = threshold_fp32(M, t);
  }
  tau = t;
  kappa = prev;
}

// Michelot's fixed point with at most one candidate per lane: x is this
// lane's candidate (-inf when it has none), n >= 1 the number of candidates
// in the group, all of them above t0.  Counts are one ballot; the fp64 sum a
// butterfly, taken only while the kept set changes.  Same sets, threshold
// predicate and result as michelot_list on the same candidates.
template <int G>
__device__ __forceinline__ void michelot_lane(float x, int n, float M, unsigned gmask, double& tau,
                                              int& kappa) {
  const double d = (double)x - (double)M;  // used only where x is kept
  double s = group_sum<G>(x > -CUDART_INF_F ? d : 0.0, gmask);
  int cnt = n;
  double t = (s - 1.0) / (double)cnt;
  for (int it = 0; it < n; ++it) {
    const float Ht = threshold_fp32(M, t);
    const bool keep = x > Ht;
    const int c = __popc(__ballot_sync(gmask, keep) & gmask);
    if (c == cnt) break;
    s = group_sum<G>(keep ? d : 0.0, gmask);
    cnt = c;
    t = (s - 1.0) / (double)cnt;
  }
  tau = t;
  kappa = cnt;
}

// Michelot's fixed point on a row held in registers (NV values per lane, G
// lanes), starting from the superset {v > t0}.  Each pass counts and sums the
// kept values; the count is reduced first (one redux.sync) and the fp64 sum
// only while the kept set changes.  A set of one element is the maximum
// alone: tau = -1 exactly, no further pass.  The threshold is never below t0,
// so the sets are nested and at most (candidates + 1) passes run.
template <int G, int NV>
__device__ __forceinline__ void michelot_regs(const float (&v)[NV], float M, float t0, unsigned gmask,
                                              double& tau, int& kappa) {
  const double Md = (double)M;
  double t = -CUDART_INF;
  float Ht = t0;
  int prev = -1;
  for (int it = 0; it <= G * NV; ++it) {
    double s = 0.0;
    int c = 0;
#pragma unroll
    for (int k = 0; k < NV; ++k)
      if (v[k] > Ht) { s += (double)v[k] - Md; ++c; }
    c = group_sum<G>(c, gmask);
    if (c == prev) break;
    prev = c;
    if (c == 1) {  // the maximum alone: h* = M - 1
      t = -1.0;
      break;
    }
    s = group_sum<G>(s, gmask);
    t = (s - 1.0) / (double)c;
    Ht = fmaxf(threshold_fp32(M, t), t0);
  }
  tau = t;
  kappa = prev;
}

// Per-row loss 1 - z_y + h* from the shifted threshold.
__device__ __forceinline__ float row_loss(float M, double tau, float zy) {
  return (float)(1.0 + ((double)M - (double)zy) + tau);
}

// Lets the kernel launched after this one on the stream as a programmatic
// dependent (the loss reduction) be scheduled before this grid ends; the
// dependent still waits (griddepcontrol.wait) for this grid to complete and
// its writes to be visible before it reads anything.  A no-op when the next
// launch is an ordinary one.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void raise_status(int32_t* status, int bits) {
  if (status) atomicOr(reinterpret_cast<int*>(status), bits);
}

// Status bit of a bounded on-chip wait that gave up (FWB_STATUS_TIMEOUT).
constexpr int kStatusTimeout = 4;

// ------------------------------------------------ mbarriers and bulk copies
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Waits at most limit_ns for the phase of the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > limit_ns) return false;
  }
}

// Non-multicast bulk copy of `bytes` (a multiple of 16, both addresses
// 16-byte aligned) from this GPU's global memory into this CTA's shared
// memory; completion is counted on `bar` (complete_tx).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Streaming 128-bit load that does not pollute L1.
__device__ __forceinline__ float4 ld_stream4(const float* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float ld_stream1(const float* p) {
  float r;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r) : "l"(p));
  return r;
}

}  // namespace fwb200
