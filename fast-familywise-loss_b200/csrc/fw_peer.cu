// Cross-GPU loss sum over peer memory: the scalar exchange of row-sharded
// data parallelism done inside the loss reduction kernel itself.
//
// Every rank (one process per GPU) owns a small exchange buffer in its own
// HBM; the ranks map each other's buffers over NVLink / NVSwitch with CUDA
// IPC (fw_peer_buffer_create / fw_peer_buffer_open, exchanged once by the
// host).  One launch of fw_loss_allreduce_kernel on every rank then
//   1. sums this rank's per-row losses in fp64 (the fixed order of
//      fw_loss_reduce's one-CTA form),
//   2. stores the partial into its own cell of every rank's buffer (plain
//      stores to peer memory, each followed by a release store of the
//      launch's epoch to that cell),
//   3. waits (bounded) until every rank's cell in its own buffer carries the
//      epoch, and adds the partials in rank order: every rank computes the
//      same fp64 total and writes scale * total.
// No NCCL call and no host round trip: one kernel of one CTA per step, where
// the library path is a reduction kernel followed by an NCCL all-reduce.
//
// Epochs: the buffer counts its own launches (device side, so a CUDA graph
// replaying the launch advances it too); all ranks make the same sequence of
// calls, so launch e of every rank uses epoch e.  Cells are double-buffered
// by epoch parity: a rank can only reach epoch e + 2 (the same parity) after
// every rank has published e + 1, which each does after finishing e, so a
// cell is never overwritten before its reader has consumed it.
//
// Peer access is plain ld/st over NVLink (no TMA, no multicast objects).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>

#include "fw_reduce.cuh"
#include "fw_host.cuh"

namespace fwb200 {

constexpr int kPeerMax = FWB_PEER_MAX;

struct PeerCell {
  double val;
  unsigned long long epoch;
};

// Layout of one rank's exchange buffer (zeroed at creation).
struct __align__(256) PeerBuffer {
  PeerCell cell[2][kPeerMax];  // [epoch parity][writing rank]
  unsigned long long launches;  // this rank's launches so far (its own kernels only)
};
static_assert(sizeof(PeerBuffer) <= FWB_PEER_BUFFER_BYTES, "exchange buffer layout");

struct PeerSet {
  PeerBuffer* buf[kPeerMax];  // rank r's buffer as mapped in this process
  int world;
  int rank;
};

namespace {

__device__ __forceinline__ void st_relaxed_sys(double* p, double v) {
  asm volatile("st.relaxed.sys.global.f64 [%0], %1;" ::"l"(p), "d"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ double ld_relaxed_sys(const double* p) {
  double v;
  asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
  return v;
}

template <class T>
__global__ void __launch_bounds__(kReduceThreads)
    fw_loss_allreduce_kernel(const T* __restrict__ loss, int64_t B, double scale, T* __restrict__ out,
                             int vec, PeerSet ps, int32_t* status, unsigned long long limit_ns) {
  constexpr int N = Vec16<T>::N;
  __shared__ double part[kReduceThreads / 32];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  double s = thread_loss_sum<T>(loss, B, 0, (B + N - 1) / N, vec);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x >= 32) return;
  double t = (threadIdx.x < kReduceThreads / 32) ? part[threadIdx.x] : 0.0;
  t = warp_sum(t);
  if (threadIdx.x != 0) return;

  PeerBuffer* own = ps.buf[ps.rank];
  const unsigned long long e = own->launches + 1;
  own->launches = e;
  const int p = (int)(e & 1ull);
  for (int r = 0; r < ps.world; ++r) {
    PeerCell* c = &ps.buf[r]->cell[p][ps.rank];
    st_relaxed_sys(&c->val, t);
    st_release_sys(&c->epoch, e);  // orders the value before the epoch
  }
  const uint64_t t0 = global_ns();
  double total = 0.0;
  for (int r = 0; r < ps.world; ++r) {
    const PeerCell* c = &own->cell[p][r];
    unsigned int spins = 0;
    while (ld_acquire_sys(&c->epoch) != e) {
      if ((++spins & 63u) == 0 && global_ns() - t0 > limit_ns) {
        // a rank did not publish in time (it failed, or did not make the
        // same call): report it; the exchange cannot be reused after this
        raise_status(status, kStatusTimeout);
        out[0] = (T)NAN;
        return;
      }
      __nanosleep(32);
    }
    total += ld_relaxed_sys(&c->val);
  }
  out[0] = (T)(total * scale);
}

template <class T>
int launch_loss_allreduce(const T* loss, int64_t B, double scale, void* const* bufs, int world, int rank,
                          T* out, int32_t* status, double timeout_s, void* stream) {
  if (B < 0) return FWB_E_SHAPE;
  if (world < 1 || world > kPeerMax) return FWB_E_CAPACITY;
  if (rank < 0 || rank >= world) return FWB_E_SHAPE;
  if (!out || !bufs || (B > 0 && !loss)) return FWB_E_POINTER;
  if (!(timeout_s > 0.0) || timeout_s > 3600.0) return FWB_E_SHAPE;
  PeerSet ps = {};
  ps.world = world;
  ps.rank = rank;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r]) return FWB_E_POINTER;
    ps.buf[r] = static_cast<PeerBuffer*>(bufs[r]);
  }
  const unsigned long long limit = (unsigned long long)(timeout_s * 1e9);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kReduceThreads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int vec = aligned16(loss) ? 1 : 0;
  return launch_status(
      cudaLaunchKernelEx(&cfg, fw_loss_allreduce_kernel<T>, loss, B, scale, out, vec, ps, status, limit));
}

}  // namespace
}  // namespace fwb200

using namespace fwb200;

extern "C" {

FWB_API int fw_peer_buffer_create(void** buf, void* handle) {
  if (!buf || !handle) return FWB_E_POINTER;
  *buf = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, FWB_PEER_BUFFER_BYTES) != cudaSuccess) return FWB_E_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, FWB_PEER_BUFFER_BYTES) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return FWB_E_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == FWB_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *buf = p;
  return FWB_OK;
}

FWB_API int fw_peer_buffer_open(const void* handle, void** peer) {
  if (!handle || !peer) return FWB_E_POINTER;
  *peer = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return FWB_E_CUDA;
  *peer = p;
  return FWB_OK;
}

FWB_API int fw_peer_buffer_close(void* peer) {
  if (!peer) return FWB_E_POINTER;
  return cudaIpcCloseMemHandle(peer) == cudaSuccess ? FWB_OK : FWB_E_CUDA;
}

FWB_API int fw_peer_buffer_destroy(void* buf) {
  if (!buf) return FWB_E_POINTER;
  return cudaFree(buf) == cudaSuccess ? FWB_OK : FWB_E_CUDA;
}

FWB_API int fw_loss_allreduce(const float* loss, int64_t B, double scale, void* const* bufs, int world, int rank,
                              float* out, int32_t* status, double timeout_s, void* stream) {
  return launch_loss_allreduce<float>(loss, B, scale, bufs, world, rank, out, status, timeout_s, stream);
}

FWB_API int fw_loss_allreduce_f64(const double* loss, int64_t B, double scale, void* const* bufs, int world,
                                  int rank, double* out, int32_t* status, double timeout_s, void* stream) {
  return launch_loss_allreduce<double>(loss, B, scale, bufs, world, rank, out, status, timeout_s, stream);
}

}  // extern "C"
