// LM-head FW-loss forward for callers that cannot allocate device memory.
//
// fw_lmhead_fused_scan writes per-(row, chunk) summary records, the
// support's local columns and the label logits into workspace that the caller
// allocates, and fw_chunks_solve reads them back.  Some callers cannot call
// cudaMalloc at all: a plugin that runs inside a host framework which owns
// every byte of device memory through its own pool and exposes no allocator
// hook, an inference server that forbids allocation once its memory plan is
// fixed, or a C / Go / Java host that only holds the buffers handed to it.
// fw_lmhead_fused_loss_noalloc runs the same two kernels with that workspace
// in a fixed array that lives in this file (a static __device__ array), so
// the caller passes only its inputs and outputs.
//
// The array costs FWB_NOALLOC_SCRATCH_BYTES (16 MiB) of device memory on
// every GPU that loads this library, held until the process exits.  The first
// call in a CUDA context looks up the array's device address
// (cudaGetSymbolAddress, with that context current) and caches it together
// with the context's unique id; a call in another context -- another device,
// or the same device after cudaDeviceReset made a new primary context -- looks
// the address up again.  Make the first call on each device before any stream
// capture.  Every call shares the array: calls whose work overlaps on the GPU
// (different streams, or different host threads on the same device without
// ordering) race on it.  Nothing in it has to start at zero: each call writes
// every word that its solve step reads before reading it, so the contents
// left behind by the previous call are never used.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/fwloss_b200.h"

namespace {

constexpr int64_t kNoAllocScratchWords = FWB_NOALLOC_SCRATCH_BYTES / 4;
constexpr int kNoAllocMaxDevices = 64;
constexpr int64_t kSegmentAlignWords = 64;  // 256-byte segment starts

// The workspace.  In host code this name is only a host-side stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocScratchWords];

// The chunk solve gathers at most this many support values per row
// (nchunks * K); it matches fw_chunks_solve's own limit, so that a problem it
// would refuse is refused here before any kernel touches the array.
constexpr int kNoAllocChunkListCap = 256;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

template <class F>
F driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return reinterpret_cast<F>(p);
}

// Unique id of the calling thread's current context (0 if there is none or
// the driver cannot say).  Ids are never reused within a process, so a
// context made by a device reset gets a new one.
unsigned long long current_context_id() {
  static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

struct ScratchSlot {
  unsigned long long ctx_id;  // context the address belongs to (0: none cached)
  int32_t* addr;
};
ScratchSlot g_scratch[kNoAllocMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of the workspace in the current context: looked up with
// that context current on the first call in it, then served from the cache
// while the same context stays current.  NULL if the lookup fails.
int32_t* scratch_on_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  const unsigned long long id = current_context_id();
  if (id != 0 && g_scratch[dev].ctx_id == id && g_scratch[dev].addr) return g_scratch[dev].addr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
    cudaGetLastError();  // clear the error so that a later call's launch check does not report it
    return nullptr;
  }
  // the lookup made the device's context current if none was; key the cache
  // by it (no id available: nothing is cached and every call looks it up)
  g_scratch[dev].ctx_id = current_context_id();
  g_scratch[dev].addr = static_cast<int32_t*>(p);
  return g_scratch[dev].addr;
}

inline int64_t round_up(int64_t n, int64_t a) { return (n + a - 1) / a * a; }

}  // namespace

extern "C" {

int fw_lmhead_fused_loss_noalloc(int dtype, const void* hidden, int64_t B, int64_t D, const void* weight,
                                 int64_t C, int nchunks, const int64_t* col_start, int K, const int64_t* y,
                                 float* H, int32_t* kappa, float* loss, int32_t* sup_cols, int32_t* fb_rows,
                                 int32_t* fb_count, int32_t* status, void* stream) {
  // Range checks first, so that the workspace arithmetic cannot overflow; the
  // shape and pointer checks of the two steps below still apply.
  if (B < 0 || B > ((int64_t)1 << 31)) return FWB_E_SHAPE;
  if (nchunks < 1 || nchunks > 16 || K < 1 || K > 64 || nchunks * K > kNoAllocChunkListCap)
    return FWB_E_CAPACITY;
  const int64_t summ_words = round_up((int64_t)nchunks * B * (4 + K), kSegmentAlignWords);
  const int64_t idx_words = round_up((int64_t)nchunks * B * K, kSegmentAlignWords);
  if (summ_words + idx_words + B > kNoAllocScratchWords) return FWB_E_CAPACITY;
  int32_t* base = scratch_on_current_device();
  if (!base) return FWB_E_LAUNCH;
  int32_t* summaries = base;
  int32_t* local_idx = base + summ_words;
  float* zy = reinterpret_cast<float*>(base + summ_words + idx_words);
  int rc = fw_lmhead_fused_scan(dtype, hidden, B, D, weight, C, nchunks, col_start, K, y, zy, summaries,
                                local_idx, status, stream);
  if (rc != FWB_OK) return rc;
  return fw_chunks_solve(summaries, local_idx, nchunks, col_start, B, K, zy, y, H, kappa, loss, sup_cols,
                         fb_rows, fb_count, status, stream);
}

}  // extern "C"
