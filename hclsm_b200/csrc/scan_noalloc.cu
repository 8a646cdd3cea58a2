// Allocation-free variant of the selective-scan backward.
//
// Some callers cannot allocate device memory at the point where they need the
// backward: code running inside a host callback or a custom allocator hook,
// hosts that forbid cudaMalloc after start-up (pre-planned memory budgets), or
// runtimes whose own allocator must not be re-entered.  For them this file
// keeps the backward's scratch in a fixed, file-scope device array instead of
// a caller-provided workspace.
//
// Limits and behaviour:
//   * the array holds kNoAllocScratchBytes (48 MiB).  It is part of this
//     library's device image, so every GPU that loads the library keeps it
//     until the process exits;
//   * arguments are validated exactly as hclsm_ssm_scan_bwd validates them
//     (same status codes); a valid call whose scratch need
//     (hclsm_ssm_scan_bwd_workspace_size) exceeds the array's size returns
//     HCLSM_ERR_WORKSPACE and launches nothing;
//   * all calls on a device share the one array, which keeps the contents of
//     the last call.  Every word the backward reads from it is written earlier
//     in the same call, so nothing has to be cleared; but calls whose kernels
//     overlap on the GPU (different streams, no ordering between them) race
//     on the array and produce wrong results;
//   * the array's device address is resolved with cudaGetSymbolAddress the
//     first time a call runs under a given CUDA context (the device's primary
//     context, or a context the caller made current through the driver API),
//     with that context current, and cached per context.  A context created
//     later, including the primary context after a device reset, gets its own
//     resolution.  Make the first call under each context before any stream
//     capture.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(48) << 20;

static __device__ __align__(256) unsigned char g_scan_bwd_scratch[kNoAllocScratchBytes];

// driver entry points fetched through the runtime (the library links no libcuda)
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

struct CacheEntry {
  unsigned long long ctx_id;
  void* ptr;
};
constexpr int kMaxCtx = 64;
CacheEntry g_cache[kMaxCtx] = {};
int g_cache_n = 0;
CtxGetCurrentFn g_get_current = nullptr;
CtxGetIdFn g_get_id = nullptr;
bool g_fns_tried = false;
std::mutex g_mu;

// Identity of the context the runtime will use for this call.  cudaFree(0)
// is not used: it would create the primary context as a side effect; the
// runtime's own cudaGetDevice already did the lazy initialisation.
bool current_ctx_id(unsigned long long* id) {
  if (!g_fns_tried) {
    g_fns_tried = true;
    cudaDriverEntryPointQueryResult q1, q2;
    void* f1 = nullptr;
    void* f2 = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f1, 12000, cudaEnableDefault, &q1) == cudaSuccess &&
        q1 == cudaDriverEntryPointSuccess &&
        cudaGetDriverEntryPointByVersion("cuCtxGetId", &f2, 12000, cudaEnableDefault, &q2) == cudaSuccess &&
        q2 == cudaDriverEntryPointSuccess) {
      g_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
      g_get_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
  }
  if (!g_get_current || !g_get_id) return false;
  CUcontext ctx = nullptr;
  if (g_get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return g_get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of the scratch array under the current context (resolved once
// per context).  Returns nullptr if it cannot be resolved.
void* scratch_for_current_context() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;  // also makes the runtime's context current
  std::lock_guard<std::mutex> lk(g_mu);
  unsigned long long id = 0;
  if (!current_ctx_id(&id)) return nullptr;
  for (int i = 0; i < g_cache_n; ++i)
    if (g_cache[i].ctx_id == id) return g_cache[i].ptr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_scan_bwd_scratch) != cudaSuccess || p == nullptr) return nullptr;
  if (g_cache_n < kMaxCtx) {
    g_cache[g_cache_n++] = {id, p};
  } else {
    // table full: overwrite the oldest entry (contexts that are gone keep their ids forever)
    for (int i = 1; i < kMaxCtx; ++i) g_cache[i - 1] = g_cache[i];
    g_cache[kMaxCtx - 1] = {id, p};
  }
  return p;
}

}  // namespace

extern "C" size_t hclsm_ssm_scan_bwd_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

extern "C" int hclsm_ssm_scan_bwd_noalloc(const void* x, const void* dt, const float* A_log, const void* B,
                                          const void* C, const float* D, const void* z, const void* dy,
                                          void* dx, void* ddt, float* dA_log, void* dB, void* dC, float* dD,
                                          void* dz, int64_t nseq, int32_t L, int32_t d_inner,
                                          int32_t d_state, int32_t dtype, int32_t clamp, void* stream) {
  const size_t need = hclsm_ssm_scan_bwd_workspace_size(nseq, L, d_inner, d_state);
  if (need > kNoAllocScratchBytes) {
    // no workspace at all: the workspace entry point runs its own argument
    // checks (returning their status for a bad call) and then reports
    // HCLSM_ERR_WORKSPACE without launching anything
    return hclsm_ssm_scan_bwd(x, dt, A_log, B, C, D, z, dy, dx, ddt, dA_log, dB, dC, dD, dz, nseq, L, d_inner,
                              d_state, dtype, clamp, nullptr, 0, stream);
  }
  void* ws = scratch_for_current_context();
  if (!ws) return HCLSM_ERR_LAUNCH;
  return hclsm_ssm_scan_bwd(x, dt, A_log, B, C, D, z, dy, dx, ddt, dA_log, dB, dC, dD, dz, nseq, L, d_inner,
                            d_state, dtype, clamp, ws, kNoAllocScratchBytes, stream);
}
