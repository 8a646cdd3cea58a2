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
//   * a call whose scratch need (hclsm_ssm_scan_bwd_workspace_size) exceeds
//     that size returns HCLSM_ERR_WORKSPACE and launches nothing;
//   * all calls on a device share the one array, which keeps the contents of
//     the last call.  Every word the backward reads from it is written earlier
//     in the same call, so nothing has to be cleared; but calls whose kernels
//     overlap on the GPU (different streams, no ordering between them) race
//     on the array and produce wrong results;
//   * the first call on each device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current).  Make that first call
//     before any stream capture.
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(48) << 20;

static __device__ __align__(256) unsigned char g_scan_bwd_scratch[kNoAllocScratchBytes];

constexpr int kMaxDev = 64;
void* g_scratch_ptr[kMaxDev] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (set up once per
// device).  Returns nullptr if the address cannot be resolved.
void* scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_scan_bwd_scratch) != cudaSuccess) return nullptr;
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" size_t hclsm_ssm_scan_bwd_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

extern "C" int hclsm_ssm_scan_bwd_noalloc(const void* x, const void* dt, const float* A_log, const void* B,
                                          const void* C, const float* D, const void* z, const void* dy,
                                          void* dx, void* ddt, float* dA_log, void* dB, void* dC, float* dD,
                                          void* dz, int64_t nseq, int32_t L, int32_t d_inner,
                                          int32_t d_state, int32_t dtype, int32_t clamp, void* stream) {
  const size_t need = hclsm_ssm_scan_bwd_workspace_size(nseq, L, d_inner, d_state);
  if (nseq > 0 && L > 0 && need == 0) return HCLSM_ERR_UNSUPPORTED;
  if (need > kNoAllocScratchBytes) return HCLSM_ERR_WORKSPACE;
  void* ws = scratch_for_current_device();
  if (!ws) return HCLSM_ERR_LAUNCH;
  return hclsm_ssm_scan_bwd(x, dt, A_log, B, C, D, z, dy, dx, ddt, dA_log, dB, dC, dD, dz, nseq, L, d_inner,
                            d_state, dtype, clamp, ws, kNoAllocScratchBytes, stream);
}
