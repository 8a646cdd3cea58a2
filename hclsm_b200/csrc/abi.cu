// Library-wide host helpers of the C ABI: version, per-device error word,
// SM count and shared-memory opt-in.
#include <mutex>

#include "common.cuh"

namespace {
// First error recorded by any kernel of this library on this device.
__device__ int g_hclsm_err = 0;

constexpr int kMaxDev = 64;
int* g_err_ptr[kMaxDev] = {};
int g_sms[kMaxDev] = {};
std::mutex g_mu;

int cur_dev() {
  int d = 0;
  cudaGetDevice(&d);
  return (d >= 0 && d < kMaxDev) ? d : 0;
}
}  // namespace

namespace hclsm {

int* device_err_ptr() {
  const int d = cur_dev();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[d]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_hclsm_err) != cudaSuccess) return nullptr;
    g_err_ptr[d] = static_cast<int*>(ptr);
  }
  return g_err_ptr[d];
}

int num_sms() {
  const int d = cur_dev();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

bool set_smem_limit(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return true;
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) == cudaSuccess;
}

}  // namespace hclsm

extern "C" int hclsm_version(void) { return 1; }

extern "C" int hclsm_device_error(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return HCLSM_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_hclsm_err, sizeof(int)) != cudaSuccess) return HCLSM_ERR_LAUNCH;
  const int zero = 0;
  cudaMemcpyToSymbol(g_hclsm_err, &zero, sizeof(int));
  return v;
}
