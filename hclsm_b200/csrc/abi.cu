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

namespace {
// Waits on an mbarrier that nothing ever completes, at most `polls` times, then
// records HCLSM_ERR_TIMEOUT and returns: the bounded-wait path every kernel of
// this library uses, exercised without a fault.
__global__ void selftest_wait_kernel(uint32_t polls, int* err, int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    hclsm::mbar_init(&bar, 1);
    hclsm::fence_mbar_init();
  }
  __syncthreads();
  const uint32_t addr = hclsm::smem_u32(&bar);
  uint32_t done = 0;
  for (uint32_t i = 0; i < polls && !done; ++i) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(0u)
        : "memory");
  }
  if (threadIdx.x == 0) {
    *status = done ? 0 : HCLSM_ERR_TIMEOUT;
    if (!done) hclsm::record_error(err, HCLSM_ERR_TIMEOUT);
  }
}
}  // namespace

extern "C" int hclsm_selftest_wait_timeout(uint32_t polls, int* status_dev, void* stream) {
  if (!status_dev) return HCLSM_ERR_NULL;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(polls, hclsm::device_err_ptr(), status_dev);
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}
