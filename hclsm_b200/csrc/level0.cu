// Level0SSM around its SSM blocks (hclsm/dynamics/level0_ssm.py:159-220):
//
//  * the global track's input, a masked mean over the objects
//      global_in[b, t, :] = sum_n mask[b, n] obj[b, n, t, :] / max(sum_n mask[b, n], 1)
//    (the plain mean over n without a mask), :175-180;
//  * the epilogue after the per-object blocks, one pass instead of four:
//      out = clamp(nan_to_num(x, 0, +100, -100), -100, 100) * mask[b, n]   :210-218
//    and its backward, g * mask * [x finite and |x| <= 100] (the gradients of
//    nan_to_num and of an inclusive clamp).
//
// Both are memory-bound element-wise passes: grid-stride loops over the
// contiguous (T * D) rows, fp32 arithmetic, fp32 or bf16 storage.
#include <algorithm>

#include "common.cuh"

namespace hclsm {
namespace level0 {

template <typename TI, typename TO>
__global__ void pool_kernel(const TI* __restrict__ obj, const float* __restrict__ mask, TO* __restrict__ out, int B,
                            int N, int64_t TD) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)B * TD;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / TD, e = i - b * TD;
    const TI* src = obj + b * N * TD + e;
    float acc = 0.0f, alive = 0.0f;
    for (int n = 0; n < N; ++n) {
      const float m = mask ? mask[b * N + n] : 1.0f;
      acc = fmaf(io<TI>::ld(src + (int64_t)n * TD), m, acc);
      alive += m;
    }
    io<TO>::st(out + i, mask ? acc / fmaxf(alive, 1.0f) : acc / (float)N);
  }
}

__device__ __forceinline__ float nan_to_num_clamp(float v) {
  v = isnan(v) ? 0.0f : v;
  return fminf(fmaxf(v, -100.0f), 100.0f);  // +-inf land on the bounds, as nan_to_num's +-100 do
}

template <typename TI, typename TO>
__global__ void epilogue_kernel(const TI* __restrict__ x, const float* __restrict__ mask, TO* __restrict__ out,
                                int64_t total, int64_t TD) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    float v = nan_to_num_clamp(io<TI>::ld(x + i));
    if (mask) v *= mask[i / TD];
    io<TO>::st(out + i, v);
  }
}

template <typename TX, typename TG>
__global__ void epilogue_bwd_kernel(const TX* __restrict__ x, const float* __restrict__ mask,
                                    const TG* __restrict__ g, TX* __restrict__ gx, int64_t total, int64_t TD) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = io<TX>::ld(x + i);
    const bool pass = isfinite(v) && v >= -100.0f && v <= 100.0f;
    float gv = pass ? io<TG>::ld(g + i) : 0.0f;
    if (mask) gv *= mask[i / TD];
    io<TX>::st(gx + i, gv);
  }
}

static unsigned blocks_for(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16));
}

}  // namespace level0
}  // namespace hclsm

using namespace hclsm;
using namespace hclsm::level0;

#define HCLSM_L0_DISPATCH2(DA, DB, CALL)                                                   \
  do {                                                                                     \
    if ((DA) == HCLSM_F32 && (DB) == HCLSM_F32) { using TA = float; using TB = float; CALL; } \
    else if ((DA) == HCLSM_F32 && (DB) == HCLSM_BF16) { using TA = float; using TB = __nv_bfloat16; CALL; } \
    else if ((DA) == HCLSM_BF16 && (DB) == HCLSM_F32) { using TA = __nv_bfloat16; using TB = float; CALL; } \
    else if ((DA) == HCLSM_BF16 && (DB) == HCLSM_BF16) { using TA = __nv_bfloat16; using TB = __nv_bfloat16; CALL; } \
    else return HCLSM_ERR_DTYPE;                                                           \
  } while (0)

extern "C" int hclsm_l0_pool(const void* obj, int32_t obj_dtype, const float* mask, void* out, int32_t out_dtype,
                             int32_t B, int32_t N, int64_t TD, void* stream) {
  if (!obj || !out) return HCLSM_ERR_NULL;
  if (B < 0 || N <= 0 || TD < 0) return HCLSM_ERR_SHAPE;
  if ((int64_t)B * TD == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = blocks_for((int64_t)B * TD);
  HCLSM_L0_DISPATCH2(obj_dtype, out_dtype,
                     return launch_pdl(pool_kernel<TA, TB>, grid, 256, 0, st, static_cast<const TA*>(obj), mask,
                                       static_cast<TB*>(out), B, N, TD));
}

extern "C" int hclsm_l0_epilogue(const void* x, int32_t x_dtype, const float* mask, void* out, int32_t out_dtype,
                                 int32_t B, int32_t N, int64_t TD, void* stream) {
  if (!x || !out) return HCLSM_ERR_NULL;
  if (B < 0 || N < 0 || TD < 0) return HCLSM_ERR_SHAPE;
  const int64_t total = (int64_t)B * N * TD;
  if (total == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HCLSM_L0_DISPATCH2(x_dtype, out_dtype,
                     return launch_pdl(epilogue_kernel<TA, TB>, blocks_for(total), 256, 0, st,
                                       static_cast<const TA*>(x), mask, static_cast<TB*>(out), total, TD));
}

extern "C" int hclsm_l0_epilogue_bwd(const void* x, int32_t x_dtype, const float* mask, const void* g,
                                     int32_t g_dtype, void* gx, int32_t B, int32_t N, int64_t TD, void* stream) {
  if (!x || !g || !gx) return HCLSM_ERR_NULL;
  if (B < 0 || N < 0 || TD < 0) return HCLSM_ERR_SHAPE;
  const int64_t total = (int64_t)B * N * TD;
  if (total == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HCLSM_L0_DISPATCH2(x_dtype, g_dtype,
                     return launch_pdl(epilogue_bwd_kernel<TA, TB>, blocks_for(total), 256, 0, st,
                                       static_cast<const TA*>(x), mask, static_cast<const TB*>(g),
                                       static_cast<TA*>(gx), total, TD));
}
