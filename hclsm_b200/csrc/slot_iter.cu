// One whole slot-attention refinement step behind one C entry point
// (hclsm_slot_attn_iter): DynamicSlotAttention._iteration_step
// (hclsm/objects/dynamic_slots.py:98-131) for bf16 weight products with fp32
// accumulation and an fp32 carried state, for callers that do not go through
// the Python layer.  The stages are this library's kernels (LayerNorm, the
// tcgen05 attention core, GRUCell + LayerNorm, residual + clamp) around five
// library GEMMs (cuBLASLt, bf16 operands, fp32 accumulation): q = LN(s) W_q^T,
// gi = upd W_ih^T, gh = s W_hh^T, m1 = relu(LN(h) W1^T + b1) (bias and ReLU in
// the GEMM's epilogue, bf16 out), m2 = m1 W2^T.  The same sequence as the
// Python path (hclsm_b200.kernels.slot_attention_iteration, bf16).
#include <cublasLt.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "common.cuh"

extern "C" int hclsm_slot_attn_core(const void* Q, const void* K, const void* V, void* out, void* attn, int32_t F,
                                    int32_t N, int32_t M, int32_t D, float scale, float clamp, float eps,
                                    int32_t dtype, int32_t attn_f32, void* stream);
extern "C" int hclsm_layernorm(const float* x, const float* w, const float* b, void* y, int64_t rows, int32_t D,
                               float eps, int32_t out_dtype, void* stream);
extern "C" int hclsm_gru_cell(const float* gi, const float* gh, const float* b_ih, const float* b_hh,
                              const float* h, float* h_out, int64_t rows, int32_t H, void* stream);
extern "C" int hclsm_gru_cell_ln(const void* gi, const void* gh, int32_t gate_dtype, const float* b_ih,
                                 const float* b_hh, const float* h, float* h_out, const float* ln_w,
                                 const float* ln_b, void* ln_out, int32_t ln_dtype, int64_t rows, int32_t H,
                                 float eps, void* stream);
extern "C" int hclsm_residual_clamp(const float* h, const float* m, const float* b, float* out, void* out_bf16,
                                    int64_t rows, int32_t C, float clamp, void* stream);

namespace hclsm {
namespace slotiter {

constexpr size_t kLtWorkspace = size_t(32) << 20;  // cuBLASLt's own scratch, inside the caller's workspace
constexpr int kMaxDev = 64;

cublasLtHandle_t g_handle[kMaxDev] = {};
std::mutex g_mu;

cublasLtHandle_t handle_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_handle[dev] && cublasLtCreate(&g_handle[dev]) != CUBLAS_STATUS_SUCCESS) g_handle[dev] = nullptr;
  return g_handle[dev];
}

size_t al256(size_t x) { return (x + 255) & ~size_t(255); }

// workspace layout (bytes)
struct Layout {
  size_t sb, sn, q, upd, gi, gh, h, mln, m1, m2, lt, total;
  Layout(int64_t R, int D) {
    size_t o = 0;
    auto take = [&](size_t b) { size_t r = o; o = al256(o + b); return r; };
    sb = take(2 * R * D);       // slots, bf16
    sn = take(2 * R * D);       // LN(slots), bf16
    q = take(2 * R * D);        // q, bf16
    upd = take(2 * R * D);      // attention updates, bf16
    gi = take(4 * R * 3 * D);   // fp32 (bf16 on the row-fused path)
    gh = take(4 * R * 3 * D);   // fp32 (bf16 on the row-fused path)
    h = take(4 * R * D);        // GRU state, fp32
    mln = take(2 * R * D);      // LN(h), bf16
    m1 = take(2 * R * 4 * D);   // relu(.. W1^T + b1), bf16
    m2 = take(4 * R * D);       // fp32
    lt = take(kLtWorkspace);
    total = o;
  }
};

// C (rows x n, row-major) = A (rows x k, row-major, bf16) @ B (k x n, row-major,
// bf16), fp32 accumulation; C in c_type; optional bias (n) with ReLU.  In
// cuBLASLt's column-major view that is C^T (n x rows) = B^T (n x k) A^T.
int gemm(cublasLtHandle_t lt, const void* A, const void* B, void* C, cudaDataType_t c_type, int64_t rows, int n,
         int k, const void* bias, void* ws, size_t ws_bytes, cudaStream_t st) {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, lc = nullptr;
  cublasLtMatmulPreference_t pref = nullptr;
  int rc = HCLSM_ERR_LAUNCH;
  do {
    if (cublasLtMatmulDescCreate(&op, CUBLAS_COMPUTE_32F, CUDA_R_32F) != CUBLAS_STATUS_SUCCESS) break;
    if (bias) {
      const cublasLtEpilogue_t epi = CUBLASLT_EPILOGUE_RELU_BIAS;
      const cudaDataType_t bt = CUDA_R_16BF;
      if (cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi, sizeof(epi)) !=
              CUBLAS_STATUS_SUCCESS ||
          cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_POINTER, &bias, sizeof(bias)) !=
              CUBLAS_STATUS_SUCCESS ||
          cublasLtMatmulDescSetAttribute(op, CUBLASLT_MATMUL_DESC_BIAS_DATA_TYPE, &bt, sizeof(bt)) !=
              CUBLAS_STATUS_SUCCESS)
        break;
    }
    // column-major: "A" = B^T as an (n x k) matrix with leading dimension n, "B" = A^T (k x rows), ld k
    if (cublasLtMatrixLayoutCreate(&la, CUDA_R_16BF, n, k, n) != CUBLAS_STATUS_SUCCESS) break;
    if (cublasLtMatrixLayoutCreate(&lb, CUDA_R_16BF, k, rows, k) != CUBLAS_STATUS_SUCCESS) break;
    if (cublasLtMatrixLayoutCreate(&lc, c_type, n, rows, n) != CUBLAS_STATUS_SUCCESS) break;
    if (cublasLtMatmulPreferenceCreate(&pref) != CUBLAS_STATUS_SUCCESS) break;
    if (cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes,
                                             sizeof(ws_bytes)) != CUBLAS_STATUS_SUCCESS)
      break;
    cublasLtMatmulHeuristicResult_t res;
    int found = 0;
    if (cublasLtMatmulAlgoGetHeuristic(lt, op, la, lb, lc, lc, pref, 1, &res, &found) != CUBLAS_STATUS_SUCCESS ||
        found == 0) {
      rc = HCLSM_ERR_UNSUPPORTED;
      break;
    }
    const float alpha = 1.0f, beta = 0.0f;
    if (cublasLtMatmul(lt, op, &alpha, B, la, A, lb, &beta, C, lc, C, lc, &res.algo, ws, ws_bytes, st) !=
        CUBLAS_STATUS_SUCCESS)
      break;
    rc = HCLSM_OK;
  } while (false);
  if (pref) cublasLtMatmulPreferenceDestroy(pref);
  if (lc) cublasLtMatrixLayoutDestroy(lc);
  if (lb) cublasLtMatrixLayoutDestroy(lb);
  if (la) cublasLtMatrixLayoutDestroy(la);
  if (op) cublasLtMatmulDescDestroy(op);
  return rc;
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __float2bfloat16_rn(x[i]);
}

}  // namespace slotiter
}  // namespace hclsm

using namespace hclsm;
using namespace hclsm::slotiter;

extern "C" size_t hclsm_slot_attn_iter_workspace_size(int32_t F, int32_t N, int32_t D) {
  if (F <= 0 || N <= 0 || D <= 0) return 0;
  return Layout((int64_t)F * N, D).total;
}

extern "C" int hclsm_slot_attn_iter(const float* slots, const void* k, const void* v,
                                    const hclsm_slot_iter_weights* w, float* slots_out, void* slots_out_bf16,
                                    int32_t F, int32_t N, int32_t M, int32_t D, void* workspace,
                                    size_t workspace_bytes, void* stream) {
  if (!slots || !k || !v || !w || !slots_out) return HCLSM_ERR_NULL;
  if (!w->wq_t || !w->w_ih_t || !w->w_hh_t || !w->b_ih || !w->b_hh || !w->w1_t || !w->b1 || !w->w2_t)
    return HCLSM_ERR_NULL;
  if (F < 0 || N <= 0 || M <= 0 || D <= 0) return HCLSM_ERR_SHAPE;
  if (D % 8 != 0) return HCLSM_ERR_UNSUPPORTED;
  if (F == 0) return HCLSM_OK;
  const int64_t R = (int64_t)F * N;
  const Layout lay(R, D);
  if (!workspace || workspace_bytes < lay.total) return HCLSM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return HCLSM_ERR_ALIGN;
  cublasLtHandle_t lt = handle_for_current_device();
  if (!lt) return HCLSM_ERR_LAUNCH;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  auto* sb = reinterpret_cast<__nv_bfloat16*>(ws + lay.sb);
  auto* sn = reinterpret_cast<__nv_bfloat16*>(ws + lay.sn);
  auto* q = reinterpret_cast<__nv_bfloat16*>(ws + lay.q);
  auto* upd = reinterpret_cast<__nv_bfloat16*>(ws + lay.upd);
  auto* gi = reinterpret_cast<float*>(ws + lay.gi);
  auto* gh = reinterpret_cast<float*>(ws + lay.gh);
  auto* h = reinterpret_cast<float*>(ws + lay.h);
  auto* mln = reinterpret_cast<__nv_bfloat16*>(ws + lay.mln);
  auto* m1 = reinterpret_cast<__nv_bfloat16*>(ws + lay.m1);
  auto* m2 = reinterpret_cast<float*>(ws + lay.m2);
  void* ltws = ws + lay.lt;
  int rc;
  // slots in bf16 for the W_hh product
  {
    const int64_t n = R * D;
    const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 32);
    f32_to_bf16_kernel<<<blocks, 256, 0, st>>>(slots, sb, n);
    if (cudaGetLastError() != cudaSuccess) return HCLSM_ERR_LAUNCH;
  }
  if ((rc = hclsm_layernorm(slots, w->ln_attn_w, w->ln_attn_b, sn, R, D, 1e-5f, HCLSM_BF16, stream))) return rc;
  if ((rc = gemm(lt, sn, w->wq_t, q, CUDA_R_16BF, R, D, D, nullptr, ltws, kLtWorkspace, st))) return rc;
  if ((rc = hclsm_slot_attn_core(q, k, v, upd, nullptr, F, N, M, D, (float)(1.0 / sqrt((double)D)), 30.0f, 0.0f, HCLSM_BF16,
                                 0, stream)))
    return rc;
  // the row-fused GRU kernel reads bf16 gate products (what the reference's
  // GRUCell receives under bf16 autocast); the separate one reads fp32
  const bool fused = D % 128 == 0 && D <= 1024;
  const cudaDataType_t gt = fused ? CUDA_R_16BF : CUDA_R_32F;
  if ((rc = gemm(lt, upd, w->w_ih_t, gi, gt, R, 3 * D, D, nullptr, ltws, kLtWorkspace, st))) return rc;
  if ((rc = gemm(lt, sb, w->w_hh_t, gh, gt, R, 3 * D, D, nullptr, ltws, kLtWorkspace, st))) return rc;
  if (fused) {
    rc = hclsm_gru_cell_ln(gi, gh, HCLSM_BF16, w->b_ih, w->b_hh, slots, h, w->ln_mlp_w, w->ln_mlp_b, mln, HCLSM_BF16,
                           R, D, 1e-5f, stream);
  } else {
    rc = hclsm_gru_cell(gi, gh, w->b_ih, w->b_hh, slots, h, R, D, stream);
    if (!rc) rc = hclsm_layernorm(h, w->ln_mlp_w, w->ln_mlp_b, mln, R, D, 1e-5f, HCLSM_BF16, stream);
  }
  if (rc) return rc;
  if ((rc = gemm(lt, mln, w->w1_t, m1, CUDA_R_16BF, R, 4 * D, D, w->b1, ltws, kLtWorkspace, st))) return rc;
  if ((rc = gemm(lt, m1, w->w2_t, m2, CUDA_R_32F, R, D, 4 * D, nullptr, ltws, kLtWorkspace, st))) return rc;
  return hclsm_residual_clamp(h, m2, w->b2, slots_out, slots_out_bf16, R, D, 50.0f, stream);
}
