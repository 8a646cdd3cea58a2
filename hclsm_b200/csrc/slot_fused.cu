// Row-fused element-wise stages of the slot-attention iteration (sm_100a):
// each kernel finishes one stage of DynamicSlotAttention._iteration_step
// (hclsm/objects/dynamic_slots.py:98-131) and applies the LayerNorm that the
// next stage starts with, so the row is read once:
//
//   gru_ln:            h = GRUCell(gi, gh, biases, h_prev)      (:123-126)
//                      m = LayerNorm_norm_slots(h)              (:128)
//   residual_clamp_ln: s = clamp(h + mlp_out + b2, +-c)         (:128-130)
//                      n = LayerNorm_norm_pre_attn(s)           (:111, next iteration)
//
// One warp per row, lane l owning the float4 columns 4 l + 128 j; rows of
// 128 to 1024 columns in multiples of 128 (others: HCLSM_ERR_UNSUPPORTED,
// use the separate kernels).
#include "common.cuh"

namespace hclsm {
namespace slotfused {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
// four gate values as fp32 from fp32 or bf16 storage (16- or 8-byte load)
__device__ __forceinline__ float4 ldg4(const float* p) { return ld4(p); }
__device__ __forceinline__ float4 ldg4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float at(const float4& v, int k) { return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w; }

// LayerNorm of a row held as NV float4 per lane (lane l owns columns
// 4 l + 128 j .. + 3), written to y (TO).
template <int NV, typename TO>
__device__ __forceinline__ void row_layernorm(const float4 (&v)[NV], int lane, const float* w, const float* b,
                                              float eps, TO* y) {
  constexpr int D = 128 * NV;
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
  const float mu = warp_sum(s) / D;
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float t = at(v[j], k) - mu;
      q += t * t;
    }
  const float rs = rsqrtf(warp_sum(q) / D + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = 4 * lane + 128 * j;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[k] = (at(v[j], k) - mu) * rs;
      if (w) o[k] *= w[c + k];
      if (b) o[k] += b[c + k];
    }
    if constexpr (sizeof(TO) == 2) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]), hi = __floats2bfloat162_rn(o[2], o[3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&lo);
      u.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(y + c) = u;
    } else {
      st4(reinterpret_cast<float*>(y) + c, make_float4(o[0], o[1], o[2], o[3]));
    }
  }
}

// torch.nn.GRUCell (gates r, z, n; gi = x W_ih^T, gh = h W_hh^T without
// biases, stored as TG = fp32 or bf16; gate arithmetic in fp32 as in
// hclsm_gru_cell), then LayerNorm of the new state.  One warp per row of
// H = 128 NV columns.
template <int NV, typename TO, typename TG>
__global__ void gru_ln_kernel(const TG* __restrict__ gi, const TG* __restrict__ gh,
                              const float* __restrict__ b_ih, const float* __restrict__ b_hh,
                              const float* __restrict__ h, float* __restrict__ h_out, const float* __restrict__ lnw,
                              const float* __restrict__ lnb, TO* __restrict__ ln_out, int64_t rows, float eps) {
  constexpr int H = 128 * NV;
  pdl_wait();
  pdl_trigger();
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const TG* gir = gi + r * 3 * H;
  const TG* ghr = gh + r * 3 * H;
  float4 v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = 4 * lane + 128 * j;
    const float4 ir = ldg4(gir + c), iz = ldg4(gir + H + c), in = ldg4(gir + 2 * H + c);
    const float4 hr = ldg4(ghr + c), hz = ldg4(ghr + H + c), hn = ldg4(ghr + 2 * H + c);
    const float4 bir = ld4(b_ih + c), biz = ld4(b_ih + H + c), bin = ld4(b_ih + 2 * H + c);
    const float4 bhr = ld4(b_hh + c), bhz = ld4(b_hh + H + c), bhn = ld4(b_hh + 2 * H + c);
    const float4 hv = ld4(h + r * H + c);
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float rg = sigmoid(at(ir, k) + at(hr, k) + (at(bir, k) + at(bhr, k)));
      const float zg = sigmoid(at(iz, k) + at(hz, k) + (at(biz, k) + at(bhz, k)));
      const float pre = at(in, k) + at(bin, k) + rg * (at(hn, k) + at(bhn, k));
      const float ng = 2.0f * sigmoid(2.0f * pre) - 1.0f;  // tanh
      o[k] = (1.0f - zg) * ng + zg * at(hv, k);
    }
    v[j] = make_float4(o[0], o[1], o[2], o[3]);
    st4(h_out + r * H + c, v[j]);
  }
  row_layernorm<NV, TO>(v, lane, lnw, lnb, eps, ln_out + r * H);
}

// s = clamp((h + m) + b, -c, c) (fp32, plus an optional bf16 copy; m stored
// as TM = fp32 or bf16), then LayerNorm of s.
template <int NV, typename TO, typename TM>
__global__ void residual_clamp_ln_kernel(const float* __restrict__ h, const TM* __restrict__ m,
                                         const float* __restrict__ b, float* __restrict__ out,
                                         __nv_bfloat16* __restrict__ out_bf16, const float* __restrict__ lnw,
                                         const float* __restrict__ lnb, TO* __restrict__ ln_out, int64_t rows, float c,
                                         float eps) {
  constexpr int C = 128 * NV;
  pdl_wait();
  pdl_trigger();
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float4 v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int col = 4 * lane + 128 * j;
    const float4 hv = ld4(h + r * C + col), mv = ldg4(m + r * C + col);
    float s[4] = {hv.x + mv.x, hv.y + mv.y, hv.z + mv.z, hv.w + mv.w};
    if (b) {
      const float4 bb = ld4(b + col);
      s[0] += bb.x; s[1] += bb.y; s[2] += bb.z; s[3] += bb.w;
    }
    if (c > 0.0f) {
#pragma unroll
      for (int k = 0; k < 4; ++k) s[k] = fminf(fmaxf(s[k], -c), c);
    }
    v[j] = make_float4(s[0], s[1], s[2], s[3]);
    st4(out + r * C + col, v[j]);
    if (out_bf16) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(s[0], s[1]), hi = __floats2bfloat162_rn(s[2], s[3]);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&lo);
      u.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(out_bf16 + r * C + col) = u;
    }
  }
  row_layernorm<NV, TO>(v, lane, lnw, lnb, eps, ln_out + r * C);
}

}  // namespace slotfused
}  // namespace hclsm

using namespace hclsm;
using namespace hclsm::slotfused;

template <typename TO, typename TG>
static int launch_gru_ln(int nv, unsigned blocks, cudaStream_t st, const TG* gi, const TG* gh, const float* b_ih,
                         const float* b_hh, const float* h, float* h_out, const float* w, const float* b, TO* y,
                         int64_t rows, float eps) {
  switch (nv) {
#define HCLSM_GRU_LN(NV) \
  case NV:                \
    return launch_pdl(gru_ln_kernel<NV, TO, TG>, blocks, 256, 0, st, gi, gh, b_ih, b_hh, h, h_out, w, b, y, rows, eps);
    HCLSM_GRU_LN(1) HCLSM_GRU_LN(2) HCLSM_GRU_LN(3) HCLSM_GRU_LN(4)
    HCLSM_GRU_LN(5) HCLSM_GRU_LN(6) HCLSM_GRU_LN(7) HCLSM_GRU_LN(8)
#undef HCLSM_GRU_LN
  }
  return HCLSM_ERR_UNSUPPORTED;
}

template <typename TO, typename TM>
static int launch_res_ln(int nv, unsigned blocks, cudaStream_t st, const float* h, const TM* m, const float* bias,
                         float* out, __nv_bfloat16* ob, const float* w, const float* b, TO* y, int64_t rows, float c,
                         float eps) {
  switch (nv) {
#define HCLSM_RES_LN(NV) \
  case NV:                \
    return launch_pdl(residual_clamp_ln_kernel<NV, TO, TM>, blocks, 256, 0, st, h, m, bias, out, ob, w, b, y, rows, c, eps);
    HCLSM_RES_LN(1) HCLSM_RES_LN(2) HCLSM_RES_LN(3) HCLSM_RES_LN(4)
    HCLSM_RES_LN(5) HCLSM_RES_LN(6) HCLSM_RES_LN(7) HCLSM_RES_LN(8)
#undef HCLSM_RES_LN
  }
  return HCLSM_ERR_UNSUPPORTED;
}

static bool al16(const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <typename TG>
static int gru_ln_dispatch(int32_t ln_dtype, int nv, unsigned blocks, cudaStream_t st, const TG* gi, const TG* gh,
                           const float* b_ih, const float* b_hh, const float* h, float* h_out, const float* ln_w,
                           const float* ln_b, void* ln_out, int64_t rows, float eps) {
  if (ln_dtype == HCLSM_BF16)
    return launch_gru_ln(nv, blocks, st, gi, gh, b_ih, b_hh, h, h_out, ln_w, ln_b,
                         static_cast<__nv_bfloat16*>(ln_out), rows, eps);
  if (ln_dtype == HCLSM_F32)
    return launch_gru_ln(nv, blocks, st, gi, gh, b_ih, b_hh, h, h_out, ln_w, ln_b, static_cast<float*>(ln_out), rows,
                         eps);
  return HCLSM_ERR_DTYPE;
}

extern "C" int hclsm_gru_cell_ln(const void* gi, const void* gh, int32_t gate_dtype, const float* b_ih,
                                 const float* b_hh, const float* h, float* h_out, const float* ln_w,
                                 const float* ln_b, void* ln_out, int32_t ln_dtype, int64_t rows, int32_t H,
                                 float eps, void* stream) {
  if (!gi || !gh || !b_ih || !b_hh || !h || !h_out || !ln_out) return HCLSM_ERR_NULL;
  if (rows < 0 || H <= 0) return HCLSM_ERR_SHAPE;
  if (H % 128 != 0 || H > 1024) return HCLSM_ERR_UNSUPPORTED;
  if (!al16(gi) || !al16(gh) || !al16(b_ih) || !al16(b_hh) || !al16(h) || !al16(h_out) || !al16(ln_out))
    return HCLSM_ERR_ALIGN;
  if (rows == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (gate_dtype == HCLSM_F32)
    return gru_ln_dispatch(ln_dtype, H / 128, blocks, st, static_cast<const float*>(gi),
                           static_cast<const float*>(gh), b_ih, b_hh, h, h_out, ln_w, ln_b, ln_out, rows, eps);
  if (gate_dtype == HCLSM_BF16)
    return gru_ln_dispatch(ln_dtype, H / 128, blocks, st, static_cast<const __nv_bfloat16*>(gi),
                           static_cast<const __nv_bfloat16*>(gh), b_ih, b_hh, h, h_out, ln_w, ln_b, ln_out, rows,
                           eps);
  return HCLSM_ERR_DTYPE;
}

template <typename TM>
static int res_ln_dispatch(int32_t ln_dtype, int nv, unsigned blocks, cudaStream_t st, const float* h, const TM* m,
                           const float* b, float* out, __nv_bfloat16* ob, const float* ln_w, const float* ln_b,
                           void* ln_out, int64_t rows, float clamp, float eps) {
  if (ln_dtype == HCLSM_BF16)
    return launch_res_ln(nv, blocks, st, h, m, b, out, ob, ln_w, ln_b, static_cast<__nv_bfloat16*>(ln_out), rows,
                         clamp, eps);
  if (ln_dtype == HCLSM_F32)
    return launch_res_ln(nv, blocks, st, h, m, b, out, ob, ln_w, ln_b, static_cast<float*>(ln_out), rows, clamp, eps);
  return HCLSM_ERR_DTYPE;
}

extern "C" int hclsm_residual_clamp_ln(const float* h, const void* m, int32_t m_dtype, const float* b, float* out,
                                       void* out_bf16, const float* ln_w, const float* ln_b, void* ln_out,
                                       int32_t ln_dtype, int64_t rows, int32_t C, float clamp, float eps,
                                       void* stream) {
  if (!h || !m || !out || !ln_out) return HCLSM_ERR_NULL;
  if (rows < 0 || C <= 0) return HCLSM_ERR_SHAPE;
  if (C % 128 != 0 || C > 1024) return HCLSM_ERR_UNSUPPORTED;
  if (!al16(h) || !al16(m) || !al16(b) || !al16(out) || !al16(out_bf16) || !al16(ln_out)) return HCLSM_ERR_ALIGN;
  if (rows == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  auto* ob = static_cast<__nv_bfloat16*>(out_bf16);
  if (m_dtype == HCLSM_F32)
    return res_ln_dispatch(ln_dtype, C / 128, blocks, st, h, static_cast<const float*>(m), b, out, ob, ln_w, ln_b,
                           ln_out, rows, clamp, eps);
  if (m_dtype == HCLSM_BF16)
    return res_ln_dispatch(ln_dtype, C / 128, blocks, st, h, static_cast<const __nv_bfloat16*>(m), b, out, ob, ln_w,
                           ln_b, ln_out, rows, clamp, eps);
  return HCLSM_ERR_DTYPE;
}
