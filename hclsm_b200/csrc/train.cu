// Backward kernels of the slot-attention iteration and of the Level-1 event
// transformer (sm_100a), so that a training step runs this library's kernels
// under autograd instead of handing the modules back to eager PyTorch.
//
// Reference semantics (paths inside RightNow-AI/hclsm), differentiated:
//   hclsm/objects/dynamic_slots.py:98-131 _iteration_step: LayerNorm, W_q,
//     logits clamp +-30, softmax over the slot axis, weighted sum, GRUCell,
//     LayerNorm-MLP residual, clamp +-50;
//   hclsm/dynamics/level1_event.py:17-54 EventTransformerBlock / SwiGLUFFN:
//     LayerNorm, nn.MultiheadAttention(bias=False) with key_padding_mask,
//     SwiGLU w2(silu(w1 x) * w3 x), residuals.
// The weight products of those modules (and their gradients) are library GEMMs;
// everything between them is here.  Gradients of clamps follow torch.clamp
// (the gradient passes where lo <= x <= hi), of ReLU torch's (x > 0).
#include <cuda_fp16.h>

#include "common.cuh"

namespace hclsm {
bool set_smem_limit(const void* fn, size_t bytes);
namespace train {

constexpr int kColChunks = 64;  // row chunks of the two-stage column sums

__device__ __forceinline__ float tanh_fast(float x) { return 2.0f * sigmoid(2.0f * x) - 1.0f; }

// ---- LayerNorm ---------------------------------------------------------------------
// Row statistics exactly as the forward (hclsm_layernorm) computes them: a warp
// per row, two passes.  Writes mu[r], rstd[r] and dx (optionally added to dx).
__global__ void ln_bwd_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                   const float* __restrict__ dy, float* __restrict__ dx, float* __restrict__ stats,
                                   int64_t rows, int D, float eps, int accumulate) {
  pdl_wait();
  pdl_trigger();
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float* xr = x + r * D;
  const float* gr = dy + r * D;
  float s = 0.0f;
  for (int i = lane; i < D; i += 32) s += xr[i];
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
  const float mu = s / D;
  float v = 0.0f;
  for (int i = lane; i < D; i += 32) {
    const float t = xr[i] - mu;
    v += t * t;
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  const float rs = rsqrtf(v / D + eps);
  // dxhat = dy * w; dx = rs * (dxhat - mean(dxhat) - xhat * mean(dxhat * xhat))
  float a = 0.0f, b = 0.0f;
  for (int i = lane; i < D; i += 32) {
    const float g = w ? gr[i] * w[i] : gr[i];
    a += g;
    b += g * (xr[i] - mu) * rs;
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, m);
    b += __shfl_xor_sync(0xffffffffu, b, m);
  }
  a /= D;
  b /= D;
  for (int i = lane; i < D; i += 32) {
    const float g = w ? gr[i] * w[i] : gr[i];
    const float xh = (xr[i] - mu) * rs;
    const float o = rs * (g - a - xh * b);
    dx[r * D + i] = accumulate ? dx[r * D + i] + o : o;
  }
  if (lane == 0 && stats) {
    stats[2 * r] = mu;
    stats[2 * r + 1] = rs;
  }
}

// Column sums over rows, first stage: block (32 columns x 8 row lanes) per
// (column tile, row chunk); part[chunk][c].  With stats, the summand is
// a * (x - mu_r) * rstd_r (LayerNorm's weight gradient), else a.
// Stage 1 of the column sums: block (column tile of 32, row chunk) sums its
// rows.  With `stats` (the LayerNorm affine gradients) it sums both dy * xhat
// (into part) and dy (into part2, when given) in the same pass over dy.
__global__ void colsum_part_kernel(const float* __restrict__ a, const float* __restrict__ x,
                                   const float* __restrict__ stats, float* __restrict__ part,
                                   float* __restrict__ part2, int64_t rows, int C, int64_t rows_per_chunk) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[2][8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  const int chunk = blockIdx.y;
  const int64_t r0 = chunk * rows_per_chunk;
  const int64_t r1 = r0 + rows_per_chunk < rows ? r0 + rows_per_chunk : rows;
  float acc = 0.0f, acc2 = 0.0f;
  if (c < C) {
#pragma unroll 4
    for (int64_t r = r0 + ty; r < r1; r += 8) {
      const float v = a[r * C + c];
      if (stats) {
        acc += v * ((x[r * C + c] - stats[2 * r]) * stats[2 * r + 1]);
        acc2 += v;
      } else {
        acc += v;
      }
    }
  }
  red[0][ty][tx] = acc;
  red[1][ty][tx] = acc2;
  __syncthreads();
  if (ty == 0) {
    float s = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      s += red[0][k][tx];
      s2 += red[1][k][tx];
    }
    if (c < C) {
      part[(int64_t)chunk * C + c] = s;
      if (part2) part2[(int64_t)chunk * C + c] = s2;
    }
  }
}

// Stage 2: out[c] = sum over the chunks' partials, fixed order.  A block takes
// 32 columns; its 8 warps each sum every 8th chunk (independent loads), then
// warp 0 adds the 8 results in order.  blockIdx.y selects (part, out) or
// (part2, out2).
__global__ void colsum_final_kernel(const float* __restrict__ part, float* __restrict__ out,
                                    const float* __restrict__ part2, float* __restrict__ out2, int nchunk, int C) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8][33];
  const float* __restrict__ src = blockIdx.y ? part2 : part;
  float* __restrict__ dst = blockIdx.y ? out2 : out;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx;
  float s = 0.0f;
  if (c < C) {
#pragma unroll
    for (int i = 0; i < kColChunks / 8; ++i) {
      const int k = ty + 8 * i;
      if (k < nchunk) s += src[(int64_t)k * C + c];
    }
  }
  red[ty][tx] = s;
  __syncthreads();
  if (ty == 0 && c < C) {
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][tx];
    dst[c] = t;
  }
}

// ---- GRUCell -----------------------------------------------------------------------
// torch.nn.GRUCell, gates (r, z, n): r = s(gi_r + b_ir + gh_r + b_hr),
// z = s(gi_z + ...), n = tanh(gi_n + b_in + r * (gh_n + b_hn)),
// h' = (1 - z) n + z h.  Given dh', writes d_gi, d_gh (rows, 3H) (the
// gradients of the two pre-bias products; the bias gradients are their column
// sums) and dh = z * dh' (the direct part of the previous state's gradient).
__global__ void gru_bwd_kernel(const float* __restrict__ gi, const float* __restrict__ gh,
                               const float* __restrict__ b_ih, const float* __restrict__ b_hh,
                               const float* __restrict__ h, const float* __restrict__ dh_new,
                               float* __restrict__ d_gi, float* __restrict__ d_gh, float* __restrict__ dh,
                               int64_t rows, int H) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * H;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int c = (int)(i % H);
    const float* gir = gi + r * 3 * H;
    const float* ghr = gh + r * 3 * H;
    const float rg = sigmoid(gir[c] + ghr[c] + (b_ih[c] + b_hh[c]));
    const float zg = sigmoid(gir[H + c] + ghr[H + c] + (b_ih[H + c] + b_hh[H + c]));
    const float hn = ghr[2 * H + c] + b_hh[2 * H + c];
    const float ng = tanh_fast(gir[2 * H + c] + b_ih[2 * H + c] + rg * hn);
    const float g = dh_new[i];
    const float dn = g * (1.0f - zg);
    const float dz = g * (h[i] - ng);
    const float dpn = dn * (1.0f - ng * ng);
    const float dpr = dpn * hn * rg * (1.0f - rg);
    const float dpz = dz * zg * (1.0f - zg);
    float* a = d_gi + r * 3 * H;
    float* b = d_gh + r * 3 * H;
    a[c] = dpr;
    b[c] = dpr;
    a[H + c] = dpz;
    b[H + c] = dpz;
    a[2 * H + c] = dpn;
    b[2 * H + c] = dpn * rg;
    dh[i] = g * zg;
  }
}

// ---- softmax over slots ------------------------------------------------------------
// dots (F, N, M) fp32 = q k^T (unscaled).  Per (frame, token) column: logits
// l = dots * scale, clamped to +-clamp (clamp > 0), softmax over the N slots
// (+eps in the denominator).  Writes attn (TA) and, given d_attn (F, N, M),
// d_dots = scale * [|l| within the clamp] * attn * (d_attn - sum_n attn d_attn)
// (TD).  One thread per column; consecutive threads take consecutive tokens.
template <typename TA, typename TD>
__global__ void slot_softmax_bwd_kernel(const float* __restrict__ dots, const float* __restrict__ d_attn,
                                        TA* __restrict__ attn, TD* __restrict__ d_dots, int F, int N, int M,
                                        float scale, float clamp, float eps) {
  pdl_wait();
  pdl_trigger();
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= (int64_t)F * M) return;
  const int f = (int)(col / M), m = (int)(col % M);
  const int64_t base = (int64_t)f * N * M + m;
  auto logit = [&](int n) {
    float l = dots[base + (int64_t)n * M] * scale;
    if (clamp > 0.0f) l = fminf(fmaxf(l, -clamp), clamp);
    return l;
  };
  float mx = -INFINITY;
  for (int n = 0; n < N; ++n) mx = fmaxf(mx, logit(n));
  float sum = 0.0f;
  for (int n = 0; n < N; ++n) sum += __expf(logit(n) - mx);
  const float inv = 1.0f / (sum + eps);
  float s = 0.0f;
  for (int n = 0; n < N; ++n) s += __expf(logit(n) - mx) * inv * d_attn[base + (int64_t)n * M];
  for (int n = 0; n < N; ++n) {
    const float raw = dots[base + (int64_t)n * M] * scale;
    const float p = __expf(logit(n) - mx) * inv;
    io<TA>::st(attn + base + (int64_t)n * M, p);
    const bool pass = clamp <= 0.0f || (raw >= -clamp && raw <= clamp);
    const float g = pass ? p * (d_attn[base + (int64_t)n * M] - s) * scale : 0.0f;
    io<TD>::st(d_dots + base + (int64_t)n * M, g);
  }
}

// ---- element-wise ------------------------------------------------------------------
// pre = (h + m) + b as hclsm_residual_clamp forms it; dpre = dout where
// -c <= pre <= c (c > 0), else 0.
__global__ void residual_clamp_bwd_kernel(const float* __restrict__ h, const float* __restrict__ m,
                                          const float* __restrict__ b, const float* __restrict__ dout,
                                          float* __restrict__ dpre, int64_t rows, int C, float c) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    float v = h[i] + m[i];
    if (b) v += b[i % C];
    dpre[i] = (v >= -c && v <= c) ? dout[i] : 0.0f;
  }
}

// dx = dy where y > 0 (y the ReLU output), in TO.
template <typename TY, typename TO>
__global__ void relu_bwd_kernel(const TY* __restrict__ y, const float* __restrict__ dy, TO* __restrict__ dx,
                                int64_t n) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    io<TO>::st(dx + i, io<TY>::ld(y + i) > 0.0f ? dy[i] : 0.0f);
}

// SwiGLU: u (rows, 2C) = [a | b], s = silu(a) * b.  Given ds (rows, C):
// da = ds * b * silu'(a), db = ds * silu(a), written as du (rows, 2C) in TO.
template <typename TO>
__global__ void swiglu_bwd_kernel(const float* __restrict__ u, const float* __restrict__ ds, TO* __restrict__ du,
                                  int64_t rows, int C) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = rows * C;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / C;
    const int c = (int)(i % C);
    const float a = u[r * 2 * C + c], bb = u[r * 2 * C + C + c];
    const float sg = sigmoid(a);
    const float g = ds[i];
    io<TO>::st(du + r * 2 * C + c, g * bb * sg * (1.0f + a * (1.0f - sg)));
    io<TO>::st(du + r * 2 * C + C + c, g * a * sg);
  }
}

// ---- multi-head attention ----------------------------------------------------------
// One block per (frame, head), everything in shared memory (T <= 64 tokens,
// head dim HD).  qkv (frames * T, 3E) rows [q | k | v], head hh at column
// hh * HD of each part; dout (frames * T, E) fp32 is the gradient of the
// attention output before out_proj.  Recomputes P = softmax(scale q k^T) with
// ignored keys at -inf (rows whose keys are all ignored give NaN, as the
// forward and PyTorch do), then dV = P^T dO, dS = P (dO V^T - rowsum(P dO V^T)),
// dQ = scale dS K, dK = scale dS^T Q; dqkv (frames * T, 3E) in TO.
template <typename TI, typename TO>
__global__ void mha_bwd_kernel(const TI* __restrict__ qkv, const uint8_t* __restrict__ key_pad,
                               const float* __restrict__ dout, TO* __restrict__ dqkv, int T, int H, int HD,
                               float scale) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm[];
  const int f = blockIdx.x / H, hh = blockIdx.x % H;
  const int E = H * HD;
  const int ld = HD + 1;
  float* Q = sm;
  float* K = Q + T * ld;
  float* V = K + T * ld;
  float* dO = V + T * ld;
  float* P = dO + T * ld;          // T x (T + 1)
  float* dP = P + T * (T + 1);     // T x (T + 1)
  const int tid = threadIdx.x, nt = blockDim.x;
  const int64_t row0 = (int64_t)f * T;
  for (int i = tid; i < T * HD; i += nt) {
    const int t = i / HD, d = i % HD;
    const TI* rp = qkv + (row0 + t) * 3 * E + hh * HD + d;
    Q[t * ld + d] = io<TI>::ld(rp);
    K[t * ld + d] = io<TI>::ld(rp + E);
    V[t * ld + d] = io<TI>::ld(rp + 2 * E);
    dO[t * ld + d] = dout[(row0 + t) * E + hh * HD + d];
  }
  __syncthreads();
  for (int i = tid; i < T * T; i += nt) {
    const int a = i / T, b = i % T;
    const bool ok = !(key_pad && key_pad[row0 + b]);
    float s = 0.0f, g = 0.0f;
    for (int d = 0; d < HD; ++d) {
      s = fmaf(Q[a * ld + d], K[b * ld + d], s);
      g = fmaf(dO[a * ld + d], V[b * ld + d], g);
    }
    P[a * (T + 1) + b] = ok ? s * scale : -INFINITY;
    dP[a * (T + 1) + b] = g;
  }
  __syncthreads();
  // row softmax and dS, a warp per row
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  for (int a = warp; a < T; a += nw) {
    float* pr = P + a * (T + 1);
    float* gr = dP + a * (T + 1);
    float mx = -INFINITY;
    for (int b = lane; b < T; b += 32) mx = fmaxf(mx, pr[b]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.0f;
    for (int b = lane; b < T; b += 32) sum += __expf(pr[b] - mx);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = 1.0f / sum;
    float dsum = 0.0f;
    for (int b = lane; b < T; b += 32) {
      const float p = __expf(pr[b] - mx) * inv;
      pr[b] = p;
      dsum += p * gr[b];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
    for (int b = lane; b < T; b += 32) gr[b] = pr[b] * (gr[b] - dsum);
  }
  __syncthreads();
  for (int i = tid; i < T * HD; i += nt) {
    const int t = i / HD, d = i % HD;
    float dq = 0.0f, dk = 0.0f, dv = 0.0f;
    for (int j = 0; j < T; ++j) {
      dq = fmaf(dP[t * (T + 1) + j], K[j * ld + d], dq);
      dk = fmaf(dP[j * (T + 1) + t], Q[j * ld + d], dk);
      dv = fmaf(P[j * (T + 1) + t], dO[j * ld + d], dv);
    }
    TO* op = dqkv + (row0 + t) * 3 * E + hh * HD + d;
    io<TO>::st(op, dq * scale);
    io<TO>::st(op + E, dk * scale);
    io<TO>::st(op + 2 * E, dv);
  }
}

}  // namespace train
}  // namespace hclsm

using namespace hclsm;
using namespace hclsm::train;

static unsigned tr_blocks(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

// out = column sums of a (rows, C), or with stats (LayerNorm row mean / rstd)
// the sums of a * xhat; out2 (only with stats, may be null) = the plain sums
// of a from the same pass.  part holds kColChunks x C floats, twice that with
// out2.
static int colsum_launch(const float* a, const float* x, const float* stats, float* part, float* out, float* out2,
                         int64_t rows, int C, cudaStream_t st) {
  const int nchunk = (int)(rows < kColChunks ? (rows > 0 ? rows : 1) : kColChunks);
  const int64_t per = (rows + nchunk - 1) / nchunk;
  float* p2 = (stats && out2) ? part + (size_t)kColChunks * C : nullptr;
  int rc = launch_pdl(colsum_part_kernel, dim3((C + 31) / 32, nchunk), 256, 0, st, a, x, stats, part, p2, rows, C,
                      per);
  if (rc != HCLSM_OK) return rc;
  return launch_pdl(colsum_final_kernel, dim3((C + 31) / 32, p2 ? 2 : 1), 256, 0, st, (const float*)part, out,
                    (const float*)p2, p2 ? out2 : (float*)nullptr, nchunk, C);
}

extern "C" size_t hclsm_colsum_workspace_size(int32_t C) {
  return C > 0 ? sizeof(float) * (size_t)kColChunks * C : 0;
}

extern "C" int hclsm_colsum(const float* a, float* out, int64_t rows, int32_t C, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!a || !out) return HCLSM_ERR_NULL;
  if (rows < 0 || C <= 0) return HCLSM_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) return cudaMemsetAsync(out, 0, sizeof(float) * C, st) == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
  if (!workspace || workspace_bytes < hclsm_colsum_workspace_size(C)) return HCLSM_ERR_WORKSPACE;
  return colsum_launch(a, nullptr, nullptr, static_cast<float*>(workspace), out, nullptr, rows, C, st);
}

extern "C" size_t hclsm_layernorm_bwd_workspace_size(int64_t rows, int32_t D) {
  if (rows < 0 || D <= 0) return 0;
  return sizeof(float) * (2 * (size_t)rows + 2 * (size_t)kColChunks * D);
}

extern "C" int hclsm_layernorm_bwd(const float* x, const float* w, const float* dy, float* dx, float* dw, float* db,
                                   int64_t rows, int32_t D, float eps, int32_t accumulate, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  if (!x || !dy || !dx) return HCLSM_ERR_NULL;
  if (rows < 0 || D <= 0) return HCLSM_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (dw) cudaMemsetAsync(dw, 0, sizeof(float) * D, st);
    if (db) cudaMemsetAsync(db, 0, sizeof(float) * D, st);
    return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
  }
  const bool need_ws = dw || db;
  if (need_ws && (!workspace || workspace_bytes < hclsm_layernorm_bwd_workspace_size(rows, D)))
    return HCLSM_ERR_WORKSPACE;
  float* stats = need_ws ? static_cast<float*>(workspace) : nullptr;
  float* part = need_ws ? stats + 2 * rows : nullptr;
  int rc = launch_pdl(ln_bwd_rows_kernel, (unsigned)((rows + 7) / 8), 256, 0, st, x, w, dy, dx, stats, rows, D, eps,
                      accumulate);
  if (rc != HCLSM_OK) return rc;
  if (dw) return colsum_launch(dy, x, stats, part, dw, db, rows, D, st);  // both sums in one pass
  if (db) rc = colsum_launch(dy, nullptr, nullptr, part, db, nullptr, rows, D, st);
  return rc;
}

extern "C" int hclsm_gru_cell_bwd(const float* gi, const float* gh, const float* b_ih, const float* b_hh,
                                  const float* h, const float* dh_new, float* d_gi, float* d_gh, float* dh,
                                  int64_t rows, int32_t H, void* stream) {
  if (!gi || !gh || !b_ih || !b_hh || !h || !dh_new || !d_gi || !d_gh || !dh) return HCLSM_ERR_NULL;
  if (rows < 0 || H <= 0) return HCLSM_ERR_SHAPE;
  if (rows == 0) return HCLSM_OK;
  return launch_pdl(gru_bwd_kernel, tr_blocks(rows * H), 256, 0, static_cast<cudaStream_t>(stream), gi, gh, b_ih,
                    b_hh, h, dh_new, d_gi, d_gh, dh, rows, H);
}

template <typename TA, typename TD>
static int launch_softmax_bwd(const float* dots, const float* d_attn, void* attn, void* d_dots, int F, int N, int M,
                              float scale, float clamp, float eps, cudaStream_t st) {
  const int64_t cols = (int64_t)F * M;
  return launch_pdl(slot_softmax_bwd_kernel<TA, TD>, (unsigned)((cols + 127) / 128), 128, 0, st, dots, d_attn,
                    static_cast<TA*>(attn), static_cast<TD*>(d_dots), F, N, M, scale, clamp, eps);
}

extern "C" int hclsm_slot_softmax_bwd(const float* dots, const float* d_attn, void* attn, void* d_dots, int32_t F,
                                      int32_t N, int32_t M, float scale, float clamp, float eps, int32_t dtype,
                                      void* stream) {
  if (!dots || !d_attn || !attn || !d_dots) return HCLSM_ERR_NULL;
  if (F < 0 || N <= 0 || M < 0) return HCLSM_ERR_SHAPE;
  if ((int64_t)F * M == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == HCLSM_F32)
    return launch_softmax_bwd<float, float>(dots, d_attn, attn, d_dots, F, N, M, scale, clamp, eps, st);
  if (dtype == HCLSM_BF16)
    return launch_softmax_bwd<__nv_bfloat16, __nv_bfloat16>(dots, d_attn, attn, d_dots, F, N, M, scale, clamp, eps,
                                                            st);
  return HCLSM_ERR_DTYPE;
}

extern "C" int hclsm_residual_clamp_bwd(const float* h, const float* m, const float* b, const float* dout,
                                        float* dpre, int64_t rows, int32_t C, float clamp, void* stream) {
  if (!h || !m || !dout || !dpre) return HCLSM_ERR_NULL;
  if (rows < 0 || C <= 0 || !(clamp > 0.0f)) return HCLSM_ERR_SHAPE;
  if (rows == 0) return HCLSM_OK;
  return launch_pdl(residual_clamp_bwd_kernel, tr_blocks(rows * C), 256, 0, static_cast<cudaStream_t>(stream), h, m,
                    b, dout, dpre, rows, C, clamp);
}

extern "C" int hclsm_relu_bwd(const void* y, int32_t y_dtype, const float* dy, void* dx, int32_t dx_dtype, int64_t n,
                              void* stream) {
  if (!y || !dy || !dx) return HCLSM_ERR_NULL;
  if (n < 0) return HCLSM_ERR_SHAPE;
  if (n == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = tr_blocks(n);
  using bf = __nv_bfloat16;
  if (y_dtype == HCLSM_F32 && dx_dtype == HCLSM_F32)
    return launch_pdl(relu_bwd_kernel<float, float>, g, 256, 0, st, static_cast<const float*>(y), dy,
                      static_cast<float*>(dx), n);
  if (y_dtype == HCLSM_BF16 && dx_dtype == HCLSM_BF16)
    return launch_pdl(relu_bwd_kernel<bf, bf>, g, 256, 0, st, static_cast<const bf*>(y), dy, static_cast<bf*>(dx), n);
  if (y_dtype == HCLSM_BF16 && dx_dtype == HCLSM_F32)
    return launch_pdl(relu_bwd_kernel<bf, float>, g, 256, 0, st, static_cast<const bf*>(y), dy,
                      static_cast<float*>(dx), n);
  return HCLSM_ERR_DTYPE;
}

extern "C" int hclsm_swiglu_bwd(const float* u, const float* ds, void* du, int64_t rows, int32_t C, int32_t out_dtype,
                                void* stream) {
  if (!u || !ds || !du) return HCLSM_ERR_NULL;
  if (rows < 0 || C <= 0) return HCLSM_ERR_SHAPE;
  if (rows == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == HCLSM_F32)
    return launch_pdl(swiglu_bwd_kernel<float>, tr_blocks(rows * C), 256, 0, st, u, ds, static_cast<float*>(du), rows,
                      C);
  if (out_dtype == HCLSM_BF16)
    return launch_pdl(swiglu_bwd_kernel<__nv_bfloat16>, tr_blocks(rows * C), 256, 0, st, u, ds,
                      static_cast<__nv_bfloat16*>(du), rows, C);
  return HCLSM_ERR_DTYPE;
}

template <typename TI, typename TO>
static int launch_mha_bwd(const void* qkv, const uint8_t* key_pad, const float* dout, void* dqkv, int frames, int T,
                          int H, int HD, float scale, size_t smem, cudaStream_t st) {
  auto fn = mha_bwd_kernel<TI, TO>;
  if (!set_smem_limit(reinterpret_cast<const void*>(fn), smem)) return HCLSM_ERR_LAUNCH;
  return launch_pdl(fn, (unsigned)(frames * H), 256, smem, st, static_cast<const TI*>(qkv), key_pad, dout,
                    static_cast<TO*>(dqkv), T, H, HD, scale);
}

extern "C" int hclsm_event_mha_bwd(const void* qkv, const uint8_t* key_pad, const float* dout, void* dqkv,
                                   int32_t frames, int32_t T, int32_t H, int32_t HD, float scale, int32_t dtype,
                                   void* stream) {
  if (!qkv || !dout || !dqkv) return HCLSM_ERR_NULL;
  if (frames < 0 || T <= 0 || H <= 0 || HD <= 0) return HCLSM_ERR_SHAPE;
  if (frames == 0) return HCLSM_OK;
  if ((int64_t)frames * H > 0x7fffffff) return HCLSM_ERR_SHAPE;
  const size_t smem = sizeof(float) * (4 * (size_t)T * (HD + 1) + 2 * (size_t)T * (T + 1));
  if (smem > 227 * 1024) return HCLSM_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == HCLSM_F32)
    return launch_mha_bwd<float, float>(qkv, key_pad, dout, dqkv, frames, T, H, HD, scale, smem, st);
  if (dtype == HCLSM_BF16)
    return launch_mha_bwd<__nv_bfloat16, __nv_bfloat16>(qkv, key_pad, dout, dqkv, frames, T, H, HD, scale, smem, st);
  return HCLSM_ERR_DTYPE;
}
