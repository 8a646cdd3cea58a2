// Sparse event attention for B200 (sm_100a): device-side compaction of the
// fired (video, t) frames, gather, the per-frame multi-head attention of
// Level1EventDynamics, SwiGLU, and a fused copy+scatter of the result.
//
// Reference semantics (paths inside RightNow-AI/hclsm):
//   hclsm/kernels/sparse_event_attn.py:35-86 naive_sparse_event_attention:
//     event timesteps of each video, ascending in time -> attn_fn -> written
//     back; other timesteps unchanged (a clone of the input).
//   hclsm/dynamics/hierarchy_manager.py:42-118 gather/scatter_events (the model
//     path; pads are zero frames, the scatter overrides at events).
//   hclsm/dynamics/level1_event.py:17-54 EventTransformerBlock / SwiGLUFFN:
//     nn.MultiheadAttention(bias=False, batch_first) with key_padding_mask,
//     SwiGLU w2(silu(w1 x) * w3 x).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"

namespace hclsm {
int* device_err_ptr();
bool set_smem_limit(const void* fn, size_t bytes);
}  // namespace hclsm

namespace hclsm {
int event_mha_tc(const void* qkv, const uint8_t* key_pad, void* out, int frames, int T, int H, int HD, float scale,
                 void* stream);
namespace event {

// ---- compaction --------------------------------------------------------------------
// One block scans the (B, T) mask as one flattened array: video-major, time
// ascending, which is the order events are numbered in.  Outputs: idx[k] =
// b*T + t of the k-th fired frame, pos[b*T + t] = k or -1, counts[b] = fired
// frames of video b, meta[0] = total, meta[1] = max over videos.
template <typename TM>
__global__ void __launch_bounds__(1024) compact_kernel(const TM* __restrict__ mask, int B, int T,
                                                       int32_t* __restrict__ idx, int32_t* __restrict__ pos,
                                                       int32_t* __restrict__ counts, int32_t* __restrict__ meta) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int64_t BT = (int64_t)B * T;
  for (int b = tid; b < B; b += nthr) counts[b] = 0;
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int64_t i0 = 0; i0 < BT; i0 += nthr) {
    const int64_t i = i0 + tid;
    const bool fired = i < BT && static_cast<float>(mask[i]) > 0.5f;
    const unsigned bal = __ballot_sync(0xffffffffu, fired);
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int before = 0, tot = 0;
    for (int w = 0; w < (nthr >> 5); ++w) {
      const int c = warp_tot[w];
      before += w < warp ? c : 0;
      tot += c;
    }
    const int rank = s_base + before + __popc(bal & ((1u << lane) - 1u));
    if (i < BT) {
      pos[i] = fired ? rank : -1;
      if (fired) {
        idx[rank] = (int32_t)i;
        atomicAdd(&counts[i / T], 1);
      }
    }
    __syncthreads();
    if (tid == 0) s_base += tot;
    __syncthreads();
  }
  // largest per-video count
  int m = 0;
  for (int b = tid; b < B; b += nthr) m = max(m, counts[b]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) warp_tot[warp] = m;
  __syncthreads();
  if (tid == 0) {
    int k = 0;
    for (int w = 0; w < (nthr >> 5); ++w) k = max(k, warp_tot[w]);
    meta[0] = s_base;
    meta[1] = k;
  }
}

// EventDetector's decision (hclsm/dynamics/event_detector.py:162-170) and the
// compaction in one block: hard[b, t] = probs[b, t] > *threshold; if any video
// has no event, t = 0 is made an event in every video (the reference's
// "always keep at least one event", decided there by a host read); then the
// same flattened scan as compact_kernel.  meta[2] = 1 when that rule fired.
__global__ void __launch_bounds__(1024) detect_kernel(const float* __restrict__ probs,
                                                      const float* __restrict__ threshold, int B, int T,
                                                      float* __restrict__ hard, int32_t* __restrict__ idx,
                                                      int32_t* __restrict__ pos, int32_t* __restrict__ counts,
                                                      int32_t* __restrict__ meta) {
  pdl_wait();
  pdl_trigger();
  __shared__ int warp_tot[32];
  __shared__ int s_base, s_empty;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int64_t BT = (int64_t)B * T;
  const float thr = *threshold;
  for (int b = tid; b < B; b += nthr) counts[b] = 0;
  if (tid == 0) { s_base = 0; s_empty = 0; }
  __syncthreads();
  for (int64_t i = tid; i < BT; i += nthr)
    if (probs[i] > thr) atomicAdd(&counts[i / T], 1);
  __syncthreads();
  for (int b = tid; b < B; b += nthr)
    if (counts[b] == 0) s_empty = 1;
  __syncthreads();
  const bool force0 = s_empty != 0;
  for (int b = tid; b < B; b += nthr) counts[b] = 0;
  __syncthreads();
  for (int64_t i0 = 0; i0 < BT; i0 += nthr) {
    const int64_t i = i0 + tid;
    bool fired = false;
    if (i < BT) {
      fired = probs[i] > thr || (force0 && i % T == 0);
      hard[i] = fired ? 1.0f : 0.0f;
    }
    const unsigned bal = __ballot_sync(0xffffffffu, fired);
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    int before = 0, tot = 0;
    for (int w = 0; w < (nthr >> 5); ++w) {
      const int c = warp_tot[w];
      before += w < warp ? c : 0;
      tot += c;
    }
    const int rank = s_base + before + __popc(bal & ((1u << lane) - 1u));
    if (i < BT) {
      pos[i] = fired ? rank : -1;
      if (fired) {
        idx[rank] = (int32_t)i;
        atomicAdd(&counts[i / T], 1);
      }
    }
    __syncthreads();
    if (tid == 0) s_base += tot;
    __syncthreads();
  }
  int m = 0;
  for (int b = tid; b < B; b += nthr) m = max(m, counts[b]);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) warp_tot[warp] = m;
  __syncthreads();
  if (tid == 0) {
    int k = 0;
    for (int w = 0; w < (nthr >> 5); ++w) k = max(k, warp_tot[w]);
    meta[0] = s_base;
    meta[1] = k;
    meta[2] = force0 ? 1 : 0;
  }
}

// out[k] = states[idx[k]] (frames of F elements, k < meta[0]); pad_k > 0 gives
// the padded (B, pad_k) layout instead: out[b, j] = j-th event of video b or 0.
template <typename T>
__global__ void gather_kernel(const T* __restrict__ states, const int32_t* __restrict__ idx,
                              const int32_t* __restrict__ counts, const int32_t* __restrict__ meta, T* __restrict__ out,
                              int64_t frame_elems, int B, int pad_k, int64_t max_frames) {
  pdl_wait();
  pdl_trigger();
  const int64_t slot = blockIdx.y;
  if (slot >= max_frames) return;
  int64_t src_frame = -1;
  if (pad_k > 0) {
    const int b = (int)(slot / pad_k), j = (int)(slot % pad_k);
    if (b < B && j < counts[b]) {
      int off = 0;
      for (int q = 0; q < b; ++q) off += counts[q];
      src_frame = idx[off + j];
    }
  } else {
    if (slot >= meta[0]) return;
    src_frame = idx[slot];
  }
  const int64_t n16 = frame_elems * (int64_t)sizeof(T) / 16;
  uint4* dst = reinterpret_cast<uint4*>(out + slot * frame_elems);
  const uint4* src = src_frame >= 0 ? reinterpret_cast<const uint4*>(states + src_frame * frame_elems) : nullptr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src ? src[i] : make_uint4(0, 0, 0, 0);
}

// out[f] = fired(f) ? upd[pos[f]] : states[f] for every frame f of the grid; with
// pad_k > 0 the updates are in the padded (B, pad_k) layout.
template <typename T>
__global__ void scatter_kernel(const T* __restrict__ states, const T* __restrict__ upd,
                               const int32_t* __restrict__ pos, const int32_t* __restrict__ counts, T* __restrict__ out,
                               int64_t frame_elems, int Tlen, int pad_k) {
  pdl_wait();
  pdl_trigger();
  const int64_t f = blockIdx.y;
  const int32_t k = pos[f];
  const T* src = states + f * frame_elems;
  if (k >= 0) {
    int64_t slot = k;
    if (pad_k > 0) {
      const int b = (int)(f / Tlen);
      int off = 0;
      for (int q = 0; q < b; ++q) off += counts[q];
      slot = (int64_t)b * pad_k + (k - off);
    }
    src = upd + slot * frame_elems;
  }
  const int64_t n16 = frame_elems * (int64_t)sizeof(T) / 16;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(out + f * frame_elems);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    d4[i] = s4[i];
}

// ---- multi-head attention within each frame ------------------------------------------
// qkv (frames*T, 3E) with q | k | v column blocks, E = H*hd; out (frames*T, E).
// key_pad (frames, T) bytes, non-zero = ignore that key (nn.MultiheadAttention's
// key_padding_mask); rows whose keys are all ignored come out NaN, as in PyTorch.
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// One warp per (frame, head).  TP: tokens padded to a multiple of 16; HD: head dim.
template <int TP, int HD>
__global__ void __launch_bounds__(32) mha_bf16_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                      const uint8_t* __restrict__ key_pad,
                                                      __nv_bfloat16* __restrict__ out, int T, int H, float scale) {
  pdl_wait();
  pdl_trigger();
  constexpr int RS = HD + 8;  // smem row stride (elements), 16-byte aligned and conflict-free
  __shared__ __align__(16) __nv_bfloat16 sq[TP * RS], sk[TP * RS], sv[TP * RS];
  const int lane = threadIdx.x;
  const int f = blockIdx.x / H, hh = blockIdx.x % H;
  const int E = H * HD;
  const __nv_bfloat16* base = qkv + (size_t)f * T * 3 * E + hh * HD;
  // stage q, k, v rows (16-byte pieces); padded rows are zero
  constexpr int P = HD / 8;
  for (int i = lane; i < TP * P; i += 32) {
    const int r = i / P, c = (i % P) * 8;
    uint4 q = make_uint4(0, 0, 0, 0), k = q, v = q;
    if (r < T) {
      const __nv_bfloat16* row = base + (size_t)r * 3 * E + c;
      q = *reinterpret_cast<const uint4*>(row);
      k = *reinterpret_cast<const uint4*>(row + E);
      v = *reinterpret_cast<const uint4*>(row + 2 * E);
    }
    *reinterpret_cast<uint4*>(sq + r * RS + c) = q;
    *reinterpret_cast<uint4*>(sk + r * RS + c) = k;
    *reinterpret_cast<uint4*>(sv + r * RS + c) = v;
  }
  __syncwarp();
  const int g = lane >> 2, t4 = lane & 3;
  const uint32_t aq = smem_u32(sq), ak = smem_u32(sk), av = smem_u32(sv);
  constexpr int MT = TP / 16, NTK = TP / 8, NTD = HD / 8;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    float s[NTK][4];
#pragma unroll
    for (int j = 0; j < NTK; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[j][c] = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < HD; k0 += 16) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(aq + (uint32_t)(((mt * 16 + (lane & 15)) * RS + k0 + (lane >> 4) * 8) * 2), a0, a1, a2, a3);
#pragma unroll
      for (int j = 0; j < NTK; ++j) {
        uint32_t b0, b1;
        ldsm_x2(ak + (uint32_t)(((j * 8 + (lane & 7)) * RS + k0 + ((lane >> 3) & 1) * 8) * 2), b0, b1);
        mma_bf16(s[j], a0, a1, a2, a3, b0, b1);
      }
    }
    // softmax over keys for rows g and g+8 of this tile
    float inv[2];
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < NTK; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = j * 8 + 2 * t4 + e;
          const bool ok = key < T && !(key_pad && key_pad[(size_t)f * T + key]);
          const float v = ok ? s[j][2 * hr + e] * scale : -INFINITY;
          s[j][2 * hr + e] = v;
          mx = fmaxf(mx, v);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      float sum = 0.0f;
#pragma unroll
      for (int j = 0; j < NTK; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float ev = (mx == -INFINITY) ? 0.0f : ex2((s[j][2 * hr + e] - mx) * kLog2e);
          s[j][2 * hr + e] = ev;
          sum += ev;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      inv[hr] = 1.0f / sum;  // all keys ignored: 1/0 -> the row becomes NaN below
    }
    // O = P V (P from registers, V via transposed ldmatrix)
    float o[NTD][4];
#pragma unroll
    for (int j = 0; j < NTD; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) o[j][c] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < TP / 16; ++kk) {
      const uint32_t a0 = pack_bf2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int j = 0; j < NTD; ++j) {
        uint32_t b0, b1;
        ldsm_x2_t(av + (uint32_t)(((kk * 16 + (lane & 15)) * RS + j * 8) * 2), b0, b1);
        mma_bf16(o[j], a0, a1, a2, a3, b0, b1);
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int r = mt * 16 + g + 8 * hr;
      if (r < T) {
        __nv_bfloat16* orow = out + ((size_t)f * T + r) * E + hh * HD;
        const float sc = inv[hr];
#pragma unroll
        for (int j = 0; j < NTD; ++j)
          *reinterpret_cast<__nv_bfloat162*>(orow + j * 8 + 2 * t4) =
              __floats2bfloat162_rn(o[j][2 * hr] * sc, o[j][2 * hr + 1] * sc);
      }
    }
  }
}

// fp32 I/O: exact fp32 arithmetic on CUDA cores, one block per (frame, head).
__global__ void mha_f32_kernel(const float* __restrict__ qkv, const uint8_t* __restrict__ key_pad,
                               float* __restrict__ out, int T, int H, int HD, float scale) {
  const int f = blockIdx.x / H, hh = blockIdx.x % H;
  const int E = H * HD;
  const float* base = qkv + (size_t)f * T * 3 * E + hh * HD;
  for (int i = threadIdx.x; i < T; i += blockDim.x) {
    const float* q = base + (size_t)i * 3 * E;
    float mx = -INFINITY;
    for (int j = 0; j < T; ++j) {
      if (key_pad && key_pad[(size_t)f * T + j]) continue;
      const float* k = base + (size_t)j * 3 * E + E;
      float a = 0.0f;
      for (int d = 0; d < HD; ++d) a = fmaf(q[d], k[d], a);
      mx = fmaxf(mx, a * scale);
    }
    float* o = out + ((size_t)f * T + i) * E + hh * HD;
    for (int d = 0; d < HD; ++d) o[d] = 0.0f;
    float sum = 0.0f;
    for (int j = 0; j < T; ++j) {
      if (key_pad && key_pad[(size_t)f * T + j]) continue;
      const float* k = base + (size_t)j * 3 * E + E;
      const float* v = base + (size_t)j * 3 * E + 2 * E;
      float a = 0.0f;
      for (int d = 0; d < HD; ++d) a = fmaf(q[d], k[d], a);
      const float p = expf(a * scale - mx);
      sum += p;
      for (int d = 0; d < HD; ++d) o[d] = fmaf(p, v[d], o[d]);
    }
    const float inv = 1.0f / sum;
    for (int d = 0; d < HD; ++d) o[d] *= inv;
  }
}

// SwiGLU: u (rows, 2C) holding [x W1^T | x W3^T] (TU = fp32 or bf16) ->
// silu(a) * b in fp32, stored as TO.  A block walks rows, its threads walk
// column pairs (one 8- or 4-byte load per half), no per-element division.
template <typename TU, typename TO>
__global__ void swiglu_kernel(const TU* __restrict__ u, TO* __restrict__ y, int64_t rows, int C) {
  pdl_wait();
  pdl_trigger();
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const TU* ur = u + r * 2 * C;
    TO* yr = y + r * C;
    if ((C & 1) == 0) {
      for (int c = 2 * threadIdx.x; c < C; c += 2 * blockDim.x) {
        const float2 a = io<TU>::ld2(ur + c), g = io<TU>::ld2(ur + C + c);
        io<TO>::st2(yr + c, a.x * sigmoid(a.x) * g.x, a.y * sigmoid(a.y) * g.y);
      }
    } else {
      for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float a = io<TU>::ld(ur + c), g = io<TU>::ld(ur + C + c);
        io<TO>::st(yr + c, a * sigmoid(a) * g);
      }
    }
  }
}

}  // namespace event
}  // namespace hclsm

using namespace hclsm;
using namespace hclsm::event;

static unsigned ew_blocks(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

extern "C" int hclsm_event_compact(const void* mask, int32_t mask_dtype, int32_t B, int32_t T, int32_t* idx,
                                   int32_t* pos, int32_t* counts, int32_t* meta, void* stream) {
  if (!mask || !idx || !pos || !counts || !meta) return HCLSM_ERR_NULL;
  if (B < 0 || T < 0) return HCLSM_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || T == 0) {
    cudaMemsetAsync(meta, 0, 2 * sizeof(int32_t), st);
    if (B > 0) cudaMemsetAsync(counts, 0, B * sizeof(int32_t), st);
    return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
  }
  const int64_t BT = (int64_t)B * T;
  const unsigned thr = (unsigned)std::min<int64_t>(1024, std::max<int64_t>(32, (BT + 31) / 32 * 32));
  if (mask_dtype == HCLSM_F32)
    return launch_pdl(compact_kernel<float>, 1, thr, 0, st, static_cast<const float*>(mask), B, T, idx, pos, counts,
                      meta);
  if (mask_dtype == HCLSM_BF16)
    return launch_pdl(compact_kernel<__nv_bfloat16>, 1, thr, 0, st, static_cast<const __nv_bfloat16*>(mask), B, T,
                      idx, pos, counts, meta);
  return HCLSM_ERR_DTYPE;
}

extern "C" int hclsm_event_detect(const float* probs, const float* threshold, int32_t B, int32_t T, float* hard,
                                  int32_t* idx, int32_t* pos, int32_t* counts, int32_t* meta, void* stream) {
  if (!probs || !threshold || !hard || !idx || !pos || !counts || !meta) return HCLSM_ERR_NULL;
  if (B <= 0 || T <= 0) return HCLSM_ERR_SHAPE;
  const int64_t BT = (int64_t)B * T;
  const unsigned thr = (unsigned)std::min<int64_t>(1024, std::max<int64_t>(32, (BT + 31) / 32 * 32));
  return launch_pdl(detect_kernel, 1, thr, 0, static_cast<cudaStream_t>(stream), probs, threshold, B, T, hard, idx,
                    pos, counts, meta);
}

extern "C" int hclsm_event_gather(const void* states, const int32_t* idx, const int32_t* counts,
                                  const int32_t* meta, void* out, int64_t frame_elems, int32_t B, int32_t pad_k,
                                  int64_t max_frames, int32_t dtype, void* stream) {
  if (!states || !idx || !counts || !meta || !out) return HCLSM_ERR_NULL;
  const size_t esz = dtype == HCLSM_F32 ? 4 : 2;
  if ((frame_elems * esz) % 16 != 0) return HCLSM_ERR_UNSUPPORTED;
  if (max_frames <= 0) return HCLSM_OK;
  if (max_frames > 65535) return HCLSM_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n16 = frame_elems * esz / 16;
  dim3 grid((unsigned)std::min<int64_t>((n16 + 255) / 256, 64), (unsigned)max_frames);
  if (dtype == HCLSM_F32)
    return launch_pdl(gather_kernel<float>, grid, 256, 0, st, static_cast<const float*>(states), idx, counts, meta,
                      static_cast<float*>(out), frame_elems, B, pad_k, max_frames);
  else if (dtype == HCLSM_BF16)
    return launch_pdl(gather_kernel<__nv_bfloat16>, grid, 256, 0, st, static_cast<const __nv_bfloat16*>(states), idx,
                      counts, meta, static_cast<__nv_bfloat16*>(out), frame_elems, B, pad_k, max_frames);
  else
    return HCLSM_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

extern "C" int hclsm_event_scatter(const void* states, const void* upd, const int32_t* pos, const int32_t* counts,
                                   void* out, int64_t frames, int64_t frame_elems, int32_t T, int32_t pad_k,
                                   int32_t dtype, void* stream) {
  if (!states || !upd || !pos || !counts || !out) return HCLSM_ERR_NULL;
  const size_t esz = dtype == HCLSM_F32 ? 4 : 2;
  if ((frame_elems * esz) % 16 != 0) return HCLSM_ERR_UNSUPPORTED;
  if (frames <= 0) return HCLSM_OK;
  if (frames > 65535) return HCLSM_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n16 = frame_elems * esz / 16;
  dim3 grid((unsigned)std::min<int64_t>((n16 + 255) / 256, 64), (unsigned)frames);
  if (dtype == HCLSM_F32)
    return launch_pdl(scatter_kernel<float>, grid, 256, 0, st, static_cast<const float*>(states),
                      static_cast<const float*>(upd), pos, counts, static_cast<float*>(out), frame_elems, T, pad_k);
  else if (dtype == HCLSM_BF16)
    return launch_pdl(scatter_kernel<__nv_bfloat16>, grid, 256, 0, st, static_cast<const __nv_bfloat16*>(states),
                      static_cast<const __nv_bfloat16*>(upd), pos, counts, static_cast<__nv_bfloat16*>(out),
                      frame_elems, T, pad_k);
  else
    return HCLSM_ERR_DTYPE;
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

template <int TP, int HD>
static void launch_mha(const void* qkv, const uint8_t* kp, void* out, int frames, int T, int H, float scale,
                       cudaStream_t st) {
  (void)launch_pdl(mha_bf16_kernel<TP, HD>, frames * H, 32, 0, st, static_cast<const __nv_bfloat16*>(qkv), kp,
                   static_cast<__nv_bfloat16*>(out), T, H, scale);
}
template <int TP>
static int launch_mha_tp(const void* qkv, const uint8_t* kp, void* out, int frames, int T, int H, int HD,
                         float scale, cudaStream_t st) {
  switch (HD) {
    case 16: launch_mha<TP, 16>(qkv, kp, out, frames, T, H, scale, st); break;
    case 32: launch_mha<TP, 32>(qkv, kp, out, frames, T, H, scale, st); break;
    case 64: launch_mha<TP, 64>(qkv, kp, out, frames, T, H, scale, st); break;
    case 128:
      if constexpr (TP <= 32) {
        launch_mha<TP, 128>(qkv, kp, out, frames, T, H, scale, st);
        break;
      }
      return HCLSM_ERR_UNSUPPORTED;
    default: return HCLSM_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

extern "C" int hclsm_event_mha(const void* qkv, const uint8_t* key_pad, void* out, int32_t frames, int32_t T,
                               int32_t H, int32_t HD, float scale, int32_t dtype, void* stream) {
  if (!qkv || !out) return HCLSM_ERR_NULL;
  if (frames < 0 || T <= 0 || H <= 0 || HD <= 0) return HCLSM_ERR_SHAPE;
  if (frames == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == HCLSM_F32) {
    mha_f32_kernel<<<frames * H, 64, 0, st>>>(static_cast<const float*>(qkv), key_pad, static_cast<float*>(out), T,
                                             H, HD, scale);
    return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
  }
  if (dtype != HCLSM_BF16) return HCLSM_ERR_DTYPE;
  if (reinterpret_cast<uintptr_t>(qkv) % 16 || reinterpret_cast<uintptr_t>(out) % 16) return HCLSM_ERR_ALIGN;
  // tcgen05 path first (head dim 64, T in {16, 32, 64}); HCLSM_EVENT_MHA=mma
  // selects the mma.sync kernel below (comparisons, tests)
  {
    const char* sel = getenv("HCLSM_EVENT_MHA");
    if (!(sel && sel[0] == 'm')) {
      const int rc = event_mha_tc(qkv, key_pad, out, frames, T, H, HD, scale, stream);
      if (rc != HCLSM_ERR_UNSUPPORTED) return rc;
    }
  }
  if (T <= 16) return launch_mha_tp<16>(qkv, key_pad, out, frames, T, H, HD, scale, st);
  if (T <= 32) return launch_mha_tp<32>(qkv, key_pad, out, frames, T, H, HD, scale, st);
  if (T <= 48) return launch_mha_tp<48>(qkv, key_pad, out, frames, T, H, HD, scale, st);
  if (T <= 64) return launch_mha_tp<64>(qkv, key_pad, out, frames, T, H, HD, scale, st);
  return HCLSM_ERR_UNSUPPORTED;
}

template <typename TU>
static int swiglu_launch(const TU* u, void* y, int64_t rows, int32_t C, int32_t out_dtype, cudaStream_t st) {
  const unsigned blocks = (unsigned)(rows < 148 * 16 ? rows : 148 * 16);
  if (out_dtype == HCLSM_BF16)
    return launch_pdl(swiglu_kernel<TU, __nv_bfloat16>, blocks, 256, 0, st, u, static_cast<__nv_bfloat16*>(y), rows,
                      C);
  if (out_dtype == HCLSM_F32)
    return launch_pdl(swiglu_kernel<TU, float>, blocks, 256, 0, st, u, static_cast<float*>(y), rows, C);
  return HCLSM_ERR_DTYPE;
}

extern "C" int hclsm_swiglu(const void* u, int32_t u_dtype, void* y, int64_t rows, int32_t C, int32_t out_dtype,
                            void* stream) {
  if (!u || !y) return HCLSM_ERR_NULL;
  if (rows < 0 || C <= 0) return HCLSM_ERR_SHAPE;
  if (rows == 0) return HCLSM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // column pairs are read and written as one word: pointers aligned to a pair
  const size_t us = u_dtype == HCLSM_BF16 ? 2 : 4, ys = out_dtype == HCLSM_BF16 ? 2 : 4;
  if ((C & 1) == 0 &&
      (reinterpret_cast<uintptr_t>(u) % (2 * us) != 0 || reinterpret_cast<uintptr_t>(y) % (2 * ys) != 0))
    return HCLSM_ERR_ALIGN;
  if (u_dtype == HCLSM_F32) return swiglu_launch(static_cast<const float*>(u), y, rows, C, out_dtype, st);
  if (u_dtype == HCLSM_BF16) return swiglu_launch(static_cast<const __nv_bfloat16*>(u), y, rows, C, out_dtype, st);
  return HCLSM_ERR_DTYPE;
}
