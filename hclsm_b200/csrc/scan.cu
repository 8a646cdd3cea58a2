// Level-0 selective SSM scan for B200 (sm_100a): forward and backward.
//
// Reference semantics: hclsm/kernels/ssm_scan_kernel.py
//   sequential_ssm_scan :42-86 (clamp=1), parallel_ssm_scan_pytorch :168-218 and
//   _ssm_scan_fwd_kernel :227-290 (clamp=0), _TritonSSMScan.backward :321-377.
//   Recurrence per (sequence, channel d, state s):
//     h_t = exp(dt_t * A_ds) * h_{t-1} + (dt_t * B_ts) * x_t ,  y_t = sum_s h_t * C_ts
//   with A = -exp(A_log) (clamp=0) or A = -clamp(exp(A_log), 1e-6, 1), dt clamped to
//   [1e-3, 1] (clamp=1).  With clamp=1, dt*A lies in [-1, 0), so the reference's
//   clamp of dt*A to [-20, 0] (:77) never binds and is not evaluated here.
//
// Layout: x, dt, z, y and their gradients are (nseq, L, d_inner) row-major, so a
// warp's 32 lanes own 32 consecutive channels and read one contiguous row segment
// per timestep.  B and C (nseq, L, d_state) are shared by every channel of a
// sequence and are broadcast from shared memory.  Every lane keeps its d_state
// fp32 states in registers; time runs sequentially inside the thread.
//
// Backward: the reverse sweep needs h_{t-1} at every step.  The kernel runs a
// forward sweep that leaves a checkpoint of h every K steps in shared memory, and
// for each K-step chunk (last to first) recomputes the chunk and parks h_t and
// exp(dt*A) for the K steps in tensor memory (TMEM: 128 lanes x 512 columns x 4 B,
// one lane per thread), then walks the chunk backwards.  Cross-channel sums (dB,
// dC) are reduced inside each warp by a halving butterfly and across warps in a
// per-chunk shared slab.  dA_log / dD are reduced over sequences by a separate,
// deterministic kernel.
#include <algorithm>
#include <cmath>
#include <vector>
#include <cstdio>

#include <cuda_fp16.h>

#include "common.cuh"

namespace hclsm {
namespace scan {

// softplus(x) = log(1 + e^x) with torch.nn.functional.softplus's default
// threshold (x > 20 returns x).  Applied to dt when the caller passes the raw
// dt projection (the flag HCLSM_SCAN_DT_SOFTPLUS).
__device__ __forceinline__ float softplus_f(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
constexpr int kFwdThreads = 128;
constexpr int kFwdTC = 64;  // timesteps of B/C staged per shared-memory pass

struct FwdParams {
  const void* x;
  const void* dt;
  const float* A_log;
  const void* B;
  const void* C;
  const float* Dp;
  const void* z;
  void* y;
  int64_t nseq;
  int L, D, S;
  // optional (bf16 pair kernel, d_state 9..16): h after every kStateEvery steps,
  // (nseq, nsnap, 4, D) float4 (state quad q of channel d at [q][d]),
  // nsnap = ceil(L / kStateEvery) - 1
  float* states;
  int softplus;  // dt is the raw projection: softplus is applied inside
};

// steps between the state snapshots the forward keeps for the backward (the
// packed backward kernel's chunk length)
constexpr int kStateEvery = 10;

template <typename T, int SP, int CPT, bool CLAMP>
__global__ void __launch_bounds__(kFwdThreads) scan_fwd_kernel(FwdParams p) {
  __shared__ float sB[kFwdTC][SP];
  __shared__ float sC[kFwdTC][SP];

  const int64_t b = blockIdx.y;
  const int D = p.D, S = p.S, L = p.L;
  const int d0 = (blockIdx.x * kFwdThreads + threadIdx.x) * CPT;
  const T* __restrict__ x = static_cast<const T*>(p.x);
  const T* __restrict__ dt = static_cast<const T*>(p.dt);
  const T* __restrict__ Bm = static_cast<const T*>(p.B);
  const T* __restrict__ Cm = static_cast<const T*>(p.C);
  const T* __restrict__ z = static_cast<const T*>(p.z);
  T* __restrict__ y = static_cast<T*>(p.y);

  bool act[CPT];
  float A2[CPT][SP], h[CPT][SP], Dv[CPT];
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    act[c] = d0 + c < D;
    Dv[c] = (p.Dp && act[c]) ? p.Dp[d0 + c] : 0.0f;
#pragma unroll
    for (int s = 0; s < SP; ++s) {
      float a2 = 0.0f;
      if (act[c] && s < S) {
        float e = ex2(p.A_log[(int64_t)(d0 + c) * S + s] * kLog2e);
        if (CLAMP) e = fminf(fmaxf(e, 1e-6f), 1.0f);
        a2 = -e * kLog2e;
      }
      A2[c][s] = a2;
      h[c][s] = 0.0f;
    }
  }
  const bool pair = (CPT == 2) && act[0] && act[CPT - 1];

  for (int t0 = 0; t0 < L; t0 += kFwdTC) {
    const int tc = min(kFwdTC, L - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < tc * SP; i += kFwdThreads) {
      const int tt = i / SP, s = i % SP;
      const int64_t row = (b * L + t0 + tt) * S;
      sB[tt][s] = s < S ? io<T>::ld(Bm + row + s) : 0.0f;
      sC[tt][s] = s < S ? io<T>::ld(Cm + row + s) : 0.0f;
    }
    __syncthreads();
#pragma unroll 2
    for (int tt = 0; tt < tc; ++tt) {
      const int64_t idx = (b * L + t0 + tt) * D + d0;
      float xv[CPT], dv[CPT];
      if (pair) {
        float2 a = io<T>::ld2(x + idx), q = io<T>::ld2(dt + idx);
        xv[0] = a.x; xv[CPT - 1] = a.y; dv[0] = q.x; dv[CPT - 1] = q.y;
      } else {
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          xv[c] = act[c] ? io<T>::ld(x + idx + c) : 0.0f;
          dv[c] = act[c] ? io<T>::ld(dt + idx + c) : 0.0f;
        }
      }
      float dtx[CPT], yv[CPT];
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        if (p.softplus) dv[c] = softplus_f(dv[c]);
        if (CLAMP) dv[c] = fminf(fmaxf(dv[c], 1e-3f), 1.0f);
        dtx[c] = dv[c] * xv[c];
        yv[c] = 0.0f;
      }
#pragma unroll
      for (int s = 0; s < SP; ++s) {
        const float bs = sB[tt][s], cs = sC[tt][s];
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          const float dA = ex2(dv[c] * A2[c][s]);
          h[c][s] = fmaf(dA, h[c][s], dtx[c] * bs);
          yv[c] = fmaf(h[c][s], cs, yv[c]);
        }
      }
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        yv[c] = fmaf(Dv[c], xv[c], yv[c]);
      }
      if (z) {
        float zv[CPT];
        if (pair) {
          float2 a = io<T>::ld2(z + idx);
          zv[0] = a.x; zv[CPT - 1] = a.y;
        } else {
#pragma unroll
          for (int c = 0; c < CPT; ++c) zv[c] = act[c] ? io<T>::ld(z + idx + c) : 0.0f;
        }
#pragma unroll
        for (int c = 0; c < CPT; ++c) yv[c] *= zv[c] * sigmoid(zv[c]);
      }
      if (pair) {
        io<T>::st2(y + idx, yv[0], yv[CPT - 1]);
      } else {
#pragma unroll
        for (int c = 0; c < CPT; ++c)
          if (act[c]) io<T>::st(y + idx + c, yv[c]);
      }
    }
  }
}

// Forward, bf16 I/O, two adjacent channels per thread (the bf16x2 word of x,
// dt, z and y).  The channel pair is processed with packed arithmetic:
//   arg  = dt2 * A2                fp32 pair (FMUL2)
//   dA   = 2^arg                   two ex2.approx.f32 (SFU)
//   h    = fma2(dA, h, dt*x*B)     fp32 pairs (FFMA2), state stays fp32
//   y   += h * C                   fp32 pairs (FFMA2)
// (An f16x2 exponential halves the SFU ops but its f16 -> f32 conversions cost
// more than that on sm_100a: measured 19.9 vs 18.4 ms at config 4.)
// x/dt/z are prefetched one 4-step block ahead in registers; B and C of 64
// steps are staged in shared memory as duplicated pairs (B, B) so that one
// 64-bit load yields an FFMA2 operand.
constexpr int kFwdBlk = 4;

__device__ __forceinline__ float2 bf2_to_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int SP, bool CLAMP>
__global__ void __launch_bounds__(kFwdThreads) scan_fwd_bf16x2_kernel(FwdParams p) {
  // B and C of a 64-step window, one float per state: a 16-byte load brings
  // four states, and each is paired with itself in registers for the packed
  // math (half the shared loads of storing the pairs; the MIO queue that the
  // loads share with the exponentials is this kernel's bound)
  __shared__ __align__(16) float sB[kFwdTC][SP];
  __shared__ __align__(16) float sC[kFwdTC][SP];

  const int64_t b = blockIdx.y;
  const int D = p.D, S = p.S, L = p.L;
  const int d0 = (blockIdx.x * kFwdThreads + threadIdx.x) * 2;
  const bool act = d0 < D;  // D is even on this path
  const uint32_t* __restrict__ x = reinterpret_cast<const uint32_t*>(p.x);
  const uint32_t* __restrict__ dt = reinterpret_cast<const uint32_t*>(p.dt);
  const uint32_t* __restrict__ z = reinterpret_cast<const uint32_t*>(p.z);
  uint32_t* __restrict__ y = reinterpret_cast<uint32_t*>(p.y);
  const __nv_bfloat16* __restrict__ Bm = static_cast<const __nv_bfloat16*>(p.B);
  const __nv_bfloat16* __restrict__ Cm = static_cast<const __nv_bfloat16*>(p.C);
  const bool has_z = z != nullptr;

  float2 A2[SP];
  float2 h[SP];
#pragma unroll
  for (int s = 0; s < SP; ++s) {
    float a0 = 0.0f, a1 = 0.0f;
    if (act && s < S) {
      float e0 = ex2(p.A_log[(int64_t)d0 * S + s] * kLog2e);
      float e1 = ex2(p.A_log[(int64_t)(d0 + 1) * S + s] * kLog2e);
      if (CLAMP) {
        e0 = fminf(fmaxf(e0, 1e-6f), 1.0f);
        e1 = fminf(fmaxf(e1, 1e-6f), 1.0f);
      }
      a0 = -e0 * kLog2e;
      a1 = -e1 * kLog2e;
    }
    A2[s] = make_float2(a0, a1);
    h[s] = make_float2(0.0f, 0.0f);
  }
  const float2 Dv = (p.Dp && act) ? make_float2(p.Dp[d0], p.Dp[d0 + 1]) : make_float2(0.0f, 0.0f);
  const int64_t row0 = b * L;
  const int64_t wD = D / 2;  // 32-bit words per row
  const int64_t col = d0 / 2;

  // state snapshots, (nsnap, 4, D) float4 per sequence: quad q of states of
  // channel d at [q][d], so that a warp's loads in the backward (one channel
  // per lane) are contiguous
  const int nsnap = (L + kStateEvery - 1) / kStateEvery - 1;
  float4* snap = (p.states && act) ? reinterpret_cast<float4*>(p.states) + (size_t)b * nsnap * D * 4 + d0 : nullptr;
  int snap_t = kStateEvery;  // step count after which the next snapshot is taken

  uint32_t cx[kFwdBlk], cd[kFwdBlk], cz[kFwdBlk];
  auto load_blk = [&](int t0, uint32_t (&ox)[kFwdBlk], uint32_t (&od)[kFwdBlk], uint32_t (&oz)[kFwdBlk]) {
#pragma unroll
    for (int j = 0; j < kFwdBlk; ++j) {
      const bool ok = act && (t0 + j < L);
      const int64_t w = (row0 + t0 + j) * wD + col;
      ox[j] = ok ? __ldcs(x + w) : 0u;
      od[j] = ok ? __ldcs(dt + w) : 0u;
      oz[j] = (ok && has_z) ? __ldcs(z + w) : 0u;
    }
  };
  load_blk(0, cx, cd, cz);

  for (int t0 = 0; t0 < L; t0 += kFwdTC) {
    const int tc = min(kFwdTC, L - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < tc * SP; i += kFwdThreads) {
      const int tt = i / SP, s = i % SP;
      const int64_t r = (row0 + t0 + tt) * S;
      const float bv = s < S ? __bfloat162float(Bm[r + s]) : 0.0f;
      const float cv = s < S ? __bfloat162float(Cm[r + s]) : 0.0f;
      sB[tt][s] = bv;
      sC[tt][s] = cv;
    }
    __syncthreads();
    for (int tb = 0; tb < tc; tb += kFwdBlk) {
      uint32_t nx[kFwdBlk], nd[kFwdBlk], nz[kFwdBlk];
      load_blk(t0 + tb + kFwdBlk, nx, nd, nz);
#pragma unroll
      for (int j = 0; j < kFwdBlk; ++j) {
        const int tt = tb + j;
        if (tt < tc) {
          float2 xv = bf2_to_f2(cx[j]);
          float2 dv = bf2_to_f2(cd[j]);
          if (p.softplus) {
            dv.x = softplus_f(dv.x);
            dv.y = softplus_f(dv.y);
          }
          if (CLAMP) {
            dv.x = fminf(fmaxf(dv.x, 1e-3f), 1.0f);
            dv.y = fminf(fmaxf(dv.y, 1e-3f), 1.0f);
          }
          const float2 dtx = __fmul2_rn(dv, xv);
          float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int s = 0; s < SP; ++s) {
            const float2 ar = __fmul2_rn(dv, A2[s]);
            const float2 dA = make_float2(ex2(ar.x), ex2(ar.y));
            const float bb = sB[tt][s], cc = sC[tt][s];
            h[s] = __ffma2_rn(dA, h[s], __fmul2_rn(dtx, make_float2(bb, bb)));
            acc = __ffma2_rn(h[s], make_float2(cc, cc), acc);
          }
          acc = __ffma2_rn(Dv, xv, acc);
          if (has_z) {
            const float2 zv = bf2_to_f2(cz[j]);
            acc.x *= zv.x * sigmoid(zv.x);
            acc.y *= zv.y * sigmoid(zv.y);
          }
          if (act) __stcs(y + (row0 + t0 + tt) * wD + col, f2_to_bf2(acc.x, acc.y));
          if constexpr (SP == 16) {
            if (t0 + tt + 1 == snap_t) {
              if (snap_t < L && snap) {
                float4* o = snap + (size_t)(snap_t / kStateEvery - 1) * D * 4;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  __stcs(o + (size_t)q * D, make_float4(h[4 * q].x, h[4 * q + 1].x, h[4 * q + 2].x, h[4 * q + 3].x));
                  __stcs(o + (size_t)q * D + 1,
                         make_float4(h[4 * q].y, h[4 * q + 1].y, h[4 * q + 2].y, h[4 * q + 3].y));
                }
              }
              snap_t += kStateEvery;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kFwdBlk; ++j) { cx[j] = nx[j]; cd[j] = nd[j]; cz[j] = nz[j]; }
    }
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
constexpr int kBwdThreads = 128;  // one thread per TMEM lane
constexpr int kTmemCols = 512;

template <typename T, int SP>
struct BwdCfg {
  static constexpr int K = (256 / SP) < 32 ? (256 / SP) : 32;  // history steps per chunk
  static constexpr int NV = 2 * SP;                             // dB and dC values per step
  static constexpr int NSTAGE = sizeof(T) == 2 ? 2 : 1;
  static constexpr int NTEN = 4;  // x, dt, dy, z tiles
  static constexpr size_t tile_elems = (size_t)K * kBwdThreads;
  static constexpr size_t stage_bytes = NTEN * tile_elems * sizeof(T);
};

struct BwdParams {
  const void* x;
  const void* dt;
  const float* A_log;
  const void* B;
  const void* C;
  const float* Dp;
  const void* z;
  const void* dy;
  void* dx;
  void* ddt;
  void* dz;
  float* dAlog_part;  // (nseq, D, S): per-sequence partial of dA_log
  float* dD_part;     // (nseq, D)
  float* dBC_ws;      // (nsplit, nseq, L, 2*SP) fp32 accumulators of dB | dC
  int64_t nseq;
  int L, D, S;
  int nck;             // number of K-step chunks
  int groups;          // number of 128-channel groups
  int groups_per_cta;  // contiguous groups handled by one CTA
  int nsplit;
  float* ckpt_ws;   // packed bf16 kernel: per-SM checkpoint slots
  int ckpt_slots;
  const float* states;  // packed bf16 kernel: the forward's snapshots (no forward sweep), or null
  int softplus;         // dt is the raw projection: softplus is applied inside
  int* err;
};

// Host and device agree on this shared-memory layout: tile stages, one chunk
// of B and C (fp32), the per-chunk dB|dC slab, barriers.  Checkpoints live in
// the workspace (one slot per SM).  The total is padded past half of the SM's
// shared memory so that one block runs per SM (the slots rely on it).
template <typename T, int SP>
struct BwdSmem {
  using Cfg = BwdCfg<T, SP>;
  __host__ __device__ static size_t tiles_off() { return 0; }
  __host__ __device__ static size_t bc_off() { return Cfg::NSTAGE * Cfg::stage_bytes; }
  __host__ __device__ static size_t slab_off() { return bc_off() + (size_t)Cfg::K * SP * 2 * sizeof(float); }
  __host__ __device__ static size_t bar_off() { return slab_off() + 4 * (size_t)Cfg::K * Cfg::NV * sizeof(float); }
  __host__ __device__ static size_t total() {
    const size_t t = bar_off() + 64;
    return t > 120 * 1024 ? t : 120 * 1024;
  }
};
// checkpoint floats per SM slot of the generic kernel
__host__ __device__ inline size_t gen_slot_floats(int nck, int SP) {
  return (size_t)(nck > 1 ? nck - 1 : 0) * SP * 128;
}

__device__ __forceinline__ uint32_t smid() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
      "%13, %14, %15, %16};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]),
        "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "f"(v[0]),
               "f"(v[1]), "f"(v[2]), "f"(v[3])
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
                 "=f"(v[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
               : "r"(taddr)
               : "memory");
}

// Stores / loads exactly SP consecutive fp32 columns of this thread's TMEM lane
// (SP a multiple of 4).  Loads are issued back to back and waited for once.
template <int SP>
__device__ __forceinline__ void tmem_store(uint32_t taddr, const float (&v)[SP]) {
#pragma unroll
  for (int q = 0; q < SP;) {
    if (SP - q >= 16) {
      float w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = v[q + i];
      tmem_st16(taddr + q, w);
      q += 16;
    } else if (SP - q >= 8) {
      tmem_st8(taddr + q, &v[q]);
      q += 8;
    } else {
      tmem_st4(taddr + q, &v[q]);
      q += 4;
    }
  }
}
template <int SP>
__device__ __forceinline__ void tmem_load_nowait(uint32_t taddr, float (&v)[SP]) {
#pragma unroll
  for (int q = 0; q < SP;) {
    if (SP - q >= 16) {
      float w[16];
      tmem_ld16(taddr + q, w);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[q + i] = w[i];
      q += 16;
    } else if (SP - q >= 8) {
      tmem_ld8(taddr + q, &v[q]);
      q += 8;
    } else {
      tmem_ld4(taddr + q, &v[q]);
      q += 4;
    }
  }
}

// Sum of v[i] over the 32 lanes.  Halving butterfly: at each level the lane
// keeps one half of its values and adds the partner's copy of that half, so 31
// shuffles reduce 32 values.  Afterwards lane l holds the total of value index
// (l >> (5 - log2 N)) in v[0] when N <= 32, or indices N/32*l ... in v[0..N/32).
template <int N, int M>
struct Halving {
  static __device__ __forceinline__ void run(float* v, int lane) {
    if constexpr (M > 0) {
      if constexpr (N > 1) {
        constexpr int HN = N / 2;
        const bool upper = (lane & M) != 0;
#pragma unroll
        for (int i = 0; i < HN; ++i) {
          const float send = upper ? v[i] : v[i + HN];
          const float keep = upper ? v[i + HN] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, M);
        }
        Halving<HN, M / 2>::run(v, lane);
      } else {
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], M);
        Halving<1, M / 2>::run(v, lane);
      }
    }
  }
};
template <int N>
__device__ __forceinline__ void warp_halving_reduce(float (&v)[N], int lane) {
  Halving<N, 16>::run(v, lane);
}

template <typename T, int SP, bool CLAMP>
__global__ void __launch_bounds__(kBwdThreads, 1) scan_bwd_kernel(BwdParams p) {
  using Cfg = BwdCfg<T, SP>;
  using Sm = BwdSmem<T, SP>;
  constexpr int K = Cfg::K, NV = Cfg::NV, NSTAGE = Cfg::NSTAGE;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint32_t s_tmem_base;
  __shared__ int s_abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = p.L, D = p.D, S = p.S, nck = p.nck;
  const int64_t b = blockIdx.x;
  const int split = blockIdx.y;
  const int g_begin = split * p.groups_per_cta;
  const int g_end = min(p.groups, g_begin + p.groups_per_cta);
  if (g_begin >= g_end) {  // no channels for this split: its dB|dC rows are zero
    float* dst = p.dBC_ws + ((int64_t)split * p.nseq + b) * L * NV;
    for (int e = tid; e < L * NV; e += kBwdThreads) dst[e] = 0.0f;
    return;
  }
  const uint32_t slot = smid();
  if (slot >= (uint32_t)p.ckpt_slots) {
    if (tid == 0) record_error(p.err, HCLSM_ERR_LAUNCH);
    return;
  }

  T* tiles = reinterpret_cast<T*>(smem + Sm::tiles_off());
  float* sBf = reinterpret_cast<float*>(smem + Sm::bc_off());  // (K, SP): this chunk's B
  float* sCf = sBf + (size_t)K * SP;                             // (K, SP): this chunk's C
  float* slab = reinterpret_cast<float*>(smem + Sm::slab_off());  // (4, K, NV)
  float4* ckpt = reinterpret_cast<float4*>(p.ckpt_ws + (size_t)slot * gen_slot_floats(nck, SP));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Sm::bar_off());
  const T* Bseq = static_cast<const T*>(p.B) + b * L * S;
  const T* Cseq = static_cast<const T*>(p.C) + b * L * S;
  // stage B and C of steps [t0, t0 + n) as fp32 (padded states zero)
  auto stage_bc = [&](int t0, int n) {
    __syncthreads();
    for (int i = tid; i < n * SP; i += kBwdThreads) {
      const int t = i / SP, s = i % SP;
      sBf[i] = s < S ? io<T>::ld(Bseq + (int64_t)(t0 + t) * S + s) : 0.0f;
      sCf[i] = s < S ? io<T>::ld(Cseq + (int64_t)(t0 + t) * S + s) : 0.0f;
    }
    __syncthreads();
  };

  const T* __restrict__ gx = static_cast<const T*>(p.x);
  const T* __restrict__ gdt = static_cast<const T*>(p.dt);
  const T* __restrict__ gdy = static_cast<const T*>(p.dy);
  const T* __restrict__ gz = static_cast<const T*>(p.z);
  const bool has_z = p.z != nullptr;
  const bool has_D = p.Dp != nullptr;

  // ---- set-up: TMEM, barriers, B/C staging -----------------------------------
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < NSTAGE; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem_base + ((uint32_t)(warp * 32) << 16);

  // ---- tile producer -----------------------------------------------------------
  // Work items, in order: for each group, nck forward chunks then nck reverse
  // chunks.  Item i uses stage i % NSTAGE.
  const int items_per_group = 2 * nck;
  const int n_items = (g_end - g_begin) * items_per_group;
  auto issue = [&](int it) {
    if (it >= n_items) return;
    const int g = g_begin + it / items_per_group;
    const int r = it % items_per_group;
    const bool rev = r >= nck;
    const int k = rev ? (items_per_group - 1 - r) : r;
    const int t0 = k * K;
    const int n = min(K, L - t0);
    const int c0 = g * kBwdThreads;
    const int w = min(kBwdThreads, D - c0);
    const uint32_t row_bytes = (uint32_t)(w * sizeof(T));
    const int nten = rev ? (has_z ? 4 : 3) : 2;
    const int stage = it % NSTAGE;
    T* st = tiles + (size_t)stage * Cfg::NTEN * Cfg::tile_elems;
    if (warp == 0) {
      if (lane == 0) mbar_expect_tx(&bars[stage], row_bytes * n * nten);
      __syncwarp();
      for (int q = lane; q < n * nten; q += 32) {
        const int ten = q / n, j = q % n;
        const T* src = ten == 0 ? gx : ten == 1 ? gdt : ten == 2 ? gdy : gz;
        src += (b * L + t0 + j) * (int64_t)D + c0;
        bulk_g2s(st + ((size_t)ten * K + j) * kBwdThreads, src, row_bytes, &bars[stage]);
      }
    }
  };
  auto wait_item = [&](int it) {
    const int stage = it % NSTAGE;
    const uint32_t parity = (it / NSTAGE) & 1;
    if (!s_abort) {
      if (!mbar_wait(&bars[stage], parity)) {
        record_error(p.err, HCLSM_ERR_TIMEOUT);
        s_abort = 1;
      }
    }
  };
  for (int i = 0; i < NSTAGE; ++i) issue(i);

  float* dbc_base = p.dBC_ws + ((int64_t)split * p.nseq + b) * L * NV;
  int it = 0;
  for (int g = g_begin; g < g_end; ++g) {
    const int d = g * kBwdThreads + tid;
    const bool act = d < D;
    float A[SP], A2[SP], fac[SP];
#pragma unroll
    for (int s = 0; s < SP; ++s) {
      A[s] = 0.0f; A2[s] = 0.0f; fac[s] = 0.0f;
      if (act && s < S) {
        const float e = ex2(p.A_log[(int64_t)d * S + s] * kLog2e);
        const float ec = CLAMP ? fminf(fmaxf(e, 1e-6f), 1.0f) : e;
        A[s] = -ec;
        A2[s] = -ec * kLog2e;
        // dA/dA_log = -exp(A_log), zero where the clamp binds
        fac[s] = (CLAMP && (e < 1e-6f || e > 1.0f)) ? 0.0f : -e;
      }
    }
    const float Dd = (has_D && act) ? p.Dp[d] : 0.0f;

    // ---- forward sweep: checkpoints ------------------------------------------
    float h[SP];
#pragma unroll
    for (int s = 0; s < SP; ++s) h[s] = 0.0f;
    for (int k = 0; k < nck; ++k, ++it) {
      wait_item(it);
      const T* st = tiles + (size_t)(it % NSTAGE) * Cfg::NTEN * Cfg::tile_elems;
      const int t0 = k * K, n = min(K, L - t0);
      stage_bc(t0, n);
      if (k > 0) {
#pragma unroll
        for (int q = 0; q < SP / 4; ++q)
          __stcg(&ckpt[((size_t)(k - 1) * (SP / 4) + q) * kBwdThreads + tid],
                 make_float4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]));
      }
      for (int j = 0; j < n; ++j) {
        float xv = act ? io<T>::ld(st + (size_t)j * kBwdThreads + tid) : 0.0f;
        float dv = act ? io<T>::ld(st + ((size_t)K + j) * kBwdThreads + tid) : 0.0f;
        if (p.softplus) dv = softplus_f(dv);
        if (CLAMP) dv = fminf(fmaxf(dv, 1e-3f), 1.0f);
        const float dtx = dv * xv;
        const float* Bt = sBf + (size_t)j * SP;
#pragma unroll
        for (int s = 0; s < SP; ++s) h[s] = fmaf(ex2(dv * A2[s]), h[s], dtx * Bt[s]);
      }
      __syncthreads();
      if (warp == 0) issue(it + NSTAGE);
    }

    // ---- reverse sweep --------------------------------------------------------
    float gcar[SP], gAcc[SP];
#pragma unroll
    for (int s = 0; s < SP; ++s) { gcar[s] = 0.0f; gAcc[s] = 0.0f; }
    float dDacc = 0.0f;
    for (int k = nck - 1; k >= 0; --k, ++it) {
      wait_item(it);
      const T* st = tiles + (size_t)(it % NSTAGE) * Cfg::NTEN * Cfg::tile_elems;
      const int t0 = k * K, n = min(K, L - t0);
      stage_bc(t0, n);
      // recompute the chunk from its checkpoint, parking h_t and dA_t in TMEM
      float hs[SP];
      if (k > 0) {
#pragma unroll
        for (int q = 0; q < SP / 4; ++q) {
          const float4 c4 = __ldcg(&ckpt[((size_t)(k - 1) * (SP / 4) + q) * kBwdThreads + tid]);
          hs[4 * q] = c4.x; hs[4 * q + 1] = c4.y; hs[4 * q + 2] = c4.z; hs[4 * q + 3] = c4.w;
        }
      } else {
#pragma unroll
        for (int s = 0; s < SP; ++s) hs[s] = 0.0f;
      }
      for (int j = 0; j < n; ++j) {
        float xv = act ? io<T>::ld(st + (size_t)j * kBwdThreads + tid) : 0.0f;
        float dv = act ? io<T>::ld(st + ((size_t)K + j) * kBwdThreads + tid) : 0.0f;
        if (p.softplus) dv = softplus_f(dv);
        if (CLAMP) dv = fminf(fmaxf(dv, 1e-3f), 1.0f);
        const float dtx = dv * xv;
        const float* Bt = sBf + (size_t)j * SP;
        float dA[SP];
#pragma unroll
        for (int s = 0; s < SP; ++s) {
          dA[s] = ex2(dv * A2[s]);
          hs[s] = fmaf(dA[s], hs[s], dtx * Bt[s]);
        }
        const uint32_t col = tmem + (uint32_t)(j * 2 * SP);
        tmem_store<SP>(col, hs);
        tmem_store<SP>(col + SP, dA);
      }
      tmem_wait_st();
      // hs == h at the last step of the chunk
      for (int j = n - 1; j >= 0; --j) {
        const int t = t0 + j;
        float xv = act ? io<T>::ld(st + (size_t)j * kBwdThreads + tid) : 0.0f;
        const float draw = act ? io<T>::ld(st + ((size_t)K + j) * kBwdThreads + tid) : 0.0f;
        float gy = act ? io<T>::ld(st + ((size_t)2 * K + j) * kBwdThreads + tid) : 0.0f;
        // dv = clamp(softplus(raw)); mdt = d dv / d raw
        float dv = draw, mdt = 1.0f;
        if (p.softplus) {
          dv = softplus_f(draw);
          mdt = sigmoid(draw);
        }
        if (CLAMP) {
          mdt = (dv >= 1e-3f && dv <= 1.0f) ? mdt : 0.0f;
          dv = fminf(fmaxf(dv, 1e-3f), 1.0f);
        }
        const float dtx = dv * xv;
        const float* Bt = sBf + (size_t)j * SP;
        const float* Ct = sCf + (size_t)j * SP;
        float dA[SP], hp[SP];
        const uint32_t col = tmem + (uint32_t)(j * 2 * SP);
        tmem_load_nowait<SP>(col + SP, dA);
        if (j > 0) {
          tmem_load_nowait<SP>(col - 2 * SP, hp);
        } else if (k > 0) {
#pragma unroll
          for (int q = 0; q < SP / 4; ++q) {
            const float4 c4 = __ldcg(&ckpt[((size_t)(k - 1) * (SP / 4) + q) * kBwdThreads + tid]);
            hp[4 * q] = c4.x; hp[4 * q + 1] = c4.y; hp[4 * q + 2] = c4.z; hp[4 * q + 3] = c4.w;
          }
        } else {
#pragma unroll
          for (int s = 0; s < SP; ++s) hp[s] = 0.0f;
        }
        tmem_wait_ld();
        float dzv = 0.0f;
        if (has_z) {
          const float zv = act ? io<T>::ld(st + ((size_t)3 * K + j) * kBwdThreads + tid) : 0.0f;
          float ys = 0.0f;
#pragma unroll
          for (int s = 0; s < SP; ++s) ys = fmaf(hs[s], Ct[s], ys);
          ys = fmaf(Dd, xv, ys);
          const float sg = sigmoid(zv);
          dzv = gy * ys * sg * (1.0f + zv * (1.0f - sg));
          gy = gy * zv * sg;
        }
        float gB = 0.0f, ddA = 0.0f;
        float pv[NV];
#pragma unroll
        for (int s = 0; s < SP; ++s) {
          const float gs = fmaf(gy, Ct[s], gcar[s]);
          gB = fmaf(gs, Bt[s], gB);
          pv[s] = gs * dtx;
          pv[SP + s] = gy * hs[s];
          const float w = dA[s] * gs;
          const float R = w * hp[s];
          ddA = fmaf(A[s], R, ddA);
          gAcc[s] = fmaf(dv, R, gAcc[s]);
          gcar[s] = w;
          hs[s] = hp[s];
        }
        dDacc = fmaf(gy, xv, dDacc);
        if (act) {
          const int64_t gi = (b * L + t) * (int64_t)D + d;
          io<T>::st(static_cast<T*>(p.dx) + gi, fmaf(dv, gB, Dd * gy));
          io<T>::st(static_cast<T*>(p.ddt) + gi, fmaf(xv, gB, ddA) * mdt);
          if (has_z) io<T>::st(static_cast<T*>(p.dz) + gi, dzv);
        }
        warp_halving_reduce<NV>(pv, lane);
        constexpr int kShift = (NV >= 32) ? 0 : (NV == 16 ? 1 : (NV == 8 ? 2 : 3));
        if (NV >= 32) {
#pragma unroll
          for (int i = 0; i < NV / 32; ++i) slab[((size_t)warp * K + j) * NV + lane * (NV / 32) + i] = pv[i];
        } else if ((lane & ((1 << kShift) - 1)) == 0) {
          slab[((size_t)warp * K + j) * NV + (lane >> kShift)] = pv[0];
        }
      }
      __syncthreads();
      // fold the four warps' partial sums into this sequence's dB|dC rows
      {
        float* dst = dbc_base + (int64_t)t0 * NV;
        const bool first = (g == g_begin);
        for (int e = tid; e < n * NV; e += kBwdThreads) {
          const int j = e / NV, v = e % NV;
          float acc = slab[((size_t)0 * K + j) * NV + v] + slab[((size_t)1 * K + j) * NV + v] +
                      slab[((size_t)2 * K + j) * NV + v] + slab[((size_t)3 * K + j) * NV + v];
          if (!first) acc += dst[e];
          dst[e] = acc;
        }
      }
      __syncthreads();
      if (warp == 0) issue(it + NSTAGE);
    }
    if (act) {
      float* da = p.dAlog_part + (b * D + d) * (int64_t)S;
#pragma unroll
      for (int s = 0; s < SP; ++s)
        if (s < S) da[s] = gAcc[s] * fac[s];
      if (has_D) p.dD_part[b * D + d] = dDacc;
    }
  }

  // ---- tear-down ---------------------------------------------------------------
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(s_tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// TMEM loads whose destination registers are tied to the wait: the values are
// consumed only after tcgen05.wait::ld, and no memory clobber is needed, so
// shared-memory traffic can be scheduled across them.
__device__ __forceinline__ void tmem_ld16_nc(uint32_t taddr, float (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]),
        "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8_nc(uint32_t taddr, float (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld_tied16(float (&a)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(a[0]), "+f"(a[1]), "+f"(a[2]), "+f"(a[3]), "+f"(a[4]), "+f"(a[5]), "+f"(a[6]), "+f"(a[7]),
                 "+f"(a[8]), "+f"(a[9]), "+f"(a[10]), "+f"(a[11]), "+f"(a[12]), "+f"(a[13]), "+f"(a[14]),
                 "+f"(a[15]));
}
__device__ __forceinline__ void tmem_wait_ld_tied(float (&a)[16], float (&b)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+f"(a[0]), "+f"(a[1]), "+f"(a[2]), "+f"(a[3]), "+f"(a[4]), "+f"(a[5]), "+f"(a[6]), "+f"(a[7]),
                 "+f"(a[8]), "+f"(a[9]), "+f"(a[10]), "+f"(a[11]), "+f"(a[12]), "+f"(a[13]), "+f"(a[14]),
                 "+f"(a[15]), "+f"(b[0]), "+f"(b[1]), "+f"(b[2]), "+f"(b[3]), "+f"(b[4]), "+f"(b[5]), "+f"(b[6]),
                 "+f"(b[7]));
}

// ---------------------------------------------------------------------------
// backward, bf16 I/O and d_state <= 16: packed variant, 8 warps
// ---------------------------------------------------------------------------
// Same algorithm as scan_bwd_kernel, reorganised for issue efficiency:
//  * a CTA has 256 threads (two warps per SM sub-partition), one channel and
//    all 16 states per thread, so per-timestep scalar work (loads, clamps,
//    stores, reductions) is shared by 16 states;
//  * warps w and w+4 share a TMEM lane quarter and split its 512 columns: 10
//    steps of history per thread, h_t as fp32 and dA_t as f16x2 (24 columns
//    per step);
//  * the sqrt(L) checkpoints of h (every 10 steps) live in a per-SM slot of
//    the workspace (blocks run one per SM, slot = %smid), which stays resident
//    in L2; the next chunk's checkpoint is fetched while a chunk is processed;
//  * per-state arithmetic runs on state pairs (FFMA2 / FMUL2); exp(dt*A) is
//    ex2.approx.f32, and dA is parked as f16x2 (one pack per pair) so that 10
//    steps fit the TMEM half (fp32 dA, 8-step chunks, measured slower);
//  * in the dB/dC warp reduction, lane l keeps state s in register slot
//    s ^ (l & 12), so the levels that exchange across lane bits 3 and 2 keep
//    slots [0, n/2) without selects.
constexpr int kW16Threads = 256;
constexpr int kW16Ch = 256;   // channels per group
constexpr int kW16K = 10;     // history steps per chunk
static_assert(kW16K == kStateEvery, "the forward's snapshots are the packed kernel's chunk boundaries");
// TMEM columns of a thread: h slots 0..K (16 fp32 each; slot 0 holds the
// chunk's starting state, slot j + 1 the state after step j), then the K
// steps' dA as f16 pairs (8 columns each)
constexpr int kW16DACol = 16 * (kW16K + 1);
static_assert(kW16DACol + 8 * kW16K <= 256, "a warp pair shares 512 TMEM columns");
constexpr int kW16MaxSlots = 1024;

struct W16Smem {
  __host__ __device__ static size_t tile_elems() { return (size_t)kW16K * kW16Ch; }
  __host__ __device__ static size_t tiles_bytes() { return 2 * 4 * tile_elems() * 2; }
  __host__ __device__ static size_t bc_off() { return tiles_bytes(); }
  __host__ __device__ static size_t slab_off(int L) { return bc_off() + (size_t)L * 16 * 2 * 4; }
  __host__ __device__ static size_t dbc_off(int L) { return slab_off(L) + 2 * 8 * (size_t)kW16K * 32 * 4; }
  __host__ __device__ static size_t bar_off(int L) { return dbc_off(L) + (size_t)L * 32 * 4; }
  // more than half of the SM's shared memory: one block per SM, which the
  // per-SM checkpoint slots rely on
  __host__ __device__ static size_t total(int L) {
    const size_t t = bar_off(L) + 64;
    return t > 120 * 1024 ? t : 120 * 1024;
  }
};
// checkpoint floats per slot
__host__ __device__ inline size_t w16_slot_floats(int nck) { return (size_t)(nck > 1 ? nck - 1 : 0) * 16 * kW16Threads; }

__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
__device__ __forceinline__ __half2 bits_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 shfl2(float2 v, int m) {
  return f2(__shfl_xor_sync(0xffffffffu, v.x, m), __shfl_xor_sync(0xffffffffu, v.y, m));
}

// bf16 store that only predicated-on lanes execute (no branch, so the step
// stays one scheduling region)
__device__ __forceinline__ void st_bf16_if(__nv_bfloat16* ptr, float v, bool pred) {
  const unsigned short u = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  asm volatile("{ .reg .pred q; setp.ne.b32 q, %2, 0; @q st.global.b16 [%0], %1; }" ::"l"(ptr), "h"(u),
               "r"((int)pred));
}

template <bool CLAMP, bool SOFTPLUS, bool HASZ>
__global__ void __launch_bounds__(kW16Threads, 1) scan_bwd_bf16_kernel(BwdParams p) {
  using T = __nv_bfloat16;
  using Sm = W16Smem;
  constexpr int K = kW16K;
  const size_t TILE = Sm::tile_elems();
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint32_t s_tmem_base;
  __shared__ int s_abort;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int perm = lane & 12;  // register slot j holds state j ^ perm
  const int pq = perm >> 1;    // the same on state pairs
  const int L = p.L, D = p.D, S = p.S, nck = p.nck;
  const int64_t b = blockIdx.x;
  const int split = blockIdx.y;
  const int g_begin = split * p.groups_per_cta;
  const int g_end = min(p.groups, g_begin + p.groups_per_cta);
  if (g_begin >= g_end) {  // no channels for this split: its dB|dC rows are zero
    float4* dst = reinterpret_cast<float4*>(p.dBC_ws + ((int64_t)split * p.nseq + b) * L * 32);
    for (int e = tid; e < L * 8; e += kW16Threads) dst[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  // with the forward's snapshots there is no forward sweep and no checkpoint slot
  const bool saved = p.states != nullptr;
  const uint32_t slot = saved ? 0u : smid();
  if (slot >= (uint32_t)p.ckpt_slots) {  // uniform over the block
    if (tid == 0) record_error(p.err, HCLSM_ERR_LAUNCH);
    return;
  }
  float4* ckpt = reinterpret_cast<float4*>(p.ckpt_ws + (size_t)slot * w16_slot_floats(nck));
  // checkpoints stay in L2; the streamed inputs should not displace them
  const uint64_t keep = policy_evict_last(), stream_pol = policy_evict_first();

  T* tiles = reinterpret_cast<T*>(smem);
  float* sBf = reinterpret_cast<float*>(smem + Sm::bc_off());
  float* sCf = sBf + (size_t)L * 16;
  float* slab0 = reinterpret_cast<float*>(smem + Sm::slab_off(L));  // 2 x (8, K, 32)
  int slab_buf = 0;
  float* dbc = reinterpret_cast<float*>(smem + Sm::dbc_off(L));    // (L, 32)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Sm::bar_off(L));

  const T* __restrict__ gx = static_cast<const T*>(p.x);
  const T* __restrict__ gdt = static_cast<const T*>(p.dt);
  const T* __restrict__ gdy = static_cast<const T*>(p.dy);
  const T* __restrict__ gz = static_cast<const T*>(p.z);
  constexpr bool has_z = HASZ;
  const bool has_D = p.Dp != nullptr;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&s_tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    s_abort = 0;
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  {
    const T* Bm = static_cast<const T*>(p.B) + b * L * S;
    const T* Cm = static_cast<const T*>(p.C) + b * L * S;
    for (int i = tid; i < L * 16; i += kW16Threads) {
      const int t = i >> 4, s = i & 15;
      sBf[i] = s < S ? __bfloat162float(Bm[(int64_t)t * S + s]) : 0.0f;
      sCf[i] = s < S ? __bfloat162float(Cm[(int64_t)t * S + s]) : 0.0f;
    }
  }
  {  // zero the tiles: the columns past a partial group's channels are never copied
    float4* z4 = reinterpret_cast<float4*>(tiles);
    for (int e = tid; e < (int)(Sm::tiles_bytes() / 16); e += kW16Threads) z4[e] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before the bulk copies overwrite them
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)((warp >> 2) * 256);

  const int items_per_group = saved ? nck : 2 * nck;
  const int n_items = (g_end - g_begin) * items_per_group;
  auto issue = [&](int it) {
    if (it >= n_items) return;
    const int g = g_end - 1 - it / items_per_group;  // groups run last to first
    const int r = it % items_per_group;
    const bool rev = saved || r >= nck;
    const int k = rev ? (items_per_group - 1 - r) : r;
    const int t0 = k * K;
    const int n = min(K, L - t0);
    const int c0 = g * kW16Ch;
    const int w = min(kW16Ch, D - c0);
    const uint32_t row_bytes = (uint32_t)(w * sizeof(T));
    const int nten = rev ? (has_z ? 4 : 3) : 2;
    const int stage = it & 1;
    T* st = tiles + (size_t)stage * 4 * TILE;
    if (warp == 0) {
      if (lane == 0) mbar_expect_tx(&bars[stage], row_bytes * n * nten);
      __syncwarp();
      for (int q = lane; q < n * nten; q += 32) {
        const int ten = q / n, j = q % n;
        const T* src = ten == 0 ? gx : ten == 1 ? gdt : ten == 2 ? gdy : gz;
        src += (b * L + t0 + j) * (int64_t)D + c0;
        bulk_g2s_hint(st + (size_t)ten * TILE + (size_t)j * kW16Ch, src, row_bytes, &bars[stage], stream_pol);
      }
    }
  };
  auto wait_item = [&](int it) {
    if (!s_abort) {
      if (!mbar_wait(&bars[it & 1], (it >> 1) & 1)) {
        record_error(p.err, HCLSM_ERR_TIMEOUT);
        s_abort = 1;
      }
    }
  };
  issue(0);
  issue(1);

  // B or C of step t in this lane's slot order: pair q holds states
  // 2*(q ^ pq) + {0, 1}
  auto load_bc = [&](const float* base, int t, float2 (&o)[8]) {
    // pairs 2m and 2m+1 of this lane's slot order are the adjacent pairs of
    // float4 m ^ (perm >> 2): four 16-byte loads instead of eight 8-byte ones
    const float4* row = reinterpret_cast<const float4*>(base + (size_t)t * 16);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float4 v = row[m ^ (perm >> 2)];
      o[2 * m] = f2(v.x, v.y);
      o[2 * m + 1] = f2(v.z, v.w);
    }
  };
  auto load_ck = [&](int k, float2 (&o)[8], int d) {  // checkpoint before chunk k (k >= 1)
    if (saved) {
      // the forward's snapshot of channel d, states in natural order: float4 m
      // holds states 4m..4m+3, which this lane keeps in pair slots
      // 2 (m ^ (perm >> 2)) and 2 (m ^ (perm >> 2)) + 1
      if (d >= D) {
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = f2(0.0f, 0.0f);
        return;
      }
      const float4* c = reinterpret_cast<const float4*>(p.states) + ((size_t)b * (nck - 1) + (k - 1)) * D * 4 + d;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float4 v = ld_hint(c + (size_t)(m ^ (perm >> 2)) * D, stream_pol);
        o[2 * m] = f2(v.x, v.y);
        o[2 * m + 1] = f2(v.z, v.w);
      }
      return;
    }
    const float4* c = ckpt + (size_t)(k - 1) * 4 * kW16Threads + tid;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v = ld_hint(c + (size_t)q * kW16Threads, keep);
      o[2 * q] = f2(v.x, v.y);
      o[2 * q + 1] = f2(v.z, v.w);
    }
  };

  int it = 0;
  // groups run last to first: only the last group of the channels can be
  // partial, and it then runs on tiles whose unused columns are still zero
  for (int g = g_end - 1; g >= g_begin; --g) {
    const int d = g * kW16Ch + tid;
    const bool act = d < D;
    float2 A[8];
    float2 A2[8];
    float fac[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int s = j ^ perm;
      float a = 0.0f, fc = 0.0f;
      if (act && s < S) {
        const float e = ex2(p.A_log[(int64_t)d * S + s] * kLog2e);
        const float ec = CLAMP ? fminf(fmaxf(e, 1e-6f), 1.0f) : e;
        a = -ec;
        fc = (CLAMP && (e < 1e-6f || e > 1.0f)) ? 0.0f : -e;
      }
      fac[j] = fc;
      if (j & 1) A[j >> 1].y = a; else A[j >> 1].x = a;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) A2[q] = f2(A[q].x * kLog2e, A[q].y * kLog2e);
    const float Dd = (has_D && act) ? p.Dp[d] : 0.0f;

    // ---- forward sweep: checkpoints (to this SM's L2-resident slot) ------------
    float2 h[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) h[q] = f2(0.0f, 0.0f);
    for (int k = 0; k < (saved ? 0 : nck); ++k, ++it) {
      wait_item(it);
      const T* st = tiles + (size_t)(it & 1) * 4 * TILE + tid;
      const int t0 = k * K, n = min(K, L - t0);
      if (k > 0) {
        float4* c = ckpt + (size_t)(k - 1) * 4 * kW16Threads + tid;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_hint(c + (size_t)q * kW16Threads, make_float4(h[2 * q].x, h[2 * q].y, h[2 * q + 1].x, h[2 * q + 1].y), keep);
      }
#pragma unroll 2
      for (int j = 0; j < n; ++j) {
        const float xv = act ? __bfloat162float(st[(size_t)j * kW16Ch]) : 0.0f;
        float dv = act ? __bfloat162float(st[TILE + (size_t)j * kW16Ch]) : 0.0f;
        if (SOFTPLUS) dv = softplus_f(dv);
        if (CLAMP) dv = fminf(fmaxf(dv, 1e-3f), 1.0f);
        const float2 dtx = f2(dv * xv, dv * xv);
        const float2 dvv2 = f2(dv, dv);
        float2 Bt[8];
        load_bc(sBf, t0 + j, Bt);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float2 ar = __fmul2_rn(dvv2, A2[q]);
          const float2 dA = f2(ex2(ar.x), ex2(ar.y));
          h[q] = __ffma2_rn(dA, h[q], __fmul2_rn(dtx, Bt[q]));
        }
      }
      __syncthreads();
      if (warp == 0) issue(it + 2);
    }

    // ---- reverse sweep --------------------------------------------------------
    float2 gcar[8], gAcc[8], hk[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) { gcar[q] = f2(0.0f, 0.0f); gAcc[q] = f2(0.0f, 0.0f); }
    float dDacc = 0.0f;
    if (nck > 1) {
      load_ck(nck - 1, hk, d);
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) hk[q] = f2(0.0f, 0.0f);
    }
    for (int k = nck - 1; k >= 0; --k, ++it) {
      wait_item(it);
      const T* st = tiles + (size_t)(it & 1) * 4 * TILE + tid;
      const int t0 = k * K, n = min(K, L - t0);
      float* slab = slab0 + (size_t)slab_buf * 8 * K * 32;
      slab_buf ^= 1;
      float2 hs[8], hnext[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) hs[q] = hk[q];
      // fetch the previous chunk's checkpoint while this chunk runs
      if (k > 1) {
        load_ck(k - 1, hnext, d);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) hnext[q] = f2(0.0f, 0.0f);
      }
      // recompute the chunk: the starting state into h slot 0, then h_t (fp32,
      // slot j + 1) and dA_t (f16 pairs) of every step into TMEM
      {
        float hv[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) { hv[2 * q] = hs[q].x; hv[2 * q + 1] = hs[q].y; }
        tmem_st16(tmem, hv);
      }
      auto rstep = [&](const int j) {
        const float xv = __bfloat162float(st[(size_t)j * kW16Ch]);
        float dv = __bfloat162float(st[TILE + (size_t)j * kW16Ch]);
        if (SOFTPLUS) dv = softplus_f(dv);
        if (CLAMP) dv = fminf(fmaxf(dv, 1e-3f), 1.0f);
        const float2 dtx = f2(dv * xv, dv * xv);
        const float2 dvv2 = f2(dv, dv);
        float2 Bt[8];
        load_bc(sBf, t0 + j, Bt);
        float hv[16], dw[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float2 ar = __fmul2_rn(dvv2, A2[q]);
          const float2 ef = f2(ex2(ar.x), ex2(ar.y));
          const __half2 e = __floats2half2_rn(ef.x, ef.y);
          hs[q] = __ffma2_rn(ef, hs[q], __fmul2_rn(dtx, Bt[q]));
          hv[2 * q] = hs[q].x;
          hv[2 * q + 1] = hs[q].y;
          dw[q] = __uint_as_float(h2_bits(e));
        }
        tmem_st16(tmem + (uint32_t)(16 * (j + 1)), hv);
        tmem_st8(tmem + (uint32_t)(kW16DACol + 8 * j), dw);
      };
      // full chunks (all but possibly the last) written out with constant step
      // indices, in the variants where that fits the register file
      constexpr bool kUnrollChunk = SOFTPLUS || (!CLAMP && !HASZ);
      if (kUnrollChunk && n == K) {
#pragma unroll
        for (int j = 0; j < K; ++j) rstep(j);
      } else {
#pragma unroll 2
        for (int j = 0; j < n; ++j) rstep(j);
      }
      tmem_wait_st();

      // reverse walk.  Step j reads h slots j + 1 (h_t) and j (h_{t-1}) and
      // dA_j; three h buffers rotate so that the prefetch of slot j - 1 lands
      // in the buffer step j + 1 finished with, and no registers are copied.
      float H0[16], H1[16], H2[16], Dc[8];
      tmem_ld16_nc(tmem + (uint32_t)(16 * n), H0);
      tmem_ld16_nc(tmem + (uint32_t)(16 * (n - 1)), H1);
      tmem_ld8_nc(tmem + (uint32_t)(kW16DACol + 8 * (n - 1)), Dc);
      tmem_wait_ld_tied16(H0);
      auto step = [&](const int j, float (&Hs)[16], float (&Hp)[16], float (&Hn)[16]) {
        const int t = t0 + j;
        tmem_wait_ld_tied(Hp, Dc);
        float2 dA[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) dA[q] = __half22float2(bits_h2(__float_as_uint(Dc[q])));
        {  // prefetch for step j - 1 (at j = 0 a harmless reload of slot 0)
          const int jn = j > 0 ? j - 1 : 0;
          tmem_ld8_nc(tmem + (uint32_t)(kW16DACol + 8 * jn), Dc);
          tmem_ld16_nc(tmem + (uint32_t)(16 * jn), Hn);
        }
        // tile columns past the group's channels stay zero, so an inactive
        // lane computes zeros without selects (its stores are skipped)
        const float xv = __bfloat162float(st[(size_t)j * kW16Ch]);
        const float draw = __bfloat162float(st[TILE + (size_t)j * kW16Ch]);
        float gy = __bfloat162float(st[2 * TILE + (size_t)j * kW16Ch]);
        // dv = clamp(softplus(raw)); mdt = d dv / d raw
        float dv = draw, mdt = 1.0f;
        if (SOFTPLUS) {
          dv = softplus_f(draw);
          mdt = sigmoid(draw);
        }
        if (CLAMP) {
          mdt = (dv >= 1e-3f && dv <= 1.0f) ? mdt : 0.0f;
          dv = fminf(fmaxf(dv, 1e-3f), 1.0f);
        }
        const float dtxs = dv * xv;
        float2 Bt[8], Ct[8];
        load_bc(sBf, t, Bt);
        load_bc(sCf, t, Ct);
        float dzv = 0.0f;
        if constexpr (HASZ) {
          const float zv = __bfloat162float(st[3 * TILE + (size_t)j * kW16Ch]);
          float2 ys2 = f2(0.0f, 0.0f);
#pragma unroll
          for (int q = 0; q < 8; ++q) ys2 = __ffma2_rn(f2(Hs[2 * q], Hs[2 * q + 1]), Ct[q], ys2);
          const float ys = fmaf(Dd, xv, ys2.x + ys2.y);
          const float sg = sigmoid(zv);
          dzv = gy * ys * sg * (1.0f + zv * (1.0f - sg));
          gy = gy * zv * sg;
        }
        const float2 gyy = f2(gy, gy), dtx = f2(dtxs, dtxs), dvv = f2(dv, dv);
        float2 gB = f2(0.0f, 0.0f), ddA = f2(0.0f, 0.0f);
        float2 vB[8], vC[8];  // dB and dC partials per state pair slot
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float2 hp = f2(Hp[2 * q], Hp[2 * q + 1]);
          const float2 gs = __ffma2_rn(gyy, Ct[q], gcar[q]);
          gB = __ffma2_rn(gs, Bt[q], gB);
          vB[q] = __fmul2_rn(gs, dtx);
          vC[q] = __fmul2_rn(gyy, f2(Hs[2 * q], Hs[2 * q + 1]));
          const float2 w = __fmul2_rn(dA[q], gs);
          const float2 R = __fmul2_rn(w, hp);
          ddA = __ffma2_rn(A[q], R, ddA);
          gAcc[q] = __ffma2_rn(dvv, R, gAcc[q]);
          gcar[q] = w;
        }
        dDacc = fmaf(gy, xv, dDacc);
        {
          const int64_t gi = (b * L + t) * (int64_t)D + d;
          const float gBs = gB.x + gB.y;
          st_bf16_if(static_cast<T*>(p.dx) + gi, fmaf(dv, gBs, Dd * gy), act);
          st_bf16_if(static_cast<T*>(p.ddt) + gi, fmaf(xv, gBs, ddA.x + ddA.y) * mdt, act);
          if constexpr (HASZ) st_bf16_if(static_cast<T*>(p.dz) + gi, dzv, act);
        }
        // reduce dB and dC over the warp's 32 channels.  Pair slot q holds
        // state pair q ^ pq (pq = lane bits 3, 2): the levels across lane bits
        // 3 and 2 keep slots [0, n/2) without selects; lane bits 1, 0 and 4
        // then pick the pair, the element and dB / dC, so that lane l ends
        // with column l of the slab row (dB of state l for l < 16, else dC of
        // state l - 16)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          vB[i] = __fadd2_rn(vB[i], shfl2(vB[i + 4], 8));
          vC[i] = __fadd2_rn(vC[i], shfl2(vC[i + 4], 8));
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          vB[i] = __fadd2_rn(vB[i], shfl2(vB[i + 2], 4));
          vC[i] = __fadd2_rn(vC[i], shfl2(vC[i + 2], 4));
        }
        {
          const bool up = (lane & 2) != 0;
          const float2 sb = up ? vB[0] : vB[1], kb = up ? vB[1] : vB[0];
          const float2 sc = up ? vC[0] : vC[1], kc = up ? vC[1] : vC[0];
          vB[0] = __fadd2_rn(kb, shfl2(sb, 2));
          vC[0] = __fadd2_rn(kc, shfl2(sc, 2));
        }
        float rB, rC;
        {
          const bool up = (lane & 1) != 0;
          const float sb = up ? vB[0].x : vB[0].y, kb = up ? vB[0].y : vB[0].x;
          const float sc = up ? vC[0].x : vC[0].y, kc = up ? vC[0].y : vC[0].x;
          rB = kb + __shfl_xor_sync(0xffffffffu, sb, 1);
          rC = kc + __shfl_xor_sync(0xffffffffu, sc, 1);
        }
        float r;
        {
          const bool up = (lane & 16) != 0;
          r = (up ? rC : rB) + __shfl_xor_sync(0xffffffffu, up ? rB : rC, 16);
        }
        slab[((size_t)warp * K + j) * 32 + lane] = r;
      };
      static_assert(K == 10, "the full-chunk walk below is written out for 10 steps");
      if (kUnrollChunk && n == K) {
        step(9, H0, H1, H2);
        step(8, H1, H2, H0);
        step(7, H2, H0, H1);
        step(6, H0, H1, H2);
        step(5, H1, H2, H0);
        step(4, H2, H0, H1);
        step(3, H0, H1, H2);
        step(2, H1, H2, H0);
        step(1, H2, H0, H1);
        step(0, H0, H1, H2);
      } else {  // blocks of three steps without branches between them, then the rest
        int j = n - 1;
        for (; j >= 2; j -= 3) {
          step(j, H0, H1, H2);
          step(j - 1, H1, H2, H0);
          step(j - 2, H2, H0, H1);
        }
        if (j >= 0) {
          step(j, H0, H1, H2);
          if (j >= 1) step(j - 1, H1, H2, H0);
        }
      }
      __syncthreads();
      {
        const bool first = (g == g_end - 1);
        for (int e = tid; e < n * 32; e += kW16Threads) {
          const int j = e >> 5, vv = e & 31;
          float acc = 0.0f;
#pragma unroll
          for (int w8 = 0; w8 < 8; ++w8) acc += slab[((size_t)w8 * K + j) * 32 + vv];
          float* dst = dbc + (size_t)t0 * 32 + e;
          *dst = first ? acc : *dst + acc;
        }
      }
      // no barrier here: the next chunk writes the other slab buffer, and the
      // barrier that ends it orders these folds before this buffer is reused
      if (warp == 0) issue(it + 2);
#pragma unroll
      for (int q = 0; q < 8; ++q) hk[q] = hnext[q];
    }
    if (act) {
      float* da = p.dAlog_part + (b * D + d) * (int64_t)S;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int s = j ^ perm;
        const float gv = (j & 1) ? gAcc[j >> 1].y : gAcc[j >> 1].x;
        if (s < S) da[s] = gv * fac[j];
      }
      if (has_D) p.dD_part[b * D + d] = dDacc;
    }
  }
  __syncthreads();
  // this sequence's dB | dC rows
  {
    float4* dst = reinterpret_cast<float4*>(p.dBC_ws + ((int64_t)split * p.nseq + b) * L * 32);
    const float4* src = reinterpret_cast<const float4*>(dbc);
    for (int e = tid; e < L * 8; e += kW16Threads) dst[e] = src[e];
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(s_tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// out[c] = sum_r part[r][c] over `rows` rows, deterministic (fixed order).
// Stage 1 sums row blocks of `rb` rows into part2[blk][c].
__global__ void colsum_stage1(const float* __restrict__ part, float* __restrict__ part2, int64_t rows,
                              int64_t cols, int64_t rb) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t blk = blockIdx.y;
  if (c >= cols) return;
  const int64_t r0 = blk * rb, r1 = min(rows, r0 + rb);
  float acc = 0.0f;
  for (int64_t r = r0; r < r1; ++r) acc += part[r * cols + c];
  part2[blk * cols + c] = acc;
}
__global__ void colsum_stage2(const float* __restrict__ part2, float* __restrict__ out, int64_t nblk,
                              int64_t cols) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float acc = 0.0f;
  for (int64_t r = 0; r < nblk; ++r) acc += part2[r * cols + c];
  out[c] = acc;
}

// dB/dC: sum the splits' fp32 accumulators and write the output dtype.
template <typename T>
__global__ void dbc_finalize(const float* __restrict__ ws, T* __restrict__ dB, T* __restrict__ dC,
                             int64_t nseq, int L, int S, int SP, int nsplit) {
  // workspace rows hold 2*SP values per timestep: dB in [0, SP), dC in [SP, 2*SP)
  const int64_t total = nseq * L * S;
  const int NV = 2 * SP;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / S;
    const int s = (int)(i % S);
    float vb = 0.0f, vc = 0.0f;
    for (int q = 0; q < nsplit; ++q) {
      const float* r = ws + ((int64_t)q * nseq * L + row) * NV;
      vb += r[s];
      vc += r[SP + s];
    }
    io<T>::st(dB + i, vb);
    io<T>::st(dC + i, vc);
  }
}

}  // namespace scan
}  // namespace hclsm

// ===========================================================================
// host side
// ===========================================================================
namespace hclsm {
int* device_err_ptr();
int num_sms();
bool set_smem_limit(const void* fn, size_t bytes);
}  // namespace hclsm

namespace hclsm {
namespace scan {

static int pad_state(int S) {
  if (S <= 4) return 4;
  if (S <= 8) return 8;
  if (S <= 16) return 16;
  if (S <= 32) return 32;
  if (S <= 64) return 64;
  return 0;
}

template <typename T, int SP, int CPT, bool CLAMP>
static int launch_fwd_t(FwdParams p, cudaStream_t st) {
  const int per_cta = kFwdThreads * CPT;
  const int gx = (p.D + per_cta - 1) / per_cta;
  const int64_t total = p.nseq;
  // grid.y is limited to 65535: launch sequence batches
  for (int64_t s0 = 0; s0 < total; s0 += 65535) {
    const int64_t ns = std::min<int64_t>(65535, total - s0);
    FwdParams q = p;
    const int64_t off = s0 * (int64_t)p.L * p.D, offs = s0 * (int64_t)p.L * p.S;
    q.x = static_cast<const T*>(p.x) + off;
    q.dt = static_cast<const T*>(p.dt) + off;
    q.z = p.z ? static_cast<const T*>(p.z) + off : nullptr;
    q.y = static_cast<T*>(p.y) + off;
    q.B = static_cast<const T*>(p.B) + offs;
    q.C = static_cast<const T*>(p.C) + offs;
    q.nseq = ns;
    scan_fwd_kernel<T, SP, CPT, CLAMP><<<dim3(gx, (unsigned)ns), kFwdThreads, 0, st>>>(q);
  }
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

template <int SP, bool CLAMP>
static int launch_fwd_bf16x2(FwdParams p, cudaStream_t st) {
  const int per_cta = kFwdThreads * 2;
  const int gx = (p.D + per_cta - 1) / per_cta;
  for (int64_t s0 = 0; s0 < p.nseq; s0 += 65535) {
    const int64_t ns = std::min<int64_t>(65535, p.nseq - s0);
    FwdParams q = p;
    const int64_t off = s0 * (int64_t)p.L * p.D, offs = s0 * (int64_t)p.L * p.S;
    using T = __nv_bfloat16;
    q.x = static_cast<const T*>(p.x) + off;
    q.dt = static_cast<const T*>(p.dt) + off;
    q.z = p.z ? static_cast<const T*>(p.z) + off : nullptr;
    q.y = static_cast<T*>(p.y) + off;
    q.B = static_cast<const T*>(p.B) + offs;
    q.C = static_cast<const T*>(p.C) + offs;
    if (p.states) q.states = p.states + s0 * (int64_t)((p.L + kStateEvery - 1) / kStateEvery - 1) * p.D * 16;
    q.nseq = ns;
    scan_fwd_bf16x2_kernel<SP, CLAMP><<<dim3(gx, (unsigned)ns), kFwdThreads, 0, st>>>(q);
  }
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

template <typename T, int SP>
static int launch_fwd_sp(const FwdParams& p, bool pairs, bool clamp, cudaStream_t st) {
  if constexpr (SP <= 16 && sizeof(T) == 2) {
    if (pairs) return clamp ? launch_fwd_bf16x2<SP, true>(p, st) : launch_fwd_bf16x2<SP, false>(p, st);
  }
  if constexpr (SP <= 16) {
    if (pairs) return clamp ? launch_fwd_t<T, SP, 2, true>(p, st) : launch_fwd_t<T, SP, 2, false>(p, st);
  }
  return clamp ? launch_fwd_t<T, SP, 1, true>(p, st) : launch_fwd_t<T, SP, 1, false>(p, st);
}

template <typename T>
static int launch_fwd(const FwdParams& p, bool clamp, cudaStream_t st) {
  const size_t pair_bytes = 2 * sizeof(T);
  auto al = [&](const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) % pair_bytes) == 0; };
  const bool pairs = (p.D % 2 == 0) && al(p.x) && al(p.dt) && al(p.z) && al(p.y);
  switch (pad_state(p.S)) {
    case 4: return launch_fwd_sp<T, 4>(p, pairs, clamp, st);
    case 8: return launch_fwd_sp<T, 8>(p, pairs, clamp, st);
    case 16: return launch_fwd_sp<T, 16>(p, pairs, clamp, st);
    case 32: return launch_fwd_sp<T, 32>(p, pairs, clamp, st);
    case 64: return launch_fwd_sp<T, 64>(p, pairs, clamp, st);
  }
  return HCLSM_ERR_SHAPE;
}

// ---- backward plan -----------------------------------------------------------
struct BwdPlan {
  int SP, K, nck, groups, nsplit, gpc, nck16, slots;
  int64_t nblk, rb;
  size_t off_dalog, off_dd, off_p2a, off_p2d, off_dbc, off_ck, total;
};

static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

static int bwd_K(int SP) { return std::min(32, 256 / SP); }

static bool plan_bwd(int64_t nseq, int L, int D, int S, BwdPlan* pl) {
  const int SP = pad_state(S);
  if (SP == 0 || nseq <= 0 || L <= 0 || D <= 0) return false;
  pl->SP = SP;
  pl->K = bwd_K(SP);
  pl->nck = (L + pl->K - 1) / pl->K;
  pl->groups = (D + 127) / 128;
  const int nsm = num_sms();
  // choose the channel split that minimises waves x work per CTA; keep the
  // smallest split within 3 % of the best
  double best = 1e30;
  std::vector<std::pair<int, double>> cand;
  for (int q = 1; q <= pl->groups; ++q) {
    const int gpc = (pl->groups + q - 1) / q;
    const int eff = (pl->groups + gpc - 1) / gpc;
    const double waves = std::ceil((double)nseq * eff / nsm);
    const double cost = waves * gpc;
    cand.push_back({eff, cost});
    best = std::min(best, cost);
  }
  pl->nsplit = pl->groups;
  for (auto& c : cand) {
    if (c.second <= best * 1.03) { pl->nsplit = c.first; break; }
  }
  pl->gpc = (pl->groups + pl->nsplit - 1) / pl->nsplit;
  pl->nsplit = (pl->groups + pl->gpc - 1) / pl->gpc;
  pl->nblk = std::min<int64_t>(nseq, 128);
  pl->rb = (nseq + pl->nblk - 1) / pl->nblk;
  pl->nblk = (nseq + pl->rb - 1) / pl->rb;
  size_t off = 0;
  pl->off_dalog = off; off = align256(off + sizeof(float) * (size_t)nseq * D * S);
  pl->off_dd = off;    off = align256(off + sizeof(float) * (size_t)nseq * D);
  pl->off_p2a = off;   off = align256(off + sizeof(float) * (size_t)pl->nblk * D * S);
  pl->off_p2d = off;   off = align256(off + sizeof(float) * (size_t)pl->nblk * D);
  pl->off_dbc = off;   off = align256(off + sizeof(float) * (size_t)pl->nsplit * nseq * L * 2 * SP);
  // checkpoint slots, one per SM: the packed bf16 kernel (d_state 9..16) or
  // the generic kernel, whichever needs more
  pl->nck16 = (L + kW16K - 1) / kW16K;
  pl->slots = std::min(nsm, kW16MaxSlots);
  const size_t per_slot =
      std::max(SP == 16 ? w16_slot_floats(pl->nck16) : (size_t)0, gen_slot_floats(pl->nck, SP));
  pl->off_ck = off;    off = align256(off + sizeof(float) * (size_t)pl->slots * per_slot);
  pl->total = off;
  return true;
}

template <typename T, int SP, bool CLAMP>
static int launch_bwd_t(const BwdParams& p, const BwdPlan& pl, cudaStream_t st) {
  const size_t smem = BwdSmem<T, SP>::total();
  if (smem > 227 * 1024) return HCLSM_ERR_UNSUPPORTED;
  auto fn = scan_bwd_kernel<T, SP, CLAMP>;
  if (!set_smem_limit(reinterpret_cast<const void*>(fn), smem)) return HCLSM_ERR_LAUNCH;
  fn<<<dim3((unsigned)p.nseq, pl.nsplit), kBwdThreads, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

template <bool CLAMP, bool SOFTPLUS, bool HASZ>
static int launch_bwd_bf16(const BwdParams& p, const BwdPlan& pl, cudaStream_t st) {
  const size_t smem = W16Smem::total(p.L);
  if (smem > 227 * 1024) return HCLSM_ERR_UNSUPPORTED;
  BwdParams q = p;
  q.nck = pl.nck16;
  q.groups = (p.D + kW16Ch - 1) / kW16Ch;
  // the channel split of the plan counts 128-channel groups; keep its CTA count
  q.groups_per_cta = (q.groups + pl.nsplit - 1) / pl.nsplit;
  auto fn = scan_bwd_bf16_kernel<CLAMP, SOFTPLUS, HASZ>;
  if (!set_smem_limit(reinterpret_cast<const void*>(fn), smem)) return HCLSM_ERR_LAUNCH;
  fn<<<dim3((unsigned)p.nseq, pl.nsplit), kW16Threads, smem, st>>>(q);
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

template <typename T>
static int launch_bwd(const BwdParams& p, const BwdPlan& pl, bool clamp, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    // the packed kernel keeps B, C and dB|dC of the whole sequence in shared
    // memory; longer sequences take the generic kernel
    if (pl.SP == 16 && W16Smem::total(p.L) <= 227 * 1024) {
      if (p.z) {
        if (p.softplus)
          return clamp ? launch_bwd_bf16<true, true, true>(p, pl, st) : launch_bwd_bf16<false, true, true>(p, pl, st);
        return clamp ? launch_bwd_bf16<true, false, true>(p, pl, st) : launch_bwd_bf16<false, false, true>(p, pl, st);
      }
      if (p.softplus)
        return clamp ? launch_bwd_bf16<true, true, false>(p, pl, st) : launch_bwd_bf16<false, true, false>(p, pl, st);
      return clamp ? launch_bwd_bf16<true, false, false>(p, pl, st)
                   : launch_bwd_bf16<false, false, false>(p, pl, st);
    }
  }
  if (p.states) return HCLSM_ERR_UNSUPPORTED;  // only the packed kernel reads snapshots
  switch (pl.SP) {
    case 4: return clamp ? launch_bwd_t<T, 4, true>(p, pl, st) : launch_bwd_t<T, 4, false>(p, pl, st);
    case 8: return clamp ? launch_bwd_t<T, 8, true>(p, pl, st) : launch_bwd_t<T, 8, false>(p, pl, st);
    case 16: return clamp ? launch_bwd_t<T, 16, true>(p, pl, st) : launch_bwd_t<T, 16, false>(p, pl, st);
    case 32: return clamp ? launch_bwd_t<T, 32, true>(p, pl, st) : launch_bwd_t<T, 32, false>(p, pl, st);
    case 64: return clamp ? launch_bwd_t<T, 64, true>(p, pl, st) : launch_bwd_t<T, 64, false>(p, pl, st);
  }
  return HCLSM_ERR_SHAPE;
}

}  // namespace scan
}  // namespace hclsm

using namespace hclsm;
using namespace hclsm::scan;

static bool aligned16(const void* q) { return q == nullptr || reinterpret_cast<uintptr_t>(q) % 16 == 0; }

extern "C" int hclsm_ssm_scan_fwd(const void* x, const void* dt, const float* A_log, const void* B,
                                  const void* C, const float* D, const void* z, void* y, int64_t nseq,
                                  int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype, int32_t clamp,
                                  void* stream) {
  if (!x || !dt || !A_log || !B || !C || !y) return HCLSM_ERR_NULL;
  if (nseq < 0 || L < 0 || d_inner < 0 || d_state <= 0 || d_state > 64) return HCLSM_ERR_SHAPE;
  if (nseq == 0 || L == 0 || d_inner == 0) return HCLSM_OK;
  if (clamp & ~(HCLSM_SCAN_CLAMP | HCLSM_SCAN_DT_SOFTPLUS)) return HCLSM_ERR_SHAPE;
  FwdParams p{x, dt, A_log, B, C, D, z, y, nseq, L, d_inner, d_state, nullptr,
              (clamp & HCLSM_SCAN_DT_SOFTPLUS) ? 1 : 0};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool cl = (clamp & HCLSM_SCAN_CLAMP) != 0;
  if (dtype == HCLSM_F32) return launch_fwd<float>(p, cl, st);
  if (dtype == HCLSM_BF16) return launch_fwd<__nv_bfloat16>(p, cl, st);
  return HCLSM_ERR_DTYPE;
}

extern "C" size_t hclsm_ssm_scan_bwd_workspace_size(int64_t nseq, int32_t L, int32_t d_inner,
                                                    int32_t d_state) {
  BwdPlan pl;
  if (!plan_bwd(nseq, L, d_inner, d_state, &pl)) return 0;
  return pl.total;
}

// the forward's state snapshots apply where both the bf16 pair forward and the
// packed backward run: bf16, 9 <= d_state <= 16, even d_inner, B/C/dB|dC of a
// sequence within shared memory
static bool states_supported(int64_t nseq, int L, int D, int S, int dtype) {
  return dtype == HCLSM_BF16 && nseq > 0 && L > 0 && D > 0 && D % 2 == 0 && pad_state(S) == 16 &&
         W16Smem::total(L) <= 227 * 1024;
}
static size_t states_bytes_for(int64_t nseq, int L, int D) {
  const int64_t nsnap = (L + kStateEvery - 1) / kStateEvery - 1;
  return std::max<size_t>(16, sizeof(float) * (size_t)nseq * nsnap * D * 16);
}

static int scan_bwd_impl(const void* x, const void* dt, const float* A_log, const void* B, const void* C,
                         const float* D, const void* z, const void* dy, void* dx, void* ddt, float* dA_log,
                         void* dB, void* dC, float* dD, void* dz, int64_t nseq, int32_t L, int32_t d_inner,
                         int32_t d_state, int32_t dtype, int32_t clamp, const float* states, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (!x || !dt || !A_log || !B || !C || !dy || !dx || !ddt || !dA_log || !dB || !dC) return HCLSM_ERR_NULL;
  if (D && !dD) return HCLSM_ERR_NULL;
  if (z && !dz) return HCLSM_ERR_NULL;
  if (nseq < 0 || L < 0 || d_inner <= 0 || d_state <= 0) return HCLSM_ERR_SHAPE;
  if (dtype != HCLSM_F32 && dtype != HCLSM_BF16) return HCLSM_ERR_DTYPE;
  if (clamp & ~(HCLSM_SCAN_CLAMP | HCLSM_SCAN_DT_SOFTPLUS)) return HCLSM_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (nseq == 0 || L == 0) {
    cudaMemsetAsync(dA_log, 0, sizeof(float) * (size_t)d_inner * d_state, st);
    if (D) cudaMemsetAsync(dD, 0, sizeof(float) * (size_t)d_inner, st);
    return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
  }
  BwdPlan pl;
  if (!plan_bwd(nseq, L, d_inner, d_state, &pl)) return HCLSM_ERR_UNSUPPORTED;
  if (nseq > 2147483647LL) return HCLSM_ERR_SHAPE;
  const size_t esz = dtype == HCLSM_F32 ? 4 : 2;
  // rows of x/dt/dy/z are fetched by 16-byte bulk copies
  if ((d_inner * esz) % 16 != 0) return HCLSM_ERR_UNSUPPORTED;
  if (!aligned16(x) || !aligned16(dt) || !aligned16(dy) || !aligned16(z)) return HCLSM_ERR_ALIGN;
  if (!workspace || workspace_bytes < pl.total) return HCLSM_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return HCLSM_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  BwdParams p;
  p.x = x; p.dt = dt; p.A_log = A_log; p.B = B; p.C = C; p.Dp = D; p.z = z; p.dy = dy;
  p.dx = dx; p.ddt = ddt; p.dz = dz;
  p.dAlog_part = reinterpret_cast<float*>(ws + pl.off_dalog);
  p.dD_part = reinterpret_cast<float*>(ws + pl.off_dd);
  p.dBC_ws = reinterpret_cast<float*>(ws + pl.off_dbc);
  p.nseq = nseq; p.L = L; p.D = d_inner; p.S = d_state;
  p.nck = pl.nck; p.groups = pl.groups; p.groups_per_cta = pl.gpc; p.nsplit = pl.nsplit;
  p.ckpt_ws = reinterpret_cast<float*>(ws + pl.off_ck);
  p.ckpt_slots = pl.slots;
  p.states = states;
  p.softplus = (clamp & HCLSM_SCAN_DT_SOFTPLUS) ? 1 : 0;
  p.err = device_err_ptr();
  const bool cl = (clamp & HCLSM_SCAN_CLAMP) != 0;
  int rc = dtype == HCLSM_F32 ? launch_bwd<float>(p, pl, cl, st) : launch_bwd<__nv_bfloat16>(p, pl, cl, st);
  if (rc != HCLSM_OK) return rc;
  // dA_log and dD: deterministic column sums over sequences
  {
    const int64_t cols = (int64_t)d_inner * d_state;
    float* p2 = reinterpret_cast<float*>(ws + pl.off_p2a);
    colsum_stage1<<<dim3((unsigned)((cols + 255) / 256), (unsigned)pl.nblk), 256, 0, st>>>(
        p.dAlog_part, p2, nseq, cols, pl.rb);
    colsum_stage2<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(p2, dA_log, pl.nblk, cols);
  }
  if (D) {
    const int64_t cols = d_inner;
    float* p2 = reinterpret_cast<float*>(ws + pl.off_p2d);
    colsum_stage1<<<dim3((unsigned)((cols + 255) / 256), (unsigned)pl.nblk), 256, 0, st>>>(
        p.dD_part, p2, nseq, cols, pl.rb);
    colsum_stage2<<<(unsigned)((cols + 255) / 256), 256, 0, st>>>(p2, dD, pl.nblk, cols);
  }
  {
    const int64_t total = nseq * (int64_t)L * d_state;
    const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
    if (dtype == HCLSM_F32)
      dbc_finalize<float><<<blocks, 256, 0, st>>>(p.dBC_ws, static_cast<float*>(dB), static_cast<float*>(dC),
                                                  nseq, L, d_state, pl.SP, pl.nsplit);
    else
      dbc_finalize<__nv_bfloat16><<<blocks, 256, 0, st>>>(p.dBC_ws, static_cast<__nv_bfloat16*>(dB),
                                                          static_cast<__nv_bfloat16*>(dC), nseq, L, d_state,
                                                          pl.SP, pl.nsplit);
  }
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}

extern "C" int hclsm_ssm_scan_bwd(const void* x, const void* dt, const float* A_log, const void* B,
                                  const void* C, const float* D, const void* z, const void* dy, void* dx,
                                  void* ddt, float* dA_log, void* dB, void* dC, float* dD, void* dz,
                                  int64_t nseq, int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype,
                                  int32_t clamp, void* workspace, size_t workspace_bytes, void* stream) {
  return scan_bwd_impl(x, dt, A_log, B, C, D, z, dy, dx, ddt, dA_log, dB, dC, dD, dz, nseq, L, d_inner, d_state,
                       dtype, clamp, nullptr, workspace, workspace_bytes, stream);
}

extern "C" size_t hclsm_ssm_scan_states_size(int64_t nseq, int32_t L, int32_t d_inner, int32_t d_state,
                                             int32_t dtype) {
  if (!states_supported(nseq, L, d_inner, d_state, dtype)) return 0;
  return states_bytes_for(nseq, L, d_inner);
}

extern "C" int hclsm_ssm_scan_fwd_states(const void* x, const void* dt, const float* A_log, const void* B,
                                         const void* C, const float* D, const void* z, void* y, int64_t nseq,
                                         int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype,
                                         int32_t clamp, float* states, size_t states_bytes, void* stream) {
  if (!x || !dt || !A_log || !B || !C || !y || !states) return HCLSM_ERR_NULL;
  if (nseq < 0 || L < 0 || d_inner < 0 || d_state <= 0 || d_state > 64) return HCLSM_ERR_SHAPE;
  if (nseq == 0 || L == 0 || d_inner == 0) return HCLSM_OK;
  if (!states_supported(nseq, L, d_inner, d_state, dtype)) return HCLSM_ERR_UNSUPPORTED;
  if (states_bytes < states_bytes_for(nseq, L, d_inner)) return HCLSM_ERR_WORKSPACE;
  auto al4 = [](const void* q) { return q == nullptr || reinterpret_cast<uintptr_t>(q) % 4 == 0; };
  if (!al4(x) || !al4(dt) || !al4(z) || !al4(y) || !aligned16(states)) return HCLSM_ERR_ALIGN;
  if (clamp & ~(HCLSM_SCAN_CLAMP | HCLSM_SCAN_DT_SOFTPLUS)) return HCLSM_ERR_SHAPE;
  FwdParams p{x, dt, A_log, B, C, D, z, y, nseq, L, d_inner, d_state, states,
              (clamp & HCLSM_SCAN_DT_SOFTPLUS) ? 1 : 0};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return (clamp & HCLSM_SCAN_CLAMP) ? launch_fwd_bf16x2<16, true>(p, st) : launch_fwd_bf16x2<16, false>(p, st);
}

extern "C" int hclsm_ssm_scan_bwd_states(const void* x, const void* dt, const float* A_log, const void* B,
                                         const void* C, const float* D, const void* z, const void* dy, void* dx,
                                         void* ddt, float* dA_log, void* dB, void* dC, float* dD, void* dz,
                                         int64_t nseq, int32_t L, int32_t d_inner, int32_t d_state,
                                         int32_t dtype, int32_t clamp, const float* states, size_t states_bytes,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  if (!states) return HCLSM_ERR_NULL;
  if (nseq > 0 && L > 0) {
    if (!states_supported(nseq, L, d_inner, d_state, dtype)) return HCLSM_ERR_UNSUPPORTED;
    if (states_bytes < states_bytes_for(nseq, L, d_inner)) return HCLSM_ERR_WORKSPACE;
    if (!aligned16(states)) return HCLSM_ERR_ALIGN;
  }
  return scan_bwd_impl(x, dt, A_log, B, C, D, z, dy, dx, ddt, dA_log, dB, dC, dD, dz, nseq, L, d_inner, d_state,
                       dtype, clamp, states, workspace, workspace_bytes, stream);
}
