// Per-frame multi-head self-attention of the Level-1 event transformer on the
// 5th-generation tensor cores (nn.MultiheadAttention(bias=False) inside
// EventTransformerBlock, hclsm/dynamics/level1_event.py:33-54), for bf16,
// head dim 64 and T in {16, 32, 64} tokens per frame.
//
// One CTA (128 threads, thread i <-> row i <-> TMEM lane i) takes 128 rows of
// the packed q|k|v matrix, i.e. 128 / T whole frames, for one head:
//   TMA (2-D tensor map, 128-byte swizzle) brings Q, K and V [128 x 64];
//   MMA 1: S [128 rows x 128 keys] = Q K^T, fp32 in TMEM; attention stays
//          inside a frame, so warp w needs only the key columns of its frames,
//          which one 32x32b TMEM load returns;
//   each thread takes the softmax over its frame's keys (key padding ignored),
//   writes its row of P (bf16, zero outside its frame's keys) as the K-major A
//   operand of MMA 2;
//   MMA 2: O [128 x 64] = P V (V as an MN-major operand), fp32 in TMEM;
//   each thread scales its row by 1 / sum and stores it (a frame whose keys
//   are all ignored yields NaN, as torch's attention does).
// One thread issues the MMAs; completion arrives on mbarriers through
// tcgen05.commit.  Every wait is bounded (HCLSM_ERR_TIMEOUT).
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace hclsm {
int* device_err_ptr();
bool set_smem_limit(const void* fn, size_t bytes);
}  // namespace hclsm

namespace hclsm {
namespace evtc {

using namespace ::hclsm::tc;

constexpr int kThreads = 128;
constexpr int kRows = 128;
constexpr int kHD = 64;
constexpr uint32_t kTile = kRows * kHD * 2;  // 16 KB: one [128 x 64] bf16 tile
// Q, K, V tiles, P [2 atoms of 64 keys][128 rows][128 B], barriers
constexpr size_t kSmem = 5 * (size_t)kTile + 64 + 1024;

struct Params {
  int R, T, E;
  float scale;
  const uint8_t* kp;  // (R / T, T) or null: non-zero = ignored key
  __nv_bfloat16* out; // (R, E)
  int* err;
};

template <int T>
__global__ void __launch_bounds__(kThreads) mha_tc_kernel(const __grid_constant__ CUtensorMap mqkv, Params p) {
  constexpr int LW = T >= 32 ? T : 32;  // key columns one warp loads
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sQ = smem;
  unsigned char* sK = sQ + kTile;
  unsigned char* sV = sK + kTile;
  unsigned char* sP = sV + kTile;  // two 16 KB atoms
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kTile);  // 0: loads, 1: MMA 1, 2: MMA 2
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = blockIdx.x * kRows, h = blockIdx.y;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 32) {
    s_abort = 0;
    for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  if (tid == 0) asm volatile("prefetch.tensormap [%0];" ::"l"(&mqkv) : "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = s_tmem;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  auto wait = [&](int b) {
    if (!s_abort && !mbar_wait(&bars[b], 0)) {
      record_error(p.err, HCLSM_ERR_TIMEOUT);
      s_abort = 1;
    }
  };

  if (tid == 0) {
    mbar_expect_tx(&bars[0], 3 * kTile);
    tma_load_2d(sQ, &mqkv, h * kHD, row0, &bars[0]);
    tma_load_2d(sK, &mqkv, p.E + h * kHD, row0, &bars[0]);
    tma_load_2d(sV, &mqkv, 2 * p.E + h * kHD, row0, &bars[0]);
  }
  wait(0);
  // ---- MMA 1: S = Q K^T ------------------------------------------------------------------
  if (tid == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t id1 = idesc_bf16(kRows, kRows, false, false);
#pragma unroll
    for (int ks = 0; ks < kHD / 16; ++ks)
      umma_bf16(tmem, smem_desc_sw128(smem_u32(sQ) + ks * 32, 16, 1024),
                smem_desc_sw128(smem_u32(sK) + ks * 32, 16, 1024), id1, ks != 0);
    umma_commit(&bars[1]);
  }
  wait(1);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

  // ---- softmax over this row's frame's keys -------------------------------------------
  const int fr = tid / T;                 // frame within the tile
  const int grow = row0 + tid;
  const bool rv = grow < p.R;
  const int col0 = T >= 32 ? (warp * 32 / T) * T : warp * 32;
  const bool hi = T == 16 && (lane >> 4) != 0;  // T = 16: lanes 16-31 hold the second frame's keys
  float s[LW];
#pragma unroll
  for (int c = 0; c < LW; c += 32) {
    float v[32];
    tmem_ld32(tmem + lane_base + (uint32_t)(col0 + c), v);
#pragma unroll
    for (int i = 0; i < 32; ++i) s[c + i] = v[i];
  }
  float ev[T];
  float mx = -INFINITY;
  const uint8_t* kp = (p.kp && rv) ? p.kp + (size_t)(grow / T) * T : nullptr;
#pragma unroll
  for (int j = 0; j < T; ++j) {
    const bool ok = rv && !(kp && kp[j]);
    const float raw = (T == 16) ? (hi ? s[(16 + j) % LW] : s[j]) : s[j];
    const float v = ok ? raw * p.scale : -INFINITY;
    ev[j] = v;
    mx = fmaxf(mx, v);
  }
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < T; ++j) {
    const float e = (mx == -INFINITY) ? 0.0f : ex2((ev[j] - mx) * kLog2e);
    ev[j] = e;
    sum += e;
  }
  const float inv = 1.0f / sum;  // all keys ignored: 1/0, the row becomes NaN below
  // P row: keys [fr T, fr T + T) carry the weights, every other key is 0.  In a
  // 64-key atom, row r's 16-byte chunk c (8 keys) sits at chunk c ^ (r & 7).
  {
    const int c_lo = fr * T / 8;
#pragma unroll
    for (int jc = 0; jc < T / 8; ++jc) {
      const int cg = c_lo + jc;
      uint4 w;
      __nv_bfloat162 a0 = __floats2bfloat162_rn(ev[8 * jc + 0], ev[8 * jc + 1]);
      __nv_bfloat162 a1 = __floats2bfloat162_rn(ev[8 * jc + 2], ev[8 * jc + 3]);
      __nv_bfloat162 a2 = __floats2bfloat162_rn(ev[8 * jc + 4], ev[8 * jc + 5]);
      __nv_bfloat162 a3 = __floats2bfloat162_rn(ev[8 * jc + 6], ev[8 * jc + 7]);
      w.x = *reinterpret_cast<uint32_t*>(&a0);
      w.y = *reinterpret_cast<uint32_t*>(&a1);
      w.z = *reinterpret_cast<uint32_t*>(&a2);
      w.w = *reinterpret_cast<uint32_t*>(&a3);
      *reinterpret_cast<uint4*>(sP + (cg >> 3) * kTile + tid * 128 + (((cg & 7) ^ (tid & 7)) << 4)) = w;
    }
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int cg = 0; cg < 16; ++cg)
      if (cg < c_lo || cg >= c_lo + T / 8)
        *reinterpret_cast<uint4*>(sP + (cg >> 3) * kTile + tid * 128 + (((cg & 7) ^ (tid & 7)) << 4)) = z;
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  // ---- MMA 2: O = P V ----------------------------------------------------------------------
  if (tid == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t id2 = idesc_bf16(kRows, kHD, false, true);
#pragma unroll
    for (int ks = 0; ks < kRows / 16; ++ks) {
      // P: K-major, 64-key atoms 16 KB apart; V: MN-major, 16 keys = 2 KB per step
      const uint64_t a = smem_desc_sw128(smem_u32(sP) + (ks >> 2) * kTile + (ks & 3) * 32, 16, 1024);
      const uint64_t b = smem_desc_sw128(smem_u32(sV) + ks * 16 * 128, kTile, 1024);
      umma_bf16(tmem + kRows, a, b, id2, ks != 0);
    }
    umma_commit(&bars[2]);
  }
  wait(2);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  // ---- epilogue: row tid of O, scaled by 1 / sum --------------------------------------
  {
    float o[kHD];
#pragma unroll
    for (int c = 0; c < kHD; c += 32) {
      float v[32];
      tmem_ld32(tmem + lane_base + (uint32_t)(kRows + c), v);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[c + i] = v[i] * inv;
    }
    if (rv && !s_abort) {
      uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)grow * p.E + h * kHD);
#pragma unroll
      for (int q = 0; q < kHD / 8; ++q) {
        __nv_bfloat162 a0 = __floats2bfloat162_rn(o[8 * q + 0], o[8 * q + 1]);
        __nv_bfloat162 a1 = __floats2bfloat162_rn(o[8 * q + 2], o[8 * q + 3]);
        __nv_bfloat162 a2 = __floats2bfloat162_rn(o[8 * q + 4], o[8 * q + 5]);
        __nv_bfloat162 a3 = __floats2bfloat162_rn(o[8 * q + 6], o[8 * q + 7]);
        uint4 w;
        w.x = *reinterpret_cast<uint32_t*>(&a0);
        w.y = *reinterpret_cast<uint32_t*>(&a1);
        w.z = *reinterpret_cast<uint32_t*>(&a2);
        w.w = *reinterpret_cast<uint32_t*>(&a3);
        dst[q] = w;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256) : "memory");
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(q);
  });
  return fn;
}

template <int T>
static int launch(const CUtensorMap& m, const Params& p, int H, cudaStream_t st) {
  auto fn = mha_tc_kernel<T>;
  if (!set_smem_limit(reinterpret_cast<const void*>(fn), kSmem)) return HCLSM_ERR_LAUNCH;
  const dim3 grid((unsigned)((p.R + kRows - 1) / kRows), (unsigned)H);
  return launch_pdl(fn, grid, kThreads, kSmem, st, m, p);
}

}  // namespace evtc

// The tcgen05 attention where it applies (bf16, head dim 64, T in {16, 32,
// 64}, 16-byte aligned rows); HCLSM_ERR_UNSUPPORTED otherwise, so the caller
// takes the mma.sync kernel.
int event_mha_tc(const void* qkv, const uint8_t* key_pad, void* out, int frames, int T, int H, int HD, float scale,
                 void* stream) {
  using namespace evtc;
  if (HD != kHD || (T != 16 && T != 32 && T != 64)) return HCLSM_ERR_UNSUPPORTED;
  const int E = H * HD;
  const int64_t R = (int64_t)frames * T;
  if (R <= 0 || R > (1 << 30)) return HCLSM_ERR_UNSUPPORTED;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return HCLSM_ERR_UNSUPPORTED;
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)(3 * E), (cuuint64_t)R};
  const cuuint64_t strides[1] = {(cuuint64_t)(3 * E) * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kHD, (cuuint32_t)kRows};
  const cuuint32_t es[2] = {1, 1};
  if (fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return HCLSM_ERR_UNSUPPORTED;
  Params p{(int)R, T, E, scale, key_pad, static_cast<__nv_bfloat16*>(out), device_err_ptr()};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (T) {
    case 16: return launch<16>(m, p, H, st);
    case 32: return launch<32>(m, p, H, st);
    default: return launch<64>(m, p, H, st);
  }
}

}  // namespace hclsm
