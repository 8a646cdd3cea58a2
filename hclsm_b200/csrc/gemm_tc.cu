// Dense GEMM on the 5th-generation tensor cores with fused epilogues:
//
//   out[m, n] = epilogue( sum_k A[m, k] * W[n, k] )      (A: M x K bf16, W: N x K bf16,
//                                                          both row-major = K-major)
//
// the weight products of DynamicSlotAttention._iteration_step
// (hclsm/objects/dynamic_slots.py:113-128) and of the Level-1 event
// transformer (hclsm/dynamics/level1_event.py:17-54), with their bias / ReLU /
// residual / clamp stages folded into the epilogue.
//
// CTA tile 128 x 128, K step 64 (one 128-byte swizzle atom), 4-stage ring.
// Warp 0 lane 0 streams A and W tiles with TMA (2-D tensor maps, 128-byte
// swizzle, no multicast); warp 1 lane 0 issues tcgen05.mma (kind::f16, fp32
// accumulator in 128 TMEM columns) and returns each stage through
// tcgen05.commit; after the last K step all four warps read the accumulator
// (thread i <-> row i of the tile) and apply the epilogue.  Rows past M arrive
// as zeros and are not stored.  Every wait is bounded (HCLSM_ERR_TIMEOUT).
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace hclsm {
int* device_err_ptr();
bool set_smem_limit(const void* fn, size_t bytes);
}  // namespace hclsm

namespace hclsm {
namespace gemm {

constexpr int kThreads = 128;
constexpr int BM = 128, BN = 128, BK = 64, kStages = 4;
constexpr size_t kStageBytes = (size_t)(BM + BN) * BK * 2;  // 32 KB

struct Params {
  int M, N, K;
  int epi;              // HCLSM_EPI_*
  const float* bias;    // (N) or null
  const float* resid;   // (M, N) fp32 or null (EPI_RESID)
  float* out_f32;       // (M, N) or null
  __nv_bfloat16* out_bf16;  // (M, N) or null
  float clamp;
  int* err;
};

__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // 8-row group stride
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;            // 128-byte swizzle
  return d;
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7]),
        "=f"(v[8]), "=f"(v[9]), "=f"(v[10]), "=f"(v[11]), "=f"(v[12]), "=f"(v[13]), "=f"(v[14]), "=f"(v[15]),
        "=f"(v[16]), "=f"(v[17]), "=f"(v[18]), "=f"(v[19]), "=f"(v[20]), "=f"(v[21]), "=f"(v[22]), "=f"(v[23]),
        "=f"(v[24]), "=f"(v[25]), "=f"(v[26]), "=f"(v[27]), "=f"(v[28]), "=f"(v[29]), "=f"(v[30]), "=f"(v[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mw, Params p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kStages], empty[kStages], done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int nk = p.K / BK;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_tmem;
  auto bounded_wait = [&](uint64_t* bar, uint32_t parity) {
    if (s_abort) return;
    if (!mbar_wait(bar, parity)) {
      record_error(p.err, HCLSM_ERR_TIMEOUT);
      s_abort = 1;
    }
  };

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ---------------------------------------------------------------
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages;
      if (kb >= kStages) bounded_wait(&empty[s], ((kb / kStages) - 1) & 1);
      unsigned char* sa = smem + (size_t)s * kStageBytes;
      unsigned char* sw = sa + (size_t)BM * BK * 2;
      mbar_expect_tx(&full[s], (uint32_t)kStageBytes);
      tma_2d(sa, &ma, kb * BK, m0, &full[s]);
      tma_2d(sw, &mw, kb * BK, n0, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer -----------------------------------------------------------------
    // kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, both
    // K-major, N = 128, M = 128
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kStages;
      bounded_wait(&full[s], (kb / kStages) & 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t sa = smem_u32(smem + (size_t)s * kStageBytes);
      const uint32_t sw = sa + BM * BK * 2;
#pragma unroll
      for (int ks = 0; ks < BK / 16; ++ks)
        mma(tmem, desc_sw128(sa + ks * 32), desc_sw128(sw + ks * 32), idesc, (kb | ks) != 0);
      commit(&empty[s]);
    }
    commit(&done);
  }
  __syncwarp();
  // ---- epilogue: thread i <-> row m0 + i ------------------------------------------------
  bounded_wait(&done, 0);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const int row = m0 + tid;
  const bool rv = row < p.M;
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    float v[32];
    tmem_ld32(taddr + c0, v);
    if (!rv) continue;
    const int n = n0 + c0;
    if (p.bias) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += p.bias[n + i];
    }
    if (p.epi == HCLSM_EPI_RELU) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
    } else if (p.epi == HCLSM_EPI_RESID) {
      const float4* r4 = reinterpret_cast<const float4*>(p.resid + (size_t)row * p.N + n);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 r = r4[i];
        v[4 * i] += r.x; v[4 * i + 1] += r.y; v[4 * i + 2] += r.z; v[4 * i + 3] += r.w;
      }
      if (p.clamp > 0.0f) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = fminf(fmaxf(v[i], -p.clamp), p.clamp);
      }
    }
    if (p.out_f32) {
      float4* o4 = reinterpret_cast<float4*>(p.out_f32 + (size_t)row * p.N + n);
#pragma unroll
      for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    if (p.out_bf16) {
      uint4* o4 = reinterpret_cast<uint4*>(p.out_bf16 + (size_t)row * p.N + n);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v[8 * i], v[8 * i + 1]);
        __nv_bfloat162 b = __floats2bfloat162_rn(v[8 * i + 2], v[8 * i + 3]);
        __nv_bfloat162 c = __floats2bfloat162_rn(v[8 * i + 4], v[8 * i + 5]);
        __nv_bfloat162 d = __floats2bfloat162_rn(v[8 * i + 6], v[8 * i + 7]);
        uint4 w;
        w.x = *reinterpret_cast<uint32_t*>(&a);
        w.y = *reinterpret_cast<uint32_t*>(&b);
        w.z = *reinterpret_cast<uint32_t*>(&c);
        w.w = *reinterpret_cast<uint32_t*>(&d);
        o4[i] = w;
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
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
// (K, rows) bf16 row-major matrix, box (64, box_rows), 128-byte swizzle, zero fill
static bool map2d(CUtensorMap* m, const void* base, int K, int rows, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {BK, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gemm
}  // namespace hclsm

using namespace hclsm;

extern "C" int hclsm_gemm_bf16(const void* A, const void* W, int32_t M, int32_t N, int32_t K, int32_t epilogue,
                               const float* bias, const float* resid, float* out_f32, void* out_bf16, float clamp,
                               void* stream) {
  using namespace hclsm::gemm;
  if (!A || !W || (!out_f32 && !out_bf16)) return HCLSM_ERR_NULL;
  if (M < 0 || N <= 0 || K <= 0) return HCLSM_ERR_SHAPE;
  if (N % BN != 0 || K % BK != 0) return HCLSM_ERR_UNSUPPORTED;
  if (epilogue == HCLSM_EPI_RESID && !resid) return HCLSM_ERR_NULL;
  if (epilogue < HCLSM_EPI_NONE || epilogue > HCLSM_EPI_RESID) return HCLSM_ERR_SHAPE;
  auto al = [](const void* q) { return q == nullptr || reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (!al(A) || !al(W) || !al(resid) || !al(out_f32) || !al(out_bf16)) return HCLSM_ERR_ALIGN;
  if (M == 0) return HCLSM_OK;
  CUtensorMap ma, mw;
  if (!map2d(&ma, A, K, M, BM) || !map2d(&mw, W, K, N, BN)) return HCLSM_ERR_LAUNCH;
  Params p{M, N, K, epilogue, bias, resid, out_f32, static_cast<__nv_bfloat16*>(out_bf16), clamp, device_err_ptr()};
  const size_t smem = kStages * kStageBytes + 1024;
  if (!set_smem_limit(reinterpret_cast<const void*>(gemm_kernel), smem)) return HCLSM_ERR_LAUNCH;
  const dim3 grid((unsigned)((M + BM - 1) / BM), (unsigned)(N / BN));
  gemm_kernel<<<grid, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(ma, mw, p);
  return cudaGetLastError() == cudaSuccess ? HCLSM_OK : HCLSM_ERR_LAUNCH;
}
