// Slot-attention core on the 5th-generation tensor cores (tcgen05, TMEM, TMA).
//
// Same contract as core_bf16_kernel in slot_attn.cu (hclsm/kernels/
// slot_attention_kernel.py:265-291: logits = Q K^T * scale, softmax over the
// SLOT axis, out = attn V), for bf16 frames with d % 64 == 0:
//
//   per frame (one CTA, 128 threads, thread i <-> TMEM lane i):
//     TMA (tensor maps, 128-byte swizzle) loads Q [N x D] once and, per tile of
//     128 tokens, K and V [128 x D] (rows past M arrive as zeros);
//     MMA 1: logits^T [128 tokens x NP slots] = K_tile . Q^T   (tcgen05.mma
//            kind::f16, bf16 in, fp32 accumulator in TMEM columns [0, NP))
//     each thread reads its token's NP logits (tcgen05.ld), clamps, masks the
//     padded slots, takes the softmax over the slots in registers and writes
//     the bf16 weights, swizzled, as the K-major B operand of MMA 2;
//     MMA 2: out^T [d x NP] += V_tile^T . attn^T  (V as an MN-major operand),
//            D/128 accumulators in TMEM, summed over token tiles;
//   finally each thread reads row d of out^T and writes out[f, :, d].
// One thread issues every MMA; completion arrives on mbarriers through
// tcgen05.commit.  Every wait is bounded (HCLSM_ERR_TIMEOUT).
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace hclsm {
int* device_err_ptr();
bool set_smem_limit(const void* fn, size_t bytes);
}  // namespace hclsm

namespace hclsm {
namespace slottc {

constexpr int kThreads = 128;
constexpr int kTok = 128;  // tokens per tile (MMA M)

struct TcParams {
  int F, N, M, D, NP;
  float scale, clamp, eps;
  void* out;   // (F, N, D) bf16
  void* attn;  // (F, N, M) or null
  int attn_f32;
  int* err;
};

// Shared memory (1024-byte aligned pieces): Q [D/64][NP rows][128 B],
// K and V [D/64][128 rows][128 B], attn [2][NP rows][128 B], barriers.
struct TcSmem {
  static __host__ __device__ size_t q_off() { return 0; }
  static __host__ __device__ size_t k_off(int NP, int D) { return q_off() + (size_t)(D / 64) * NP * 128; }
  static __host__ __device__ size_t v_off(int NP, int D) { return k_off(NP, D) + (size_t)(D / 64) * kTok * 128; }
  static __host__ __device__ size_t a_off(int NP, int D) { return v_off(NP, D) + (size_t)(D / 64) * kTok * 128; }
  static __host__ __device__ size_t bar_off(int NP, int D) { return a_off(NP, D) + 2 * (size_t)NP * 128; }
  static __host__ __device__ size_t total(int NP, int D) { return bar_off(NP, D) + 64 + 1024; }  // + alignment
};

using namespace ::hclsm::tc;

// NP: slots padded to a multiple of 32 (<= 64); DB: D / 64 k-blocks.
template <int NP, int DB>
__global__ void __launch_bounds__(kThreads, 1)
    core_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                   const __grid_constant__ CUtensorMap mv, TcParams p) {
  constexpr int D = DB * 64;
  constexpr int MB = D / 128;  // output blocks of 128 rows of out^T
  constexpr uint32_t kCols = (NP * (1 + MB) <= 128) ? 128 : 256;
  static_assert(NP * (1 + MB) <= 256, "TMEM columns");
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int f = blockIdx.x;
  const int N = p.N, M = p.M;
  unsigned char* sQ = smem + TcSmem::q_off();
  unsigned char* sK = smem + TcSmem::k_off(NP, D);
  unsigned char* sV = smem + TcSmem::v_off(NP, D);
  unsigned char* sA = smem + TcSmem::a_off(NP, D);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::bar_off(NP, D));  // 0: K(+Q) 1: V 2: MMA1 3: MMA2

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    s_abort = 0;
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = s_tmem;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  auto wait = [&](int b, uint32_t parity) {
    if (!s_abort && !mbar_wait(&bars[b], parity)) {
      record_error(p.err, HCLSM_ERR_TIMEOUT);
      s_abort = 1;
    }
  };
  const uint32_t id1 = idesc_bf16(128, NP, false, false);  // K-major A (K tile), K-major B (Q)
  const uint32_t id2 = idesc_bf16(128, NP, true, false);   // MN-major A (V^T), K-major B (attn^T)
  const int ntiles = (M + kTok - 1) / kTok;
  const uint32_t tile_bytes = (uint32_t)DB * kTok * 128;
  const uint32_t q_bytes = (uint32_t)DB * NP * 128;

  // K of tile ti is fetched as soon as MMA 1 of tile ti - 1 has released the K
  // buffer (so it overlaps that tile's softmax and MMA 2); V of tile ti once MMA
  // 2 of tile ti - 1 has released the V buffer
  auto load_k = [&](int ti) {
    mbar_expect_tx(&bars[0], tile_bytes + (ti == 0 ? q_bytes : 0));
    for (int kb = 0; kb < DB; ++kb) {
      if (ti == 0) tma_load_3d(sQ + (size_t)kb * NP * 128, &mq, kb * 64, 0, f, &bars[0]);
      tma_load_3d(sK + (size_t)kb * kTok * 128, &mk, kb * 64, ti * kTok, f, &bars[0]);
    }
  };
  auto load_v = [&](int ti) {
    mbar_expect_tx(&bars[1], tile_bytes);
    for (int kb = 0; kb < DB; ++kb) tma_load_3d(sV + (size_t)kb * kTok * 128, &mv, kb * 64, ti * kTok, f, &bars[1]);
  };
  if (tid == 0) {
    load_k(0);
    load_v(0);
  }
  for (int ti = 0; ti < ntiles; ++ti) {
    const uint32_t par = ti & 1;
    // ---- MMA 1: logits^T = K_tile . Q^T -----------------------------------------------
    wait(0, par);
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int kb = 0; kb < DB; ++kb)
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t a = smem_desc_sw128(smem_u32(sK + (size_t)kb * kTok * 128) + ks * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(smem_u32(sQ + (size_t)kb * NP * 128) + ks * 32, 16, 1024);
          umma_bf16(tmem, a, b, id1, (kb | ks) != 0);
        }
      umma_commit(&bars[2]);
    }
    wait(2, par);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (tid == 0 && ti + 1 < ntiles) load_k(ti + 1);
    // ---- softmax over the slots of this thread's token ------------------------------
    {
      float lg[NP];
#pragma unroll
      for (int c = 0; c < NP; c += 32) {
        float v[32];
        tmem_ld32(tmem + lane_base + c, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) lg[c + i] = v[i];
      }
      const int tok = ti * kTok + tid;
      float mx = -INFINITY;
#pragma unroll
      for (int s = 0; s < NP; ++s) {
        float v = lg[s] * p.scale;
        if (p.clamp > 0.0f) v = fminf(fmaxf(v, -p.clamp), p.clamp);
        v = s < N ? v : -INFINITY;
        lg[s] = v;
        mx = fmaxf(mx, v);
      }
      float sum = 0.0f;
#pragma unroll
      for (int s = 0; s < NP; ++s) {
        const float e = ex2((lg[s] - mx) * kLog2e);
        lg[s] = e;
        sum += e;
      }
      const float inv = 1.0f / (sum + p.eps);
      const bool tv = tok < M;
      // attn^T as the K-major, 128-byte-swizzled B operand: row = slot, column = token
      const int kb2 = tid >> 6, tc = tid & 63;
      unsigned char* ab = sA + (size_t)kb2 * NP * 128;
#pragma unroll
      for (int s = 0; s < NP; ++s) {
        const float a = tv ? lg[s] * inv : 0.0f;
        const uint32_t off = (uint32_t)s * 128 + ((((tc >> 3) ^ (s & 7)) << 4)) + (tc & 7) * 2;
        *reinterpret_cast<__nv_bfloat16*>(ab + off) = __float2bfloat16_rn(a);
        if (p.attn && tv && s < N) {
          const size_t gi = ((size_t)f * N + s) * M + tok;
          if (p.attn_f32) static_cast<float*>(p.attn)[gi] = a;
          else static_cast<__nv_bfloat16*>(p.attn)[gi] = __float2bfloat16_rn(a);
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    // ---- MMA 2: out^T += V_tile^T . attn^T -------------------------------------------
    wait(1, par);
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      for (int mb = 0; mb < MB; ++mb)
        for (int ks = 0; ks < kTok / 16; ++ks) {
          // V^T, MN-major: 64-d atoms are the tile's 64-column TMA boxes (16 KB
          // apart), 8-token row groups 1 KB apart
          const uint64_t a =
              smem_desc_sw128(smem_u32(sV + (size_t)(2 * mb) * kTok * 128) + ks * 16 * 128, kTok * 128, 1024);
          const uint64_t b = smem_desc_sw128(smem_u32(sA + (size_t)(ks >> 2) * NP * 128) + (ks & 3) * 32, 16, 1024);
          umma_bf16(tmem + (uint32_t)(NP * (1 + mb)), a, b, id2, (ti | ks) != 0);
        }
      umma_commit(&bars[3]);
    }
    wait(3, par);  // the V and attn buffers are free again
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (tid == 0 && ti + 1 < ntiles) load_v(ti + 1);
  }
  // ---- epilogue: row d of out^T -> out[f, :, d] --------------------------------------
  __nv_bfloat16* gO = static_cast<__nv_bfloat16*>(p.out) + (size_t)f * N * D;
#pragma unroll
  for (int mb = 0; mb < MB; ++mb) {
    const int d = mb * 128 + tid;
#pragma unroll
    for (int c = 0; c < NP; c += 32) {
      float v[32];
      tmem_ld32(tmem + lane_base + (uint32_t)(NP * (1 + mb) + c), v);
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c + i < N) gO[(size_t)(c + i) * D + d] = __float2bfloat16_rn(v[i]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
}

// ---- host: tensor maps -----------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// (D, rows, F) bf16 tensor, box (64, box_rows, 1), 128-byte swizzle, zero fill
static bool make_map(CUtensorMap* m, const void* base, int D, int rows, int F, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)F};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)D * rows * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NP, int DB>
static int launch_tc(const void* Q, const void* K, const void* V, const TcParams& p, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!make_map(&mq, Q, p.D, p.N, p.F, NP) || !make_map(&mk, K, p.D, p.M, p.F, kTok) ||
      !make_map(&mv, V, p.D, p.M, p.F, kTok))
    return HCLSM_ERR_UNSUPPORTED;
  const size_t smem = TcSmem::total(NP, p.D);
  auto fn = core_tc_kernel<NP, DB>;
  if (!set_smem_limit(reinterpret_cast<const void*>(fn), smem)) return HCLSM_ERR_LAUNCH;
  return launch_pdl(fn, p.F, kThreads, smem, st, mq, mk, mv, p);
}

}  // namespace slottc

// Tensor-core (tcgen05) core for bf16, D in {64, 128, 192, 256, 320, 384}
// (D % 128 == 0 for the output blocks: 128, 256, 384), N <= 64.  Returns
// HCLSM_ERR_UNSUPPORTED for other shapes (the caller then uses the
// mma.sync core).
int slot_core_tc(const void* Q, const void* K, const void* V, void* out, void* attn, int F, int N, int M, int D,
                 float scale, float clamp, float eps, int attn_f32, cudaStream_t st) {
  using namespace slottc;
  if (D % 128 != 0 || D > 384 || N > 64 || M <= 0) return HCLSM_ERR_UNSUPPORTED;
  auto al = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (!al(Q) || !al(K) || !al(V)) return HCLSM_ERR_UNSUPPORTED;
  const int NP = N <= 32 ? 32 : 64;
  if (TcSmem::total(NP, D) > 227 * 1024) return HCLSM_ERR_UNSUPPORTED;
  TcParams p{F, N, M, D, NP, scale, clamp, eps, out, attn, attn_f32, device_err_ptr()};
  if (NP == 32) {
    if (D == 128) return launch_tc<32, 2>(Q, K, V, p, st);
    if (D == 256) return launch_tc<32, 4>(Q, K, V, p, st);
    if (D == 384) return launch_tc<32, 6>(Q, K, V, p, st);
  } else {
    if (D == 128) return launch_tc<64, 2>(Q, K, V, p, st);
    if (D == 256) return launch_tc<64, 4>(Q, K, V, p, st);
  }
  return HCLSM_ERR_UNSUPPORTED;
}

}  // namespace hclsm
