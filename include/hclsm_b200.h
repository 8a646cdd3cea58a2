/*
 * hclsm_b200 — C ABI of the B200 (sm_100a) kernels behind HCLSM's data-parallel
 * hot path: the Level-0 selective SSM scan (forward and backward), the fused
 * slot-attention iteration and the sparse event attention.
 *
 * Conventions for every entry point:
 *   - pointers are device pointers unless stated; tensors are dense row-major;
 *   - `stream` is a cudaStream_t passed as void*; every call is stream-ordered,
 *     never synchronises and allocates nothing (callers pass workspaces);
 *   - the return value is an hclsm_status; nothing traps.  A kernel whose
 *     bounded wait ran out records HCLSM_ERR_TIMEOUT in a per-device error
 *     word that hclsm_device_error() reads (that call synchronises).
 *
 * Reference interfaces (paths inside the RightNow-AI/hclsm project):
 *   hclsm/kernels/ssm_scan_kernel.py, slot_attention_kernel.py,
 *   sparse_event_attn.py; hclsm/objects/dynamic_slots.py;
 *   hclsm/dynamics/level1_event.py, hierarchy_manager.py.
 */
#ifndef HCLSM_B200_H_
#define HCLSM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  HCLSM_OK = 0,
  HCLSM_ERR_SHAPE = 1,       /* a size is out of the supported range */
  HCLSM_ERR_DTYPE = 2,       /* unknown dtype code */
  HCLSM_ERR_ALIGN = 3,       /* a pointer is not aligned as required */
  HCLSM_ERR_WORKSPACE = 4,   /* workspace missing or too small */
  HCLSM_ERR_LAUNCH = 5,      /* a CUDA launch failed (see cudaGetLastError) */
  HCLSM_ERR_TIMEOUT = 6,     /* a device-side bounded wait ran out */
  HCLSM_ERR_UNSUPPORTED = 7, /* valid input this build does not handle */
  HCLSM_ERR_NULL = 8         /* a required pointer is NULL */
} hclsm_status;

typedef enum { HCLSM_F32 = 0, HCLSM_BF16 = 1 } hclsm_dtype;

/* Flags of the scan entry points' `clamp` argument (0 and 1 keep their
 * meaning: the unclamped and the clamped arithmetic). */
typedef enum { HCLSM_SCAN_CLAMP = 1, HCLSM_SCAN_DT_SOFTPLUS = 2 } hclsm_scan_flags;

/* Library version and the per-device error word.  hclsm_device_error
 * synchronises the device, returns the first recorded error code (0 if none)
 * and clears it. */
int hclsm_version(void);
int hclsm_device_error(void);

/* Self-test of the bounded device-side wait (no reference counterpart): one
 * block polls an mbarrier that nothing completes `polls` times, then writes
 * HCLSM_ERR_TIMEOUT to *status_dev (device int) and to the error word. */
int hclsm_selftest_wait_timeout(uint32_t polls, int* status_dev, void* stream);

/* ---------------------------------------------------------------------------
 * Selective SSM scan, forward.
 * Replaces hclsm/kernels/ssm_scan_kernel.py:394 ssm_scan_fn (the dispatcher),
 * with the arithmetic of sequential_ssm_scan :42-86 (clamp=1) or of
 * parallel_ssm_scan_pytorch :168-218 / _ssm_scan_fwd_kernel :227-290 (clamp=0).
 *   x, dt, y, z : (nseq, L, d_inner)   dtype
 *   B, C        : (nseq, L, d_state)   dtype
 *   A_log       : (d_inner, d_state)   f32
 *   D           : (d_inner,)           f32, optional (NULL)
 *   z           : optional (NULL); when given y = (scan + D*x) * silu(z)
 *   clamp       : flags, HCLSM_SCAN_CLAMP for the clamped arithmetic and/or
 *                 HCLSM_SCAN_DT_SOFTPLUS when dt is the raw projection and
 *                 softplus(dt) (torch's threshold 20) is applied inside, as
 *                 SimplifiedSSMBlock does before its scan (level0_ssm.py:76);
 *                 the backward then returns the gradient of the raw dt
 * d_state <= 64.  State and arithmetic are fp32 for both dtypes.
 * ------------------------------------------------------------------------- */
int hclsm_ssm_scan_fwd(const void* x, const void* dt, const float* A_log, const void* B,
                       const void* C, const float* D, const void* z, void* y, int64_t nseq,
                       int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype, int32_t clamp,
                       void* stream);

/* ---------------------------------------------------------------------------
 * Selective SSM scan, backward.
 * Replaces hclsm/kernels/ssm_scan_kernel.py:321-377 _TritonSSMScan.backward
 * (clamp=0) and the autograd of sequential_ssm_scan (clamp=1).
 * Inputs as for the forward plus dy (nseq, L, d_inner).  Outputs:
 *   dx, ddt, dz : (nseq, L, d_inner) dtype  (dz only when z != NULL)
 *   dB, dC      : (nseq, L, d_state) dtype
 *   dA_log      : (d_inner, d_state) f32
 *   dD          : (d_inner,)         f32  (only when D != NULL)
 * `workspace` must hold hclsm_ssm_scan_bwd_workspace_size(...) bytes.
 * Supported: d_state <= 64, any L; d_inner * element size a multiple of 16
 * bytes; x, dt, dy, z 16-byte aligned.  bf16 with 9 <= d_state <= 16 and
 * L <= ~600 takes the packed fast kernel.
 * ------------------------------------------------------------------------- */
size_t hclsm_ssm_scan_bwd_workspace_size(int64_t nseq, int32_t L, int32_t d_inner, int32_t d_state);
int hclsm_ssm_scan_bwd(const void* x, const void* dt, const float* A_log, const void* B, const void* C,
                       const float* D, const void* z, const void* dy, void* dx, void* ddt,
                       float* dA_log, void* dB, void* dC, float* dD, void* dz, int64_t nseq,
                       int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype, int32_t clamp,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Scan forward that keeps state snapshots for the backward, and the backward
 * that uses them.  No counterpart in the reference (its backward,
 * ssm_scan_kernel.py:321-377, re-runs the whole forward recurrence): the
 * forward writes h after every 10 steps, (nseq, ceil(L/10) - 1, 4, d_inner)
 * float4 of fp32 (quad q = states 4q..4q+3 of a channel), and the backward starts each 10-step chunk from those snapshots
 * instead of sweeping the recurrence a second time.  Results are identical to
 * hclsm_ssm_scan_fwd / hclsm_ssm_scan_bwd.
 * hclsm_ssm_scan_states_size returns the snapshot bytes, or 0 where the path
 * does not apply (it needs bf16, 9 <= d_state <= 16, even d_inner, and the
 * packed backward's L limit); then call the plain entry points.
 * x, dt, z, y 4-byte aligned; states 16-byte aligned.
 * ------------------------------------------------------------------------- */
size_t hclsm_ssm_scan_states_size(int64_t nseq, int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype);
int hclsm_ssm_scan_fwd_states(const void* x, const void* dt, const float* A_log, const void* B, const void* C,
                              const float* D, const void* z, void* y, int64_t nseq, int32_t L, int32_t d_inner,
                              int32_t d_state, int32_t dtype, int32_t clamp, float* states, size_t states_bytes,
                              void* stream);
int hclsm_ssm_scan_bwd_states(const void* x, const void* dt, const float* A_log, const void* B, const void* C,
                              const float* D, const void* z, const void* dy, void* dx, void* ddt, float* dA_log,
                              void* dB, void* dC, float* dD, void* dz, int64_t nseq, int32_t L, int32_t d_inner,
                              int32_t d_state, int32_t dtype, int32_t clamp, const float* states,
                              size_t states_bytes, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Level0SSM around its blocks (hclsm/dynamics/level0_ssm.py:159-220).
 *   obj / x : (B, N, T*D) contiguous, obj_dtype / x_dtype f32 or bf16
 *   mask    : (B, N) f32, optional (NULL)
 * hclsm_l0_pool: out (B, T*D) = sum_n mask obj / max(sum_n mask, 1), or the
 *   mean over n without a mask (the global track's input, :175-180).
 * hclsm_l0_epilogue: out = clamp(nan_to_num(x, 0, 100, -100), -100, 100) * mask
 *   in one pass (:210-218).
 * hclsm_l0_epilogue_bwd: gx (x's dtype) = g * mask * [x finite, |x| <= 100].
 * ------------------------------------------------------------------------- */
int hclsm_l0_pool(const void* obj, int32_t obj_dtype, const float* mask, void* out, int32_t out_dtype, int32_t B,
                  int32_t N, int64_t TD, void* stream);
int hclsm_l0_epilogue(const void* x, int32_t x_dtype, const float* mask, void* out, int32_t out_dtype, int32_t B,
                      int32_t N, int64_t TD, void* stream);
int hclsm_l0_epilogue_bwd(const void* x, int32_t x_dtype, const float* mask, const void* g, int32_t g_dtype,
                          void* gx, int32_t B, int32_t N, int64_t TD, void* stream);

/* ---------------------------------------------------------------------------
 * Slot attention core: out = softmax_over_slots(clamp(Q K^T * scale)) V.
 * Replaces hclsm/kernels/slot_attention_kernel.py:324 slot_attention_fn (the
 * arithmetic of naive_slot_attention :265-291 with eps=0, of the Triton path
 * :42-236 with eps=1e-8) and the attention lines of
 * hclsm/objects/dynamic_slots.py:110-121 (clamp=30).
 *   Q (F, N, D), K and V (F, M, D), out (F, N, D): dtype (f32 or bf16)
 *   attn (F, N, M): optional (NULL); f32 when attn_f32, else dtype
 * clamp <= 0 disables the logit clamp.  bf16: N <= 64, D % 16 == 0, D <= 512,
 * 16-byte aligned rows; tensor-core MMA with fp32 accumulation.  f32: exact
 * fp32 arithmetic on CUDA cores.
 * ------------------------------------------------------------------------- */
int hclsm_slot_attn_core(const void* Q, const void* K, const void* V, void* out, void* attn, int32_t F,
                         int32_t N, int32_t M, int32_t D, float scale, float clamp, float eps, int32_t dtype,
                         int32_t attn_f32, void* stream);

/* Fused element-wise stages of DynamicSlotAttention._iteration_step
 * (hclsm/objects/dynamic_slots.py:111-130).  Matrices are (rows, C), fp32
 * unless an out_dtype is given.
 *   hclsm_layernorm:      y = LayerNorm(x) * w + b   (nn.LayerNorm, :111, :128)
 *   hclsm_gru_cell:       nn.GRUCell from gi = x W_ih^T, gh = h W_hh^T (:123-126)
 *   hclsm_bias_act:       y = act(x + b), act 0 = identity, 1 = ReLU (:128 MLP)
 *   hclsm_residual_clamp: out = clamp(h + m + b, -clamp, clamp), optional bf16 copy (:128-130) */
int hclsm_layernorm(const float* x, const float* w, const float* b, void* y, int64_t rows, int32_t D, float eps,
                    int32_t out_dtype, void* stream);
int hclsm_gru_cell(const float* gi, const float* gh, const float* b_ih, const float* b_hh, const float* h,
                   float* h_out, int64_t rows, int32_t H, void* stream);
int hclsm_bias_act(const float* x, const float* b, void* y, int64_t rows, int32_t C, int32_t act,
                   int32_t out_dtype, void* stream);
int hclsm_residual_clamp(const float* h, const float* m, const float* b, float* out, void* out_bf16, int64_t rows,
                         int32_t C, float clamp, void* stream);

/* ---------------------------------------------------------------------------
 * Sparse event attention.  Replaces the gather / scatter of
 * hclsm/kernels/sparse_event_attn.py:35-188 and
 * hclsm/dynamics/hierarchy_manager.py:42-118, and the attention and SwiGLU of
 * hclsm/dynamics/level1_event.py:17-54.
 *   hclsm_event_compact: (B, T) mask (f32/bf16, fired > 0.5) -> idx[k] =
 *       b*T + t of the k-th fired frame (video-major, time ascending),
 *       pos[b*T + t] = k or -1, counts[b], meta = {total, max per video}.
 *       Runs on the device; nothing is read back.
 *   hclsm_event_gather: frames (frame_elems elements each) of the fired
 *       timesteps: compact (pad_k = 0, rows >= meta[0] untouched) or padded
 *       (B, pad_k) with zero pad frames.
 *   hclsm_event_scatter: out = states with every fired frame replaced by its
 *       update (the reference's clone + scatter in one pass).
 *   hclsm_event_mha: per-frame multi-head self-attention of
 *       nn.MultiheadAttention(bias=False) on a packed (frames*T, 3E) q|k|v
 *       matrix; key_pad (frames, T) bytes, non-zero = ignored key (NULL: none).
 *       bf16: T <= 64, head dim in {16, 32, 64, 128}, tensor cores.
 *   hclsm_swiglu: y = silu(u[:, :C]) * u[:, C:] (SwiGLUFFN, level1_event.py:28);
 *     u fp32 or bf16 (u_dtype), arithmetic fp32.
 * frame_elems * element size must be a multiple of 16 bytes.
 * ------------------------------------------------------------------------- */
int hclsm_event_compact(const void* mask, int32_t mask_dtype, int32_t B, int32_t T, int32_t* idx, int32_t* pos,
                        int32_t* counts, int32_t* meta, void* stream);
int hclsm_event_gather(const void* states, const int32_t* idx, const int32_t* counts, const int32_t* meta,
                       void* out, int64_t frame_elems, int32_t B, int32_t pad_k, int64_t max_frames,
                       int32_t dtype, void* stream);
int hclsm_event_scatter(const void* states, const void* upd, const int32_t* pos, const int32_t* counts, void* out,
                        int64_t frames, int64_t frame_elems, int32_t T, int32_t pad_k, int32_t dtype,
                        void* stream);
int hclsm_event_mha(const void* qkv, const uint8_t* key_pad, void* out, int32_t frames, int32_t T, int32_t H,
                    int32_t HD, float scale, int32_t dtype, void* stream);
int hclsm_swiglu(const void* u, int32_t u_dtype, void* y, int64_t rows, int32_t C, int32_t out_dtype, void* stream);

/* EventDetector's hard decision and the compaction in one launch
 * (hclsm/dynamics/event_detector.py:162-170 feeding hierarchy_manager.py:42-77):
 * hard[b, t] = probs[b, t] > *threshold (f32, the learned threshold read on the
 * device); if any video has no event, t = 0 becomes an event in every video
 * (the reference's rule, decided there by a host read); idx / pos / counts as
 * hclsm_event_compact, meta[0] = events, meta[1] = max per video, meta[2] = 1
 * when the t = 0 rule fired (meta holds 3 ints).  probs and hard (B, T) f32. */
int hclsm_event_detect(const float* probs, const float* threshold, int32_t B, int32_t T, float* hard, int32_t* idx,
                       int32_t* pos, int32_t* counts, int32_t* meta, void* stream);

/* ---------------------------------------------------------------------------
 * One whole slot-attention refinement step: DynamicSlotAttention._iteration_step
 * (hclsm/objects/dynamic_slots.py:98-131), the slot-attention entry point of
 * the reference's hot path as one call.  bf16 weight products (fp32
 * accumulation, library GEMMs), fp32 carried state:
 *   slots (F, N, D) f32 -> slots_out (F, N, D) f32 (+ an optional bf16 copy);
 *   k, v (F, M, D) bf16 (the module's k / v projections of its inputs).
 * Weights are transposed for x @ W^T ((in, out) row-major, bf16); biases and
 * LayerNorm affines f32 (b1 bf16: it is the epilogue bias of the MLP's first
 * product; affines and b2 may be NULL).  Workspace:
 * hclsm_slot_attn_iter_workspace_size(F, N, D) bytes, 256-byte aligned.
 * D % 8 == 0; the attention core's limits apply (N <= 64, D <= 512).
 * ------------------------------------------------------------------------- */
typedef struct hclsm_slot_iter_weights {
  const void* wq_t;          /* (D, D) bf16: project_q.weight^T */
  const void* w_ih_t;        /* (D, 3D) bf16: gru.weight_ih^T */
  const void* w_hh_t;        /* (D, 3D) bf16: gru.weight_hh^T */
  const float* b_ih;         /* (3D) */
  const float* b_hh;         /* (3D) */
  const void* w1_t;          /* (D, 4D) bf16: mlp.0.weight^T */
  const void* b1;            /* (4D) bf16: mlp.0.bias */
  const void* w2_t;          /* (4D, D) bf16: mlp.2.weight^T */
  const float* b2;           /* (D): mlp.2.bias */
  const float* ln_attn_w;    /* norm_pre_attn */
  const float* ln_attn_b;
  const float* ln_mlp_w;     /* norm_slots */
  const float* ln_mlp_b;
} hclsm_slot_iter_weights;

size_t hclsm_slot_attn_iter_workspace_size(int32_t F, int32_t N, int32_t D);
int hclsm_slot_attn_iter(const float* slots, const void* k, const void* v, const hclsm_slot_iter_weights* w,
                         float* slots_out, void* slots_out_bf16, int32_t F, int32_t N, int32_t M, int32_t D,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------
 * Row-fused stages of the slot-attention iteration (dynamic_slots.py:98-131):
 * one warp per row, rows of 128 to 1024 columns in multiples of 128 (else
 * HCLSM_ERR_UNSUPPORTED), 16-byte aligned rows.
 *   hclsm_gru_cell_ln: hclsm_gru_cell, then LayerNorm (w, b may be NULL,
 *     eps) of the new state into ln_out (ln_dtype) -- the GRUCell of :123-126
 *     and the norm_slots LayerNorm of :128 in one pass.  The gate products gi
 *     and gh are HCLSM_F32 or HCLSM_BF16 (gate_dtype; bf16 is what the
 *     reference's GRUCell sees under bf16 autocast); the gate arithmetic and
 *     the state are fp32.
 *   hclsm_residual_clamp_ln: hclsm_residual_clamp, then LayerNorm of the
 *     result into ln_out -- the residual and clamp of :128-130 and the next
 *     iteration's norm_pre_attn LayerNorm (:111) in one pass.  m (the MLP
 *     output) is HCLSM_F32 or HCLSM_BF16 (m_dtype); the sum is fp32.
 * ------------------------------------------------------------------------- */
int hclsm_gru_cell_ln(const void* gi, const void* gh, int32_t gate_dtype, const float* b_ih, const float* b_hh,
                      const float* h, float* h_out, const float* ln_w, const float* ln_b, void* ln_out,
                      int32_t ln_dtype, int64_t rows, int32_t H, float eps, void* stream);
int hclsm_residual_clamp_ln(const float* h, const void* m, int32_t m_dtype, const float* b, float* out,
                            void* out_bf16, const float* ln_w, const float* ln_b, void* ln_out, int32_t ln_dtype,
                            int64_t rows, int32_t C, float clamp, float eps, void* stream);

/* ---------------------------------------------------------------------------
 * Training-mode backward of the slot-attention iteration and of the Level-1
 * event transformer (the gradients autograd takes through
 * hclsm/objects/dynamic_slots.py:98-131 _iteration_step and
 * hclsm/dynamics/level1_event.py:17-133, EventTransformerBlock / SwiGLUFFN).
 * The weight-product gradients are library GEMMs; these are the stages between
 * them.  All fp32 unless a dtype code says otherwise.
 *
 *   hclsm_colsum: out[c] = sum_r a[r, c] (deterministic two-stage sum; the
 *     bias gradients of nn.Linear / nn.GRUCell).  Workspace
 *     hclsm_colsum_workspace_size(C) bytes.
 *   hclsm_layernorm_bwd: nn.LayerNorm backward from x and dy (statistics
 *     recomputed as hclsm_layernorm forms them): dx (written, or added when
 *     accumulate != 0), dw / db (may be NULL).  Workspace
 *     hclsm_layernorm_bwd_workspace_size(rows, D) bytes when dw or db is given.
 *   hclsm_gru_cell_bwd: nn.GRUCell backward (gates r, z, n) from the forward's
 *     pre-bias products gi, gh (rows, 3H), its biases and input state h:
 *     d_gi, d_gh (rows, 3H) and dh = z * dh_new (the state's direct term).
 *   hclsm_slot_softmax_bwd: softmax over the slot axis (dim=1 of (F, N, M))
 *     with the +-clamp logit clamp, recomputed from dots = q k^T (unscaled):
 *     writes attn and d_dots = d(q k^T), both in dtype.
 *   hclsm_residual_clamp_bwd: dpre = dout where -c <= (h + m) + b <= c.
 *   hclsm_relu_bwd: dx = dy where y > 0 (y the ReLU output).
 *   hclsm_swiglu_bwd: du (rows, 2C) of y = silu(u[:, :C]) * u[:, C:].
 *   hclsm_event_mha_bwd: nn.MultiheadAttention core backward per (frame,
 *     head), recomputing the probabilities from qkv (frames * T, 3E) and
 *     key_pad; dout (frames * T, E) fp32; dqkv (frames * T, 3E) in dtype.
 * ------------------------------------------------------------------------- */
size_t hclsm_colsum_workspace_size(int32_t C);
int hclsm_colsum(const float* a, float* out, int64_t rows, int32_t C, void* workspace, size_t workspace_bytes,
                 void* stream);
size_t hclsm_layernorm_bwd_workspace_size(int64_t rows, int32_t D);
int hclsm_layernorm_bwd(const float* x, const float* w, const float* dy, float* dx, float* dw, float* db, int64_t rows,
                        int32_t D, float eps, int32_t accumulate, void* workspace, size_t workspace_bytes,
                        void* stream);
int hclsm_gru_cell_bwd(const float* gi, const float* gh, const float* b_ih, const float* b_hh, const float* h,
                       const float* dh_new, float* d_gi, float* d_gh, float* dh, int64_t rows, int32_t H,
                       void* stream);
int hclsm_slot_softmax_bwd(const float* dots, const float* d_attn, void* attn, void* d_dots, int32_t F, int32_t N,
                           int32_t M, float scale, float clamp, float eps, int32_t dtype, void* stream);
int hclsm_residual_clamp_bwd(const float* h, const float* m, const float* b, const float* dout, float* dpre,
                             int64_t rows, int32_t C, float clamp, void* stream);
int hclsm_relu_bwd(const void* y, int32_t y_dtype, const float* dy, void* dx, int32_t dx_dtype, int64_t n,
                   void* stream);
int hclsm_swiglu_bwd(const float* u, const float* ds, void* du, int64_t rows, int32_t C, int32_t out_dtype,
                     void* stream);
int hclsm_event_mha_bwd(const void* qkv, const uint8_t* key_pad, const float* dout, void* dqkv, int32_t frames,
                        int32_t T, int32_t H, int32_t HD, float scale, int32_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Selective SSM scan, backward, without a caller workspace.
 * No counterpart in the reference: an addition for callers that cannot
 * allocate device memory when they run the backward (host callbacks, allocator
 * hooks, runtimes with a fixed memory plan).  Same arguments and outputs as
 * hclsm_ssm_scan_bwd minus the workspace; the scratch lives in a fixed device
 * array of hclsm_ssm_scan_bwd_noalloc_max_scratch() bytes (48 MiB) that every
 * GPU loading the library holds until exit.  Arguments are checked as
 * hclsm_ssm_scan_bwd checks them (same status codes); a valid problem that
 * needs more scratch than that returns HCLSM_ERR_WORKSPACE.  Calls on one
 * device share the array: calls that overlap on the GPU race.  The array's
 * address is resolved on the first call under each CUDA context (primary or
 * caller-created; a device reset makes a new one) and cached per context;
 * make that first call before any stream capture.
 * ------------------------------------------------------------------------- */
size_t hclsm_ssm_scan_bwd_noalloc_max_scratch(void);
int hclsm_ssm_scan_bwd_noalloc(const void* x, const void* dt, const float* A_log, const void* B,
                               const void* C, const float* D, const void* z, const void* dy, void* dx,
                               void* ddt, float* dA_log, void* dB, void* dC, float* dD, void* dz,
                               int64_t nseq, int32_t L, int32_t d_inner, int32_t d_state, int32_t dtype,
                               int32_t clamp, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HCLSM_B200_H_ */
