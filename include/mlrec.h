/*
 * mlrec.h - C ABI of the B200 scan library (libmlrec.so).
 *
 * One forward and one backward entry point per scan plug-in of
 * mlx-recurrence v0.3.0. Each pair replaces one reference plug-in's Metal
 * kernel launch plus its MLX epilogue:
 *
 *   mr_ssd_fwd     <- mlx_recurrence/ssd.py:54-135     (_ssd_forward_kernel)
 *   mr_ssd_bwd     <- mlx_recurrence/ssd.py:142-307    (_ssd_backward_kernel + mx.sum epilogue)
 *   mr_gla_fwd     <- mlx_recurrence/gla.py:49-123     (_gla_forward_kernel)
 *   mr_gla_bwd     <- mlx_recurrence/gla.py:130-270    (_gla_backward_kernel + mx.sum epilogue)
 *   mr_rglru_fwd   <- mlx_recurrence/rglru.py:64-123   (_rglru_forward_kernel)
 *   mr_rglru_bwd   <- mlx_recurrence/rglru.py:130-203  (_rglru_backward_kernel)
 *   mr_rotlru_fwd  <- mlx_recurrence/rotlru.py:80-146  (_rotlru_forward_kernel)
 *   mr_rotlru_bwd  <- mlx_recurrence/rotlru.py:153-266 (_rotlru_backward_kernel)
 *   mr_check_segment_shape <- mlx_recurrence/_chassis.py:92-115 (check_segment_shape)
 *
 * Conventions (all entry points):
 *   - Every data pointer is a CUDA device pointer owned by the caller;
 *     tensors are dense row-major in the shapes given below.
 *   - `dtype` selects the element type of the primal inputs and of the
 *     gradients written for them: MR_F32, MR_BF16 or MR_F16. Outputs y,
 *     h_ckpt and every state are float32, as in the reference (its
 *     output_dtypes are always mx.float32, e.g. ssd.py:128). All state
 *     and accumulation is float32.
 *   - `stream` is a cudaStream_t (passed as void*). Work is enqueued on it;
 *     no entry point synchronises the device or allocates memory.
 *   - Return value: MR_OK, or an MR_E_* code with a message available from
 *     mr_last_error() (thread-local). Shape errors are detected on the host
 *     before any launch, with the reference's messages.
 *   - Checkpoints h_ckpt hold the state at the end of every `seg`-step
 *     segment, in the reference's layouts; the last one is the final state.
 *   - `grad_final` (nullable) is the cotangent of the final state. The
 *     reference's VJPs drop it (ssd.py:334, gla.py:293, rglru.py:226,
 *     rotlru.py:288); here it seeds the adjoint, matching the reference's
 *     pure per-step loops.
 */
#ifndef MLREC_H_
#define MLREC_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MR_API __attribute__((visibility("default")))
#else
#define MR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MR_OK = 0,
  MR_E_SHAPE = 1,     /* shape rule violated (reference: ValueError)        */
  MR_E_DTYPE = 2,     /* unsupported dtype code                             */
  MR_E_ALIGN = 3,     /* a pointer is not 16-byte aligned                   */
  MR_E_LAUNCH = 4,    /* a CUDA launch failed                               */
  MR_E_WORKSPACE = 5, /* workspace missing or smaller than required         */
  MR_E_DEVICE = 6     /* no usable sm_100 device                             */
};

enum { MR_F32 = 0, MR_BF16 = 1, MR_F16 = 2 };

/* ABI revision of this header. */
MR_API int mr_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
MR_API const char* mr_last_error(void);

/* Number of kernels this library has launched in this process (all threads). */
MR_API uint64_t mr_launch_count(void);

/* Device-side error word of the current device's kernels: 0 = none,
 * 1 = a bounded wait on an asynchronous copy timed out (results invalid),
 * -1 = the word could not be read. Synchronises with the device; clear != 0
 * resets the word. While the word is set, every later wait that does not
 * complete at once gives up immediately (so a kernel whose copies stopped
 * arriving ends in about one 2 s limit), and results stay void until the
 * word is cleared. For diagnostics and tests. */
MR_API int mr_device_error_status(int clear);

/* Diagnostic (no reference counterpart): `ctas` CTAs each wait on a shared-memory
 * barrier that nothing completes, first with a `limit_ns` time limit, then with
 * the kernels' standard 2 s limit, and write both waits' durations (ns) to
 * elapsed_ns[2*cta], elapsed_ns[2*cta + 1] (device memory, uint64). The first
 * wait to run out sets the device error word; every wait after it gives up at
 * once. Checks the bounded-wait path without a fault: the context stays
 * usable, and mr_device_error_status(1) reads and clears the word. */
MR_API int mr_selftest_wait_timeout(int ctas, uint64_t limit_ns, uint64_t* elapsed_ns, void* stream);

/* Diagnostic (no reference counterpart): one 128x128x128 bf16 tcgen05 tile
 * per shared-memory operand form the chunked kernels use. A, Bk, Amn are
 * [128,128] bf16, Bmn [128,64] bf16 (row-major); D1 = A*Bk^T [128,128],
 * D2 = A*Bmn [128,64], D3 = Amn^T*Bmn [128,64], all f32. */
MR_API int mr_selftest_umma(const void* A, const void* Bk, const void* Bmn, const void* Amn,
                            float* D1, float* D2, float* D3, void* stream);

/* Shape rule of the checkpoint/recompute pattern: seg > 0, L % seg == 0 and
 * lane_dim % 32 == 0 (mlx_recurrence/_chassis.py:92-115). lane_name names
 * lane_dim in the message. Host-only, launches nothing. */
MR_API int mr_check_segment_shape(int64_t L, int64_t seg, int64_t lane_dim, const char* lane_name);

/* ---------------------------------------------------------------- SSD ---
 * u [B,L,H,Dh], delta [B,L,H], Bm/Cm [B,L,H,N] in `dtype`;
 * A_neg float32, element (h,n) at A_neg[h*a_stride_h + n*a_stride_n]
 *   (a_stride_n == 0: one decay rate per head, the Mamba-2 case);
 * y [B,L,H,Dh] f32; h_ckpt [B,L/seg,H,N,Dh] f32 (reference layout, ssd.py:67). */
MR_API int mr_ssd_fwd(const void* u, const void* delta, const void* Bm, const void* Cm,
               const float* A_neg, int64_t a_stride_h, int64_t a_stride_n, int dtype,
               int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t N, int64_t seg,
               float* y, float* h_ckpt, void* stream);

/* Checkpoint spacing to pass to mr_ssd_fwd/mr_ssd_bwd for the fastest path
 * when the caller only needs the segment rule L % seg == 0 and the final
 * state: the tensor-core chunk length (128) when seg divides it and the
 * chunked path applies (bf16/fp16, Dh = 64, N = 128, a_stride_n == 0,
 * L % 128 == 0), else seg unchanged. Host-only. */
MR_API int64_t mr_ssd_preferred_seg(int dtype, int64_t L, int64_t Dh, int64_t N, int64_t seg,
                                    int64_t a_stride_n);

/* Bytes of device workspace mr_ssd_bwd needs for these arguments. */
MR_API size_t mr_ssd_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                                  int64_t N, int64_t seg, int64_t a_stride_n);

/* grad_y [B,L,H,Dh] f32; grad_final [B,H,Dh,N] f32 or NULL;
 * grad_u/grad_delta/grad_B/grad_C in `dtype`; grad_A [H,N] f32 (summed over
 * the batch, ssd.py:305). With a_stride_n == 0 (one rate per head) row h of
 * grad_A holds d loss / d A_h divided evenly over its N entries, so that its
 * sum over n is the derivative for the per-head rate. */
MR_API int mr_ssd_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt,
               const void* u, const void* delta, const void* Bm, const void* Cm,
               const float* A_neg, int64_t a_stride_h, int64_t a_stride_n, int dtype,
               int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t N, int64_t seg,
               void* grad_u, void* grad_delta, void* grad_B, void* grad_C, float* grad_A,
               void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free SSD backward. No counterpart in the reference: it exists
 * for callers that cannot allocate device memory when the backward runs
 * (code inside an allocator's callback, where allocating would re-enter the
 * allocator, or embedders that own all device memory and only hand over
 * pre-placed buffers). Same arguments and results as mr_ssd_bwd
 * without the workspace; covers the tensor-core path only (bf16/f16, Dh=64,
 * N=128, a_stride_n == 0, seg == 128, L % 128 == 0; else MR_E_SHAPE). Its
 * scratch is a built-in 256 KiB device array per GPU (batch*H <= 65,536,
 * else MR_E_WORKSPACE). The first call in each CUDA context (the device's
 * primary context, or one the caller created and made current) looks up that
 * array's address in the context and caches it by the context's unique id
 * (make that call before any stream capture); all calls on a device share
 * the array, so calls that overlap on the GPU race. */
MR_API int mr_ssd_bwd_noalloc(const float* grad_y, const float* grad_final, const float* h_ckpt,
                              const void* u, const void* delta, const void* Bm, const void* Cm,
                              const float* A_neg, int64_t a_stride_h, int64_t a_stride_n, int dtype,
                              int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t N, int64_t seg,
                              void* grad_u, void* grad_delta, void* grad_B, void* grad_C, float* grad_A,
                              void* stream);

/* ---------------------------------------------------------------- GLA ---
 * q,k,v [B,L,H,Dh], gates [B,L,H] in `dtype`; y [B,L,H,Dh] f32;
 * h_ckpt [B,L/seg,H,Dh(i),Dh(j)] f32 (gla.py:62).
 * bf16/fp16 with Dh = 64, L % 128 == 0 and seg % 128 == 0 run on the tensor
 * cores (chunks of 128 steps); units (batch row, head) with a gate outside
 * [1e-3, 1] are then recomputed step by step, so every input gets the
 * per-step result. */
MR_API int mr_gla_fwd(const void* q, const void* k, const void* v, const void* gates, int dtype,
               int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg,
               float* y, float* h_ckpt, void* stream);

/* Checkpoint spacing for the fastest GLA path when the caller only needs the
 * segment rule and the final state: 128 when seg divides it and the
 * tensor-core path applies (bf16/fp16, Dh = 64, L % 128 == 0), else seg.
 * No reference counterpart (the reference always checkpoints at seg). Host-only. */
MR_API int64_t mr_gla_preferred_seg(int dtype, int64_t L, int64_t Dh, int64_t seg);

MR_API size_t mr_gla_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                                  int64_t seg);

/* grad_y [B,L,H,Dh] f32; grad_final [B,H,Dh,Dh] f32 or NULL; grads in `dtype`. */
MR_API int mr_gla_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt,
               const void* q, const void* k, const void* v, const void* gates, int dtype,
               int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg,
               void* grad_q, void* grad_k, void* grad_v, void* grad_gates,
               void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- RG-LRU ---
 * a, x [B,L,D] in `dtype`; y [B,L,D] f32; h_ckpt [B,L/seg,D] f32 (rglru.py:76). */
MR_API int mr_rglru_fwd(const void* a, const void* x, int dtype, int64_t batch, int64_t L, int64_t D,
                 int64_t seg, float* y, float* h_ckpt, void* stream);

/* Bytes of device workspace mr_rglru_bwd needs (0 unless seg > 64). */
MR_API size_t mr_rglru_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t D, int64_t seg);

/* grad_y [B,L,D] f32; grad_final [B,D] f32 or NULL; grad_a, grad_x in `dtype`.
 * workspace may be NULL when mr_rglru_bwd_workspace_bytes() returns 0. */
MR_API int mr_rglru_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt,
                 const void* a, const void* x, int dtype, int64_t batch, int64_t L, int64_t D,
                 int64_t seg, void* grad_a, void* grad_x, void* workspace,
                 size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- rotLRU ---
 * a, cs, sn [B,L,Dp], x [B,L,2*Dp] (pairs interleaved) in `dtype`;
 * y [B,L,2*Dp] f32; h_ckpt [B,L/seg,2*Dp] f32 (rotlru.py:87, 145). */
MR_API int mr_rotlru_fwd(const void* a, const void* cs, const void* sn, const void* x, int dtype,
                  int64_t batch, int64_t L, int64_t Dp, int64_t seg,
                  float* y, float* h_ckpt, void* stream);

/* Bytes of device workspace mr_rotlru_bwd needs (0 unless seg > 64). */
MR_API size_t mr_rotlru_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t Dp, int64_t seg);

/* grad_y [B,L,2Dp] f32; grad_final [B,2Dp] f32 or NULL; grads in `dtype`.
 * workspace may be NULL when mr_rotlru_bwd_workspace_bytes() returns 0. */
MR_API int mr_rotlru_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt,
                  const void* a, const void* cs, const void* sn, const void* x, int dtype,
                  int64_t batch, int64_t L, int64_t Dp, int64_t seg,
                  void* grad_a, void* grad_cs, void* grad_sn, void* grad_x,
                  void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------ initial state ---
 * No counterpart in the reference, which starts every scan from a zero state
 * and cannot resume from a returned final state (ssd.py:365-375). These
 * variants take the same arguments as the entry points above plus
 *   h0       the initial state, float32, in the final state's layout
 *            ([B,H,Dh,N] SSD, [B,H,Dh,Dh] GLA, [B,D] RG-LRU, [B,2Dp] rotLRU),
 *            or NULL for zero; forward and backward must get the same h0;
 *   grad_h0  (backward) the gradient of the loss w.r.t. h0, float32, same
 *            layout, or NULL when not wanted.
 * Passing the final state of one call as h0 of the next continues the scan
 * (chunked prefill). The plain entry points equal these with NULLs. */
MR_API int mr_ssd_fwd_h0(const void* u, const void* delta, const void* Bm, const void* Cm, const float* A_neg,
                         int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t L, int64_t H,
                         int64_t Dh, int64_t N, int64_t seg, float* y, float* h_ckpt, const float* h0,
                         void* stream);
MR_API int mr_ssd_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* u,
                         const void* delta, const void* Bm, const void* Cm, const float* A_neg,
                         int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t L, int64_t H,
                         int64_t Dh, int64_t N, int64_t seg, void* grad_u, void* grad_delta, void* grad_B,
                         void* grad_C, float* grad_A, void* workspace, size_t workspace_bytes, const float* h0,
                         float* grad_h0, void* stream);
MR_API int mr_gla_fwd_h0(const void* q, const void* k, const void* v, const void* gates, int dtype,
                         int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* h_ckpt,
                         const float* h0, void* stream);
MR_API int mr_gla_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* q,
                         const void* k, const void* v, const void* gates, int dtype, int64_t batch, int64_t L,
                         int64_t H, int64_t Dh, int64_t seg, void* grad_q, void* grad_k, void* grad_v,
                         void* grad_gates, void* workspace, size_t workspace_bytes, const float* h0,
                         float* grad_h0, void* stream);
MR_API int mr_rglru_fwd_h0(const void* a, const void* x, int dtype, int64_t batch, int64_t L, int64_t D,
                           int64_t seg, float* y, float* h_ckpt, const float* h0, void* stream);
MR_API int mr_rglru_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* a,
                           const void* x, int dtype, int64_t batch, int64_t L, int64_t D, int64_t seg,
                           void* grad_a, void* grad_x, void* workspace, size_t workspace_bytes,
                           const float* h0, float* grad_h0, void* stream);
MR_API int mr_rotlru_fwd_h0(const void* a, const void* cs, const void* sn, const void* x, int dtype,
                            int64_t batch, int64_t L, int64_t Dp, int64_t seg, float* y, float* h_ckpt,
                            const float* h0, void* stream);
MR_API int mr_rotlru_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* a,
                            const void* cs, const void* sn, const void* x, int dtype, int64_t batch, int64_t L,
                            int64_t Dp, int64_t seg, void* grad_a, void* grad_cs, void* grad_sn, void* grad_x,
                            void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0,
                            void* stream);

/* ------------------------------------------------------ Gated DeltaNet ---
 * A recurrence the reference carries as a design only
 * (docs/DESIGN_gated_deltanet.md), built from its pinned recurrence
 * (section 1, R1''/R2') and adjoint (section 4): per (batch row, head) a state
 * S [Dh(i), Dh(j)] with
 *   S_t = alpha_t (I - beta_t k_t k_t^T) S_{t-1} + beta_t k_t v_t^T,
 *   y_t = S_t^T q_t.
 * q, k, v [B,L,H,Dh] (q, k L2-normalised by the caller) and alpha, beta [B,L,H]
 * (already activated: alpha in (0,1], beta in (0,1) for a contraction) in
 * `dtype`; y [B,L,H,Dh] float32; h_ckpt [B, L/seg, H, Dh, Dh] float32 (the state
 * after each segment, i-major; the last is the final state); h0 / grad_h0
 * [B,H,Dh,Dh] float32 or NULL. Dh must be 32 or 64 and L a multiple of seg.
 * step_cache [B,L,H,Dh] float32 receives, per step, w_t = beta (v - alpha
 * S_{t-1}^T k) (NULL in the forward: not kept); the backward reads it
 * (required there) so that it replays states without the dot products.
 * With 2-byte inputs, Dh = 64, L a multiple of 128, seg a multiple of 64 and
 * fewer (batch, head) units than twice the device's SMs, the forward runs in
 * chunkwise (WY) form when given mr_gdn_fwd_workspace_bytes of device workspace
 * (0 bytes when it does not apply; NULL or too small: the per-step form, same
 * results within the parity tolerance). The backward writes grad_q, grad_k, grad_v, grad_alpha,
 * grad_beta in `dtype` and needs mr_gdn_bwd_workspace_bytes of device scratch. */
MR_API int mr_gdn_fwd(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int dtype,
                      int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* h_ckpt,
                      float* step_cache, const float* h0, void* workspace, size_t workspace_bytes, void* stream);
MR_API size_t mr_gdn_fwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg);
MR_API size_t mr_gdn_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg);
MR_API int mr_gdn_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const float* step_cache,
                      const void* q, const void* k, const void* v, const void* alpha, const void* beta, int dtype, int64_t batch,
                      int64_t L, int64_t H, int64_t Dh, int64_t seg, void* grad_q, void* grad_k, void* grad_v,
                      void* grad_alpha, void* grad_beta, void* workspace, size_t workspace_bytes, const float* h0,
                      float* grad_h0, void* stream);

/* One Gated DeltaNet decode step: state [B,H,Dh,Dh] float32 (the final state's
 * layout) advanced in place by one step of the recurrence above; q, k, v
 * [B,H,Dh] and alpha, beta [B,H] in `dtype`; y [B,H,Dh] float32. */
MR_API int mr_gdn_step(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int dtype,
                       int64_t batch, int64_t H, int64_t Dh, float* state, float* y, void* stream);

/* ------------------------------------------------- rotLRU, angle input ---
 * The rotLRU scan taking the rotation angle theta [B,L,Dp] in place of cs, sn
 * (no counterpart in the reference, which forms cos and sin in MLX host code
 * and passes both through HBM, rotlru.py:18-22): the kernels form
 * cos(theta), sin(theta) in float32 as they load each tile, so the scan reads
 * four streams instead of five and the backward writes grad_theta =
 * cos(theta) grad_sn - sin(theta) grad_cs directly. Everything else (layout,
 * h_ckpt, h0, workspace size from mr_rotlru_bwd_workspace_bytes) is as in
 * mr_rotlru_fwd_h0 / mr_rotlru_bwd_h0; h0 and grad_h0 may be NULL. */
MR_API int mr_rotlru_angle_fwd(const void* a, const void* theta, const void* x, int dtype, int64_t batch,
                               int64_t L, int64_t Dp, int64_t seg, float* y, float* h_ckpt, const float* h0,
                               void* stream);
MR_API int mr_rotlru_angle_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* a,
                               const void* theta, const void* x, int dtype, int64_t batch, int64_t L,
                               int64_t Dp, int64_t seg, void* grad_a, void* grad_theta, void* grad_x,
                               void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0,
                               void* stream);

/* ------------------------------------------------------ gated RG-LRU ---
 * The RG-LRU scan with its input gating folded in (no counterpart in the
 * reference, which leaves the gating to MLX host code, rglru.py:8-27, and
 * takes a, b through HBM): inputs x, r (activated recurrence gate), i
 * (activated input gate) [B,L,D] in `dtype` and lam [D] float32;
 *   a_t = sigmoid(lam)^(c r_t),  b_t = sqrt(1 - a_t^2) i_t x_t,
 *   h_t = a_t h_{t-1} + b_t,     y_t = h_t.
 * y, h_ckpt, h0 as in mr_rglru_fwd(_h0). The backward returns the gradients of
 * x, r, i (in `dtype`) and of lam (float32 [D], summed over batch and time). */
MR_API int mr_rglru_gated_fwd(const void* x, const void* r, const void* i, const float* lam, float c, int dtype,
                              int64_t batch, int64_t L, int64_t D, int64_t seg, float* y, float* h_ckpt,
                              const float* h0, void* stream);
MR_API size_t mr_rglru_gated_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t D, int64_t seg);
MR_API int mr_rglru_gated_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* x,
                              const void* r, const void* i, const float* lam, float c, int dtype, int64_t batch,
                              int64_t L, int64_t D, int64_t seg, void* grad_x, void* grad_r, void* grad_i,
                              float* grad_lam, void* workspace, size_t workspace_bytes, const float* h0,
                              float* grad_h0, void* stream);

/* -------------------------------------------------------- decode steps ---
 * No counterpart in the reference (a decode step there is a scan of length 1,
 * one Metal dispatch per call). One time step of the recurrence for a batch of
 * sequences: `state` (float32, the final state's layout, as above) is advanced
 * in place and y receives the step's output (float32). Inputs are one token's
 * slices in `dtype`:
 *   SSD:    u [B,H,Dh], delta [B,H], Bm/Cm [B,H,N], A_neg as in mr_ssd_fwd
 *           (N <= 128); y [B,H,Dh]
 *   GLA:    q,k,v [B,H,Dh], gates [B,H] (Dh <= 128); y [B,H,Dh]
 *   RG-LRU: a, x [B,D]; y [B,D]
 *   rotLRU: a, cs, sn [B,Dp], x [B,2Dp]; y [B,2Dp]
 * The update is one step of the reference's pure loops (ssd.py:382-394,
 * gla.py:336-346, rglru.py:274-282, rotlru.py:338-351). */
MR_API int mr_ssd_step(const void* u, const void* delta, const void* Bm, const void* Cm, const float* A_neg,
                       int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t H, int64_t Dh,
                       int64_t N, float* state, float* y, void* stream);
MR_API int mr_gla_step(const void* q, const void* k, const void* v, const void* gates, int dtype, int64_t batch,
                       int64_t H, int64_t Dh, float* state, float* y, void* stream);
MR_API int mr_rglru_step(const void* a, const void* x, int dtype, int64_t batch, int64_t D, float* state,
                         float* y, void* stream);
MR_API int mr_rotlru_step(const void* a, const void* cs, const void* sn, const void* x, int dtype,
                          int64_t batch, int64_t Dp, float* state, float* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLREC_H_ */
