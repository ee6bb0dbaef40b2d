// extern "C" entry points of libmlrec.so (declared in include/mlrec.h):
// host-side validation with the reference's messages, dtype dispatch and
// launch of the scan kernels. Nothing here allocates or synchronises.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "common.cuh"

namespace mr {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<uint64_t> g_launches{0};

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MR_E_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return MR_OK;
}

// ---- launchers defined in the kernel translation units ----------------------
// (h0: initial state or NULL; gh0: its gradient or NULL; both in the final state's layout)
template <typename T> int rglru_fwd_launch(const void*, const void*, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int rglru_bwd_launch(const float*, const float*, const float*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, void*, void*, float*, const float*, float*, cudaStream_t);
template <typename T> int rotlru_fwd_launch(const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int rotlru_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, float*, const float*, float*, cudaStream_t);
template <typename T> int ssd_seq_fwd_launch(const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t, int);
template <typename T> int ssd_seq_bwd_marked_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, float*, void*, const float*, float*, cudaStream_t);
size_t ssd_fallback_ws_bytes(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t);
bool ssd_dense_chunk_supported(int dtype, int64_t L, int64_t Dh, int64_t N, int64_t seg, int64_t a_stride_n);
template <typename T> int ssd_dense_chunk_fwd_launch(const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int ssd_dense_chunk_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, float*, const float*, float*, cudaStream_t);
template <typename T> int ssd_seq_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, float*, void*, const float*, float*, cudaStream_t);
template <typename T> int gla_seq_fwd_launch(const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t, int);
template <typename T> int gla_seq_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, void*, const float*, float*, cudaStream_t, int);
template <typename T> int gla_chunk_fwd_launch(const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int gla_chunk_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, const float*, float*, cudaStream_t);
bool gla_chunk_supported(int dtype, int64_t L, int64_t Dh, int64_t seg);
size_t gla_fallback_ws_bytes(int64_t, int64_t, int64_t, int64_t, int64_t);
size_t rglru_bwd_ws_bytes(int64_t, int64_t, int64_t, int64_t);
size_t rotlru_bwd_ws_bytes(int64_t, int64_t, int64_t, int64_t);
size_t ssd_seq_bwd_ws_bytes(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t);
size_t gla_seq_bwd_ws_bytes(int64_t, int64_t, int64_t, int64_t, int64_t);
bool ssd_seq_supported(int64_t Dh, int64_t N);
bool gla_seq_supported(int64_t Dh);
int diag_device_error(bool clear);
int selftest_device_error(bool clear);
int ssdc_device_error(bool clear);
bool ssd_chunk_supported(int dtype, int64_t L, int64_t Dh, int64_t N, int64_t seg, int64_t a_stride_n);
bool ssd_chunk_bwd_supported(int dtype, int64_t L, int64_t Dh, int64_t N, int64_t seg, int64_t a_stride_n);
int ssd_chunk_len();
size_t ssd_chunk_bwd_ws_bytes(int64_t batch, int64_t H);
int ssd_chunk_bwd_noalloc(int dtype, const float*, const float*, const float*, const void*, const void*,
                          const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                          void*, void*, void*, void*, float*, cudaStream_t);
template <typename T> int ssd_chunk_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, float*, float*, const float*, float*, cudaStream_t);
template <typename T> int ssd_chunk_fwd_launch(const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int ssd_step_launch(const void*, const void*, const void*, const void*, const float*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, cudaStream_t);
template <typename T> int gla_step_launch(const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, float*, float*, cudaStream_t);
template <typename T> int rglru_step_launch(const void*, const void*, int64_t, int64_t, float*, float*, cudaStream_t);
template <typename T> int rotlru_step_launch(const void*, const void*, const void*, const void*, int64_t, int64_t, float*, float*, cudaStream_t);
template <typename T> int rglru_gated_fwd_launch(const void*, const void*, const void*, const float*, float, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int rglru_gated_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, const float*, float, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, float*, void*, const float*, float*, cudaStream_t);
size_t rglru_gated_bwd_ws_bytes(int64_t, int64_t, int64_t, int64_t);
template <typename T> int gdn_fwd_launch(const void*, const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, int64_t, float*, float*, float*, const float*, void*, size_t, cudaStream_t);
size_t gdn_fwd_ws_bytes(int, int64_t, int64_t, int64_t, int64_t, int64_t);
template <typename T> int gdn_bwd_launch(const float*, const float*, const float*, const float*, const void*, const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, void*, void*, void*, const float*, float*, cudaStream_t);
size_t gdn_bwd_ws_bytes(int64_t, int64_t, int64_t, int64_t, int64_t);
template <typename T> int gdn_step_launch(const void*, const void*, const void*, const void*, const void*, int64_t, int64_t, int64_t, float*, float*, cudaStream_t);
template <typename T> int rotlru_angle_fwd_launch(const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, float*, float*, const float*, cudaStream_t);
template <typename T> int rotlru_angle_bwd_launch(const float*, const float*, const float*, const void*, const void*, const void*, int64_t, int64_t, int64_t, int64_t, void*, void*, void*, float*, const float*, float*, cudaStream_t);
int umma_selftest_launch(const void*, const void*, const void*, const void*, float*, float*, float*,
                         cudaStream_t);
int wait_selftest_launch(int, uint64_t, uint64_t*, cudaStream_t);

// ---- validation helpers -----------------------------------------------------
static int check_seg(int64_t L, int64_t seg, int64_t lane_dim, const char* lane_name) {
  // messages: mlx_recurrence/_chassis.py:104-115
  if (seg <= 0) return set_error(MR_E_SHAPE, "seg must be positive, got %lld", (long long)seg);
  if (L % seg != 0)
    return set_error(MR_E_SHAPE,
                     "sequence length L=%lld must be divisible by seg=%lld (segment-checkpoint "
                     "pattern tiles L into L/seg segments)",
                     (long long)L, (long long)seg);
  if (lane_dim % 32 != 0)
    return set_error(MR_E_SHAPE,
                     "%s=%lld must be a multiple of 32 (fused gradient reductions use 32-lane "
                     "simdgroups)",
                     lane_name, (long long)lane_dim);
  return MR_OK;
}

static int check_dims(const char* what, int64_t batch, int64_t L, int64_t other) {
  if (batch <= 0 || L <= 0 || other <= 0)
    return set_error(MR_E_SHAPE, "%s: every dimension must be positive", what);
  if (L > (int64_t)INT32_MAX / 2) return set_error(MR_E_SHAPE, "%s: L=%lld too large", what, (long long)L);
  if (batch > 65535) return set_error(MR_E_SHAPE, "%s: batch=%lld exceeds 65535", what, (long long)batch);
  return MR_OK;
}

static int check_dtype(int dtype) {
  if (dtype != MR_F32 && dtype != MR_BF16 && dtype != MR_F16)
    return set_error(MR_E_DTYPE, "unsupported dtype code %d (0=f32, 1=bf16, 2=f16)", dtype);
  return MR_OK;
}

static int check_ptrs(const char* what, std::initializer_list<const void*> ps) {
  int i = 0;
  for (const void* p : ps) {
    if (p == nullptr) return set_error(MR_E_ALIGN, "%s: pointer argument %d is NULL", what, i);
    if (((uintptr_t)p) & 15u)
      return set_error(MR_E_ALIGN, "%s: pointer argument %d is not 16-byte aligned", what, i);
    ++i;
  }
  return MR_OK;
}

static int check_opt_ptr(const char* what, const void* p) {
  if (p != nullptr && (((uintptr_t)p) & 15u))
    return set_error(MR_E_ALIGN, "%s: optional pointer is not 16-byte aligned", what);
  return MR_OK;
}

#define MR_TRY(x)              \
  do {                         \
    const int rc_ = (x);       \
    if (rc_ != MR_OK) return rc_; \
  } while (0)

#define MR_DTYPE_SWITCH(dtype, CALL)                 \
  switch (dtype) {                                   \
    case MR_F32: { using T = float; return CALL; }   \
    case MR_BF16: { using T = __nv_bfloat16; return CALL; } \
    default: { using T = __half; return CALL; }      \
  }

}  // namespace mr

using namespace mr;

extern "C" {

// 2: the _h0 (initial state) entry points; 3: the decode steps; 4: the gated RG-LRU scan
int mr_abi_version(void) { return 7; }

const char* mr_last_error(void) { return g_err; }

uint64_t mr_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int mr_device_error_status(int clear) {
  const int words[] = {diag_device_error(clear != 0), selftest_device_error(clear != 0),
                       ssdc_device_error(clear != 0)};
  int r = 0;
  for (int w : words) {
    if (w < 0) return -1;
    if (r == 0) r = w;
  }
  return r;
}

int mr_selftest_umma(const void* A, const void* Bk, const void* Bmn, const void* Amn, float* D1,
                     float* D2, float* D3, void* stream) {
  g_err[0] = 0;
  MR_TRY(check_ptrs("mr_selftest_umma", {A, Bk, Bmn, Amn, D1, D2, D3}));
  return umma_selftest_launch(A, Bk, Bmn, Amn, D1, D2, D3, (cudaStream_t)stream);
}

int mr_selftest_wait_timeout(int ctas, uint64_t limit_ns, uint64_t* elapsed_ns, void* stream) {
  g_err[0] = 0;
  if (ctas <= 0 || ctas > 1024) return set_error(MR_E_SHAPE, "mr_selftest_wait_timeout: ctas must be 1..1024");
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return set_error(MR_E_SHAPE, "mr_selftest_wait_timeout: limit_ns must be 1..1e9");
  MR_TRY(check_ptrs("mr_selftest_wait_timeout", {elapsed_ns}));
  return wait_selftest_launch(ctas, limit_ns, elapsed_ns, (cudaStream_t)stream);
}

int mr_check_segment_shape(int64_t L, int64_t seg, int64_t lane_dim, const char* lane_name) {
  g_err[0] = 0;
  return check_seg(L, seg, lane_dim, lane_name ? lane_name : "lane dimension");
}

// ------------------------------------------------------------------ RG-LRU ---
int mr_rglru_fwd(const void* a, const void* x, int dtype, int64_t batch, int64_t L, int64_t D,
                 int64_t seg, float* y, float* h_ckpt, void* stream) {
  return mr_rglru_fwd_h0(a, x, dtype, batch, L, D, seg, y, h_ckpt, nullptr, stream);
}

int mr_rglru_fwd_h0(const void* a, const void* x, int dtype, int64_t batch, int64_t L, int64_t D,
                    int64_t seg, float* y, float* h_ckpt, const float* h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rglru_fwd", batch, L, D));
  MR_TRY(check_seg(L, seg, D, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rglru_fwd", {a, x, y, h_ckpt}));
  cudaStream_t st = (cudaStream_t)stream;
  MR_TRY(check_opt_ptr("mr_rglru_fwd", h0));
  MR_DTYPE_SWITCH(dtype, rglru_fwd_launch<T>(a, x, batch, L, D, seg, y, h_ckpt, h0, st));
}

size_t mr_rglru_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t D, int64_t seg) {
  (void)dtype;
  if (batch <= 0 || L <= 0 || D <= 0 || seg <= 0) return 0;
  return rglru_bwd_ws_bytes(batch, L, D, seg);
}

int mr_rglru_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt,
                    const void* a, const void* x, int dtype, int64_t batch, int64_t L, int64_t D,
                    int64_t seg, void* grad_a, void* grad_x, void* workspace,
                    size_t workspace_bytes, void* stream) {
  return mr_rglru_bwd_h0(grad_y, grad_final, h_ckpt, a, x, dtype, batch, L, D, seg, grad_a, grad_x, workspace,
                         workspace_bytes, nullptr, nullptr, stream);
}

int mr_rglru_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* a,
                    const void* x, int dtype, int64_t batch, int64_t L, int64_t D, int64_t seg, void* grad_a,
                    void* grad_x, void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0,
                    void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rglru_bwd", batch, L, D));
  MR_TRY(check_seg(L, seg, D, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rglru_bwd", {grad_y, h_ckpt, a, x, grad_a, grad_x}));
  MR_TRY(check_opt_ptr("mr_rglru_bwd", grad_final));
  const size_t need = rglru_bwd_ws_bytes(batch, L, D, seg);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(MR_E_WORKSPACE, "mr_rglru_bwd: workspace of %zu bytes required, got %zu",
                     need, workspace_bytes);
  MR_TRY(check_opt_ptr("mr_rglru_bwd", workspace));
  MR_TRY(check_opt_ptr("mr_rglru_bwd", h0));
  MR_TRY(check_opt_ptr("mr_rglru_bwd", grad_h0));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rglru_bwd_launch<T>(grad_y, grad_final, h_ckpt, a, x, batch, L, D, seg,
                                             grad_a, grad_x, (float*)workspace, h0, grad_h0, st));
}

int mr_rglru_gated_fwd(const void* x, const void* r, const void* i, const float* lam, float c, int dtype,
                       int64_t batch, int64_t L, int64_t D, int64_t seg, float* y, float* h_ckpt, const float* h0,
                       void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rglru_gated_fwd", batch, L, D));
  MR_TRY(check_seg(L, seg, D, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rglru_gated_fwd", {x, r, i, lam, y, h_ckpt}));
  MR_TRY(check_opt_ptr("mr_rglru_gated_fwd", h0));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rglru_gated_fwd_launch<T>(x, r, i, lam, c, batch, L, D, seg, y, h_ckpt, h0, st));
}

size_t mr_rglru_gated_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t D, int64_t seg) {
  (void)dtype;
  if (batch <= 0 || L <= 0 || D <= 0 || seg <= 0) return 0;
  return rglru_gated_bwd_ws_bytes(batch, L, D, seg);
}

int mr_rglru_gated_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* x,
                       const void* r, const void* i, const float* lam, float c, int dtype, int64_t batch, int64_t L,
                       int64_t D, int64_t seg, void* grad_x, void* grad_r, void* grad_i, float* grad_lam,
                       void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rglru_gated_bwd", batch, L, D));
  MR_TRY(check_seg(L, seg, D, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rglru_gated_bwd", {grad_y, h_ckpt, x, r, i, lam, grad_x, grad_r, grad_i, grad_lam}));
  MR_TRY(check_opt_ptr("mr_rglru_gated_bwd", grad_final));
  MR_TRY(check_opt_ptr("mr_rglru_gated_bwd", h0));
  MR_TRY(check_opt_ptr("mr_rglru_gated_bwd", grad_h0));
  const size_t need = rglru_gated_bwd_ws_bytes(batch, L, D, seg);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(MR_E_WORKSPACE, "mr_rglru_gated_bwd: workspace of %zu bytes required, got %zu", need,
                     workspace_bytes);
  MR_TRY(check_opt_ptr("mr_rglru_gated_bwd", workspace));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rglru_gated_bwd_launch<T>(grad_y, grad_final, h_ckpt, x, r, i, lam, c, batch, L, D, seg,
                                                   grad_x, grad_r, grad_i, grad_lam, workspace, h0, grad_h0, st));
}

// ------------------------------------------------------------------ rotLRU ---
int mr_rotlru_fwd(const void* a, const void* cs, const void* sn, const void* x, int dtype,
                  int64_t batch, int64_t L, int64_t Dp, int64_t seg, float* y, float* h_ckpt,
                  void* stream) {
  return mr_rotlru_fwd_h0(a, cs, sn, x, dtype, batch, L, Dp, seg, y, h_ckpt, nullptr, stream);
}

int mr_rotlru_fwd_h0(const void* a, const void* cs, const void* sn, const void* x, int dtype, int64_t batch,
                     int64_t L, int64_t Dp, int64_t seg, float* y, float* h_ckpt, const float* h0,
                     void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rotlru_fwd", batch, L, Dp));
  MR_TRY(check_seg(L, seg, 2 * Dp, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rotlru_fwd", {a, cs, sn, x, y, h_ckpt}));
  cudaStream_t st = (cudaStream_t)stream;
  MR_TRY(check_opt_ptr("mr_rotlru_fwd", h0));
  MR_DTYPE_SWITCH(dtype, rotlru_fwd_launch<T>(a, cs, sn, x, batch, L, Dp, seg, y, h_ckpt, h0, st));
}

size_t mr_rotlru_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t Dp, int64_t seg) {
  (void)dtype;
  if (batch <= 0 || L <= 0 || Dp <= 0 || seg <= 0) return 0;
  return rotlru_bwd_ws_bytes(batch, L, Dp, seg);
}

int mr_rotlru_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt,
                     const void* a, const void* cs, const void* sn, const void* x, int dtype,
                     int64_t batch, int64_t L, int64_t Dp, int64_t seg, void* grad_a,
                     void* grad_cs, void* grad_sn, void* grad_x, void* workspace,
                     size_t workspace_bytes, void* stream) {
  return mr_rotlru_bwd_h0(grad_y, grad_final, h_ckpt, a, cs, sn, x, dtype, batch, L, Dp, seg, grad_a, grad_cs,
                          grad_sn, grad_x, workspace, workspace_bytes, nullptr, nullptr, stream);
}

int mr_rotlru_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* a,
                     const void* cs, const void* sn, const void* x, int dtype, int64_t batch, int64_t L,
                     int64_t Dp, int64_t seg, void* grad_a, void* grad_cs, void* grad_sn, void* grad_x,
                     void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0,
                     void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rotlru_bwd", batch, L, Dp));
  MR_TRY(check_seg(L, seg, 2 * Dp, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rotlru_bwd", {grad_y, h_ckpt, a, cs, sn, x, grad_a, grad_cs, grad_sn, grad_x}));
  MR_TRY(check_opt_ptr("mr_rotlru_bwd", grad_final));
  const size_t need = rotlru_bwd_ws_bytes(batch, L, Dp, seg);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(MR_E_WORKSPACE, "mr_rotlru_bwd: workspace of %zu bytes required, got %zu",
                     need, workspace_bytes);
  MR_TRY(check_opt_ptr("mr_rotlru_bwd", workspace));
  MR_TRY(check_opt_ptr("mr_rotlru_bwd", h0));
  MR_TRY(check_opt_ptr("mr_rotlru_bwd", grad_h0));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rotlru_bwd_launch<T>(grad_y, grad_final, h_ckpt, a, cs, sn, x, batch, L,
                                              Dp, seg, grad_a, grad_cs, grad_sn, grad_x,
                                              (float*)workspace, h0, grad_h0, st));
}

int mr_rotlru_angle_fwd(const void* a, const void* theta, const void* x, int dtype, int64_t batch, int64_t L,
                        int64_t Dp, int64_t seg, float* y, float* h_ckpt, const float* h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rotlru_angle_fwd", batch, L, Dp));
  MR_TRY(check_seg(L, seg, 2 * Dp, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rotlru_angle_fwd", {a, theta, x, y, h_ckpt}));
  MR_TRY(check_opt_ptr("mr_rotlru_angle_fwd", h0));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rotlru_angle_fwd_launch<T>(a, theta, x, batch, L, Dp, seg, y, h_ckpt, h0, st));
}

int mr_rotlru_angle_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* a,
                        const void* theta, const void* x, int dtype, int64_t batch, int64_t L, int64_t Dp,
                        int64_t seg, void* grad_a, void* grad_theta, void* grad_x, void* workspace,
                        size_t workspace_bytes, const float* h0, float* grad_h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(check_dims("mr_rotlru_angle_bwd", batch, L, Dp));
  MR_TRY(check_seg(L, seg, 2 * Dp, "D"));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rotlru_angle_bwd", {grad_y, h_ckpt, a, theta, x, grad_a, grad_theta, grad_x}));
  MR_TRY(check_opt_ptr("mr_rotlru_angle_bwd", grad_final));
  const size_t need = rotlru_bwd_ws_bytes(batch, L, Dp, seg);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return set_error(MR_E_WORKSPACE, "mr_rotlru_angle_bwd: workspace of %zu bytes required, got %zu", need,
                     workspace_bytes);
  MR_TRY(check_opt_ptr("mr_rotlru_angle_bwd", workspace));
  MR_TRY(check_opt_ptr("mr_rotlru_angle_bwd", h0));
  MR_TRY(check_opt_ptr("mr_rotlru_angle_bwd", grad_h0));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rotlru_angle_bwd_launch<T>(grad_y, grad_final, h_ckpt, a, theta, x, batch, L, Dp, seg,
                                                    grad_a, grad_theta, grad_x, (float*)workspace, h0, grad_h0,
                                                    st));
}

// ---------------------------------------------------------- Gated DeltaNet ---
static int gdn_common_checks(const char* what, int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                             int64_t seg) {
  MR_TRY(check_dims(what, batch, L, H));
  if (Dh != 32 && Dh != 64)
    return set_error(MR_E_SHAPE, "%s: Dh=%lld is not supported (32 or 64)", what, (long long)Dh);
  MR_TRY(check_seg(L, seg, Dh, "Dh"));
  if (batch * H > (int64_t)INT32_MAX) return set_error(MR_E_SHAPE, "%s: batch*H too large", what);
  return check_dtype(dtype);
}

int mr_gdn_fwd(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int dtype,
               int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* h_ckpt,
               float* step_cache, const float* h0, void* workspace, size_t workspace_bytes, void* stream) {
  g_err[0] = 0;
  MR_TRY(gdn_common_checks("mr_gdn_fwd", dtype, batch, L, H, Dh, seg));
  MR_TRY(check_ptrs("mr_gdn_fwd", {q, k, v, alpha, beta, y, h_ckpt}));
  MR_TRY(check_opt_ptr("mr_gdn_fwd", step_cache));
  MR_TRY(check_opt_ptr("mr_gdn_fwd", h0));
  MR_TRY(check_opt_ptr("mr_gdn_fwd", workspace));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, gdn_fwd_launch<T>(q, k, v, alpha, beta, batch, L, H, Dh, seg, y, h_ckpt, step_cache, h0,
                                           workspace, workspace_bytes, st));
}

size_t mr_gdn_fwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  if (batch <= 0 || L <= 0 || H <= 0 || Dh <= 0 || seg <= 0) return 0;
  if (dtype != MR_F32 && dtype != MR_BF16 && dtype != MR_F16) return 0;
  return gdn_fwd_ws_bytes(dtype == MR_F32 ? 4 : 2, batch, L, H, Dh, seg);
}

size_t mr_gdn_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg) {
  (void)dtype;
  if (batch <= 0 || L <= 0 || H <= 0 || Dh <= 0 || seg <= 0) return 0;
  return gdn_bwd_ws_bytes(batch, L, H, Dh, seg);
}

int mr_gdn_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const float* step_cache,
               const void* q, const void* k,
               const void* v, const void* alpha, const void* beta, int dtype, int64_t batch, int64_t L, int64_t H,
               int64_t Dh, int64_t seg, void* grad_q, void* grad_k, void* grad_v, void* grad_alpha,
               void* grad_beta, void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0,
               void* stream) {
  g_err[0] = 0;
  MR_TRY(gdn_common_checks("mr_gdn_bwd", dtype, batch, L, H, Dh, seg));
  MR_TRY(check_ptrs("mr_gdn_bwd", {grad_y, h_ckpt, step_cache, q, k, v, alpha, beta, grad_q, grad_k, grad_v,
                                   grad_alpha, grad_beta, workspace}));
  MR_TRY(check_opt_ptr("mr_gdn_bwd", grad_final));
  MR_TRY(check_opt_ptr("mr_gdn_bwd", h0));
  MR_TRY(check_opt_ptr("mr_gdn_bwd", grad_h0));
  const size_t need = gdn_bwd_ws_bytes(batch, L, H, Dh, seg);
  if (workspace_bytes < need)
    return set_error(MR_E_WORKSPACE, "mr_gdn_bwd: workspace of %zu bytes required, got %zu", need,
                     workspace_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, gdn_bwd_launch<T>(grad_y, grad_final, h_ckpt, step_cache, q, k, v, alpha, beta, batch, L, H, Dh, seg,
                                           grad_q, grad_k, grad_v, grad_alpha, grad_beta, workspace, h0, grad_h0,
                                           st));
}

int mr_gdn_step(const void* q, const void* k, const void* v, const void* alpha, const void* beta, int dtype,
                int64_t batch, int64_t H, int64_t Dh, float* state, float* y, void* stream) {
  g_err[0] = 0;
  MR_TRY(gdn_common_checks("mr_gdn_step", dtype, batch, 1, H, Dh, 1));
  MR_TRY(check_ptrs("mr_gdn_step", {q, k, v, alpha, beta, state, y}));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, gdn_step_launch<T>(q, k, v, alpha, beta, batch, H, Dh, state, y, st));
}

// --------------------------------------------------------------------- SSD ---
static int ssd_common_checks(const char* what, int dtype, int64_t batch, int64_t L, int64_t H,
                             int64_t Dh, int64_t N, int64_t seg) {
  MR_TRY(check_dims(what, batch, L, H));
  if (Dh <= 0 || N <= 0) return set_error(MR_E_SHAPE, "%s: every dimension must be positive", what);
  MR_TRY(check_seg(L, seg, Dh, "Dh"));
  MR_TRY(check_dtype(dtype));
  if (!ssd_seq_supported(Dh, N))
    return set_error(MR_E_SHAPE, "%s: this build supports Dh in {32,64,96,128} and N <= 128, got Dh=%lld N=%lld",
                     what, (long long)Dh, (long long)N);
  if (batch * H > (int64_t)INT32_MAX) return set_error(MR_E_SHAPE, "%s: batch*H too large", what);
  return MR_OK;
}

int mr_ssd_fwd(const void* u, const void* delta, const void* Bm, const void* Cm, const float* A_neg,
               int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t L,
               int64_t H, int64_t Dh, int64_t N, int64_t seg, float* y, float* h_ckpt,
               void* stream) {
  return mr_ssd_fwd_h0(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, dtype, batch, L, H, Dh, N, seg, y, h_ckpt,
                       nullptr, stream);
}

int mr_ssd_fwd_h0(const void* u, const void* delta, const void* Bm, const void* Cm, const float* A_neg,
                  int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t L, int64_t H,
                  int64_t Dh, int64_t N, int64_t seg, float* y, float* h_ckpt, const float* h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(ssd_common_checks("mr_ssd_fwd", dtype, batch, L, H, Dh, N, seg));
  MR_TRY(check_ptrs("mr_ssd_fwd", {u, delta, Bm, Cm, y, h_ckpt}));
  if (A_neg == nullptr) return set_error(MR_E_ALIGN, "mr_ssd_fwd: A_neg is NULL");
  MR_TRY(check_opt_ptr("mr_ssd_fwd", h0));
  cudaStream_t st = (cudaStream_t)stream;
  if (ssd_chunk_supported(dtype, L, Dh, N, seg, a_stride_n)) {
    if (dtype == MR_BF16)
      return ssd_chunk_fwd_launch<__nv_bfloat16>(u, delta, Bm, Cm, A_neg, a_stride_h, batch, L, H, seg, y,
                                                 h_ckpt, h0, st);
    return ssd_chunk_fwd_launch<__half>(u, delta, Bm, Cm, A_neg, a_stride_h, batch, L, H, seg, y, h_ckpt, h0,
                                        st);
  }
  if (ssd_dense_chunk_supported(dtype, L, Dh, N, seg, a_stride_n)) {
    // dense A_neg on the tensor cores, then the per-step kernel for the units it marked
    if (dtype == MR_BF16) {
      MR_TRY(ssd_dense_chunk_fwd_launch<__nv_bfloat16>(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, batch, L,
                                                        H, seg, y, h_ckpt, h0, st));
      return ssd_seq_fwd_launch<__nv_bfloat16>(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, batch, L, H, Dh,
                                               N, seg, y, h_ckpt, h0, st, 1);
    }
    MR_TRY(ssd_dense_chunk_fwd_launch<__half>(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, batch, L, H, seg,
                                               y, h_ckpt, h0, st));
    return ssd_seq_fwd_launch<__half>(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, batch, L, H, Dh, N, seg,
                                      y, h_ckpt, h0, st, 1);
  }
  MR_DTYPE_SWITCH(dtype, ssd_seq_fwd_launch<T>(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n,
                                               batch, L, H, Dh, N, seg, y, h_ckpt, h0, st, 0));
}

// the backward's tensor-core path with a dense A_neg needs a checkpoint at every chunk start
static bool ssd_dense_chunk_bwd(int dtype, int64_t L, int64_t Dh, int64_t N, int64_t seg, int64_t a_stride_n) {
  return ssd_dense_chunk_supported(dtype, L, Dh, N, seg, a_stride_n) && seg == ssd_chunk_len();
}

size_t mr_ssd_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                                  int64_t N, int64_t seg, int64_t a_stride_n) {
  if (batch <= 0 || L <= 0 || H <= 0 || Dh <= 0 || N <= 0 || seg <= 0) return 0;
  if (ssd_chunk_bwd_supported(dtype, L, Dh, N, seg, a_stride_n)) return ssd_chunk_bwd_ws_bytes(batch, H);
  if (ssd_dense_chunk_bwd(dtype, L, Dh, N, seg, a_stride_n)) return ssd_fallback_ws_bytes(batch, L, H, Dh, N, seg);
  return ssd_seq_bwd_ws_bytes(batch, L, H, Dh, N, seg);
}

int64_t mr_ssd_preferred_seg(int dtype, int64_t L, int64_t Dh, int64_t N, int64_t seg, int64_t a_stride_n) {
  const int64_t q = ssd_chunk_len();
  if (seg > 0 && L % q == 0 && q % seg == 0 &&
      (ssd_chunk_bwd_supported(dtype, L, Dh, N, q, a_stride_n) || ssd_dense_chunk_bwd(dtype, L, Dh, N, q, a_stride_n)))
    return q;
  return seg;
}

int mr_ssd_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* u,
               const void* delta, const void* Bm, const void* Cm, const float* A_neg,
               int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t L,
               int64_t H, int64_t Dh, int64_t N, int64_t seg, void* grad_u, void* grad_delta,
               void* grad_B, void* grad_C, float* grad_A, void* workspace,
               size_t workspace_bytes, void* stream) {
  return mr_ssd_bwd_h0(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, dtype, batch,
                       L, H, Dh, N, seg, grad_u, grad_delta, grad_B, grad_C, grad_A, workspace, workspace_bytes,
                       nullptr, nullptr, stream);
}

int mr_ssd_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* u,
                  const void* delta, const void* Bm, const void* Cm, const float* A_neg, int64_t a_stride_h,
                  int64_t a_stride_n, int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t N,
                  int64_t seg, void* grad_u, void* grad_delta, void* grad_B, void* grad_C, float* grad_A,
                  void* workspace, size_t workspace_bytes, const float* h0, float* grad_h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(ssd_common_checks("mr_ssd_bwd", dtype, batch, L, H, Dh, N, seg));
  MR_TRY(check_ptrs("mr_ssd_bwd", {grad_y, h_ckpt, u, delta, Bm, Cm, grad_u, grad_delta, grad_B, grad_C}));
  MR_TRY(check_opt_ptr("mr_ssd_bwd", grad_final));
  if (A_neg == nullptr || grad_A == nullptr)
    return set_error(MR_E_ALIGN, "mr_ssd_bwd: A_neg / grad_A is NULL");
  const bool chunk = ssd_chunk_bwd_supported(dtype, L, Dh, N, seg, a_stride_n);
  const bool dense = !chunk && ssd_dense_chunk_bwd(dtype, L, Dh, N, seg, a_stride_n);
  const size_t need = chunk   ? ssd_chunk_bwd_ws_bytes(batch, H)
                      : dense ? ssd_fallback_ws_bytes(batch, L, H, Dh, N, seg)
                              : ssd_seq_bwd_ws_bytes(batch, L, H, Dh, N, seg);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(MR_E_WORKSPACE, "mr_ssd_bwd: workspace of %zu bytes required, got %zu", need,
                     workspace_bytes);
  MR_TRY(check_opt_ptr("mr_ssd_bwd", workspace));
  MR_TRY(check_opt_ptr("mr_ssd_bwd", h0));
  MR_TRY(check_opt_ptr("mr_ssd_bwd", grad_h0));
  cudaStream_t st = (cudaStream_t)stream;
  if (chunk) {
    if (dtype == MR_BF16)
      return ssd_chunk_bwd_launch<__nv_bfloat16>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg, a_stride_h,
                                                 batch, L, H, seg, grad_u, grad_delta, grad_B, grad_C, grad_A,
                                                 (float*)workspace, h0, grad_h0, st);
    return ssd_chunk_bwd_launch<__half>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg, a_stride_h, batch, L,
                                        H, seg, grad_u, grad_delta, grad_B, grad_C, grad_A, (float*)workspace, h0,
                                        grad_h0, st);
  }
  if (dense) {
    // dense A_neg on the tensor cores (per-unit grad A partials at the start of the workspace),
    // then the per-step kernel for the units it marked, then the sum over the batch
    if (dtype == MR_BF16) {
      MR_TRY(ssd_dense_chunk_bwd_launch<__nv_bfloat16>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg,
                                                        a_stride_h, a_stride_n, batch, L, H, seg, grad_u,
                                                        grad_delta, grad_B, grad_C, (float*)workspace, h0, grad_h0,
                                                        st));
      return ssd_seq_bwd_marked_launch<__nv_bfloat16>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg,
                                                      a_stride_h, a_stride_n, batch, L, H, Dh, N, seg, grad_u,
                                                      grad_delta, grad_B, grad_C, grad_A, workspace, h0, grad_h0,
                                                      st);
    }
    MR_TRY(ssd_dense_chunk_bwd_launch<__half>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg, a_stride_h,
                                               a_stride_n, batch, L, H, seg, grad_u, grad_delta, grad_B, grad_C,
                                               (float*)workspace, h0, grad_h0, st));
    return ssd_seq_bwd_marked_launch<__half>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg, a_stride_h,
                                             a_stride_n, batch, L, H, Dh, N, seg, grad_u, grad_delta, grad_B, grad_C,
                                             grad_A, workspace, h0, grad_h0, st);
  }
  MR_DTYPE_SWITCH(dtype, ssd_seq_bwd_launch<T>(grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg,
                                               a_stride_h, a_stride_n, batch, L, H, Dh, N, seg,
                                               grad_u, grad_delta, grad_B, grad_C, grad_A,
                                               workspace, h0, grad_h0, st));
}

int mr_ssd_bwd_noalloc(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* u,
                       const void* delta, const void* Bm, const void* Cm, const float* A_neg,
                       int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t L,
                       int64_t H, int64_t Dh, int64_t N, int64_t seg, void* grad_u, void* grad_delta,
                       void* grad_B, void* grad_C, float* grad_A, void* stream) {
  g_err[0] = 0;
  MR_TRY(ssd_common_checks("mr_ssd_bwd_noalloc", dtype, batch, L, H, Dh, N, seg));
  MR_TRY(check_ptrs("mr_ssd_bwd_noalloc", {grad_y, h_ckpt, u, delta, Bm, Cm, grad_u, grad_delta, grad_B, grad_C}));
  MR_TRY(check_opt_ptr("mr_ssd_bwd_noalloc", grad_final));
  if (A_neg == nullptr || grad_A == nullptr)
    return set_error(MR_E_ALIGN, "mr_ssd_bwd_noalloc: A_neg / grad_A is NULL");
  if (!ssd_chunk_bwd_supported(dtype, L, Dh, N, seg, a_stride_n))
    return set_error(MR_E_SHAPE,
                     "mr_ssd_bwd_noalloc covers the tensor-core path only (bf16/f16, Dh=64, N=128, one rate "
                     "per head, seg=128, L %% 128 == 0); use mr_ssd_bwd with a workspace otherwise");
  return ssd_chunk_bwd_noalloc(dtype, grad_y, grad_final, h_ckpt, u, delta, Bm, Cm, A_neg, a_stride_h, batch,
                               L, H, seg, grad_u, grad_delta, grad_B, grad_C, grad_A, (cudaStream_t)stream);
}

// --------------------------------------------------------------------- GLA ---
static int gla_common_checks(const char* what, int dtype, int64_t batch, int64_t L, int64_t H,
                             int64_t Dh, int64_t seg) {
  MR_TRY(check_dims(what, batch, L, H));
  if (Dh <= 0) return set_error(MR_E_SHAPE, "%s: every dimension must be positive", what);
  MR_TRY(check_seg(L, seg, Dh, "Dh"));
  MR_TRY(check_dtype(dtype));
  if (!gla_seq_supported(Dh))
    return set_error(MR_E_SHAPE, "%s: this build supports Dh in {32,64,96,128}, got Dh=%lld", what,
                     (long long)Dh);
  if (batch * H > (int64_t)INT32_MAX) return set_error(MR_E_SHAPE, "%s: batch*H too large", what);
  return MR_OK;
}

int mr_gla_fwd(const void* q, const void* k, const void* v, const void* gates, int dtype,
               int64_t batch, int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y,
               float* h_ckpt, void* stream) {
  return mr_gla_fwd_h0(q, k, v, gates, dtype, batch, L, H, Dh, seg, y, h_ckpt, nullptr, stream);
}

int mr_gla_fwd_h0(const void* q, const void* k, const void* v, const void* gates, int dtype, int64_t batch,
                  int64_t L, int64_t H, int64_t Dh, int64_t seg, float* y, float* h_ckpt, const float* h0,
                  void* stream) {
  g_err[0] = 0;
  MR_TRY(gla_common_checks("mr_gla_fwd", dtype, batch, L, H, Dh, seg));
  MR_TRY(check_ptrs("mr_gla_fwd", {q, k, v, gates, y, h_ckpt}));
  MR_TRY(check_opt_ptr("mr_gla_fwd", h0));
  cudaStream_t st = (cudaStream_t)stream;
  if (gla_chunk_supported(dtype, L, Dh, seg)) {
    // tensor-core chunks for every unit, then the per-step kernel redoes the
    // units with a gate outside [1e-3, 1]
    if (dtype == MR_BF16) {
      MR_TRY(gla_chunk_fwd_launch<__nv_bfloat16>(q, k, v, gates, batch, L, H, seg, y, h_ckpt, h0, st));
      return gla_seq_fwd_launch<__nv_bfloat16>(q, k, v, gates, batch, L, H, Dh, seg, y, h_ckpt, h0, st, 1);
    }
    MR_TRY(gla_chunk_fwd_launch<__half>(q, k, v, gates, batch, L, H, seg, y, h_ckpt, h0, st));
    return gla_seq_fwd_launch<__half>(q, k, v, gates, batch, L, H, Dh, seg, y, h_ckpt, h0, st, 1);
  }
  MR_DTYPE_SWITCH(dtype, gla_seq_fwd_launch<T>(q, k, v, gates, batch, L, H, Dh, seg, y, h_ckpt, h0, st, 0));
}

int64_t mr_gla_preferred_seg(int dtype, int64_t L, int64_t Dh, int64_t seg) {
  const int64_t q = ssd_chunk_len();
  if (seg > 0 && L % q == 0 && q % seg == 0 && gla_chunk_supported(dtype, L, Dh, q)) return q;
  return seg;
}

// the backward's tensor-core path needs a checkpoint at every chunk start
static bool gla_chunk_bwd(int dtype, int64_t L, int64_t Dh, int64_t seg) {
  return gla_chunk_supported(dtype, L, Dh, seg) && seg == ssd_chunk_len();
}

size_t mr_gla_bwd_workspace_bytes(int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                                  int64_t seg) {
  if (batch <= 0 || L <= 0 || H <= 0 || Dh <= 0 || seg <= 0) return 0;
  if (gla_chunk_bwd(dtype, L, Dh, seg)) return gla_fallback_ws_bytes(batch, L, H, Dh, seg);
  return gla_seq_bwd_ws_bytes(batch, L, H, Dh, seg);
}

int mr_gla_bwd(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* q,
               const void* k, const void* v, const void* gates, int dtype, int64_t batch,
               int64_t L, int64_t H, int64_t Dh, int64_t seg, void* grad_q, void* grad_k,
               void* grad_v, void* grad_gates, void* workspace, size_t workspace_bytes,
               void* stream) {
  return mr_gla_bwd_h0(grad_y, grad_final, h_ckpt, q, k, v, gates, dtype, batch, L, H, Dh, seg, grad_q, grad_k,
                       grad_v, grad_gates, workspace, workspace_bytes, nullptr, nullptr, stream);
}

int mr_gla_bwd_h0(const float* grad_y, const float* grad_final, const float* h_ckpt, const void* q, const void* k,
                  const void* v, const void* gates, int dtype, int64_t batch, int64_t L, int64_t H, int64_t Dh,
                  int64_t seg, void* grad_q, void* grad_k, void* grad_v, void* grad_gates, void* workspace,
                  size_t workspace_bytes, const float* h0, float* grad_h0, void* stream) {
  g_err[0] = 0;
  MR_TRY(gla_common_checks("mr_gla_bwd", dtype, batch, L, H, Dh, seg));
  MR_TRY(check_ptrs("mr_gla_bwd", {grad_y, h_ckpt, q, k, v, gates, grad_q, grad_k, grad_v, grad_gates}));
  MR_TRY(check_opt_ptr("mr_gla_bwd", grad_final));
  const bool chunk = gla_chunk_bwd(dtype, L, Dh, seg);
  const size_t need = chunk ? gla_fallback_ws_bytes(batch, L, H, Dh, seg) : gla_seq_bwd_ws_bytes(batch, L, H, Dh, seg);
  if (workspace == nullptr || workspace_bytes < need)
    return set_error(MR_E_WORKSPACE, "mr_gla_bwd: workspace of %zu bytes required, got %zu", need,
                     workspace_bytes);
  MR_TRY(check_opt_ptr("mr_gla_bwd", workspace));
  MR_TRY(check_opt_ptr("mr_gla_bwd", h0));
  MR_TRY(check_opt_ptr("mr_gla_bwd", grad_h0));
  cudaStream_t st = (cudaStream_t)stream;
  if (chunk) {
    // tensor-core chunks for every unit, then the per-step kernel redoes the
    // units with a gate outside [1e-3, 1] (workspace: its scratch slots)
    if (dtype == MR_BF16) {
      MR_TRY(gla_chunk_bwd_launch<__nv_bfloat16>(grad_y, grad_final, h_ckpt, q, k, v, gates, batch, L, H, seg,
                                                 grad_q, grad_k, grad_v, grad_gates, h0, grad_h0, st));
      return gla_seq_bwd_launch<__nv_bfloat16>(grad_y, grad_final, h_ckpt, q, k, v, gates, batch, L, H, Dh, seg,
                                               grad_q, grad_k, grad_v, grad_gates, workspace, h0, grad_h0, st, 1);
    }
    MR_TRY(gla_chunk_bwd_launch<__half>(grad_y, grad_final, h_ckpt, q, k, v, gates, batch, L, H, seg, grad_q,
                                        grad_k, grad_v, grad_gates, h0, grad_h0, st));
    return gla_seq_bwd_launch<__half>(grad_y, grad_final, h_ckpt, q, k, v, gates, batch, L, H, Dh, seg, grad_q,
                                      grad_k, grad_v, grad_gates, workspace, h0, grad_h0, st, 1);
  }
  MR_DTYPE_SWITCH(dtype, gla_seq_bwd_launch<T>(grad_y, grad_final, h_ckpt, q, k, v, gates, batch, L,
                                               H, Dh, seg, grad_q, grad_k, grad_v, grad_gates,
                                               workspace, h0, grad_h0, st, 0));
}

// ------------------------------------------------------------ decode steps ---
static int step_dims(const char* what, std::initializer_list<int64_t> dims) {
  for (int64_t d : dims)
    if (d <= 0) return set_error(MR_E_SHAPE, "%s: every dimension must be positive", what);
  return MR_OK;
}

int mr_ssd_step(const void* u, const void* delta, const void* Bm, const void* Cm, const float* A_neg,
                int64_t a_stride_h, int64_t a_stride_n, int dtype, int64_t batch, int64_t H, int64_t Dh,
                int64_t N, float* state, float* y, void* stream) {
  g_err[0] = 0;
  MR_TRY(step_dims("mr_ssd_step", {batch, H, Dh, N}));
  if (N > 128) return set_error(MR_E_SHAPE, "mr_ssd_step: N <= 128 supported, got N=%lld", (long long)N);
  if (batch * H > (int64_t)INT32_MAX) return set_error(MR_E_SHAPE, "mr_ssd_step: batch*H too large");
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_ssd_step", {u, delta, Bm, Cm, state, y}));
  if (A_neg == nullptr) return set_error(MR_E_ALIGN, "mr_ssd_step: A_neg is NULL");
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, ssd_step_launch<T>(u, delta, Bm, Cm, A_neg, a_stride_h, a_stride_n, batch, H, Dh, N,
                                            state, y, st));
}

int mr_gla_step(const void* q, const void* k, const void* v, const void* gates, int dtype, int64_t batch,
                int64_t H, int64_t Dh, float* state, float* y, void* stream) {
  g_err[0] = 0;
  MR_TRY(step_dims("mr_gla_step", {batch, H, Dh}));
  if (Dh > 128) return set_error(MR_E_SHAPE, "mr_gla_step: Dh <= 128 supported, got Dh=%lld", (long long)Dh);
  if (batch * H > (int64_t)INT32_MAX) return set_error(MR_E_SHAPE, "mr_gla_step: batch*H too large");
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_gla_step", {q, k, v, gates, state, y}));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, gla_step_launch<T>(q, k, v, gates, batch, H, Dh, state, y, st));
}

int mr_rglru_step(const void* a, const void* x, int dtype, int64_t batch, int64_t D, float* state, float* y,
                  void* stream) {
  g_err[0] = 0;
  MR_TRY(step_dims("mr_rglru_step", {batch, D}));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rglru_step", {a, x, state, y}));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rglru_step_launch<T>(a, x, batch, D, state, y, st));
}

int mr_rotlru_step(const void* a, const void* cs, const void* sn, const void* x, int dtype, int64_t batch,
                   int64_t Dp, float* state, float* y, void* stream) {
  g_err[0] = 0;
  MR_TRY(step_dims("mr_rotlru_step", {batch, Dp}));
  MR_TRY(check_dtype(dtype));
  MR_TRY(check_ptrs("mr_rotlru_step", {a, cs, sn, x, state, y}));
  cudaStream_t st = (cudaStream_t)stream;
  MR_DTYPE_SWITCH(dtype, rotlru_step_launch<T>(a, cs, sn, x, batch, Dp, state, y, st));
}

}  // extern "C"
