// C ABI and host context of libnova_winograd (sm_100a).
//
// Replaces the reference's host class NovaWinogradF63 and its extern "C" block
// (Jayluci4/nova-wino-amd csrc/nova_winograd.hip:456-611, 681-756) and the
// fused-dispatch class NovaWinogradFused (csrc/nova_winograd_fused.hip:446-654).
// Differences that matter to callers, all deliberate:
//   * no process exit on error: status codes + last-error string;
//   * the transform constants are compiled in, so nova_create uploads nothing;
//   * the handle remembers its device and switches to it for every call;
//   * forward paths allocate nothing and never synchronize (nova_forward keeps a
//     grow-only workspace in the handle instead of malloc/free per call);
//   * tiles that lie wholly in the padding (the reference's over-tiling, see
//     compute_tiling) are skipped; nova_compute_tiling still returns the
//     reference's values and workspaces are still sized by them.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "../../include/nova_winograd.h"
#include "nova_internal.h"

#define NOVA_EXPORT extern "C" __attribute__((visibility("default")))

namespace nova {

__global__ void u_to_ref_layout_kernel(const __half* __restrict__ Uint, __half* __restrict__ Uref,
                                       int K, int C) {
  // [64][K][C] -> [64][C][K]
  const long long KC = (long long)K * C;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 64 * KC) return;
  const int pos = (int)(i / KC);
  const long long r = i % KC;
  const int k = (int)(r % K);
  const int c = (int)(r / K);
  Uref[i] = Uint[pos * KC + (long long)k * C + c];
}

namespace {

// 0 until the fused kernel beats the 3-pass path at some batch (it is opt-in via
// nova_set_path(h, 3) meanwhile).
constexpr long long kFusedMaxBpDefault = 0;

thread_local std::string t_err_msg = "no error";
thread_local int t_err_code = NOVA_OK;

struct Context {
  int device = -1;
  int num_sms = 148;
  int K = 0, C = 0;
  bool has_weights = false;
  __half* U = nullptr;  // [64][K][C]
  long long U_elems = 0;
  __half* U_ref = nullptr;  // [64][C][K], on request
  bool U_ref_valid = false;
  TcGemmPlan plan;
  bool tc_ok = false;
  FusedPlan fplan;
  bool fused_ok = false;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int* d_status = nullptr;
  int forced_path = 0;
  int last_path = 0;
  int last_error = NOVA_OK;
};

int fail(Context* ctx, int code, const std::string& msg) {
  t_err_code = code;
  t_err_msg = msg;
  if (ctx) ctx->last_error = code;
  return code;
}

int ok(Context* ctx) {
  t_err_code = NOVA_OK;
  if (ctx) ctx->last_error = NOVA_OK;
  return NOVA_OK;
}

int cuda_fail(Context* ctx, cudaError_t e, const char* where) {
  return fail(ctx, NOVA_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

// Switches to the handle's device for the duration of a call.
struct DeviceGuard {
  int prev = -1;
  bool switched = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != dev && dev >= 0) {
      switched = cudaSetDevice(dev) == cudaSuccess;
    }
  }
  ~DeviceGuard() {
    if (switched) cudaSetDevice(prev);
  }
};

void live_tiling(int H, int W, int pad, int* nh, int* nw, int* H_out, int* W_out) {
  *H_out = H + 2 * pad - 2;
  *W_out = W + 2 * pad - 2;
  *nh = (*H_out + 5) / 6;
  *nw = (*W_out + 5) / 6;
}

void ref_tiling(int H, int W, int pad, int* nh, int* nw, int* H_out, int* W_out) {
  // Formula of the reference's compute_tiling (csrc/nova_winograd.hip:617-631):
  // pad the output extent by n-1 = 7 and round up so (extent - 8) % 6 == 0.
  const int m = 6, n = 8;
  *H_out = H + 2 * pad - 2;
  *W_out = W + 2 * pad - 2;
  int Hp = *H_out + n - 1, Wp = *W_out + n - 1;
  Hp += (m - (Hp - n) % m) % m;
  Wp += (m - (Wp - n) % m) % m;
  *nh = (Hp - n) / m + 1;
  *nw = (Wp - n) / m + 1;
}

Context* create_context() {
  Context* ctx = new Context();
  if (cudaGetDevice(&ctx->device) != cudaSuccess) {
    delete ctx;
    fail(nullptr, NOVA_ERR_CUDA, "nova_create: no CUDA device");
    return nullptr;
  }
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, ctx->device);
  cudaError_t e = cudaMalloc(&ctx->d_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, sizeof(int));
  if (e != cudaSuccess) {
    delete ctx;
    cuda_fail(nullptr, e, "nova_create");
    return nullptr;
  }
  ok(nullptr);
  return ctx;
}

void destroy_context(Context* ctx) {
  if (!ctx) return;
  DeviceGuard g(ctx->device);
  if (ctx->U) cudaFree(ctx->U);
  if (ctx->U_ref) cudaFree(ctx->U_ref);
  if (ctx->ws) cudaFree(ctx->ws);
  if (ctx->d_status) cudaFree(ctx->d_status);
  delete ctx;
}

int set_weights(Context* ctx, const void* w, int K, int C, cudaStream_t s) {
  if (!ctx) return fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "set_weights: null handle");
  if (!w || K <= 0 || C <= 0)
    return fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "set_weights: null weight or non-positive K/C");
  DeviceGuard g(ctx->device);
  const long long elems = 64ll * K * C;
  if (elems != ctx->U_elems) {
    if (ctx->U) cudaFree(ctx->U);
    if (ctx->U_ref) cudaFree(ctx->U_ref);
    ctx->U = nullptr;
    ctx->U_ref = nullptr;
    ctx->U_elems = 0;
    cudaError_t e = cudaMalloc(&ctx->U, elems * sizeof(__half));
    if (e != cudaSuccess) {
      ctx->has_weights = false;
      return fail(ctx, NOVA_ERR_ALLOC, "set_weights: cudaMalloc(U) failed");
    }
    ctx->U_elems = elems;
  }
  ctx->K = K;
  ctx->C = C;
  ctx->U_ref_valid = false;
  cudaError_t e = launch_filter_transform(static_cast<const float*>(w), ctx->U, K, C, false, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "set_weights: filter transform");
  ctx->tc_ok = false;
  if (tc_gemm_supported(C, K)) {
    const char* why = nullptr;
    ctx->tc_ok = tc_gemm_plan(&ctx->plan, ctx->U, K, C, &why) == cudaSuccess;
  }
  ctx->fused_ok = false;
  if (fused_supported(C, K)) {
    const char* why = nullptr;
    ctx->fused_ok = fused_plan(&ctx->fplan, ctx->U, K, C, &why) == cudaSuccess;
  }
  ctx->has_weights = true;
  return ok(ctx);
}

int check_forward_args(Context* ctx, const void* x, const void* y, int B, int H, int W, int pad) {
  if (!ctx) return fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "forward: null handle");
  if (!ctx->has_weights)
    return fail(ctx, NOVA_ERR_NO_WEIGHTS, "forward: call set_weights() before forward()");
  if (B < 0 || H <= 0 || W <= 0 || pad < 0)
    return fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "forward: bad batch/H/W/pad");
  if (H + 2 * pad - 2 <= 0 || W + 2 * pad - 2 <= 0)
    return fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "forward: output would be empty (H+2*pad < 3)");
  if (B > 0 && (!x || !y)) return fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "forward: null tensor");
  return NOVA_OK;
}

// Largest live-tile count BP = B*ceil(H_out/6)*ceil(W_out/6) for which the
// automatic dispatch runs the fused kernel (NOVA_FUSED_MAX_BP overrides).
long long fused_max_bp() {
  static const long long v = [] {
    const char* env = std::getenv("NOVA_FUSED_MAX_BP");
    return env ? std::atoll(env) : kFusedMaxBpDefault;
  }();
  return v;
}

// Path ids: 1 = 3-pass with the tcgen05 GEMM, 2 = 3-pass with the SIMT GEMM,
// 3 = fused single kernel.  BP < 0 asks for a GEMM-only path.
int choose_path(Context* ctx, long long BP = -1) {
  if (ctx->forced_path == 3 && BP >= 0) return 3;
  if (ctx->forced_path == 0 && BP >= 0 && ctx->fused_ok && BP <= fused_max_bp()) return 3;
  if (ctx->forced_path == 1 || ctx->forced_path == 3 || (ctx->forced_path == 0 && ctx->tc_ok))
    return ctx->tc_ok ? 1 : 2;
  return 2;
}

// The three passes.  V and M hold at least 64*C*BP and 64*K*BP halves with
// BP = B * ceil(H_out/6) * ceil(W_out/6).
// L2 budget for one window's V + M (bytes), from NOVA_L2_WINDOW_MB; unset or 0
// = a single window over the whole batch.  Off by default: measured on B200 at
// batch 128, windows of 24-80 MB were 0-40 % slower than one window because the
// transforms are not HBM-bound and every window adds kernel drain / fill.
size_t l2_window_bytes() {
  static const size_t bytes = [] {
    const char* env = std::getenv("NOVA_L2_WINDOW_MB");
    long mb = env ? std::atol(env) : 0;
    if (mb < 0) mb = 0;
    return (size_t)mb << 20;
  }();
  return bytes;
}

// Tile rows (row = b*nh + th) per window so that the window's V and M fit the
// L2 budget.
long long window_rows(const Context* ctx, int nw, long long total_rows) {
  const size_t budget = l2_window_bytes();
  if (budget == 0) return total_rows;
  const size_t per_row = 64ull * (size_t)(ctx->C + ctx->K) * 2 * (size_t)nw;
  long long r = (long long)(budget / per_row);
  if (r < 1) r = 1;
  return std::min(r, total_rows);
}

// The three passes.  V and M hold at least 64*C*BP and 64*K*BP halves with
// BP = B * ceil(H_out/6) * ceil(W_out/6).  For even channel counts the batch
// is cut into windows of whole tile rows whose V and M fit in L2; each window
// runs its three passes back to back on the front of the workspace, so V and M
// are written and re-read in L2 instead of HBM.
int run_forward(Context* ctx, const void* x, void* y, void* V, void* M, int B, int H, int W,
                int pad, cudaStream_t s) {
  if (B == 0) return ok(ctx);
  int nh, nw, H_out, W_out;
  live_tiling(H, W, pad, &nh, &nw, &H_out, &W_out);
  const __half* xh = static_cast<const __half*>(x);
  __half* Vh = static_cast<__half*>(V);
  __half* Mh = static_cast<__half*>(M);
  __half* yh = static_cast<__half*>(y);
  const int path = choose_path(ctx, (long long)B * nh * nw);
  if (path == 3) {
    const char* why = "";
    cudaError_t e = fused_run(ctx->fplan, xh, yh, B, H, W, pad, ctx->d_status, ctx->num_sms, s, &why);
    if (e != cudaSuccess) return fail(ctx, NOVA_ERR_CUDA, std::string("forward: fused: ") + why);
    ctx->last_path = 3;
    return ok(ctx);
  }
  const bool even = ctx->C % 2 == 0 && ctx->K % 2 == 0;
  const long long total_rows = (long long)B * nh;
  const long long per_window = even ? window_rows(ctx, nw, total_rows) : total_rows;
  for (long long r0 = 0; r0 < total_rows; r0 += per_window) {
    const long long nrows = std::min(per_window, total_rows - r0);
    const long long BPw = nrows * nw;
    cudaError_t e =
        even ? launch_input_transform_fast(xh, Vh, B, ctx->C, H, W, pad, nh, nw, r0, nrows, BPw, s)
             : launch_input_transform(xh, Vh, B, ctx->C, H, W, pad, nh, nw, BPw, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "forward: input transform");
    if (path == 1) {
      const char* why = "";
      e = tc_gemm_run(ctx->plan, Vh, Mh, BPw, ctx->d_status, ctx->num_sms, s, &why);
      if (e != cudaSuccess)
        return fail(ctx, NOVA_ERR_CUDA, std::string("forward: tcgen05 GEMM: ") + why);
    } else {
      e = launch_gemm_simt(Vh, ctx->U, Mh, BPw, ctx->C, ctx->K, s);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "forward: SIMT GEMM");
    }
    e = even ? launch_output_transform_fast(Mh, yh, ctx->K, H_out, W_out, nh, nw, r0, nrows, BPw,
                                            s)
             : launch_output_transform(Mh, yh, B, ctx->K, H_out, W_out, nh, nw, BPw, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "forward: output transform");
  }
  ctx->last_path = path;
  return ok(ctx);
}

// The three passes on channels-last activations: x [B][H][W][C] and
// y [B][H_out][W_out][K], C and K even; never the fused kernel.
int run_forward_nhwc(Context* ctx, const void* x, void* y, void* V, void* M, int B, int H, int W,
                     int pad, cudaStream_t s) {
  if (B == 0) return ok(ctx);
  if (ctx->C % 8 || ctx->K % 2)
    return fail(ctx, NOVA_ERR_INVALID_ARGUMENT,
                "forward_nhwc: C must be a multiple of 8 and K even");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 4)
    return fail(ctx, NOVA_ERR_INVALID_ARGUMENT,
                "forward_nhwc: x must be 16-byte and y 4-byte aligned");
  int nh, nw, H_out, W_out;
  live_tiling(H, W, pad, &nh, &nw, &H_out, &W_out);
  const long long BP = (long long)B * nh * nw;
  __half* Vh = static_cast<__half*>(V);
  __half* Mh = static_cast<__half*>(M);
  cudaError_t e = launch_input_transform_nhwc(static_cast<const __half*>(x), Vh, B, ctx->C, H, W,
                                              pad, nh, nw, BP, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "forward_nhwc: input transform");
  const int path = choose_path(ctx);
  if (path == 1) {
    const char* why = "";
    e = tc_gemm_run(ctx->plan, Vh, Mh, BP, ctx->d_status, ctx->num_sms, s, &why);
    if (e != cudaSuccess)
      return fail(ctx, NOVA_ERR_CUDA, std::string("forward_nhwc: tcgen05 GEMM: ") + why);
  } else {
    e = launch_gemm_simt(Vh, ctx->U, Mh, BP, ctx->C, ctx->K, s);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "forward_nhwc: SIMT GEMM");
  }
  e = launch_output_transform_nhwc(Mh, static_cast<__half*>(y), B, ctx->K, H_out, W_out, nh, nw,
                                   BP, s);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "forward_nhwc: output transform");
  ctx->last_path = path;
  return ok(ctx);
}

size_t live_workspace_bytes(const Context* ctx, int B, int H, int W, int pad) {
  int nh, nw, H_out, W_out;
  live_tiling(H, W, pad, &nh, &nw, &H_out, &W_out);
  const size_t BP = (size_t)B * nh * nw;
  // V then M, M aligned to 256 bytes.
  const size_t v = (64 * (size_t)ctx->C * BP * 2 + 255) & ~size_t(255);
  return v + 64 * (size_t)ctx->K * BP * 2;
}

int forward_internal_ws(Context* ctx, const void* x, void* y, int B, int H, int W, int pad,
                        cudaStream_t s, bool nhwc = false) {
  int rc = check_forward_args(ctx, x, y, B, H, W, pad);
  if (rc) return rc;
  DeviceGuard g(ctx->device);
  const size_t need = live_workspace_bytes(ctx, B, H, W, pad);
  if (need > ctx->ws_bytes) {
    if (ctx->ws) cudaFree(ctx->ws);
    ctx->ws = nullptr;
    ctx->ws_bytes = 0;
    if (cudaMalloc(&ctx->ws, need) != cudaSuccess)
      return fail(ctx, NOVA_ERR_ALLOC, "forward: cudaMalloc(workspace) failed");
    ctx->ws_bytes = need;
  }
  int nh, nw, H_out, W_out;
  live_tiling(H, W, pad, &nh, &nw, &H_out, &W_out);
  const size_t BP = (size_t)B * nh * nw;
  const size_t voff = (64 * (size_t)ctx->C * BP * 2 + 255) & ~size_t(255);
  void* Mp = static_cast<char*>(ctx->ws) + voff;
  return nhwc ? run_forward_nhwc(ctx, x, y, ctx->ws, Mp, B, H, W, pad, s)
              : run_forward(ctx, x, y, ctx->ws, Mp, B, H, W, pad, s);
}

int forward_caller_ws(Context* ctx, const void* x, void* y, void* V, void* M, int B, int H, int W,
                      int pad, int nh, int nw, cudaStream_t s, bool nhwc = false) {
  int rc = check_forward_args(ctx, x, y, B, H, W, pad);
  if (rc) return rc;
  if (B > 0 && (!V || !M)) return fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "forward: null workspace");
  int lnh, lnw, H_out, W_out;
  live_tiling(H, W, pad, &lnh, &lnw, &H_out, &W_out);
  if ((long long)nh * nw < (long long)lnh * lnw)
    return fail(ctx, NOVA_ERR_WORKSPACE,
                "forward_workspace: nh*nw smaller than the tiles the output needs");
  DeviceGuard g(ctx->device);
  return nhwc ? run_forward_nhwc(ctx, x, y, V, M, B, H, W, pad, s)
              : run_forward(ctx, x, y, V, M, B, H, W, pad, s);
}

}  // namespace

int record_error(int code, const std::string& msg) { return fail(nullptr, code, msg); }

}  // namespace nova

using nova::Context;

static Context* as_ctx(nova_handle_t h) { return static_cast<Context*>(h); }
static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// Reference-compatible entry points.
// ---------------------------------------------------------------------------
NOVA_EXPORT nova_handle_t nova_create(void) { return nova::create_context(); }

NOVA_EXPORT void nova_destroy(nova_handle_t h) { nova::destroy_context(as_ctx(h)); }

NOVA_EXPORT void nova_set_weights(nova_handle_t h, const void* d_weight, int K, int C) {
  nova::set_weights(as_ctx(h), d_weight, K, C, nullptr);
}

NOVA_EXPORT void nova_forward(nova_handle_t h, const void* d_input, void* d_output, int batch,
                              int H, int W, int pad) {
  nova::forward_internal_ws(as_ctx(h), d_input, d_output, batch, H, W, pad, nullptr);
}

NOVA_EXPORT void nova_forward_workspace(nova_handle_t h, const void* d_input, void* d_output,
                                        void* d_V_gemm, void* d_M_gemm, int batch, int H, int W,
                                        int pad, int nh, int nw) {
  nova::forward_caller_ws(as_ctx(h), d_input, d_output, d_V_gemm, d_M_gemm, batch, H, W, pad, nh,
                          nw, nullptr);
}

NOVA_EXPORT void nova_compute_tiling(int H, int W, int pad, int* nh, int* nw, int* H_out,
                                     int* W_out) {
  if (!nh || !nw || !H_out || !W_out) {
    nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "compute_tiling: null output pointer");
    return;
  }
  nova::ref_tiling(H, W, pad, nh, nw, H_out, W_out);
}

NOVA_EXPORT int nova_filter_transform_v2(const void* d_weight, void* d_U_gemm, int K, int C,
                                         void* stream) {
  if (!d_weight || !d_U_gemm || K <= 0 || C <= 0)
    return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "filter_transform: bad arguments");
  cudaError_t e = nova::launch_filter_transform(static_cast<const float*>(d_weight),
                                                static_cast<__half*>(d_U_gemm), K, C, true,
                                                as_stream(stream));
  if (e != cudaSuccess) return nova::cuda_fail(nullptr, e, "filter_transform");
  return nova::ok(nullptr);
}

NOVA_EXPORT void nova_filter_transform(const void* d_weight, void* d_U_gemm, int K, int C) {
  if (nova_filter_transform_v2(d_weight, d_U_gemm, K, C, nullptr) == NOVA_OK) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) nova::cuda_fail(nullptr, e, "filter_transform: synchronize");
  }
}

NOVA_EXPORT int nova_input_transform_v2(const void* d_input, void* d_V_gemm, int batch, int C,
                                        int H, int W, int pad, int nh, int nw, int BP,
                                        void* stream) {
  if (!d_input || !d_V_gemm || batch <= 0 || C <= 0 || H <= 0 || W <= 0 || pad < 0 || nh <= 0 ||
      nw <= 0 || (long long)BP < (long long)batch * nh * nw)
    return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "input_transform: bad arguments");
  cudaError_t e = nova::launch_input_transform(static_cast<const __half*>(d_input),
                                               static_cast<__half*>(d_V_gemm), batch, C, H, W, pad,
                                               nh, nw, BP, as_stream(stream));
  if (e != cudaSuccess) return nova::cuda_fail(nullptr, e, "input_transform");
  return nova::ok(nullptr);
}

NOVA_EXPORT void nova_input_transform(const void* d_input, void* d_V_gemm, int batch, int C,
                                      int H, int W, int pad, int nh, int nw, int BP) {
  nova_input_transform_v2(d_input, d_V_gemm, batch, C, H, W, pad, nh, nw, BP, nullptr);
}

NOVA_EXPORT int nova_output_transform_v2(const void* d_M_gemm, void* d_output, int batch, int K,
                                         int H_out, int W_out, int nh, int nw, int BP,
                                         void* stream) {
  if (!d_M_gemm || !d_output || batch <= 0 || K <= 0 || H_out <= 0 || W_out <= 0 || nh <= 0 ||
      nw <= 0 || (long long)BP < (long long)batch * nh * nw)
    return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "output_transform: bad arguments");
  cudaError_t e = nova::launch_output_transform(static_cast<const __half*>(d_M_gemm),
                                                static_cast<__half*>(d_output), batch, K, H_out,
                                                W_out, nh, nw, BP, as_stream(stream));
  if (e != cudaSuccess) return nova::cuda_fail(nullptr, e, "output_transform");
  return nova::ok(nullptr);
}

NOVA_EXPORT void nova_output_transform(const void* d_M_gemm, void* d_output, int batch, int K,
                                       int H_out, int W_out, int nh, int nw, int BP) {
  nova_output_transform_v2(d_M_gemm, d_output, batch, K, H_out, W_out, nh, nw, BP, nullptr);
}

NOVA_EXPORT int nova_get_K(nova_handle_t h) { return h ? as_ctx(h)->K : 0; }
NOVA_EXPORT int nova_get_C(nova_handle_t h) { return h ? as_ctx(h)->C : 0; }

NOVA_EXPORT void* nova_get_U_gemm(nova_handle_t h) {
  Context* ctx = as_ctx(h);
  if (!ctx || !ctx->has_weights) {
    nova::fail(ctx, NOVA_ERR_NO_WEIGHTS, "get_U_gemm: no weights set");
    return nullptr;
  }
  if (!ctx->U_ref_valid) {
    nova::DeviceGuard g(ctx->device);
    if (!ctx->U_ref && cudaMalloc(&ctx->U_ref, ctx->U_elems * sizeof(__half)) != cudaSuccess) {
      ctx->U_ref = nullptr;
      nova::fail(ctx, NOVA_ERR_ALLOC, "get_U_gemm: cudaMalloc failed");
      return nullptr;
    }
    const unsigned blocks = (unsigned)((ctx->U_elems + 255) / 256);
    nova::u_to_ref_layout_kernel<<<blocks, 256>>>(ctx->U, ctx->U_ref, ctx->K, ctx->C);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      nova::cuda_fail(ctx, e, "get_U_gemm");
      return nullptr;
    }
    ctx->U_ref_valid = true;
  }
  return ctx->U_ref;
}

// ---------------------------------------------------------------------------
// Fused-dispatch names (csrc/nova_winograd_fused.hip:619-652).
// ---------------------------------------------------------------------------
NOVA_EXPORT nova_handle_t nova_fused_create(void) { return nova_create(); }
NOVA_EXPORT void nova_fused_destroy(nova_handle_t h) { nova_destroy(h); }
NOVA_EXPORT void nova_fused_set_weights(nova_handle_t h, const void* d_weight, int K, int C) {
  nova_set_weights(h, d_weight, K, C);
}
NOVA_EXPORT void nova_fused_forward(nova_handle_t h, const void* d_input, void* d_output,
                                    int batch, int H, int W, int pad) {
  nova_forward(h, d_input, d_output, batch, H, W, pad);
}
NOVA_EXPORT void nova_fused_compute_tiling(int H, int W, int pad, int* nh, int* nw, int* H_out,
                                           int* W_out) {
  nova_compute_tiling(H, W, pad, nh, nw, H_out, W_out);
}

// ---------------------------------------------------------------------------
// Additions.
// ---------------------------------------------------------------------------
NOVA_EXPORT int nova_get_last_error(nova_handle_t h) {
  return h ? as_ctx(h)->last_error : nova::t_err_code;
}

NOVA_EXPORT const char* nova_last_error_string(void) { return nova::t_err_msg.c_str(); }

NOVA_EXPORT int nova_set_weights_v2(nova_handle_t h, const void* d_weight, int K, int C,
                                    void* stream) {
  return nova::set_weights(as_ctx(h), d_weight, K, C, as_stream(stream));
}

NOVA_EXPORT int nova_forward_v2(nova_handle_t h, const void* d_input, void* d_output, int batch,
                                int H, int W, int pad, void* stream) {
  return nova::forward_internal_ws(as_ctx(h), d_input, d_output, batch, H, W, pad,
                                   as_stream(stream));
}

NOVA_EXPORT int nova_forward_workspace_v2(nova_handle_t h, const void* d_input, void* d_output,
                                          void* d_V_gemm, void* d_M_gemm, int batch, int H, int W,
                                          int pad, int nh, int nw, void* stream) {
  return nova::forward_caller_ws(as_ctx(h), d_input, d_output, d_V_gemm, d_M_gemm, batch, H, W,
                                 pad, nh, nw, as_stream(stream));
}

NOVA_EXPORT int nova_forward_nhwc_v2(nova_handle_t h, const void* d_input, void* d_output,
                                     int batch, int H, int W, int pad, void* stream) {
  return nova::forward_internal_ws(as_ctx(h), d_input, d_output, batch, H, W, pad,
                                   as_stream(stream), true);
}

NOVA_EXPORT int nova_forward_workspace_nhwc_v2(nova_handle_t h, const void* d_input,
                                               void* d_output, void* d_V_gemm, void* d_M_gemm,
                                               int batch, int H, int W, int pad, int nh, int nw,
                                               void* stream) {
  return nova::forward_caller_ws(as_ctx(h), d_input, d_output, d_V_gemm, d_M_gemm, batch, H, W,
                                 pad, nh, nw, as_stream(stream), true);
}

NOVA_EXPORT int nova_input_transform_nhwc_v2(const void* d_input, void* d_V_gemm, int batch, int C,
                                             int H, int W, int pad, int nh, int nw, int BP,
                                             void* stream) {
  if (!d_input || !d_V_gemm || batch <= 0 || C <= 0 || C % 8 || H <= 0 || W <= 0 || pad < 0 ||
      nh <= 0 || nw <= 0 || (long long)BP < (long long)batch * nh * nw ||
      reinterpret_cast<uintptr_t>(d_input) % 16)
    return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "input_transform_nhwc: bad arguments");
  cudaError_t e = nova::launch_input_transform_nhwc(static_cast<const __half*>(d_input),
                                                    static_cast<__half*>(d_V_gemm), batch, C, H, W,
                                                    pad, nh, nw, BP, as_stream(stream));
  if (e != cudaSuccess) return nova::cuda_fail(nullptr, e, "input_transform_nhwc");
  return nova::ok(nullptr);
}

NOVA_EXPORT int nova_output_transform_nhwc_v2(const void* d_M_gemm, void* d_output, int batch,
                                              int K, int H_out, int W_out, int nh, int nw, int BP,
                                              void* stream) {
  if (!d_M_gemm || !d_output || batch <= 0 || K <= 0 || K % 2 || H_out <= 0 || W_out <= 0 ||
      nh <= 0 || nw <= 0 || (long long)BP < (long long)batch * nh * nw ||
      reinterpret_cast<uintptr_t>(d_output) % 4)
    return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "output_transform_nhwc: bad arguments");
  cudaError_t e = nova::launch_output_transform_nhwc(static_cast<const __half*>(d_M_gemm),
                                                     static_cast<__half*>(d_output), batch, K,
                                                     H_out, W_out, nh, nw, BP, as_stream(stream));
  if (e != cudaSuccess) return nova::cuda_fail(nullptr, e, "output_transform_nhwc");
  return nova::ok(nullptr);
}

NOVA_EXPORT int nova_batched_gemm_v2(nova_handle_t h, const void* d_V_gemm, void* d_M_gemm,
                                     int BP, void* stream) {
  Context* ctx = as_ctx(h);
  if (!ctx) return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "batched_gemm: null handle");
  if (!ctx->has_weights) return nova::fail(ctx, NOVA_ERR_NO_WEIGHTS, "batched_gemm: no weights");
  if (BP < 0 || (BP > 0 && (!d_V_gemm || !d_M_gemm)))
    return nova::fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "batched_gemm: bad arguments");
  if (BP == 0) return nova::ok(ctx);
  nova::DeviceGuard g(ctx->device);
  const __half* V = static_cast<const __half*>(d_V_gemm);
  __half* M = static_cast<__half*>(d_M_gemm);
  const int path = nova::choose_path(ctx);
  cudaError_t e;
  if (path == 1) {
    const char* why = "";
    e = nova::tc_gemm_run(ctx->plan, V, M, BP, ctx->d_status, ctx->num_sms, as_stream(stream),
                          &why);
    if (e != cudaSuccess)
      return nova::fail(ctx, NOVA_ERR_CUDA, std::string("batched_gemm: tcgen05 GEMM: ") + why);
  } else {
    e = nova::launch_gemm_simt(V, ctx->U, M, BP, ctx->C, ctx->K, as_stream(stream));
    if (e != cudaSuccess) return nova::cuda_fail(ctx, e, "batched_gemm: SIMT GEMM");
  }
  ctx->last_path = path;
  return nova::ok(ctx);
}

NOVA_EXPORT long long nova_workspace_bytes(nova_handle_t h, int batch, int H, int W, int pad) {
  Context* ctx = as_ctx(h);
  if (!ctx || !ctx->has_weights || batch < 0) return -1;
  int nh, nw, H_out, W_out;
  nova::ref_tiling(H, W, pad, &nh, &nw, &H_out, &W_out);
  const long long BP = (long long)batch * nh * nw;
  return (64ll * ctx->C * BP + 64ll * ctx->K * BP) * 2;
}

NOVA_EXPORT int nova_set_path(nova_handle_t h, int path) {
  Context* ctx = as_ctx(h);
  if (!ctx) return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "set_path: null handle");
  if (path < 0 || path > 3)
    return nova::fail(ctx, NOVA_ERR_INVALID_ARGUMENT, "set_path: unknown path");
  if (path == 3 && !ctx->fused_ok)
    return nova::fail(ctx, NOVA_ERR_INVALID_ARGUMENT,
                      "set_path: fused kernel needs C in {16, 32, 48, 64} and K <= 64");
  if (path == 1 && !ctx->tc_ok)
    return nova::fail(ctx, NOVA_ERR_INVALID_ARGUMENT,
                      "set_path: tcgen05 GEMM needs C % 8 == 0 and K % 16 == 0");
  ctx->forced_path = path;
  return nova::ok(ctx);
}

NOVA_EXPORT int nova_get_path(nova_handle_t h) { return h ? as_ctx(h)->last_path : 0; }

NOVA_EXPORT int nova_device_status(nova_handle_t h) {
  Context* ctx = as_ctx(h);
  if (!ctx) return nova::fail(nullptr, NOVA_ERR_INVALID_ARGUMENT, "device_status: null handle");
  nova::DeviceGuard g(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return nova::cuda_fail(ctx, e, "device_status: synchronize");
  int st = 0;
  e = cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return nova::cuda_fail(ctx, e, "device_status: read");
  if (st != 0) {
    cudaMemset(ctx->d_status, 0, sizeof(int));
    return nova::fail(ctx, NOVA_ERR_DEVICE_TIMEOUT,
                      "device_status: a kernel's bounded wait expired (code " +
                          std::to_string(st) + ")");
  }
  return nova::ok(ctx);
}

NOVA_EXPORT const char* nova_version(void) { return "nova-winograd-b200 0.1.0 (sm_100a)"; }
