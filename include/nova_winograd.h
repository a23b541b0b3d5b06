/*
 * libnova_winograd -- NOVA F(6,3) Winograd 3x3 stride-1 FP16 convolution forward
 * for NVIDIA B200 (sm_100a).  Plain C ABI: raw device pointers, int sizes, no
 * CUDA or torch types.  A stream argument is a cudaStream_t passed as void*
 * (NULL = the legacy default stream, which is what every reference entry point
 * uses).
 *
 * Reference: Jayluci4/nova-wino-amd.  Each declaration names the reference
 * entry point it replaces (file:line).  The first block keeps the reference's
 * exact names and signatures so its ctypes bridge (nova_winograd/ops.py:66-114)
 * binds unchanged.
 *
 * Error behaviour.  The reference prints and calls exit(1) on any HIP/rocBLAS
 * error (csrc/nova_winograd.hip:27-41).  This library never exits the process:
 * the void entry points record the error, which nova_get_last_error() /
 * nova_last_error_string() report; the *_v2 entry points return it.
 *
 * Tensor layouts (element offsets):
 *   x  [B][C][H][W]            FP16, NCHW, contiguous
 *   w  [K][C][3][3]            FP32
 *   y  [B][K][H_out][W_out]    FP16
 *   V  workspace, 64*C*B*nh*nw FP16 (reference V_gemm size)
 *   M  workspace, 64*K*B*nh*nw FP16 (reference M_gemm size)
 *   U  [64][C][K]              FP16, U[pos][c][k] at pos*K*C + c*K + k
 *      (the reference's U_gemm layout, csrc/nova_winograd.hip:254)
 */
#ifndef NOVA_WINOGRAD_H
#define NOVA_WINOGRAD_H

#ifdef __cplusplus
extern "C" {
#endif

typedef void* nova_handle_t;

/* Status codes returned by the *_v2 entry points and nova_get_last_error(). */
enum {
  NOVA_OK = 0,
  NOVA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, unsupported shape     */
  NOVA_ERR_NO_WEIGHTS = 2,       /* forward before set_weights                    */
  NOVA_ERR_WORKSPACE = 3,        /* workspace too small for the tiling            */
  NOVA_ERR_CUDA = 4,             /* a CUDA runtime call or launch failed          */
  NOVA_ERR_DEVICE_TIMEOUT = 5,   /* a kernel's bounded wait expired               */
  NOVA_ERR_WRONG_DEVICE = 6,     /* handle used on another device than created on */
  NOVA_ERR_ALLOC = 7             /* device allocation failed                      */
};

/* ---- Reference-compatible entry points (same names and signatures) ------- */

/* csrc/nova_winograd.hip:686-690.  Creates a context on the current device. */
nova_handle_t nova_create(void);
/* csrc/nova_winograd.hip:692-694. */
void nova_destroy(nova_handle_t h);
/* csrc/nova_winograd.hip:696-698.  Transforms w (device, FP32 [K][C][3][3])
 * into the handle's cached U; asynchronous on the default stream. */
void nova_set_weights(nova_handle_t h, const void* d_weight, int K, int C);
/* csrc/nova_winograd.hip:700-706.  Forward with library-managed workspace
 * (grow-only cache inside the handle instead of malloc/free per call). */
void nova_forward(nova_handle_t h, const void* d_input, void* d_output, int batch, int H, int W,
                  int pad);
/* csrc/nova_winograd.hip:708-717.  Forward with caller-owned workspace sized
 * from nova_compute_tiling: V >= 64*C*batch*nh*nw, M >= 64*K*batch*nh*nw FP16.
 * Allocates nothing, never synchronizes. */
void nova_forward_workspace(nova_handle_t h, const void* d_input, void* d_output, void* d_V_gemm,
                            void* d_M_gemm, int batch, int H, int W, int pad, int nh, int nw);
/* csrc/nova_winograd.hip:719-721 (formula :617-631).  Pure host. */
void nova_compute_tiling(int H, int W, int pad, int* nh, int* nw, int* H_out, int* W_out);
/* csrc/nova_winograd.hip:724-728.  U (reference layout) from w; synchronizes
 * the device like the reference. */
void nova_filter_transform(const void* d_weight, void* d_U_gemm, int K, int C);
/* csrc/nova_winograd.hip:731-739.  Stage entry: V[pos][bp][c] for the given
 * tiling (nh, nw, BP = batch*nh*nw), default stream. */
void nova_input_transform(const void* d_input, void* d_V_gemm, int batch, int C, int H, int W,
                          int pad, int nh, int nw, int BP);
/* csrc/nova_winograd.hip:742-750.  Stage entry: y from M[pos][bp][k]. */
void nova_output_transform(const void* d_M_gemm, void* d_output, int batch, int K, int H_out,
                           int W_out, int nh, int nw, int BP);
/* csrc/nova_winograd.hip:752-754. */
int nova_get_K(nova_handle_t h);
int nova_get_C(nova_handle_t h);
/* csrc/nova_winograd.hip:754.  The handle's U in the reference layout
 * [64][C][K] (materialised on first request after set_weights). */
void* nova_get_U_gemm(nova_handle_t h);

/* ---- Fused-dispatch entry points ---------------------------------------- */
/* csrc/nova_winograd_fused.hip:619-652 (nova_fused_*).  Same context as
 * nova_create; forward runs the library's path dispatch. */
nova_handle_t nova_fused_create(void);
void nova_fused_destroy(nova_handle_t h);
void nova_fused_set_weights(nova_handle_t h, const void* d_weight, int K, int C);
void nova_fused_forward(nova_handle_t h, const void* d_input, void* d_output, int batch, int H,
                        int W, int pad);
void nova_fused_compute_tiling(int H, int W, int pad, int* nh, int* nw, int* H_out, int* W_out);

/* ---- Additions: status returns, explicit streams ------------------------- */
/* No counterpart in the reference (which exits on error): status of the last
 * call on this handle (or on this thread for handle-less calls when h is NULL). */
int nova_get_last_error(nova_handle_t h);
/* Human-readable text of the last error recorded on the calling thread. */
const char* nova_last_error_string(void);

/* Stream-aware, status-returning forms of nova_set_weights / nova_forward /
 * nova_forward_workspace / the stage entries.  stream is a cudaStream_t. */
int nova_set_weights_v2(nova_handle_t h, const void* d_weight, int K, int C, void* stream);
int nova_forward_v2(nova_handle_t h, const void* d_input, void* d_output, int batch, int H, int W,
                    int pad, void* stream);
int nova_forward_workspace_v2(nova_handle_t h, const void* d_input, void* d_output,
                              void* d_V_gemm, void* d_M_gemm, int batch, int H, int W, int pad,
                              int nh, int nw, void* stream);
int nova_filter_transform_v2(const void* d_weight, void* d_U_gemm, int K, int C, void* stream);
int nova_input_transform_v2(const void* d_input, void* d_V_gemm, int batch, int C, int H, int W,
                            int pad, int nh, int nw, int BP, void* stream);
int nova_output_transform_v2(const void* d_M_gemm, void* d_output, int batch, int K, int H_out,
                             int W_out, int nh, int nw, int BP, void* stream);

/* Stage entry for the 64-way batched GEMM the reference ran through rocBLAS
 * gemm_strided_batched_ex (csrc/nova_winograd.hip:534-548):
 * M[pos][bp][k] = sum_c V[pos][bp][c] * U[pos][c][k], FP16 in, FP32 accumulate,
 * FP16 out, on the handle's U, with the path nova_set_path selects. */
int nova_batched_gemm_v2(nova_handle_t h, const void* d_V_gemm, void* d_M_gemm, int BP,
                         void* stream);

/* Channels-last (NHWC) forward.  No reference counterpart: the reference takes
 * NCHW activations only (csrc/nova_winograd.hip:141-205, 264-328).
 * d_input is [batch][H][W][C] (16-byte aligned, C % 8 == 0) and d_output
 * [batch][H_out][W_out][K] (4-byte aligned, K even), FP16; V and M have the NCHW path's layout and size
 * (nova_workspace_bytes), and the GEMM is the same, so outputs equal the NCHW
 * path's (up to the sign of an exact zero).  Never takes the fused path.
 * Returns NOVA_ERR_INVALID_ARGUMENT for other C, K or alignments. */
int nova_forward_nhwc_v2(nova_handle_t h, const void* d_input, void* d_output, int batch, int H,
                         int W, int pad, void* stream);
int nova_forward_workspace_nhwc_v2(nova_handle_t h, const void* d_input, void* d_output,
                                   void* d_V_gemm, void* d_M_gemm, int batch, int H, int W,
                                   int pad, int nh, int nw, void* stream);
/* Stage entries of the NHWC path (the layouts of V and M as nova_input_transform_v2 /
 * nova_output_transform_v2). */
int nova_input_transform_nhwc_v2(const void* d_input, void* d_V_gemm, int batch, int C, int H,
                                 int W, int pad, int nh, int nw, int BP, void* stream);
int nova_output_transform_nhwc_v2(const void* d_M_gemm, void* d_output, int batch, int K,
                                  int H_out, int W_out, int nh, int nw, int BP, void* stream);

/* Bytes of caller workspace nova_forward_workspace needs (V + M), the
 * reference's sizing (csrc/nova_winograd_fused.hip:524-534 for the 3-pass case). */
long long nova_workspace_bytes(nova_handle_t h, int batch, int H, int W, int pad);

/* Path selection.  0 = automatic dispatch, 1 = 3-pass with the tcgen05 GEMM,
 * 2 = 3-pass with the SIMT GEMM, 3 = the fused single kernel (transform ->
 * tcgen05 MMA -> inverse, no V/M in HBM; C in {16, 32, 48, 64} and K <= 64,
 * the fused path of csrc/nova_winograd_fused.hip:511).  The automatic dispatch
 * takes the fused kernel for those shapes up to a live-tile count and the
 * tcgen05 3-pass beyond it.  Stage entries (nova_batched_gemm_v2) treat 3 as 1.
 * Returns NOVA_ERR_INVALID_ARGUMENT for a path the current weights cannot take.  nova_get_path reports the path the last
 * forward on this handle ran. */
int nova_set_path(nova_handle_t h, int path);
int nova_get_path(nova_handle_t h);

/* Synchronizes the handle's device and returns NOVA_ERR_DEVICE_TIMEOUT if any
 * kernel launched through this handle hit a bounded-wait expiry since the last
 * call (and clears the flag); NOVA_OK otherwise. */
int nova_device_status(nova_handle_t h);

/* Forward that allocates nothing -- no counterpart in the reference.  For
 * callers that may not allocate device memory where they run the convolution
 * (a plugin inside a runtime that owns all device memory, an allocation-free
 * real-time loop): no handle, the caller passes x, the transformed filter U in
 * the reference layout [64][C][K] (fill it once with nova_filter_transform into
 * memory the caller owns) and y.  V and M live in one fixed 32 MiB device array
 * inside the library (held by every GPU that loads it): shapes whose
 * 64*(C+K)*batch*ceil(H_out/6)*ceil(W_out/6) FP16 values exceed it are refused
 * with NOVA_ERR_WORKSPACE.  The first call on a device looks the array's address
 * up (make it before any stream capture); calls that overlap on the GPU share
 * the array and race.  Returns a NOVA_* status. */
int nova_forward_noalloc(const void* d_input, const void* d_U_gemm, void* d_output, int batch,
                         int C, int K, int H, int W, int pad, void* stream);

/* Weight gradient of the 3x3 stride-1 convolution by the NOVA F(6,3) Winograd
 * algorithm, replacing the reference's FP32 per-sample unfold loop
 * (nova_winograd/conv2d.py:131-141 and the custom-op backward :66-80):
 * dW[K][C][3][3] (FP32) from the FP16 input x [B][C][H][W] and output gradient
 * dy [B][K][H_out][W_out].  dW = G^T [sum over tiles (A^T dY A) . (B^T d B)] G:
 * both transforms stored FP16, the per-position sums over tiles on the tensor
 * cores with FP32 accumulation.  C must be a multiple of 16.  The caller passes
 * a 256-byte aligned device workspace of nova_weight_grad_workspace_bytes()
 * bytes; nothing is allocated.  Runs on `stream`; returns a NOVA_* status. */
long long nova_weight_grad_workspace_bytes(int batch, int C, int K, int H, int W, int pad);
int nova_weight_grad_v2(const void* d_input, const void* d_grad_output, void* d_grad_weight,
                        void* d_workspace, long long workspace_bytes, int batch, int C, int K,
                        int H, int W, int pad, void* stream);

/* Library version string. */
const char* nova_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NOVA_WINOGRAD_H */
