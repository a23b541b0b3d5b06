// Internal declarations shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "nova_common.cuh"

#include <cstdlib>
#include <utility>

namespace nova {

// Per-thread cache of encoded TMA descriptors.  A descriptor depends only on
// the base address, the dims / strides and the box, all of which are in the
// key, so a hit is always the descriptor a fresh encode would produce.  The
// workspaces (V, M) keep their addresses across calls, which saves their
// host-side encodes on every forward.
template <typename Encode>
bool cached_tensor_map(CUtensorMap* map, const void* ptr, long long k0, long long k1,
                       long long k2, int tag, Encode&& encode) {
  struct Entry {
    const void* ptr;
    long long k0, k1, k2;
    int tag;
    CUtensorMap map;
  };
  constexpr int kEntries = 16;
  thread_local Entry cache[kEntries] = {};
  thread_local int next = 0;
  for (const Entry& e : cache)
    if (e.ptr == ptr && ptr != nullptr && e.k0 == k0 && e.k1 == k1 && e.k2 == k2 && e.tag == tag) {
      *map = e.map;
      return true;
    }
  if (!encode(map)) return false;
  cache[next] = Entry{ptr, k0, k1, k2, tag, *map};
  next = (next + 1) % kEntries;
  return true;
}

// Programmatic dependent launch for the hot-path kernels.  Kinds: 1 = input
// transform, 2 = tensor-core GEMM, 4 = output transform, 8 = fused kernel;
// NOVA_PDL_MASK (default: all) selects which kinds launch with it.  The kernel
// must call pdl_wait() before touching global memory.
enum PdlKind : int { kPdlInput = 1, kPdlGemm = 2, kPdlOutput = 4, kPdlFused = 8 };
inline bool pdl_enabled(int kind) {
  static const int mask = [] {
    const char* e = std::getenv("NOVA_PDL_MASK");
    return e ? std::atoi(e) : 15;
  }();
  return (mask & kind) != 0;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(int kind, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled(kind) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Records code + message as the calling thread's last error (handle-less
// entry points); returns code.
int record_error(int code, const std::string& msg);

// Device-side status codes written by kernels whose waits are bounded.
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutProducer = 1,  // TMA producer gave up waiting for a free stage
  kDevTimeoutMma = 2,       // MMA issuer gave up waiting for operands / accumulator
  kDevTimeoutEpilogue = 3,  // epilogue gave up waiting for an accumulator
  kDevTimeoutFused = 4,     // fused kernel gave up waiting for U or its MMAs
};

cudaError_t launch_filter_transform(const float* w, __half* U, int K, int C, bool ref_layout,
                                    cudaStream_t s);
cudaError_t launch_input_transform(const __half* x, __half* V, int B, int C, int H, int W,
                                   int pad, int nh, int nw, long long BP, cudaStream_t s);
cudaError_t launch_output_transform(const __half* M, __half* y, int B, int K, int H_out,
                                    int W_out, int nh, int nw, long long BP, cudaStream_t s);
// Even channel counts: the fast kernels, over the tile rows [row0, row0+nrows)
// (row = b*nh + th); inside V / M, bp = (row - row0)*nw + tw and BP is the
// tensors' bp extent.
cudaError_t launch_input_transform_fast(const __half* x, __half* V, int B, int C, int H, int W,
                                        int pad, int nh, int nw, long long row0, long long nrows,
                                        long long BP, cudaStream_t s);
cudaError_t launch_output_transform_fast(const __half* M, __half* y, int K, int H_out, int W_out,
                                         int nh, int nw, long long row0, long long nrows,
                                         long long BP, cudaStream_t s);
cudaError_t launch_gemm_simt(const __half* V, const __half* U, __half* M, long long BP, int C,
                             int K, cudaStream_t s);
// cuTensorMapEncodeTiled through the runtime's driver entry point (null if
// the driver does not provide it); defined in nova_gemm_tc.cu.
using TensorMapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                       const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                       const cuuint32_t*, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion,
                                       CUtensorMapFloatOOBfill);
TensorMapEncodeFn tensor_map_encode_fn();

// Channels-last (NHWC) activations, whole batch (nova_nhwc.cu): the same V / M
// layouts as the NCHW kernels.  Input transform: C % 8 == 0 and x 16-byte
// aligned (TMA box loads); output transform: K even, y 4-byte aligned.
cudaError_t launch_input_transform_nhwc(const __half* x, __half* V, int B, int C, int H, int W,
                                        int pad, int nh, int nw, long long BP, cudaStream_t s);
cudaError_t launch_output_transform_nhwc(const __half* M, __half* y, int B, int K, int H_out,
                                         int W_out, int nh, int nw, long long BP, cudaStream_t s);

// Tensor-core (tcgen05 + TMA) batched GEMM.
struct TcGemmPlan {
  CUtensorMap tmU;       // U internal layout [64][K][C], box {64 c, BN k, 1}
  CUtensorMap tmU_half;  // the same with box {64 c, BN/2 k, 1} (BN > 128 only)
  CUtensorMap tmU_pair;  // the same with box {64 c, BN/2 k, 1}: one CTA's half of
                         // a pair tile (SM-pair GEMM, BN % 64 == 0 only)
  int BN = 0;            // output channels per tile (MMA N)
  int K = 0, C = 0;
  bool has_half = false;
  bool has_pair = false;
  bool valid = false;
};

// True when (C, K) is a shape the tcgen05 path takes.
bool tc_gemm_supported(int C, int K);
// Builds the weight-side tensor map for U (call when the weights change).
cudaError_t tc_gemm_plan(TcGemmPlan* plan, const __half* U, int K, int C, const char** why);
// M[pos][bp][k] = sum_c V[pos][bp][c] U[pos][k][c] on the tensor cores.
cudaError_t tc_gemm_run(const TcGemmPlan& plan, const __half* V, __half* M, long long BP,
                        int* dev_status, int num_sms, cudaStream_t s, const char** why);

// The same GEMM on SM pairs (tcgen05 cta_group::2, 256 x BN pair tiles):
// eligible launches and the launch itself (nova_gemm_tc2.cu).
bool tc2_gemm_eligible(const TcGemmPlan& plan, long long BP);
cudaError_t tc2_gemm_run(const TcGemmPlan& plan, const __half* V, __half* M, long long BP,
                         int* dev_status, int num_sms, cudaStream_t s, const char** why);

// Weight-gradient GEMM: Ug[pos][K][C] = sum_bp A[pos][K][bp] * Bop[pos][C][bp]
// (rows `pitch` halves apart, bp < BP valid), FP32.  The reduction is split
// over CTAs when the output tiles alone cannot fill the GPU: split s writes
// its partial sums to Ug + s * 64 * K * C, and the caller adds the
// tc_gemm_wgrad_splits() slices.
constexpr int kWgradMaxSplits = 8;
int tc_gemm_wgrad_splits(int K, int C, long long BP, int num_sms);
cudaError_t tc_gemm_wgrad_run(const __half* A, const __half* Bop, float* Ug, int K, int C,
                              long long BP, long long pitch, int* dev_status, int num_sms,
                              cudaStream_t s, const char** why);

// 3-D FP16 tensor map over [64][rows][C] (C fastest), box {64, box_rows, 1},
// SWIZZLE_128B: the layout of the UMMA K-major operands.
bool tc_encode_operand_map(CUtensorMap* map, const void* ptr, int C, long long rows,
                           int box_rows);

// Single-kernel forward (transform -> tcgen05 MMA -> inverse) for C, K <= 64.
struct FusedPlan {
  CUtensorMap tmU;  // U internal layout [64][K][C], box {64 c, 64 k, 1}
  int K = 0, C = 0;
  bool valid = false;
};

// True when (C, K) is a shape the fused kernel takes: C in {16, 32, 48, 64}, K <= 64.
bool fused_supported(int C, int K);
cudaError_t fused_plan(FusedPlan* plan, const __half* U, int K, int C, const char** why);
// y = conv(x) for the whole batch; no workspace.
cudaError_t fused_run(const FusedPlan& plan, const __half* x, __half* y, int B, int H, int W,
                      int pad, int* dev_status, int num_sms, cudaStream_t s, const char** why);

}  // namespace nova
