// nova_forward_noalloc: a forward that performs no device allocation at all.
//
// Who needs it: callers that may not allocate device memory at the point where
// they run the convolution -- plugins inside an inference runtime that owns all
// device memory and forbids allocation in its enqueue step, code that runs
// under an allocation-free real-time budget, or hosts whose memory is carved up
// once at start-up.  Such a caller cannot create a handle either (nova_create
// and nova_set_weights allocate), so this entry point takes no handle: the
// caller passes x, the transformed filter U (reference layout [64][C][K],
// produced once by nova_filter_transform into memory the caller owns) and y.
//
// The V / M intermediates live in one file-scope device array of fixed size
// (kNoAllocScratchBytes), which every GPU that loads the library holds until
// the process exits.  Its host-side name is only a stand-in for the symbol, so
// its device address is looked up with cudaGetSymbolAddress once per device,
// on the first call made on that device (make that first call before any
// stream capture).  Every call on a device shares the array: calls that overlap
// on the GPU (different streams, no ordering) race on it.  Nothing in the array
// needs clearing: each call writes every V and M element it later reads.
#include <atomic>
#include <string>

#include "../../include/nova_winograd.h"
#include "nova_internal.h"

namespace nova {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;  // 32 MiB for V + M

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// M[pos][bp][k] = sum_c V[pos][bp][c] * U[pos][c][k] with U in the reference
// layout (k fastest); FP32 accumulate, FP16 store.
__global__ void __launch_bounds__(256) gemm_uref_kernel(const __half* __restrict__ V,
                                                        const __half* __restrict__ U,
                                                        __half* __restrict__ M, long long BP,
                                                        int C, int K) {
  constexpr int T = 64, SC = 16;
  __shared__ float As[SC][T + 1];
  __shared__ float Bs[SC][T + 1];
  const int pos = blockIdx.z;
  const long long bp0 = (long long)blockIdx.x * T;
  const int k0 = blockIdx.y * T;
  const __half* Vp = V + (long long)pos * BP * C;
  const __half* Up = U + (long long)pos * K * C;
  __half* Mp = M + (long long)pos * BP * K;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int c0 = 0; c0 < C; c0 += SC) {
    for (int i = threadIdx.x; i < SC * T; i += 256) {
      const int a_cl = i % SC, a_r = i / SC;  // V: c fastest
      const int b_r = i % T, b_cl = i / T;    // U: k fastest
      const long long bp = bp0 + a_r;
      As[a_cl][a_r] = (c0 + a_cl < C && bp < BP) ? __half2float(Vp[bp * C + c0 + a_cl]) : 0.f;
      Bs[b_cl][b_r] = (c0 + b_cl < C && k0 + b_r < K)
                          ? __half2float(Up[(long long)(c0 + b_cl) * K + k0 + b_r])
                          : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int cl = 0; cl < SC; ++cl) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[cl][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[cl][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const long long bp = bp0 + ty * 4 + i;
    if (bp >= BP) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + tx * 4 + j;
      if (k < K) Mp[bp * K + k] = __float2half_rn(acc[i][j]);
    }
  }
}

namespace {
// Errors are reported through the library's last-error string
// (nova_last_error_string).
int noalloc_fail(int code, const std::string& msg) { return record_error(code, msg); }

// Device address of the scratch array on the current device (looked up once).
// Host threads may make their first calls concurrently: the slots are atomic,
// and a racing lookup stores the same address.
unsigned char* scratch_address(int* rc) {
  static std::atomic<unsigned char*> addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *rc = noalloc_fail(NOVA_ERR_CUDA, "forward_noalloc: no usable current device");
    return nullptr;
  }
  unsigned char* known = addr[dev].load(std::memory_order_relaxed);
  if (!known) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *rc = noalloc_fail(NOVA_ERR_CUDA, std::string("forward_noalloc: cudaGetSymbolAddress: ") +
                                            cudaGetErrorString(e));
      return nullptr;
    }
    known = static_cast<unsigned char*>(p);
    addr[dev].store(known, std::memory_order_relaxed);
  }
  *rc = NOVA_OK;
  return known;
}
}  // namespace

}  // namespace nova

extern "C" __attribute__((visibility("default"))) int nova_forward_noalloc(
    const void* d_input, const void* d_U_gemm, void* d_output, int batch, int C, int K, int H,
    int W, int pad, void* stream) {
  using namespace nova;
  if (batch < 0 || C <= 0 || K <= 0 || H <= 0 || W <= 0 || pad < 0 || H + 2 * pad - 2 <= 0 ||
      W + 2 * pad - 2 <= 0)
    return noalloc_fail(NOVA_ERR_INVALID_ARGUMENT, "forward_noalloc: bad sizes");
  if (batch == 0) return NOVA_OK;
  if (!d_input || !d_U_gemm || !d_output)
    return noalloc_fail(NOVA_ERR_INVALID_ARGUMENT, "forward_noalloc: null pointer");
  const int H_out = H + 2 * pad - 2, W_out = W + 2 * pad - 2;
  const int nh = (H_out + 5) / 6, nw = (W_out + 5) / 6;
  const long long BP = (long long)batch * nh * nw;
  const size_t v_bytes = ((size_t)64 * C * BP * 2 + 255) & ~size_t(255);
  const size_t m_bytes = (size_t)64 * K * BP * 2;
  if (v_bytes + m_bytes > kNoAllocScratchBytes)
    return noalloc_fail(NOVA_ERR_WORKSPACE,
                        "forward_noalloc: V + M need " + std::to_string(v_bytes + m_bytes) +
                            " bytes, more than the fixed " +
                            std::to_string(kNoAllocScratchBytes) +
                            "-byte scratch; use nova_forward_workspace with caller memory");
  int rc = NOVA_OK;
  unsigned char* base = scratch_address(&rc);
  if (!base) return rc;
  __half* V = reinterpret_cast<__half*>(base);
  __half* M = reinterpret_cast<__half*>(base + v_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_input_transform(static_cast<const __half*>(d_input), V, batch, C, H, W,
                                         pad, nh, nw, BP, s);
  if (e == cudaSuccess) {
    dim3 grid((unsigned)((BP + 63) / 64), (K + 63) / 64, 64);
    gemm_uref_kernel<<<grid, 256, 0, s>>>(V, static_cast<const __half*>(d_U_gemm), M, BP, C, K);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess)
    e = launch_output_transform(M, static_cast<__half*>(d_output), batch, K, H_out, W_out, nh, nw,
                                BP, s);
  if (e != cudaSuccess)
    return noalloc_fail(NOVA_ERR_CUDA, std::string("forward_noalloc: ") + cudaGetErrorString(e));
  return NOVA_OK;
}
