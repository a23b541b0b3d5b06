// Weight gradient of the NOVA F(6,3) convolution by the same Winograd algorithm.
//
// The reference computes grad_weight with a per-sample unfold loop in FP32
// PyTorch (Jayluci4/nova-wino-amd nova_winograd/conv2d.py:131-141 and the
// custom-op backward :66-80).  The forward is y = A [ (G w G^T) . (B^T d B) ] A^T
// per tile; differentiating it with respect to w gives, summed over tiles,
//
//   dW[k][c] = G^T [ sum_tiles (A^T dY_k A) . (B^T d_c B) ] G
//
// (dY_k = the tile's 6x6 output gradient, zero past H_out / W_out; d_c = the
// same 8x8 input windows as the forward).  Three steps:
//
// 1. V^T[pos][c][bp] = B^T d B and G'^T[pos][k][bp] = A^T dY A, FP32 arithmetic
//    stored FP16 (as the forward stores V), with the tile index bp contiguous:
//    one lane per tile, so each warp store is 32 consecutive tiles of one
//    (position, channel).
// 2. Ug[pos][k][c] = sum_bp G'^T[pos][k][bp] V^T[pos][c][bp]: the tcgen05 GEMM
//    with the tile index as its reduction, split over CTAs, FP32 atomic adds.
// 3. dW[k][c] = G^T Ug[.][k][c] G in FP32.
//
// In exact arithmetic this is the exact gradient of the convolution; with the
// FP16 storage of V and G' its error is of the order of the forward's.
#include <string>

#include "../../include/nova_winograd.h"
#include "nova_internal.h"

namespace nova {
namespace wgrad {

constexpr int kChanPerBlock = 4;  // one channel per warp, the same 32 tiles

// G for runtime-indexed rows (the same FP32 table as kG).
__constant__ float c_G[8][3] = {
    {kG(0, 0), kG(0, 1), kG(0, 2)}, {kG(1, 0), kG(1, 1), kG(1, 2)},
    {kG(2, 0), kG(2, 1), kG(2, 2)}, {kG(3, 0), kG(3, 1), kG(3, 2)},
    {kG(4, 0), kG(4, 1), kG(4, 2)}, {kG(5, 0), kG(5, 1), kG(5, 2)},
    {kG(6, 0), kG(6, 1), kG(6, 2)}, {kG(7, 0), kG(7, 1), kG(7, 2)}};

// m[n] = sum_i A[i][n] g[i]  (6 -> 8, the transpose of a_1d): the columns of A
// pair up as n = 1/2, 3/4, 5/6 (even part +- odd part); n = 0 and 7 are g[0]
// and g[5].
__device__ __forceinline__ void at_1d(const float g[6], float m[8]) {
  const float e1 = fmaf(kA036, g[2], fmaf(kA01296, g[4], g[0]));
  const float o1 = fmaf(kA06, g[1], fmaf(kA0216, g[3], kA00778 * g[5]));
  const float e2 = g[0] + g[2] + g[4];
  const float o2 = g[1] + g[3] + g[5];
  const float e3 = fmaf(kA1361, g[2], fmaf(kA1853, g[4], g[0]));
  const float o3 = fmaf(kA1167, g[1], fmaf(kA1588, g[3], kA2161 * g[5]));
  m[0] = g[0];
  m[1] = e1 + o1;
  m[2] = e1 - o1;
  m[3] = e2 + o2;
  m[4] = e2 - o2;
  m[5] = e3 + o3;
  m[6] = e3 - o3;
  m[7] = g[5];
}

// One 2-byte global store kept in program order (as plain stores, the compiler
// gathers all 64 of a tile with their 64-bit addresses and spills).
__device__ __forceinline__ void st_global_f16(__half* p, float v) {
  const __half h = __float2half_rn(v);
  asm volatile("st.global.b16 [%0], %1;" ::"l"(p), "h"(__half_as_ushort(h)) : "memory");
}

struct TArgs {
  int Cn, H, W, pad;  // channels of the tensor read; its spatial size; input padding
  int nh, nw;
  long long BP, pitch;
};

// V^T[pos][c][bp] = (B^T d B)[pos] for tile bp, channel c.  Block: 32
// consecutive tiles (one per lane) x kChanPerBlock channels (one per warp).
__global__ void __launch_bounds__(128) input_transform_t(const __half* __restrict__ x,
                                                         __half* __restrict__ VT, const TArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long bp = (long long)blockIdx.x * 32 + lane;
  const int c0 = blockIdx.y * kChanPerBlock + warp;
  if (bp >= a.BP || c0 >= a.Cn) return;
  const int P = a.nh * a.nw;
  const int b = (int)(bp / P);
  const int tp = (int)(bp - (long long)b * P);
  const int th = tp / a.nw, tw = tp - th * a.nw;
  const int h0 = th * 6 - a.pad, w0 = tw * 6 - a.pad;
  const long long plane = (long long)a.H * a.W;
  // Lane-constant row offsets and column validity of the 8x8 window.
  int roff[8];
  unsigned cmask = 0;  // bit j: column w0 + j exists
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int h = h0 + i;
    roff[i] = (h >= 0 && h < a.H) ? h * a.W : -1;
    const int w = w0 + i;
    if (w >= 0 && w < a.W) cmask |= 1u << i;
  }
  {
    const int c = c0;
    const __half* xc = x + ((long long)b * a.Cn + c) * plane + w0;
    // The window, packed in column pairs (32 registers).
    __half2 pr[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const bool ok = roff[i] >= 0;
        const __half lo = (ok && ((cmask >> (2 * q)) & 1u)) ? __ldg(xc + roff[i] + 2 * q)
                                                            : __ushort_as_half(0);
        const __half hi = (ok && ((cmask >> (2 * q + 1)) & 1u)) ? __ldg(xc + roff[i] + 2 * q + 1)
                                                                : __ushort_as_half(0);
        pr[i][q] = __halves2half2(lo, hi);
      }
    __half* const vt = VT + (long long)c * a.pitch + bp;
    const long long step = (long long)a.Cn * a.pitch;  // one position
    // Column pass in two halves of its output rows ({0,1,2,7}, {3,4,5,6}).
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      float tt[4][8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // columns: tmp[.][j] = B^T d[.][j]
        float v[8], f[4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = (j & 1) ? __high2float(pr[i][j >> 1]) : __low2float(pr[i][j >> 1]);
        if (half == 0)
          bt_1d_a(v, f);
        else
          bt_1d_b(v, f);
#pragma unroll
        for (int i = 0; i < 4; ++i) tt[i][j] = f[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // rows: V[r][.] = tmp[r][.] B
        const int r = half == 0 ? (i < 3 ? i : 7) : 3 + i;
        float f[8];
        bt_1d(tt[i], f);
        __half* out = vt + (long long)(r * 8) * step;
#pragma unroll
        for (int s2 = 0; s2 < 8; ++s2) {
          st_global_f16(out, f[s2]);
          out += step;
        }
      }
    }
  }
}

// G'^T[pos][k][bp] = (A^T dY A)[pos] for tile bp, output channel k (dY zero past
// H_out x W_out, which are a.H x a.W here).
__global__ void __launch_bounds__(128, 4) grad_output_transform_t(const __half* __restrict__ dy,
                                                               __half* __restrict__ GT,
                                                               const TArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long bp = (long long)blockIdx.x * 32 + lane;
  const int k0 = blockIdx.y * kChanPerBlock + warp;
  if (bp >= a.BP || k0 >= a.Cn) return;
  const int P = a.nh * a.nw;
  const int b = (int)(bp / P);
  const int tp = (int)(bp - (long long)b * P);
  const int th = tp / a.nw, tw = tp - th * a.nw;
  const int h0 = th * 6, w0 = tw * 6;
  const long long plane = (long long)a.H * a.W;
  {
    const int k = k0;
    const __half* gk = dy + ((long long)b * a.Cn + k) * plane;
    float tt[8][6];
#pragma unroll
    for (int j = 0; j < 6; ++j) {  // columns: tmp[.][j] = A^T g[.][j]
      float g[6], m[8];
      const int w = w0 + j;
#pragma unroll
      for (int i = 0; i < 6; ++i) {
        const int h = h0 + i;
        g[i] = (h < a.H && w < a.W) ? __half2float(__ldg(gk + h * a.W + w)) : 0.f;
      }
      at_1d(g, m);
#pragma unroll
      for (int n = 0; n < 8; ++n) tt[n][j] = m[n];
    }
    __half* out = GT + (long long)k * a.pitch + bp;
    const long long step = (long long)a.Cn * a.pitch;
#pragma unroll
    for (int n = 0; n < 8; ++n) {  // rows: G'[n][.] = tmp[n][.] A
      float m[8];
      at_1d(tt[n], m);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        st_global_f16(out, m[q]);
        out += step;
      }
    }
  }
}

// dW[k][c][u][v] = sum_{n,m} G[n][u] G[m][v] Ug[n*8+m][k][c], FP32.  Ug holds
// n_split slices of partial sums over the tiles, added here in slice order.
// Block: 32 consecutive (k, c) pairs (one per lane) x the 8 position rows n
// (one per warp): warp n forms G[n][u] sum_m Ug[n][m] G[m][v] for its rows,
// and the 8 partial 3x3 results are added through shared memory in n order.
__global__ void __launch_bounds__(256) filter_back_transform(const float* __restrict__ Ug,
                                                             float* __restrict__ dw, int K,
                                                             int C, int n_split) {
  // Block: 128 consecutive (k, c) pairs, four per lane (16-byte loads; K * C is
  // a multiple of 4 since C is a multiple of 16), x the 8 position rows n (one
  // per warp).
  __shared__ float part[8][9][132];
  const int lane = threadIdx.x & 31, n = threadIdx.x >> 5;
  const long long stride = (long long)K * C;
  const long long kc0 = (long long)blockIdx.x * 128 + lane * 4;
  if (kc0 < stride) {
    float4 u[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const float* q = Ug + (n * 8 + m) * stride + kc0;
      float4 acc = *reinterpret_cast<const float4*>(q);
      for (int sp = 1; sp < n_split; ++sp) {
        const float4 t = *reinterpret_cast<const float4*>(q + (long long)sp * 64 * stride);
        acc.x += t.x;
        acc.y += t.y;
        acc.z += t.z;
        acc.w += t.w;
      }
      u[m] = acc;
    }
#pragma unroll
    for (int v = 0; v < 3; ++v) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);  // sum_m Ug[n][m] G[m][v]
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        t.x = fmaf(u[m].x, kG(m, v), t.x);
        t.y = fmaf(u[m].y, kG(m, v), t.y);
        t.z = fmaf(u[m].z, kG(m, v), t.z);
        t.w = fmaf(u[m].w, kG(m, v), t.w);
      }
#pragma unroll
      for (int uu = 0; uu < 3; ++uu) {
        const float g = c_G[n][uu];
        float* dst = &part[n][uu * 3 + v][lane * 4];
        dst[0] = g * t.x;
        dst[1] = g * t.y;
        dst[2] = g * t.z;
        dst[3] = g * t.w;
      }
    }
  }
  __syncthreads();
  // 128 pairs x 9 outputs: consecutive threads write consecutive floats of dW.
  for (int i = threadIdx.x; i < 128 * 9; i += blockDim.x) {
    const int l = i / 9, e = i - (i / 9) * 9;
    const long long kcl = (long long)blockIdx.x * 128 + l;
    if (kcl >= stride) continue;
    float acc = 0.f;
#pragma unroll
    for (int nn = 0; nn < 8; ++nn) acc += part[nn][e][l];
    dw[kcl * 9 + e] = acc;
  }
}

struct Layout {
  int nh, nw, H_out, W_out;
  long long BP, pitch;
  int splits;  // slices of partial sums the GEMM writes (device-dependent)
  size_t vt_bytes, gt_bytes, ug_bytes, total;  // total includes a 256-byte status word
};

static size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

static int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess &&
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    sms = 148;
  return sms;
}

static bool layout(int B, int C, int K, int H, int W, int pad, Layout* L) {
  if (B <= 0 || C <= 0 || K <= 0 || H <= 0 || W <= 0 || pad < 0) return false;
  L->H_out = H + 2 * pad - 2;
  L->W_out = W + 2 * pad - 2;
  if (L->H_out <= 0 || L->W_out <= 0) return false;
  L->nh = (L->H_out + 5) / 6;
  L->nw = (L->W_out + 5) / 6;
  L->BP = (long long)B * L->nh * L->nw;
  L->pitch = (L->BP + 7) / 8 * 8;  // 16-byte row pitch for the GEMM's tensor maps
  L->vt_bytes = align256((size_t)64 * C * L->pitch * 2);
  L->gt_bytes = align256((size_t)64 * K * L->pitch * 2);
  L->splits = tc_gemm_wgrad_splits(K, C, L->BP, device_sms());
  L->ug_bytes = align256((size_t)L->splits * 64 * K * C * 4);
  L->total = L->vt_bytes + L->gt_bytes + L->ug_bytes + 256;
  return true;
}

}  // namespace wgrad
}  // namespace nova

extern "C" __attribute__((visibility("default"))) long long nova_weight_grad_workspace_bytes(
    int batch, int C, int K, int H, int W, int pad) {
  nova::wgrad::Layout L;
  if (!nova::wgrad::layout(batch, C, K, H, W, pad, &L)) return -1;
  return (long long)L.total;
}

extern "C" __attribute__((visibility("default"))) int nova_weight_grad_v2(
    const void* d_input, const void* d_grad_output, void* d_grad_weight, void* d_workspace,
    long long workspace_bytes, int batch, int C, int K, int H, int W, int pad, void* stream) {
  using namespace nova;
  using namespace nova::wgrad;
  Layout L;
  if (!layout(batch, C, K, H, W, pad, &L))
    return record_error(NOVA_ERR_INVALID_ARGUMENT, "weight_grad: bad sizes");
  if (!d_input || !d_grad_output || !d_grad_weight || !d_workspace)
    return record_error(NOVA_ERR_INVALID_ARGUMENT, "weight_grad: null pointer");
  if (C % 16 != 0)
    return record_error(NOVA_ERR_INVALID_ARGUMENT,
                        "weight_grad: C must be a multiple of 16 (the GEMM's N)");
  if (reinterpret_cast<uintptr_t>(d_workspace) % 256)
    return record_error(NOVA_ERR_INVALID_ARGUMENT, "weight_grad: workspace not 256-byte aligned");
  if (workspace_bytes < (long long)L.total)
    return record_error(NOVA_ERR_WORKSPACE, "weight_grad: workspace needs " +
                                                std::to_string(L.total) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* ws = static_cast<unsigned char*>(d_workspace);
  __half* VT = reinterpret_cast<__half*>(ws);
  __half* GT = reinterpret_cast<__half*>(ws + L.vt_bytes);
  float* Ug = reinterpret_cast<float*>(ws + L.vt_bytes + L.gt_bytes);
  // The GEMM's bounded waits record an expiry here (never read by this call).
  int* status = reinterpret_cast<int*>(ws + L.vt_bytes + L.gt_bytes + L.ug_bytes);
  const int sms = device_sms();
  cudaError_t e = cudaMemsetAsync(status, 0, 256, s);
  const unsigned gx = (unsigned)((L.BP + 31) / 32);
  if (e == cudaSuccess) {
    TArgs ai{C, H, W, pad, L.nh, L.nw, L.BP, L.pitch};
    input_transform_t<<<dim3(gx, (C + kChanPerBlock - 1) / kChanPerBlock), 128, 0, s>>>(
        static_cast<const __half*>(d_input), VT, ai);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    TArgs ag{K, L.H_out, L.W_out, 0, L.nh, L.nw, L.BP, L.pitch};
    grad_output_transform_t<<<dim3(gx, (K + kChanPerBlock - 1) / kChanPerBlock), 128, 0, s>>>(
        static_cast<const __half*>(d_grad_output), GT, ag);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess)
    return record_error(NOVA_ERR_CUDA, std::string("weight_grad: ") + cudaGetErrorString(e));
  const char* why = "";
  e = tc_gemm_wgrad_run(GT, VT, Ug, K, C, L.BP, L.pitch, status, sms, s, &why);
  if (e != cudaSuccess) return record_error(NOVA_ERR_CUDA, std::string("weight_grad: ") + why);
  const long long kc = (long long)K * C;
  filter_back_transform<<<(unsigned)((kc + 127) / 128), 256, 0, s>>>(
      Ug, static_cast<float*>(d_grad_weight), K, C, L.splits);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return record_error(NOVA_ERR_CUDA, std::string("weight_grad: ") + cudaGetErrorString(e));
  return NOVA_OK;
}
