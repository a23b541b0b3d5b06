// Winograd transform kernels (CUDA cores) and the SIMT batched GEMM used for
// shapes the tensor-core GEMM does not take.
//
// Layouts (element offsets, FP16 unless stated):
//   x  NCHW [B][C][H][W]
//   V  [64 pos][BP][C]   at pos*BP*C + bp*C + c        (c fastest)
//   U  internal [64 pos][K][C] at pos*K*C + k*C + c    (c fastest, K-major GEMM operand)
//   U  reference [64 pos][C][K] at pos*K*C + c*K + k   (k fastest)
//   M  [64 pos][BP][K]   at pos*BP*K + bp*K + k        (k fastest), FP16
//   y  NCHW [B][K][H_out][W_out]
// with bp = (b*nh + th)*nw + tw.  V and M are exactly the reference's V_gemm /
// M_gemm layouts (csrc/nova_winograd.hip:391 and :434 of Jayluci4/nova-wino-amd)
// when nh, nw are the reference tiling.

#include "nova_internal.h"

namespace nova {

// ---------------------------------------------------------------------------
// Filter transform: U = G w G^T in FP32, stored FP16.
// Reference: filter_transform_kernel, csrc/nova_winograd.hip:214-255.
// One thread per (k, c); the fast thread index follows the fast axis of the
// output layout so the 64 stores of a warp are coalesced.
// ---------------------------------------------------------------------------
template <bool kRefLayout>
__global__ void __launch_bounds__(256) filter_transform_kernel(const float* __restrict__ w,
                                                               __half* __restrict__ U, int K,
                                                               int C) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long KC = (long long)K * C;
  if (idx >= KC) return;
  int k, c;
  if (kRefLayout) {
    k = (int)(idx % K);
    c = (int)(idx / K);
  } else {
    c = (int)(idx % C);
    k = (int)(idx / C);
  }
  const float* wp = w + ((long long)k * C + c) * 9;
  float g[3][3];
#pragma unroll
  for (int i = 0; i < 9; ++i) g[i / 3][i % 3] = wp[i];
  float t[8][3];  // t = G w
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int q = 0; q < 3; ++q)
      t[i][q] = kG(i, 0) * g[0][q] + kG(i, 1) * g[1][q] + kG(i, 2) * g[2][q];
  const long long off = kRefLayout ? ((long long)c * K + k) : ((long long)k * C + c);
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float u = t[i][0] * kG(j, 0) + t[i][1] * kG(j, 1) + t[i][2] * kG(j, 2);
      U[(long long)(i * 8 + j) * KC + off] = __float2half_rn(u);
    }
}

// ---------------------------------------------------------------------------
// Input transform: V = B^T d B per (b, c, tile), zero padding fused.
// Reference: input_transform_kernel(_mt), csrc/nova_winograd.hip:141-205, 338-392.
//
// A block owns one tile row th of one image, kTW consecutive tiles along w and
// 32 channels.  The 8 input rows it needs are staged once in shared memory with
// loads that run along w (coalesced), laid out [row][col][channel] with a
// 17-word channel pitch so both the staging stores and the per-tile reads are
// bank-conflict free.  A warp then transforms one tile for 32 channels (lane =
// channel) and its 64 stores per position are one contiguous 64-byte run of V.
// ---------------------------------------------------------------------------
constexpr int kTW = 8;                 // tiles per block along w
constexpr int kCG = 32;                // channels per block
constexpr int kCols = kTW * 6 + 2;     // staged input columns
constexpr int kCPad = 34;              // halves per staged (row, col) cell

__global__ void __launch_bounds__(256) input_transform_kernel(
    const __half* __restrict__ x, __half* __restrict__ V, int C, int H, int W, int pad, int nh,
    int nw, long long BP, int n_twc) {
  __shared__ __half xs[8][kCols][kCPad];
  const int cg = blockIdx.x / n_twc;
  const int twc = blockIdx.x % n_twc;
  const int th = blockIdx.y;
  const int b = blockIdx.z;
  const int c0 = cg * kCG;
  const int tw0 = twc * kTW;
  const int ntw = min(kTW, nw - tw0);
  const int cols = ntw * 6 + 2;
  const int h0 = th * 6 - pad;
  const int w0 = tw0 * 6 - pad;

  const int total = kCG * 8 * cols;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int col = i % cols;
    const int r = (i / cols) & 7;
    const int cl = i / (cols * 8);
    const int c = c0 + cl, h = h0 + r, ww = w0 + col;
    __half v = __float2half_rn(0.f);
    if (c < C && h >= 0 && h < H && ww >= 0 && ww < W)
      v = x[(((long long)b * C + c) * H + h) * W + ww];
    xs[r][col][cl] = v;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = c0 + lane;
  const long long plane = BP * (long long)C;
  for (int t = warp; t < ntw; t += blockDim.x >> 5) {
    float tmp[8][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // columns: tmp[.][j] = B^T d[.][j]
      float v[8], f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __half2float(xs[i][t * 6 + j][lane]);
      bt_1d(v, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) tmp[i][j] = f[i];
    }
    if (c < C) {
      const long long bp = ((long long)b * nh + th) * nw + tw0 + t;
      __half* out = V + bp * C + c;
#pragma unroll
      for (int r = 0; r < 8; ++r) {  // rows: V[r][.] = tmp[r][.] B
        float f[8];
        bt_1d(tmp[r], f);
#pragma unroll
        for (int s = 0; s < 8; ++s) out[(long long)(r * 8 + s) * plane] = __float2half_rn(f[s]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Output transform: Y = A M A^T (6x6 of 8x8), bounds-checked NCHW store.
// Reference: output_transform_kernel(_mt), csrc/nova_winograd.hip:264-328, 398-450.
//
// Mirror image of the input transform: a warp reads the 64 positions of one
// tile for 32 output channels (64-byte runs of M), transforms in registers and
// parks the 6x6 results in shared memory; the block then writes whole output
// row segments along w.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) output_transform_kernel(
    const __half* __restrict__ M, __half* __restrict__ y, int K, int H_out, int W_out, int nh,
    int nw, long long BP, int n_twc) {
  __shared__ __half ys[6][kTW * 6][kCPad];
  const int kg = blockIdx.x / n_twc;
  const int twc = blockIdx.x % n_twc;
  const int th = blockIdx.y;
  const int b = blockIdx.z;
  const int k0 = kg * kCG;
  const int tw0 = twc * kTW;
  const int ntw = min(kTW, nw - tw0);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k = k0 + lane;
  const long long plane = BP * (long long)K;
  for (int t = warp; t < ntw; t += blockDim.x >> 5) {
    const long long bp = ((long long)b * nh + th) * nw + tw0 + t;
    const __half* in = M + bp * K + k;
    float tmp[6][8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // columns: tmp[.][q] = A m[.][q]
      float m[8], g[6];
#pragma unroll
      for (int p = 0; p < 8; ++p)
        m[p] = (k < K) ? __half2float(in[(long long)(p * 8 + q) * plane]) : 0.f;
      a_1d(m, g);
#pragma unroll
      for (int i = 0; i < 6; ++i) tmp[i][q] = g[i];
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) {  // rows: Y[i][.] = tmp[i][.] A^T
      float g[6];
      a_1d(tmp[i], g);
#pragma unroll
      for (int j = 0; j < 6; ++j) ys[i][t * 6 + j][lane] = __float2half_rn(g[j]);
    }
  }
  __syncthreads();

  const int cols = ntw * 6;
  const int total = kCG * 6 * cols;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int col = i % cols;
    const int r = (i / cols) % 6;
    const int kl = i / (cols * 6);
    const int kk = k0 + kl, h = th * 6 + r, ww = tw0 * 6 + col;
    if (kk < K && h < H_out && ww < W_out)
      y[(((long long)b * K + kk) * H_out + h) * W_out + ww] = ys[r][col][kl];
  }
}

// ---------------------------------------------------------------------------
// SIMT batched GEMM: M[pos][bp][k] = sum_c V[pos][bp][c] U[pos][k][c], FP32
// accumulate, FP16 store.  Used when C % 8 != 0 or K % 16 != 0 (shapes the
// tensor-core path's TMA / MMA granularity does not cover, e.g. C = 3).
// ---------------------------------------------------------------------------
constexpr int kST = 64, kSC = 16;

__global__ void __launch_bounds__(256) gemm_simt_kernel(const __half* __restrict__ V,
                                                        const __half* __restrict__ U,
                                                        __half* __restrict__ M, long long BP, int C,
                                                        int K) {
  __shared__ float As[kSC][kST + 1];
  __shared__ float Bs[kSC][kST + 1];
  const int pos = blockIdx.z;
  const long long bp0 = (long long)blockIdx.x * kST;
  const int k0 = blockIdx.y * kST;
  const __half* Vp = V + (long long)pos * BP * C;
  const __half* Up = U + (long long)pos * K * C;
  __half* Mp = M + (long long)pos * BP * K;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int c0 = 0; c0 < C; c0 += kSC) {
    for (int i = threadIdx.x; i < kSC * kST; i += 256) {
      const int cl = i % kSC, r = i / kSC;
      const int c = c0 + cl;
      const long long bp = bp0 + r;
      const int k = k0 + r;
      As[cl][r] = (c < C && bp < BP) ? __half2float(Vp[bp * C + c]) : 0.f;
      Bs[cl][r] = (c < C && k < K) ? __half2float(Up[(long long)k * C + c]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int cl = 0; cl < kSC; ++cl) {
      float a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[cl][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Bs[cl][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
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

// ---------------------------------------------------------------------------
// Launchers.
// ---------------------------------------------------------------------------
cudaError_t launch_filter_transform(const float* w, __half* U, int K, int C, bool ref_layout,
                                    cudaStream_t s) {
  const long long n = (long long)K * C;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (ref_layout)
    filter_transform_kernel<true><<<blocks, 256, 0, s>>>(w, U, K, C);
  else
    filter_transform_kernel<false><<<blocks, 256, 0, s>>>(w, U, K, C);
  return cudaGetLastError();
}

cudaError_t launch_input_transform(const __half* x, __half* V, int B, int C, int H, int W,
                                   int pad, int nh, int nw, long long BP, cudaStream_t s) {
  if (C % 2 == 0)
    return launch_input_transform_fast(x, V, B, C, H, W, pad, nh, nw, 0, (long long)B * nh, BP, s);
  const int n_twc = (nw + kTW - 1) / kTW;
  const int n_cg = (C + kCG - 1) / kCG;
  dim3 grid(n_twc * n_cg, nh, B);
  input_transform_kernel<<<grid, 256, 0, s>>>(x, V, C, H, W, pad, nh, nw, BP, n_twc);
  return cudaGetLastError();
}

cudaError_t launch_output_transform(const __half* M, __half* y, int B, int K, int H_out,
                                    int W_out, int nh, int nw, long long BP, cudaStream_t s) {
  if (K % 2 == 0)
    return launch_output_transform_fast(M, y, K, H_out, W_out, nh, nw, 0, (long long)B * nh, BP,
                                        s);
  const int n_twc = (nw + kTW - 1) / kTW;
  const int n_kg = (K + kCG - 1) / kCG;
  dim3 grid(n_twc * n_kg, nh, B);
  output_transform_kernel<<<grid, 256, 0, s>>>(M, y, K, H_out, W_out, nh, nw, BP, n_twc);
  return cudaGetLastError();
}

cudaError_t launch_gemm_simt(const __half* V, const __half* U, __half* M, long long BP, int C,
                             int K, cudaStream_t s) {
  dim3 grid((unsigned)((BP + kST - 1) / kST), (K + kST - 1) / kST, 64);
  gemm_simt_kernel<<<grid, 256, 0, s>>>(V, U, M, BP, C, K);
  return cudaGetLastError();
}

}  // namespace nova
