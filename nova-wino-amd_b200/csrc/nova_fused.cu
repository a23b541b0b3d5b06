// Single-kernel NOVA F(6,3) forward for small channel counts (C, K <= 64):
// input transform -> tcgen05 MMA -> output transform, with V in shared memory
// and M in tensor memory, so neither touches HBM.
//
// Replaces the reference's fused_winograd_mfma_kernel
// (Jayluci4/nova-wino-amd csrc/nova_winograd_fused.hip:283-440), which keeps V
// and M in LDS for blocks of 16 tiles and rounds M to FP16 there (:405).  The
// numerics here are the same: V = B^T d B in FP32 stored FP16, M accumulated
// in FP32 by the tensor core and rounded to FP16, Y = A M A^T in FP32 stored
// FP16.
//
// Shape of one CTA (8 tiles, all K output channels, 256 threads, 2 CTAs/SM):
//
// * Input transform.  Input channels go in passes of 32: the 8x8 patches of
//   the CTA's 8 tiles are staged in shared memory ([tile][channel][64], odd
//   word pitch), then warp w transforms tile w with lane = channel and writes
//   V straight into the UMMA operand layout: one 1024-byte SWIZZLE_128B atom
//   per position (8 tile rows x 64 channels).
// * GEMM.  Per position p, D_p[k][t] = sum_c U_p[k][c] V_p[t][c] is one
//   M=64 x N=8 MMA chain (K = C in steps of 16); U_p (64 x 64 FP16, 8 KB) is
//   streamed by TMA through a 4-slot ring that reuses the staging memory.
//   M=64 accumulators fill half of each 32-lane TMEM sub-partition, so even
//   positions go to lanes 0-15 and odd positions to lanes 16-31 of the same
//   columns: 64 positions x 8 tiles fit in 256 columns.
// * Output transform.  The thread at TMEM lane 32q + l owns output channel
//   k = 16q + (l & 15) and the positions of parity l >> 4.  It applies A along
//   the position rows it holds completely (i), swaps half of the partial sums
//   with lane l ^ 16, and applies A along j for three of the six output rows.
//
// Waits on mbarriers are bounded (2 s); on expiry the kernel records
// kDevTimeoutFused in the device status word, skips its stores and frees TMEM.
#include "nova_internal.h"
#include "nova_tc_ptx.cuh"

namespace nova {
namespace fused {

using namespace tc;

constexpr int kT = 8;                        // tiles per CTA (MMA N)
constexpr int kThreads = 256;
constexpr int kCPass = 32;                   // input channels staged per pass
constexpr int kXsPitch = 66;                 // halves per staged (tile, channel) patch
constexpr int kUStages = 4;
constexpr int kUBytes = 64 * 64 * 2;         // U of one position: 64 k rows x 128 B
constexpr int kTmemCols = 256;
constexpr int kVsBytes = 64 * kT * 128;      // 64 KB
constexpr int kXsBytes = kT * kCPass * kXsPitch * 2;
constexpr int kRingBytes = kUStages * kUBytes;
constexpr int kUnionBytes = kXsBytes > kRingBytes ? kXsBytes : kRingBytes;
constexpr int kMetaBytes = 256;
constexpr int kSmemBytes = 1024 + kVsBytes + kUnionBytes + kMetaBytes;

#ifdef NOVA_FUSED_TRACE
// Debug builds only: per-CTA globaltimer stamps at the phase boundaries.
constexpr int kTraceCtas = 8192;
__device__ unsigned long long g_fused_trace[kTraceCtas * 4];
#define FUSED_MARK(i)                                   \
  if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) \
    g_fused_trace[blockIdx.x * 4 + (i)] = globaltimer();
#else
#define FUSED_MARK(i)
#endif

struct Params {
  const __half* x;
  __half* y;
  int C, K, H, W, pad, H_out, W_out, nh, nw;
  long long BP;
  int* status;
};

__device__ __forceinline__ void tmem_ld_x2(uint32_t taddr, uint32_t& a, uint32_t& b) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
               : "=r"(a), "=r"(b)
               : "r"(taddr));
}

// Waits for this thread's outstanding TMEM loads.  The registers pass through
// the asm so no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld32(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
        "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
        "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, __half v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(__half_as_ushort(v)) : "memory");
}

__device__ __forceinline__ float round_f16(uint32_t bits) {
  return __half2float(__float2half_rn(__uint_as_float(bits)));
}

__global__ void __launch_bounds__(kThreads, 2)
    fused_forward_kernel(const __grid_constant__ CUtensorMap tmU, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* Vs = base;
  uint8_t* ring = base + kVsBytes;  // staged input during the transform, then the U ring
  __half* Xs = reinterpret_cast<__half*>(ring);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kUnionBytes);
  uint64_t* ufull = bars;
  uint64_t* uempty = bars + kUStages;
  uint64_t* done = bars + 2 * kUStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* t_n = const_cast<int*>(abort_flag + 1);  // image of tile t, -1 past BP
  int* t_h0 = t_n + kT;                         // 6*th - pad
  int* t_w0 = t_h0 + kT;                        // 6*tw - pad

  FUSED_MARK(0);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const long long bp0 = (long long)blockIdx.x * kT;

  if (threadIdx.x < kT) {
    const long long bp = bp0 + threadIdx.x;
    int n = -1, th = 0, tw = 0;
    if (bp < p.BP) {
      tw = (int)(bp % p.nw);
      const long long r = bp / p.nw;
      th = (int)(r % p.nh);
      n = (int)(r / p.nh);
    }
    t_n[threadIdx.x] = n;
    t_h0[threadIdx.x] = th * 6 - p.pad;
    t_w0[threadIdx.x] = tw * 6 - p.pad;
  }
  if (threadIdx.x == 32 * 2) {
    for (int s = 0; s < kUStages; ++s) {
      mbar_init(smem_u32(&ufull[s]), 1);
      mbar_init(smem_u32(&uempty[s]), 1);
    }
    mbar_init(smem_u32(done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // ---------------- Input transform: V into the operand layout ----------------
  const long long HW = (long long)p.H * p.W;
  const uint32_t vs_addr = smem_u32(Vs);
  // Staging: thread (r, cc) of each 64-thread group loads patch element (r, cc)
  // of channels cl0, cl0 + 4, ... for every tile; a warp covers 4 rows x 8
  // columns of one channel.  Loads are issued 32 at a time before any store.
  const int st_cc = threadIdx.x & 7, st_r = (threadIdx.x >> 3) & 7, st_cl0 = threadIdx.x >> 6;
  for (int cbase = 0; cbase < p.C; cbase += kCPass) {
#pragma unroll
    for (int tb = 0; tb < kT; tb += 4) {
      __half v[4][kCPass / 4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = tb + u;
        const int n = t_n[t];
        const int h = t_h0[t] + st_r, w = t_w0[t] + st_cc;
        const bool in = n >= 0 && (unsigned)h < (unsigned)p.H && (unsigned)w < (unsigned)p.W;
        const __half* src =
            p.x + ((long long)(in ? n : 0) * p.C + cbase + st_cl0) * HW + (in ? h * p.W + w : 0);
#pragma unroll
        for (int j = 0; j < kCPass / 4; ++j) {
          const bool ok = in && cbase + st_cl0 + 4 * j < p.C;
          v[u][j] = ok ? __ldg(src + (long long)(4 * j) * HW) : __float2half_rn(0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < kCPass / 4; ++j)
          Xs[((tb + u) * kCPass + st_cl0 + 4 * j) * kXsPitch + st_r * 8 + st_cc] = v[u][j];
    }
    __syncthreads();
    {
      const int t = warp;
      const int c = cbase + lane;
      const __half2* xp = reinterpret_cast<const __half2*>(Xs + (t * kCPass + lane) * kXsPitch);
      float d[8][8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          const float2 f = __half22float2(xp[i * 4 + j2]);
          d[i][2 * j2] = f.x;
          d[i][2 * j2 + 1] = f.y;
        }
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // columns: d[.][j] <- B^T d[.][j]
        float v[8], f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = d[i][j];
        bt_1d(v, f);
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i][j] = f[i];
      }
      if (c < p.C) {
        // Byte offset of (pos, tile t, channel c) in the SWIZZLE_128B atoms.
        const uint32_t row = vs_addr + t * 128 + (c & 7) * 2;
        const uint32_t chunk = (uint32_t)(((c >> 3) ^ t) << 4);
#pragma unroll
        for (int r = 0; r < 8; ++r) {  // rows: V[r][.] = d[r][.] B
          float f[8];
          bt_1d(d[r], f);
#pragma unroll
          for (int s = 0; s < 8; ++s)
            st_shared_u16(row + (uint32_t)(r * 8 + s) * 1024u + chunk, __float2half_rn(f[s]));
        }
      }
    }
    __syncthreads();
  }
  fence_async_smem();  // V (and the freed staging memory) visible to the async proxy
  __syncthreads();
  FUSED_MARK(1);

  // ---------------- GEMM: 64 positions of M=64 x N=8 MMAs ----------------
  const int nks = p.C / 16;
  if (warp == 0) {
    if (lane == 0) {
      for (int pos = 0; pos < 64; ++pos) {
        const int s = pos % kUStages;
        const uint32_t ph = (uint32_t)(pos / kUStages) & 1u;
        if (!mbar_wait(smem_u32(&uempty[s]), ph ^ 1u, abort_flag, p.status, kDevTimeoutFused))
          break;
        const uint32_t fb = smem_u32(&ufull[s]);
        mbar_expect_tx(fb, kUBytes);
        tma_load_3d(smem_u32(ring + s * kUBytes), &tmU, 0, 0, pos, fb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | ((uint32_t)(kT >> 3) << 17) | ((uint32_t)(64 >> 4) << 24);
      for (int pos = 0; pos < 64; ++pos) {
        const int s = pos % kUStages;
        const uint32_t ph = (uint32_t)(pos / kUStages) & 1u;
        if (!mbar_wait(smem_u32(&ufull[s]), ph, abort_flag, p.status, kDevTimeoutFused)) break;
        tc_fence_after();
        const uint64_t ad = smem_desc_sw128(smem_u32(ring + s * kUBytes));
        const uint64_t bd = smem_desc_sw128(vs_addr + (uint32_t)pos * 1024u);
        const uint32_t dt = tmem_base + ((uint32_t)((pos & 1) * 16) << 16) + (uint32_t)(pos >> 1) * kT;
        for (int ks = 0; ks < nks; ++ks) umma_f16(dt, ad + 2ull * ks, bd + 2ull * ks, idesc, ks);
        umma_commit(smem_u32(&uempty[s]));
      }
      // Fires once every MMA issued above has completed (also after an abort).
      umma_commit(smem_u32(done));
    }
  }
  __syncwarp();

  // ---------------- Output transform from TMEM ----------------
  const bool got = mbar_wait(smem_u32(done), 0, abort_flag, p.status, kDevTimeoutFused) &&
                   *abort_flag == 0;
  tc_fence_after();
  FUSED_MARK(2);
  if (got) {
    const int q = warp & 3;
    const int h = lane >> 4;
    const int k = q * 16 + (lane & 15);
    const long long plane = (long long)p.H_out * p.W_out;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(q * 32) << 16);
    for (int tp = 0; tp < 2; ++tp) {
      const int t0 = (warp >> 2) * 4 + tp * 2;
      // mv[u][m] = M at position 2m + h of tile t0 + u.
      float mv[2][32];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
#pragma unroll
        for (int m = 0; m < 16; ++m)
          tmem_ld_x2(lane_addr + (uint32_t)(half * 16 + m) * kT + t0, r[2 * m], r[2 * m + 1]);
        tmem_wait_ld32(r);
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          mv[0][half * 16 + m] = round_f16(r[2 * m]);
          mv[1][half * 16 + m] = round_f16(r[2 * m + 1]);
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = t0 + u;
        // Position p = 8i + j with j = 2jj + h, i.e. m = 4i + jj.
        float z[6][4];  // z[a][jj] = sum_i A[a][i] M[i][2jj + h]
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float v[8], g[6];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = mv[u][4 * i + jj];
          a_1d(v, g);
#pragma unroll
          for (int a = 0; a < 6; ++a) z[a][jj] = g[a];
        }
        // Lane h = 0 keeps output rows 0-2, lane h = 1 rows 3-5.
        float other[3][4];
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
            other[a][jj] = __shfl_xor_sync(0xffffffffu, h ? z[a][jj] : z[a + 3][jj], 16);
        const int n = t_n[t];
        if (n < 0 || k >= p.K) continue;
        const int oh0 = t_h0[t] + p.pad, ow0 = t_w0[t] + p.pad;
        __half* yk = p.y + ((long long)n * p.K + k) * plane;
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          const int ar = a + 3 * h;
          float row[8], g[6];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            row[2 * jj] = h ? other[a][jj] : z[a][jj];
            row[2 * jj + 1] = h ? z[a + 3][jj] : other[a][jj];
          }
          a_1d(row, g);
          const int oh = oh0 + ar;
          if (oh >= p.H_out) continue;
          __half* yr = yk + (long long)oh * p.W_out + ow0;
          const int nb = min(6, p.W_out - ow0);
          if ((p.W_out & 1) == 0) {
#pragma unroll
            for (int b = 0; b < 6; b += 2)
              if (b < nb)  // nb is even when W_out is
                *reinterpret_cast<__half2*>(yr + b) = __floats2half2_rn(g[b], g[b + 1]);
          } else {
#pragma unroll
            for (int b = 0; b < 6; ++b)
              if (b < nb) yr[b] = __float2half_rn(g[b]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  FUSED_MARK(3);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace fused

#ifdef NOVA_FUSED_TRACE
extern "C" __attribute__((visibility("default"))) int nova_debug_fused_trace(
    unsigned long long* out, int n_ctas) {
  if (n_ctas > fused::kTraceCtas) n_ctas = fused::kTraceCtas;
  return (int)cudaMemcpyFromSymbol(out, fused::g_fused_trace,
                                   sizeof(unsigned long long) * 4 * (size_t)n_ctas);
}
#endif

bool fused_supported(int C, int K) {
  return C >= 16 && C <= 64 && C % 16 == 0 && K >= 1 && K <= 64;
}

cudaError_t fused_plan(FusedPlan* plan, const __half* U, int K, int C, const char** why) {
  plan->valid = false;
  if (!fused_supported(C, K)) {
    *why = "shape not supported by the fused kernel";
    return cudaErrorInvalidValue;
  }
  // Box of 64 k rows even when K < 64: the rows past K read as zeros.
  if (!tc_encode_operand_map(&plan->tmU, U, C, K, 64)) {
    *why = "cuTensorMapEncodeTiled failed for U";
    return cudaErrorInvalidValue;
  }
  plan->K = K;
  plan->C = C;
  plan->valid = true;
  return cudaSuccess;
}

cudaError_t fused_run(const FusedPlan& plan, const __half* x, __half* y, int B, int H, int W,
                      int pad, int* dev_status, cudaStream_t s, const char** why) {
  if (!plan.valid) {
    *why = "fused plan not built";
    return cudaErrorInvalidValue;
  }
  fused::Params p;
  p.x = x;
  p.y = y;
  p.C = plan.C;
  p.K = plan.K;
  p.H = H;
  p.W = W;
  p.pad = pad;
  p.H_out = H + 2 * pad - 2;
  p.W_out = W + 2 * pad - 2;
  p.nh = (p.H_out + 5) / 6;
  p.nw = (p.W_out + 5) / 6;
  p.BP = (long long)B * p.nh * p.nw;
  p.status = dev_status;
  if (p.BP <= 0) return cudaSuccess;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fused::fused_forward_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         fused::kSmemBytes);
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed";
      return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const long long grid = (p.BP + fused::kT - 1) / fused::kT;
  fused::fused_forward_kernel<<<(unsigned)grid, fused::kThreads, fused::kSmemBytes, s>>>(plan.tmU,
                                                                                         p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) *why = "fused kernel launch failed";
  return e;
}

}  // namespace nova
