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
// Work split.  A group of 8 consecutive tiles (bp) is one MMA N = 8.  Its 64
// Winograd positions are split over a cluster of CS CTAs (CS = 1, 2 or 4): CTA
// rank r owns the position rows i in [r*8/CS, (r+1)*8/CS), i.e. 64/CS
// positions, and with them 1/CS of the U stream, of the MMAs and of the output
// transform.  Each CTA (one per SM, 256 threads):
//
// * prefetches its U_p (64 x 64 FP16 = 8 KB each, TMA, no multicast) into a
//   ring at kernel start, so the weight stream overlaps the input transform;
// * stages the 8x8 input patches of the 8 tiles for all channels in shared
//   memory ([tile][channel][64], odd word pitch), applies B^T along the patch
//   rows for every row and B along the columns only for its own position rows,
//   and writes V straight into the UMMA operand layout: one 1024-byte
//   SWIZZLE_128B atom per position (8 tile rows x 64 channels);
// * per position, D_p[k][t] = sum_c U_p[k][c] V_p[t][c] is one M=64 x N=8 MMA
//   chain (K = C in steps of 16).  M=64 accumulators fill half of each 32-lane
//   TMEM sub-partition, so even positions go to lanes 0-15 and odd positions to
//   lanes 16-31 of the same columns;
// * output transform: the thread at TMEM lane 32q + l owns output channel
//   k = 16q + (l & 15) and the positions of parity l >> 4.  With CS = 1 it
//   applies A along i, swaps half of the partial sums with lane l ^ 16 and
//   applies A along j, writing y.  With CS > 1 it applies A along j (swapping
//   half with lane l ^ 16) and then A along its own rows i, leaving a partial
//   6x6 tile in shared memory; after a cluster barrier each CTA sums the CS
//   partials of 8/CS tiles through distributed shared memory and writes y.
//
// Waits on mbarriers are bounded (2 s); on expiry the kernel records
// kDevTimeoutFused in the device status word, skips its stores and frees TMEM.
#include <cstdlib>

#include "nova_internal.h"
#include "nova_tc_ptx.cuh"

namespace nova {
namespace fused {

using namespace tc;

constexpr int kT = 8;                  // tiles per group (MMA N)
constexpr int kThreads = 256;
constexpr int kXsPitch = 66;           // halves per staged (tile, channel) patch
constexpr int kUBytes = 64 * 64 * 2;   // U of one position: 64 k rows x 128 B
constexpr int kMetaBytes = 512;
constexpr int kSmemMax = 227 * 1024;
constexpr int kYsPitch = 40;           // floats per (tile, k) partial tile: 2 x 20

template <int CS>
struct Cfg {
  static constexpr int kPos = 64 / CS;   // positions per CTA
  static constexpr int kRows = 8 / CS;   // position rows per CTA
  static constexpr int kVsBytes = kPos * 1024;
  static constexpr int kTmemCols = kPos * 4 < 32 ? 32 : kPos * 4;
  static constexpr int kXsBytes = kT * 64 * kXsPitch * 2;
  static constexpr int kFixed = 1024 + kVsBytes + kXsBytes + kMetaBytes;
  static constexpr int kFit = (kSmemMax - kFixed) / kUBytes;
  static constexpr int kStages = kFit < kPos ? kFit : kPos;
  static constexpr int kRingBytes = kStages * kUBytes;
  static constexpr int kSmemBytes = kFixed + kRingBytes;
  static_assert(CS == 1 || kRingBytes >= kT * 64 * kYsPitch * 4, "partials must fit the ring");
};

__constant__ float c_A[6][8];  // A (6 x 8), FP16-rounded entries

#ifdef NOVA_FUSED_TRACE
// Debug builds only: per-CTA globaltimer stamps at the phase boundaries.
constexpr int kTraceCtas = 8192;
constexpr int kTraceSlots = 8;
__device__ unsigned long long g_fused_trace[kTraceCtas * kTraceSlots];
#define FUSED_MARK(i)                              \
  if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) \
    g_fused_trace[blockIdx.x * kTraceSlots + (i)] = globaltimer();
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

__device__ __forceinline__ void tmem_ld_x4(uint32_t taddr, uint32_t& a, uint32_t& b, uint32_t& c,
                                           uint32_t& d) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
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

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Six outputs of one row of a 6x6 tile, bounds-checked, into y.
__device__ __forceinline__ void store_row6(__half* yr, int nb, bool even_w, const float g[6]) {
  if (even_w) {
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

template <int CS>
__global__ void __launch_bounds__(kThreads, 1)
    fused_forward_kernel(const __grid_constant__ CUtensorMap tmU, const Params p) {
  using Cf = Cfg<CS>;
  constexpr int kPos = Cf::kPos, kStages = Cf::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* Vs = base;
  uint8_t* ring = Vs + Cf::kVsBytes;  // U ring; after the MMAs, the partial tiles (CS > 1)
  __half* Xs = reinterpret_cast<__half*>(ring + Cf::kRingBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + Cf::kRingBytes + Cf::kXsBytes);
  uint64_t* ufull = bars;
  uint64_t* uempty = bars + kStages;
  uint64_t* done = bars + 2 * kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* t_n = const_cast<int*>(abort_flag + 1);  // image of tile t, -1 past BP
  int* t_h0 = t_n + kT;                         // 6*th - pad
  int* t_w0 = t_h0 + kT;                        // 6*tw - pad

  FUSED_MARK(0);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = CS > 1 ? (int)cluster_ctarank() : 0;
  const long long bp0 = (long long)(blockIdx.x / CS) * kT;
  const int i0 = rank * Cf::kRows;  // first position row of this CTA
  const int pos0 = i0 * 8;

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
    for (int s = 0; s < kStages; ++s) {
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
                 "r"(Cf::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // x and U come from earlier kernels in the stream

  // U prefetch: the ring starts empty, so its first kStages loads need no wait.
  if (threadIdx.x == 0) {
    for (int lp = 0; lp < kStages; ++lp) {
      const uint32_t fb = smem_u32(&ufull[lp]);
      mbar_expect_tx(fb, kUBytes);
      tma_load_3d(smem_u32(ring + lp * kUBytes), &tmU, 0, 0, pos0 + lp, fb);
    }
  }
  __syncwarp();

  // ---------------- Input transform: V into the operand layout ----------------
  const long long HW = (long long)p.H * p.W;
  const uint32_t vs_addr = smem_u32(Vs);
  {
    // Thread (r, cc) of each 64-thread quarter loads patch element (r, cc) of
    // channels cl0 + 4j for every tile: a warp covers 4 rows x 8 columns of
    // one channel.  All 128 loads are issued before the first store.
    const int st_cc = threadIdx.x & 7, st_r = (threadIdx.x >> 3) & 7, st_cl0 = threadIdx.x >> 6;
    unsigned short v[kT][16];
#pragma unroll
    for (int t = 0; t < kT; ++t) {
      const int n = t_n[t];
      const int h = t_h0[t] + st_r, w = t_w0[t] + st_cc;
      const bool in = n >= 0 && (unsigned)h < (unsigned)p.H && (unsigned)w < (unsigned)p.W;
      const unsigned short* src = reinterpret_cast<const unsigned short*>(p.x) +
                                  ((long long)(in ? n : 0) * p.C + st_cl0) * HW +
                                  (in ? h * p.W + w : 0);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const bool ok = in && st_cl0 + 4 * j < p.C;
        v[t][j] = ok ? __ldg(src + (long long)(4 * j) * HW) : (unsigned short)0;
      }
    }
    unsigned short* xs16 = reinterpret_cast<unsigned short*>(Xs);
#pragma unroll
    for (int t = 0; t < kT; ++t)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        xs16[(t * 64 + st_cl0 + 4 * j) * kXsPitch + st_r * 8 + st_cc] = v[t][j];
  }
  __syncthreads();
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    const int t = warp;
    const int c = half * 32 + lane;
    if (half * 32 >= p.C) break;
    const __half2* xp = reinterpret_cast<const __half2*>(Xs + (t * 64 + c) * kXsPitch);
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
      float vv[8], f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) vv[i] = d[i][j];
      bt_1d(vv, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i][j] = f[i];
    }
    if (c < p.C) {
      // Byte offset of (local position, tile t, channel c) in the SWIZZLE_128B atoms.
      const uint32_t row = vs_addr + t * 128 + (c & 7) * 2;
      const uint32_t chunk = (uint32_t)(((c >> 3) ^ t) << 4);
#pragma unroll
      for (int r = 0; r < 8; ++r) {  // rows: V[r][.] = d[r][.] B, own rows only
        if (r < i0 || r >= i0 + Cf::kRows) continue;
        float f[8];
        bt_1d(d[r], f);
#pragma unroll
        for (int s = 0; s < 8; ++s)
          st_shared_u16(row + (uint32_t)((r - i0) * 8 + s) * 1024u + chunk, __float2half_rn(f[s]));
      }
    }
  }
  fence_async_smem();  // V visible to the async proxy
  __syncthreads();
  FUSED_MARK(1);

  // ---------------- GEMM: kPos positions of M=64 x N=8 MMAs ----------------
  const int nks = p.C / 16;
  if (warp == 0) {
    if (lane == 0) {
      for (int lp = kStages; lp < kPos; ++lp) {
        const int s = lp % kStages;
        const uint32_t ph = (uint32_t)(lp / kStages) & 1u;
        if (!mbar_wait(smem_u32(&uempty[s]), ph ^ 1u, abort_flag, p.status, kDevTimeoutFused))
          break;
        const uint32_t fb = smem_u32(&ufull[s]);
        mbar_expect_tx(fb, kUBytes);
        tma_load_3d(smem_u32(ring + s * kUBytes), &tmU, 0, 0, pos0 + lp, fb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | ((uint32_t)(kT >> 3) << 17) | ((uint32_t)(64 >> 4) << 24);
      // Positions go in batches of kBatch with the k-step as the outer loop, so
      // consecutive MMAs write different accumulators.
      constexpr int kBatch = kStages >= 4 ? 4 : 1;
      bool ok = true;
      for (int lb = 0; lb < kPos && ok; lb += kBatch) {
        for (int b = 0; b < kBatch; ++b) {
          const int lp = lb + b;
          if (!mbar_wait(smem_u32(&ufull[lp % kStages]), (uint32_t)(lp / kStages) & 1u,
                         abort_flag, p.status, kDevTimeoutFused)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        tc_fence_after();
        for (int ks = 0; ks < nks; ++ks) {
#pragma unroll
          for (int b = 0; b < kBatch; ++b) {
            const int lp = lb + b;
            const uint64_t ad = smem_desc_sw128(smem_u32(ring + (lp % kStages) * kUBytes));
            const uint64_t bd = smem_desc_sw128(vs_addr + (uint32_t)lp * 1024u);
            const uint32_t dt =
                tmem_base + ((uint32_t)((lp & 1) * 16) << 16) + (uint32_t)(lp >> 1) * kT;
            umma_f16(dt, ad + 2ull * ks, bd + 2ull * ks, idesc, ks);
          }
        }
        for (int b = 0; b < kBatch; ++b) {
          const int lp = lb + b;
          if (lp + kStages < kPos) umma_commit(smem_u32(&uempty[lp % kStages]));
        }
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
  const int q = warp & 3;
  const int h = lane >> 4;
  const int k = q * 16 + (lane & 15);
  const long long plane = (long long)p.H_out * p.W_out;
  const bool even_w = (p.W_out & 1) == 0;
  const uint32_t lane_addr = tmem_base + ((uint32_t)(q * 32) << 16);
  if constexpr (CS == 1) {
    if (got) {
      for (int tp = 0; tp < 2; ++tp) {
        const int t0 = (warp >> 2) * 4 + tp * 2;
        // mv[u][m] = M at position 2m + h of tile t0 + u.
        float mv[2][32];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t r[32];
          __syncwarp();
#pragma unroll
          for (int m = 0; m < 16; ++m)
            tmem_ld_x2(lane_addr + (uint32_t)(hh * 16 + m) * kT + t0, r[2 * m], r[2 * m + 1]);
          tmem_wait_ld32(r);
#pragma unroll
          for (int m = 0; m < 16; ++m) {
            mv[0][hh * 16 + m] = round_f16(r[2 * m]);
            mv[1][hh * 16 + m] = round_f16(r[2 * m + 1]);
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int t = t0 + u;
          // Position p = 8i + j with j = 2jj + h, i.e. m = 4i + jj.
          float z[6][4];  // z[a][jj] = sum_i A[a][i] M[i][2jj + h]
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            float vv[8], g[6];
#pragma unroll
            for (int i = 0; i < 8; ++i) vv[i] = mv[u][4 * i + jj];
            a_1d(vv, g);
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
            store_row6(yk + (long long)oh * p.W_out + ow0, min(6, p.W_out - ow0), even_w, g);
          }
        }
      }
    }
  } else {
    // Partial tiles.  Tile t is finished by cluster rank t / kTilesOwn; every
    // CTA stores its partial of t into that rank's shared memory, slot
    // Yr[src][t % kTilesOwn][k][h*20 + a*3 + x] (b = 3h + x), with 16-byte
    // remote stores that need no round trip.
    constexpr int kTilesOwn = kT / CS;
    float* Yr = reinterpret_cast<float*>(ring);
    // The slots reuse the U ring: no CTA stores into a peer before that
    // peer's MMAs have finished reading it.
    __syncwarp();
    cluster_sync();
    const uint32_t yr_addr = smem_u32(Yr);
    constexpr int kTpl = CS == 4 ? 4 : 2;       // tiles per TMEM load
    constexpr int kM = kPos / 2;                // positions of one parity
    static_assert(kTpl * kM == 32, "one 32-register TMEM batch per tile chunk");
    for (int tc = 0; tc < 4 / kTpl; ++tc) {
      const int t0 = (warp >> 2) * 4 + tc * kTpl;
      uint32_t r[32];
      __syncwarp();
#pragma unroll
      for (int m = 0; m < kM; ++m) {
        if (kTpl == 4)
          tmem_ld_x4(lane_addr + (uint32_t)m * kT + t0, r[4 * m], r[4 * m + 1], r[4 * m + 2],
                     r[4 * m + 3]);
        else
          tmem_ld_x2(lane_addr + (uint32_t)m * kT + t0, r[2 * m], r[2 * m + 1]);
      }
      tmem_wait_ld32(r);
#pragma unroll
      for (int u = 0; u < kTpl; ++u) {
        const int t = t0 + u;
        float yp[6][3];
#pragma unroll
        for (int a = 0; a < 6; ++a)
#pragma unroll
          for (int x = 0; x < 3; ++x) yp[a][x] = 0.f;
#pragma unroll
        for (int il = 0; il < Cf::kRows; ++il) {
          // zp[b] = sum over own j (parity h) of A[b][j] M[i][j]
          float zp[6];
#pragma unroll
          for (int b = 0; b < 6; ++b) zp[b] = 0.f;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const float mval = got ? round_f16(r[(4 * il + jj) * kTpl + u]) : 0.f;
#pragma unroll
            for (int b = 0; b < 6; ++b)
              zp[b] = fmaf(h ? kA(b, 2 * jj + 1) : kA(b, 2 * jj), mval, zp[b]);
          }
          // Lane h keeps columns b = 3h .. 3h+2 and adds the partner's share.
          float zb[3];
#pragma unroll
          for (int x = 0; x < 3; ++x) {
            const float other = __shfl_xor_sync(0xffffffffu, h ? zp[x] : zp[x + 3], 16);
            zb[x] = (h ? zp[x + 3] : zp[x]) + other;
          }
#pragma unroll
          for (int a = 0; a < 6; ++a) {
            const float ca = c_A[a][i0 + il];
#pragma unroll
            for (int x = 0; x < 3; ++x) yp[a][x] = fmaf(ca, zb[x], yp[a][x]);
          }
        }
        const uint32_t owner = (uint32_t)(t / kTilesOwn);
        const uint32_t local = yr_addr + 4u * (uint32_t)((((rank * kTilesOwn + t % kTilesOwn) * 64 +
                                                            k) * kYsPitch) + h * 20);
        uint32_t remote;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(owner));
        float flat[20];
#pragma unroll
        for (int a = 0; a < 6; ++a)
#pragma unroll
          for (int x = 0; x < 3; ++x) flat[a * 3 + x] = yp[a][x];
        flat[18] = flat[19] = 0.f;
#pragma unroll
        for (int v = 0; v < 5; ++v)
          asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(remote + 16u * v),
                       "f"(flat[4 * v]), "f"(flat[4 * v + 1]), "f"(flat[4 * v + 2]),
                       "f"(flat[4 * v + 3])
                       : "memory");
      }
    }
    FUSED_MARK(4);
    __syncwarp();
    cluster_sync();  // all partials of this CTA's tiles have landed here
    FUSED_MARK(5);
    for (int idx = threadIdx.x; idx < kTilesOwn * 64 * 6; idx += kThreads) {
      const int kk = idx & 63;
      const int a = (idx >> 6) % 6;
      const int tl = idx / 384;
      const int t = rank * kTilesOwn + tl;
      float g[6];
#pragma unroll
      for (int b = 0; b < 6; ++b) g[b] = 0.f;
#pragma unroll
      for (int src = 0; src < CS; ++src) {
        const float* e = Yr + ((src * kTilesOwn + tl) * 64 + kk) * kYsPitch + a * 3;
#pragma unroll
        for (int x = 0; x < 3; ++x) {
          g[x] += e[x];
          g[3 + x] += e[20 + x];
        }
      }
      const int n = t_n[t];
      if (!got || n < 0 || kk >= p.K) continue;
      const int oh = t_h0[t] + p.pad + a, ow0 = t_w0[t] + p.pad;
      if (oh >= p.H_out) continue;
      store_row6(p.y + ((long long)n * p.K + kk) * plane + (long long)oh * p.W_out + ow0,
                 min(6, p.W_out - ow0), even_w, g);
    }
    FUSED_MARK(6);
  }

  tc_fence_before();
  __syncthreads();
  pdl_trigger();  // after the whole CTA is done
  FUSED_MARK(3);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(Cf::kTmemCols)
                 : "memory");
  }
}

template <int CS>
cudaError_t launch(const CUtensorMap& tmU, const Params& p, long long groups, cudaStream_t s,
                   const char** why) {
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fused_forward_kernel<CS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         Cfg<CS>::kSmemBytes);
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed";
      return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups * CS), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg<CS>::kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled(kPdlFused) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fused_forward_kernel<CS>, tmU, p);
  if (e != cudaSuccess) *why = "fused kernel launch failed";
  return e;
}

// Cluster size: split positions further while the groups alone leave SMs idle.
int pick_cs(long long groups, int num_sms) {
  static const int forced = [] {
    const char* env = std::getenv("NOVA_FUSED_CS");
    return env ? std::atoi(env) : 0;
  }();
  if (forced == 1 || forced == 2 || forced == 4) return forced;
  if (groups * 2 <= num_sms) return 4;
  if (groups <= num_sms) return 2;
  return 1;
}

}  // namespace fused

#ifdef NOVA_FUSED_TRACE
extern "C" __attribute__((visibility("default"))) int nova_debug_fused_trace(
    unsigned long long* out, int n_ctas) {
  if (n_ctas > fused::kTraceCtas) n_ctas = fused::kTraceCtas;
  return (int)cudaMemcpyFromSymbol(out, fused::g_fused_trace,
                                   sizeof(unsigned long long) * fused::kTraceSlots *
                                       (size_t)n_ctas);
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
  static bool constants_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !constants_set[dev]) {
    float a[6][8];
    for (int i = 0; i < 6; ++i)
      for (int j = 0; j < 8; ++j) a[i][j] = kA(i, j);
    if (cudaMemcpyToSymbol(fused::c_A, a, sizeof(a)) != cudaSuccess) {
      *why = "cudaMemcpyToSymbol(A) failed";
      return cudaErrorInvalidValue;
    }
    if (dev >= 0 && dev < 64) constants_set[dev] = true;
  }
  plan->K = K;
  plan->C = C;
  plan->valid = true;
  return cudaSuccess;
}

cudaError_t fused_run(const FusedPlan& plan, const __half* x, __half* y, int B, int H, int W,
                      int pad, int* dev_status, int num_sms, cudaStream_t s, const char** why) {
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
  const long long groups = (p.BP + fused::kT - 1) / fused::kT;
  switch (fused::pick_cs(groups, num_sms)) {
    case 4:
      return fused::launch<4>(plan.tmU, p, groups, s, why);
    case 2:
      return fused::launch<2>(plan.tmU, p, groups, s, why);
    default:
      return fused::launch<1>(plan.tmU, p, groups, s, why);
  }
}

}  // namespace nova
