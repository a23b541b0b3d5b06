// Input / output transform kernels for even channel counts (the hot path).
//
// Geometry: a block owns one tile row (row = b*nh + th), a chunk of TPC
// consecutive tiles along w (TPC is a template parameter, so every shared-memory
// offset below is a compile-time immediate) and 64*G channels.  Work item =
// (tile, 64 channels) for one warp; each lane owns two adjacent channels, so
// every access a warp makes to one position of V or M is one aligned half2 per
// lane = one full 128-byte line.
//
// Input transform:  image rows staged in shared memory, then V = B^T d B in
//   registers.  With W % 8 == 0 (mode 1) the rows arrive by one TMA tile load
//   and are transposed with ldmatrix.trans into [col][channel][row]; with
//   W % 4 == 0 and even H (mode 2) they arrive as pair rows and are repacked
//   into [row][col][channel] (66-half cell pitch = 33 words, odd:
//   conflict-free).  In both TMA modes the V tiles go back out through shared
//   memory by TMA tile stores; otherwise (mode 0) the rows are staged with
//   plain loads and V is written straight to V[pos][bp][c].
// Output transform: the block's M tiles arrive by TMA tile loads (or 64
//   independent loads per lane when M cannot be described by a tensor map),
//   Y = A M A^T in registers, parked in shared memory as [pixel][k].  With
//   W_out % 8 == 0 the tile rows are transposed into a dense [k][row][col] box
//   and leave by one TMA tile store; otherwise they are written as whole output
//   row segments along w (warp per channel, lane per column).
// Reference: input_transform_kernel(_mt) and output_transform_kernel(_mt),
// Jayluci4/nova-wino-amd csrc/nova_winograd.hip:141-205, 264-328, 338-450.
#include <algorithm>
#include <cstdlib>

#include "nova_internal.h"
#include "nova_tc_ptx.cuh"

namespace nova {
namespace fast {

#ifdef NOVA_FAST_TRACE
// Debug builds only: globaltimer stamps per block of the input transform.
constexpr int kFtBlocks = 16384, kFtSlots = 4;
__device__ unsigned long long g_fast_trace[kFtBlocks * kFtSlots];
#define FAST_MARK(i)                                                                  \
  {                                                                                   \
    const unsigned _b = blockIdx.x + gridDim.x * blockIdx.y;                          \
    if (threadIdx.x == 0 && _b < kFtBlocks) {                                         \
      unsigned long long _t;                                                          \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(_t));                          \
      g_fast_trace[_b * kFtSlots + (i)] = _t;                                         \
    }                                                                                 \
  }
#else
#define FAST_MARK(i)
#endif

constexpr int kMaxTPC = 6;
#ifndef NOVA_IT_CHAN_IN_FLIGHT
#define NOVA_IT_CHAN_IN_FLIGHT 2
#endif
#ifndef NOVA_IT_MIN_BLOCKS
#define NOVA_IT_MIN_BLOCKS 3  // 128 registers: 3 blocks of 5 warps per SM
#endif
#ifndef NOVA_PLANE_PAIR_CH
#define NOVA_PLANE_PAIR_CH 6  // channels per round of the cell-pair plane loader (4: 28.6 us, 6: 26.7, 8: 26.6 at conv4_x batch 128)
#endif
#ifndef NOVA_OT_MIN_BLOCKS
#define NOVA_OT_MIN_BLOCKS 3
#endif
constexpr long long kMaxGridY = 65535;

// Dynamic shared memory above 48 KB is a per-device, per-kernel opt-in.
// static_bytes: the kernel's static shared memory; the opt-in is needed once
// static + dynamic exceeds 48 KB.
template <const void* (*Fn)()>
static bool smem_optin_once(size_t bytes, size_t static_bytes = 0) {
  static bool done[64] = {};
  if (bytes + static_bytes <= 48 * 1024) return true;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (done[dev]) return true;
  done[dev] = cudaFuncSetAttribute(Fn(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)bytes) == cudaSuccess;
  return done[dev];
}

struct Args {
  int C, H, W, pad;  // C = channels of this tensor (C for input, K for output)
  int B;             // batch
  int nh, nw;
  long long row0;    // first global tile row of the window
  long long lrow0;   // window-relative tile row of blockIdx.y == 0
  long long BP;      // bp extent (plane stride) of V / M
  int n_twc;         // chunks along w
};

template <int TPC, int G>
struct Geo {
  static constexpr int kCGN = 64 * G;            // channels per block
  static constexpr int kPitch = kCGN + 2;        // halves per staged cell (odd words)
  static constexpr int kInCols = TPC * 6 + 2;    // staged image columns
  static constexpr int kOutCols = TPC * 6;       // output columns per chunk
  static constexpr int kWarps = TPC * G < 2 ? 2 : TPC * G;
  static constexpr size_t kInSmem = 8 * kInCols * kPitch * 2;
  static constexpr size_t kOutSmem = 6 * kOutCols * kPitch * 2;
  // TMA staging (W % 8 == 0): box {kBoxW, 8 rows, kCGN channels, 1 image}
  // starting at the multiple of 8 at or below w0, landed as [c][r][w].
  static constexpr int kBoxW = ((kInCols + 7 + 7) / 8) * 8;
  static constexpr size_t kLandBytes = (size_t)kCGN * 8 * kBoxW * 2;
  // TMA path staging [col][channel slot][8 rows]: column pitch kCGN*8 + 8
  // halves (= 4 mod 32 words, so the transposing stores are conflict-free).
  static constexpr int kColPitch = kCGN * 8 + 8;
  static constexpr size_t kInSmemCol = (size_t)kInCols * kColPitch * 2;
  static constexpr size_t kInSmemTma = 128 + kLandBytes + kInSmemCol;
  // V tiles staged for the TMA stores: [tile][pos][kCGN].
  static constexpr size_t kVStage = (size_t)TPC * 64 * kCGN * 2;
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(src)
      : "memory");
}

// Bounded mbarrier wait (2 s of globaltimer); false on expiry.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 255u) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t0 == 0) t0 = t;
      else if (t - t0 > 2000000000ull) return false;
    }
  }
}

__device__ __forceinline__ void block_coords(const Args& a, long long& lrow, int& b, int& th,
                                             int& twc, int& cg) {
  twc = blockIdx.x % a.n_twc;
  cg = blockIdx.x / a.n_twc;
  lrow = a.lrow0 + blockIdx.y;
  // Tile rows (b * nh + th) stay below 2^31: 32-bit division, not the long
  // emulated 64-bit one.
  const uint32_t grow = (uint32_t)(a.row0 + lrow);
  b = (int)(grow / (uint32_t)a.nh);
  th = (int)(grow - (uint32_t)b * (uint32_t)a.nh);
}

template <int TPC, int G>
__host__ __device__ inline size_t pair_land_bytes(int W) {
  const size_t pair = (((size_t)Geo<TPC, G>::kCGN * 5 * 2 * W * 2 + 127) / 128) * 128;
  return pair > Geo<TPC, G>::kVStage ? pair : Geo<TPC, G>::kVStage;
}

// 16-byte slot of channel c inside a staged column: channels rotate within
// each octet by the octet index, so the 16-byte reads of 8 consecutive lanes
// (channels 2l or 2l + 1) fall on 8 different bank groups.
__device__ __forceinline__ int chan_slot(int c) { return (c & ~7) | ((c + (c >> 3)) & 7); }

// kMode: 0 = staged with plain loads; 1 = one TMA tile load of 8 image rows
// (W % 8 == 0); 2 = one TMA tile load of 5 "pair rows" (2 image rows each, for
// W % 4 == 0 and even H, where single rows are not 16-byte strided).
template <int TPC, int G, int kMode>
__global__ void __launch_bounds__(32 * Geo<TPC, G>::kWarps, NOVA_IT_MIN_BLOCKS)
    input_transform_fast(const __half* __restrict__ x, __half* __restrict__ V,
                         const __grid_constant__ CUtensorMap map_x,
                         const __grid_constant__ CUtensorMap map_v, const Args a) {
  using Gm = Geo<TPC, G>;
  extern __shared__ uint8_t it_raw[];
  uint8_t* it_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(it_raw) + 127) &
                                                ~uintptr_t(127));
  // TMA landing buffer [kCGN][8][kBoxW] (TMA path only), then [8][kInCols][kPitch].
  const __half* land = reinterpret_cast<const __half*>(it_base);
  // The landing buffer also holds the V tiles for the TMA stores once the
  // staging has been repacked out of it.
  const size_t land_bytes =
      kMode == 1 ? Gm::kLandBytes
                 : (kMode == 2 ? pair_land_bytes<TPC, G>(a.W) : 0);
  __half* xs = reinterpret_cast<__half*>(it_base + land_bytes);
  const uint32_t land_s = static_cast<uint32_t>(__cvta_generic_to_shared(land));
  __shared__ uint64_t land_bar;
  long long lrow;
  int b, th, twc, cg;
  block_coords(a, lrow, b, th, twc, cg);
  const int C = a.C, H = a.H, W = a.W;
  const int c0 = cg * Gm::kCGN;
  const int tw0 = twc * TPC;
  const int ntw = min(TPC, a.nw - tw0);
  const int h0 = th * 6 - a.pad;
  const int w0 = tw0 * 6 - a.pad;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();

  if constexpr (kMode == 2) {
    // Pair rows: row pr of the landing buffer holds image rows 2(p0+pr) and
    // 2(p0+pr)+1 back to back (2W halves), zero-filled outside the tensor.
    const int p0 = h0 >= 0 ? h0 / 2 : -((-h0 + 1) / 2);
    const int W2 = 2 * W;
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&land_bar));
    if (threadIdx.x == 0) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                   "r"((uint32_t)(Gm::kCGN * 5 * W2 * 2))
                   : "memory");
      tma_load_4d(static_cast<uint32_t>(__cvta_generic_to_shared(land)), &map_x, 0, p0, c0, b,
                  bar);
    }
    __syncthreads();
    if (!mbar_wait_bounded(bar, 0)) return;
    const bool ok0 = lane < Gm::kInCols && w0 + lane >= 0 && w0 + lane < W;
    const bool ok1 = lane + 32 < Gm::kInCols && w0 + lane + 32 >= 0 && w0 + lane + 32 < W;
    // Offset of image row h0 + r inside one channel's landing rows, per r.
    int rowoff[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int h = h0 + r;
      const int hp = h >= 0 ? h / 2 : -((-h + 1) / 2);
      rowoff[r] = (hp - p0) * W2 + (h - 2 * hp) * W + w0 + lane;
    }
    const __half z = __ushort_as_half(0);
    // A warp takes whole channel pairs and walks their 8 rows.
    for (int p2 = warp; p2 < Gm::kCGN / 2; p2 += Gm::kWarps) {
      const __half* s0 = land + (2 * p2) * 5 * W2;
      const __half* s1 = s0 + 5 * W2;
      __half* dst = xs + lane * Gm::kPitch + 2 * p2;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (lane < Gm::kInCols)
          *reinterpret_cast<__half2*>(dst + r * Gm::kInCols * Gm::kPitch) =
              ok0 ? __halves2half2(s0[rowoff[r]], s1[rowoff[r]]) : __halves2half2(z, z);
        if (lane + 32 < Gm::kInCols)
          *reinterpret_cast<__half2*>(dst + (r * Gm::kInCols + 32) * Gm::kPitch) =
              ok1 ? __halves2half2(s0[rowoff[r] + 32], s1[rowoff[r] + 32]) : __halves2half2(z, z);
      }
    }
  } else if constexpr (kMode == 1) {
    // One TMA tile load brings rows h0..h0+7, columns x0..x0+kBoxW-1 of the
    // block's channels, zero-filled outside the tensor, as [channel][row][col];
    // ldmatrix.trans then turns it into [col][channel slot][row].
    FAST_MARK(0);
    const int x0 = w0 >= 0 ? (w0 & ~7) : -((-w0 + 7) & ~7);
    const int d = w0 - x0;
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&land_bar));
    if (threadIdx.x == 0) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                   "r"((uint32_t)Gm::kLandBytes)
                   : "memory");
      tma_load_4d(static_cast<uint32_t>(__cvta_generic_to_shared(land)), &map_x, x0, h0, c0, b,
                  bar);
    }
    __syncthreads();
    if (!mbar_wait_bounded(bar, 0)) return;
    FAST_MARK(1);
    // Transpose [channel][row][col] into [col][channel slot][row] with
    // ldmatrix.trans: one 8x8 matrix = (channel, rows 0-7, 8 columns); lane T
    // gets rows 2(T%4), 2(T%4)+1 of column T/4, i.e. one 32-bit word of the
    // destination.
    constexpr int kChunks = Gm::kBoxW / 8;
    constexpr int kQuads = Gm::kCGN / 4;
    const uint32_t xs_s = static_cast<uint32_t>(__cvta_generic_to_shared(xs));
    // A warp owns whole 8-column chunks and walks every channel quad of them:
    // all per-quad offsets (source rows, destination slots) are immediates.
    const uint32_t src_lane =
        land_s + (uint32_t)((((lane >> 3) * 8 + (lane & 7)) * Gm::kBoxW) * 2);
    for (int chunk = warp; chunk < kChunks; chunk += Gm::kWarps) {
      const int col = chunk * 8 + (lane >> 2) - d;
      const bool in = col >= 0 && col < Gm::kInCols;
      const uint32_t src = src_lane + (uint32_t)(chunk * 16);
      const uint32_t dst = xs_s + (uint32_t)(((in ? col : 0) * Gm::kColPitch + 2 * (lane & 3)) * 2);
#pragma unroll
      for (int cq = 0; cq < kQuads; ++cq) {
        uint32_t rg[4];
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(rg[0]), "=r"(rg[1]), "=r"(rg[2]), "=r"(rg[3])
                     : "r"(src + (uint32_t)(cq * 4 * 8 * Gm::kBoxW * 2))
                     : "memory");
        if (in) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst + (uint32_t)chan_slot(cq * 4 + i) * 16u),
                         "r"(rg[i])
                         : "memory");
        }
      }
    }
  } else {
  // Stage rows h0..h0+7 of the block's channels, columns w0..w0+kInCols-1.
  // A warp takes whole channels (kChanInFlight at a time: 16 loads per channel
  // per lane in flight); the 8 rows of a channel are one base pointer plus
  // per-block row offsets, and every shared-memory offset is an immediate.
  {
    const bool ok0 = lane < Gm::kInCols && w0 + lane >= 0 && w0 + lane < W;
    const bool ok1 = lane + 32 < Gm::kInCols && w0 + lane + 32 >= 0 && w0 + lane + 32 < W;
    unsigned rmask = 0;  // bit r: image row h0 + r exists
    int roff[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int h = h0 + r;
      if (h >= 0 && h < H) rmask |= 1u << r;
      roff[r] = (h >= 0 && h < H ? h : 0) * W;
    }
    const long long plane_x = (long long)H * W;
    const __half* xb = x + ((long long)b * C + c0) * plane_x + w0;
    __half* sbase = xs + lane * Gm::kPitch;
    constexpr int kChanInFlight = NOVA_IT_CHAN_IN_FLIGHT;
    for (int cl0 = warp; cl0 < Gm::kCGN; cl0 += Gm::kWarps * kChanInFlight) {
      __half2 v[kChanInFlight][8];
#pragma unroll
      for (int u = 0; u < kChanInFlight; ++u) {
        const int cl = cl0 + u * Gm::kWarps;
        const bool cok = cl < Gm::kCGN && c0 + cl < C;
        const __half* cp = xb + (cok ? cl : 0) * plane_x;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const bool rok = cok && ((rmask >> r) & 1u);
          v[u][r].x = (rok && ok0) ? cp[roff[r] + lane] : __ushort_as_half(0);
          v[u][r].y = (rok && ok1) ? cp[roff[r] + lane + 32] : __ushort_as_half(0);
        }
      }
#pragma unroll
      for (int u = 0; u < kChanInFlight; ++u) {
        const int cl = cl0 + u * Gm::kWarps;
        if (cl < Gm::kCGN) {
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            if (lane < Gm::kInCols) sbase[r * Gm::kInCols * Gm::kPitch + cl] = v[u][r].x;
            if (lane + 32 < Gm::kInCols)
              sbase[(r * Gm::kInCols + 32) * Gm::kPitch + cl] = v[u][r].y;
          }
        }
      }
    }
  }
  }
  __syncthreads();
  if (kMode == 1) FAST_MARK(2);

  const long long plane = a.BP * (long long)C;
  for (int it = warp; it < TPC * G; it += Gm::kWarps) {
    const int t = it / G, g = it % G;
    if (t >= ntw) break;
    const int cl = g * 64 + 2 * lane;
    const int c = c0 + cl;
    float2 tt[8][8];  // the lane's channel pair, paired in every operation
#pragma unroll
    for (int j = 0; j < 8; ++j) {  // columns: tmp[.][j] = B^T d[.][j]
      float2 v[8], f[8];
      if constexpr (kMode == 1) {
        const __half* colp = xs + (t * 6 + j) * Gm::kColPitch;
        const uint4 wa = *reinterpret_cast<const uint4*>(colp + chan_slot(cl) * 8);
        const uint4 wb = *reinterpret_cast<const uint4*>(colp + chan_slot(cl + 1) * 8);
        const uint32_t ua[4] = {wa.x, wa.y, wa.z, wa.w}, ub[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i2 = 0; i2 < 4; ++i2) {
          const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&ua[i2]));
          const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&ub[i2]));
          v[2 * i2] = make_float2(fa.x, fb.x);
          v[2 * i2 + 1] = make_float2(fa.y, fb.y);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          v[i] = __half22float2(*reinterpret_cast<const __half2*>(
              xs + (i * Gm::kInCols + t * 6 + j) * Gm::kPitch + cl));
      }
      bt_1d2(v, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) tt[i][j] = f[i];
    }
    if constexpr (kMode == 1 || kMode == 2) {
      // V tile [pos][kCGN] into the landing buffer, which the repack has freed;
      // channels past C are clipped by the TMA store.
      const uint32_t vrow = land_s + (uint32_t)((t * 64 * Gm::kCGN + cl) * 2);
#pragma unroll
      for (int r = 0; r < 8; ++r) {  // rows: V[r][.] = tmp[r][.] B
        float2 f[8];
        bt_1d2(tt[r], f);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const __half2 hv = __float22half2_rn(f[s]);
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(vrow + (uint32_t)((r * 8 + s) *
                                                                         Gm::kCGN * 2)),
                       "r"(*reinterpret_cast<const uint32_t*>(&hv))
                       : "memory");
        }
      }
    } else {
      if (c >= C) continue;  // C is even: the pair is wholly in or out
      __half2* out = reinterpret_cast<__half2*>(V + (lrow * a.nw + tw0 + t) * C + c);
#pragma unroll
      for (int r = 0; r < 8; ++r) {  // rows: V[r][.] = tmp[r][.] B
        float2 f[8];
        bt_1d2(tt[r], f);
#pragma unroll
        for (int s = 0; s < 8; ++s) out[(long long)(r * 8 + s) * (plane >> 1)] = __float22half2_rn(f[s]);
      }
    }
  }
  if constexpr (kMode == 1 || kMode == 2) {
    tc::fence_async_smem();  // the staged V tiles are visible to the TMA unit
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int t = 0; t < ntw; ++t)
        tc::tma_store_3d(&map_v, land_s + (uint32_t)(t * 64 * Gm::kCGN * 2), c0,
                         (int)(lrow * a.nw + tw0 + t), 0);
      tc::bulk_commit();
      tc::bulk_wait_read_all();  // shared memory stays valid until the stores read it
    }
  }
  __syncthreads();
  pdl_trigger();  // after the whole block is done
#ifdef NOVA_FAST_TRACE
  __syncthreads();
  if (kMode == 1) FAST_MARK(3);
#endif
}

// ---------------------------------------------------------------------------
// Streaming input transform (W % 8 == 0, one 64-channel group per item).
//
// The block-per-item kernel above serialises, per block, TMA load -> transpose
// -> transform -> store, and an SM holds three such blocks: its warps wait on
// DRAM and on block barriers more than they compute.  This persistent kernel
// (one CTA per SM) decouples the two.  Warp 0 streams the items' 8-row x
// 64-channel landings by TMA into a ring of kSlots buffers; kGroups consumer
// groups of TPC warps (one warp per tile) take items in turn: a group
// transposes its landing into its own [col][channel slot][row] staging (the
// landing slot is released right after, so the producer refills it while the
// group computes), transforms one tile per warp and writes V with coalesced
// 128-byte stores.  Items are (tile row, chunk of TPC tiles, 64 channels) in
// the order of the block-per-item kernel's blocks.
// ---------------------------------------------------------------------------
// One 4-byte global store, kept in program order: as a plain C++ store the
// compiler batches the 64 stores of a tile together with their 64-bit
// addresses and spills at the 128-register cap.
__device__ __forceinline__ void st_global_h2(__half2* p, __half2 v) {
  asm volatile("st.global.b32 [%0], %1;" ::"l"(p), "r"(*reinterpret_cast<const uint32_t*>(&v))
               : "memory");
}

template <int TPC>
struct StreamGeo {
  using Gm = Geo<TPC, 1>;
  static constexpr int kGroups = 15 / TPC;       // 128 registers: 16 warps per SM
  static constexpr int kWarps = 1 + kGroups * TPC;
  static constexpr int kSlots = 3;
  static constexpr size_t kLand = (Gm::kLandBytes + 127) / 128 * 128;
  static constexpr size_t kXs = (Gm::kInSmemCol + 127) / 128 * 128;
  static constexpr size_t kBars = 128;
  static constexpr size_t kSmem = 128 + kSlots * kLand + kGroups * kXs + kBars;
};

template <int TPC>
__global__ void __launch_bounds__(32 * StreamGeo<TPC>::kWarps, 1)
    input_transform_stream(__half* __restrict__ V, const __grid_constant__ CUtensorMap map_x,
                           const Args a, long long n_items) {
  using Gm = Geo<TPC, 1>;
  using Sg = StreamGeo<TPC>;
  extern __shared__ uint8_t st_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(st_raw) + 127) &
                                             ~uintptr_t(127));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + Sg::kSlots * Sg::kLand +
                                               Sg::kGroups * Sg::kXs);
  uint64_t* full = bars;
  uint64_t* empty = bars + Sg::kSlots;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = a.C;
  const int per_row = a.n_twc * ((C + Gm::kCGN - 1) / Gm::kCGN);
  if (threadIdx.x == 0) {
    for (int i = 0; i < Sg::kSlots; ++i) {
      tc::mbar_init(tc::smem_u32(&full[i]), 1);
      tc::mbar_init(tc::smem_u32(&empty[i]), 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      long long j = 0;
      for (long long item = blockIdx.x; item < n_items; item += gridDim.x, ++j) {
        const int sl = (int)(j % Sg::kSlots);
        const uint32_t ph = (uint32_t)((j / Sg::kSlots) & 1);
        if (!mbar_wait_bounded(tc::smem_u32(&empty[sl]), ph ^ 1u)) break;
        const long long lrow = (uint32_t)item / (uint32_t)per_row;  // items < 2^31
        const int bx = (int)(item - lrow * per_row);
        const int twc = bx % a.n_twc, cg = bx / a.n_twc;
        const long long grow = a.row0 + lrow;
        const int b = (int)((uint32_t)grow / (uint32_t)a.nh),
                  th = (int)(grow - (long long)b * a.nh);
        const int w0 = twc * TPC * 6 - a.pad;
        const int x0 = w0 >= 0 ? (w0 & ~7) : -((-w0 + 7) & ~7);
        const uint32_t fb = tc::smem_u32(&full[sl]);
        tc::mbar_expect_tx(fb, (uint32_t)Gm::kLandBytes);
        tma_load_4d(tc::smem_u32(base + sl * Sg::kLand), &map_x, x0, th * 6 - a.pad,
                    cg * Gm::kCGN, b, fb);
      }
    }
  } else {
    // ---------------- consumer groups ----------------
    const int g = (warp - 1) / TPC, wg = (warp - 1) % TPC;
    const uint32_t named = 1u + (uint32_t)g;  // barrier 0 is __syncthreads
    __half* xs = reinterpret_cast<__half*>(base + Sg::kSlots * Sg::kLand + g * Sg::kXs);
    const uint32_t xs_s = tc::smem_u32(xs);
    const long long plane = a.BP * (long long)C;
    long long j = 0;
    for (long long item = blockIdx.x; item < n_items; item += gridDim.x, ++j) {
      if ((int)(j % Sg::kGroups) != g) continue;
      const int sl = (int)(j % Sg::kSlots);
      const uint32_t ph = (uint32_t)((j / Sg::kSlots) & 1);
      const long long lrow = (uint32_t)item / (uint32_t)per_row;  // items < 2^31
      const int bx = (int)(item - lrow * per_row);
      const int twc = bx % a.n_twc, cg = bx / a.n_twc;
      const int c0 = cg * Gm::kCGN;
      const int tw0 = twc * TPC;
      const int ntw = min(TPC, a.nw - tw0);
      const int w0 = tw0 * 6 - a.pad;
      const int x0 = w0 >= 0 ? (w0 & ~7) : -((-w0 + 7) & ~7);
      const int d = w0 - x0;
      // Every warp of the group waits (bounded) for the landing, then the group
      // agrees on the outcome through the named barrier, so after an expiry the
      // whole group leaves together and no warp is left at a later barrier.
      {
        const uint32_t ok = mbar_wait_bounded(tc::smem_u32(&full[sl]), ph) ? 1u : 0u;
        uint32_t all;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\t"
            "setp.ne.u32 p, %1, 0;\n\t"
            "bar.red.and.pred q, %2, %3, p;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(all)
            : "r"(ok), "r"(named), "r"(32 * TPC)
            : "memory");
        if (!all) break;
      }
      // Transpose the landing [channel][row][col] into [col][channel slot][row]
      // (as in input_transform_fast, mode 1), 8-column chunks over the group.
      constexpr int kChunks = Gm::kBoxW / 8;
      constexpr int kQuads = Gm::kCGN / 4;
      const uint32_t land_s = tc::smem_u32(base + sl * Sg::kLand);
      const uint32_t src_lane =
          land_s + (uint32_t)((((lane >> 3) * 8 + (lane & 7)) * Gm::kBoxW) * 2);
      for (int chunk = wg; chunk < kChunks; chunk += TPC) {
        const int col = chunk * 8 + (lane >> 2) - d;
        const bool in = col >= 0 && col < Gm::kInCols;
        const uint32_t src = src_lane + (uint32_t)(chunk * 16);
        const uint32_t dst =
            xs_s + (uint32_t)(((in ? col : 0) * Gm::kColPitch + 2 * (lane & 3)) * 2);
#pragma unroll
        for (int cq = 0; cq < kQuads; ++cq) {
          uint32_t rg[4];
          asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                       : "=r"(rg[0]), "=r"(rg[1]), "=r"(rg[2]), "=r"(rg[3])
                       : "r"(src + (uint32_t)(cq * 4 * 8 * Gm::kBoxW * 2))
                       : "memory");
          if (in) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              asm volatile("st.shared.b32 [%0], %1;" ::"r"(dst + (uint32_t)chan_slot(cq * 4 + i) * 16u),
                           "r"(rg[i])
                           : "memory");
          }
        }
      }
      asm volatile("bar.sync %0, %1;" ::"r"(named), "r"(32 * TPC) : "memory");
      if (wg == 0 && lane == 0) tc::mbar_arrive(tc::smem_u32(&empty[sl]));  // landing read
      const int t = wg;
      if (t < ntw && c0 + 2 * lane < C) {  // C is even: a lane's pair is wholly in or out
        const int cl = 2 * lane;
        __half2* const vt = reinterpret_cast<__half2*>(V + (lrow * a.nw + tw0 + t) * C + c0 + cl);
        const long long step = plane >> 1;  // one position plane of V, in half2
        // The column pass in two halves of its output rows ({0,1,2,7} then
        // {3,4,5,6}): 64 live registers for the intermediate instead of 128,
        // at the cost of reading the staged columns twice.
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          float2 tt[4][8];
#pragma unroll
          for (int jc = 0; jc < 8; ++jc) {  // columns: tmp[.][jc] = B^T d[.][jc]
            float2 v[8], f[4];
            const __half* colp = xs + (t * 6 + jc) * Gm::kColPitch;
            const uint4 wa = *reinterpret_cast<const uint4*>(colp + chan_slot(cl) * 8);
            const uint4 wb = *reinterpret_cast<const uint4*>(colp + chan_slot(cl + 1) * 8);
            const uint32_t ua[4] = {wa.x, wa.y, wa.z, wa.w}, ub[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int i2 = 0; i2 < 4; ++i2) {
              const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&ua[i2]));
              const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&ub[i2]));
              v[2 * i2] = make_float2(fa.x, fb.x);
              v[2 * i2 + 1] = make_float2(fa.y, fb.y);
            }
            if (half == 0)
              bt_1d2_a(v, f);
            else
              bt_1d2_b(v, f);
#pragma unroll
            for (int i = 0; i < 4; ++i) tt[i][jc] = f[i];
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {  // rows: V[r][.] = tmp[r][.] B
            const int r = half == 0 ? (i < 3 ? i : 7) : 3 + i;
            float2 f[8];
            bt_1d2(tt[i], f);
            __half2* out = vt + (long long)(r * 8) * step;
#pragma unroll
            for (int s2 = 0; s2 < 8; ++s2) {
              st_global_h2(out, __float22half2_rn(f[s2]));
              out += step;
            }
          }
        }
      }
      // The staging is read by every warp of the group before the next item
      // overwrites it.
      asm volatile("bar.sync %0, %1;" ::"r"(named), "r"(32 * TPC) : "memory");
    }
  }
  __syncthreads();
  pdl_trigger();
}

template <int TPC>
const void* it_stream_fn() { return (const void*)input_transform_stream<TPC>; }

// kTmaIn: the block's M tiles ([pos][channels] each) arrive by TMA tile loads
// into shared memory instead of 64 scattered 4-byte loads per lane.
// kYTma (needs kTmaIn; W_out % 8 == 0 and TPC = 4, so every chunk starts on a
// 48-byte boundary): the staged 6 x 6*TPC output rows are transposed with
// ldmatrix.trans into a dense [channel][row][col] box in the freed M buffer
// and leave by one TMA tile store per block.
template <int TPC, int G, bool kTmaIn, bool kYTma = false>
__global__ void __launch_bounds__(32 * Geo<TPC, G>::kWarps, NOVA_OT_MIN_BLOCKS)
    output_transform_fast(const __half* __restrict__ M, __half* __restrict__ y,
                          const __grid_constant__ CUtensorMap map_m,
                          const __grid_constant__ CUtensorMap map_y, const Args a) {
  using Gm = Geo<TPC, G>;
  constexpr int kYP = kYTma ? Gm::kCGN + 8 : Gm::kPitch;  // halves per staged pixel
  __shared__ __align__(16) __half ys[6 * Gm::kOutCols * kYP];
  extern __shared__ uint8_t ot_raw[];
  __shared__ uint64_t m_bar;
  long long lrow;
  int b, th, twc, kg;
  block_coords(a, lrow, b, th, twc, kg);
  const int K = a.C, H_out = a.H, W_out = a.W;
  const int k0 = kg * Gm::kCGN;
  const int tw0 = twc * TPC;
  const int ntw = min(TPC, a.nw - tw0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  const long long plane = a.BP * (long long)K;
  const __half* mtiles = reinterpret_cast<const __half*>(
      (reinterpret_cast<uintptr_t>(ot_raw) + 127) & ~uintptr_t(127));
  if constexpr (kTmaIn) {
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&m_bar));
    if (threadIdx.x == 0) {
      const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(mtiles));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      tc::mbar_expect_tx(bar, (uint32_t)(ntw * 64 * Gm::kCGN * 2));
      for (int t = 0; t < ntw; ++t)
        tc::tma_load_3d(dst + (uint32_t)(t * 64 * Gm::kCGN * 2), &map_m, k0,
                        (int)(lrow * a.nw + tw0 + t), 0, bar);
    }
    __syncthreads();
    if (!mbar_wait_bounded(bar, 0)) return;
  }

  for (int it = warp; it < TPC * G; it += Gm::kWarps) {
    const int t = it / G, g = it % G;
    if (t >= ntw) break;
    const int kl = g * 64 + 2 * lane;
    const int k = k0 + kl;
    const bool kok = k < K;
    const __half2* in =
        reinterpret_cast<const __half2*>(M + (lrow * a.nw + tw0 + t) * K + (kok ? k : 0));
    const __half* mt = mtiles + t * 64 * Gm::kCGN + kl;
    float2 tt[6][8];  // the lane's channel pair, paired in every operation
#pragma unroll
    for (int q = 0; q < 8; ++q) {  // columns: tmp[.][q] = A m[.][q]
      float2 m[8], g[6];
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        if constexpr (kTmaIn)
          m[p] = __half22float2(*reinterpret_cast<const __half2*>(mt + (p * 8 + q) * Gm::kCGN));
        else
          m[p] = kok ? __half22float2(in[(long long)(p * 8 + q) * (plane >> 1)])
                     : make_float2(0.f, 0.f);
      }
      a_1d2(m, g);
#pragma unroll
      for (int i = 0; i < 6; ++i) tt[i][q] = g[i];
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) {  // rows: Y[i][.] = tmp[i][.] A^T
      float2 g[6];
      a_1d2(tt[i], g);
#pragma unroll
      for (int j = 0; j < 6; ++j)
        *reinterpret_cast<__half2*>(ys + (i * Gm::kOutCols + t * 6 + j) * kYP + kl) =
            __float22half2_rn(g[j]);
    }
  }
  __syncthreads();

  if constexpr (kYTma) {
    static_assert(kTmaIn && Gm::kOutCols % 8 == 0, "dense y box needs the M buffer and 8-col groups");
    constexpr int kGroups = Gm::kOutCols / 8;
    constexpr int kQuads = Gm::kCGN / 32;
    const uint32_t ys_s = static_cast<uint32_t>(__cvta_generic_to_shared(ys));
    const uint32_t yd_s = static_cast<uint32_t>(__cvta_generic_to_shared(mtiles));
    // Lane L addresses pixel L%8 of channel octet L/8 of an 8-pixel x 32-channel
    // block and receives pixels 2(L%4), 2(L%4)+1 of channel L/4 of each octet.
    const uint32_t lane_src = ys_s + (uint32_t)(((lane & 7) * kYP + (lane >> 3) * 8) * 2);
    const uint32_t lane_dst = yd_s + (uint32_t)(((lane >> 2) * 6 * Gm::kOutCols + 2 * (lane & 3)) * 2);
    for (int item = warp; item < 6 * kGroups * kQuads; item += Gm::kWarps) {
      const int r = item / (kGroups * kQuads);
      const int rem = item - r * (kGroups * kQuads);
      const int g = rem / kQuads, o4 = rem - (rem / kQuads) * kQuads;
      uint32_t rg[4];
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                   : "=r"(rg[0]), "=r"(rg[1]), "=r"(rg[2]), "=r"(rg[3])
                   : "r"(lane_src + (uint32_t)(((r * Gm::kOutCols + 8 * g) * kYP + o4 * 32) * 2))
                   : "memory");
#pragma unroll
      for (int i = 0; i < 4; ++i)
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(
                         lane_dst + (uint32_t)((((o4 * 32 + 8 * i) * 6 + r) * Gm::kOutCols + 8 * g) * 2)),
                     "r"(rg[i])
                     : "memory");
    }
    tc::fence_async_smem();  // the dense box is visible to the TMA unit
    __syncthreads();
    if (threadIdx.x == 0) {
      // Rows past H_out, columns past W_out and channels past K are clipped.
      tma_store_4d(&map_y, yd_s, tw0 * 6, th * 6, k0, b);
      tc::bulk_commit();
      tc::bulk_wait_read_all();
    }
    __syncthreads();
    pdl_trigger();  // after the whole block is done
    return;
  }

  // Write output rows: warp per channel (6 rows each), lane per column.
  const int wcols = min(ntw * 6, W_out - tw0 * 6);
  const int hrows = min(6, H_out - th * 6);
  const long long plane_y = (long long)H_out * W_out;
  __half* yb = y + ((long long)b * K + k0) * plane_y + (long long)(th * 6) * W_out + tw0 * 6;
  // Lane-constant parts once: row offsets in y, validity of the lane's two
  // columns; the channel loop then only advances two pointers.
  const bool c0ok = lane < wcols, c1ok = lane + 32 < wcols;
  int roff[6];
#pragma unroll
  for (int r = 0; r < 6; ++r) roff[r] = r < hrows ? r * W_out : -1;
  const __half* sp = ys + lane * kYP + warp;
  __half* dst = yb + lane + (long long)warp * plane_y;
  const long long dstep = (long long)Gm::kWarps * plane_y;
  for (int kl = warp; kl < Gm::kCGN; kl += Gm::kWarps, sp += Gm::kWarps, dst += dstep) {
    if (k0 + kl >= K) break;
#pragma unroll
    for (int r = 0; r < 6; ++r) {
      if (roff[r] >= 0) {
        if (c0ok) dst[roff[r]] = sp[r * Gm::kOutCols * kYP];
        if (c1ok) dst[roff[r] + 32] = sp[(r * Gm::kOutCols + 32) * kYP];
      }
    }
  }
  __syncthreads();
  pdl_trigger();  // after the whole block is done
}

// ---------------------------------------------------------------------------
// Plane mode: images of at most 3x3 tiles (e.g. 14x14, 7x7).  A block owns a
// whole image for 64 channels.  Row-wise staging would leave most lanes idle on
// 7- or 14-wide rows, so lanes walk the contiguous image plane instead (each
// lane's plane elements and their shared-memory cells are computed once per
// block), and the output is written back as whole contiguous planes.
// ---------------------------------------------------------------------------
// kW > 0 fixes the warps per block (small batches: one warp per tile, so a
// block finishes its image in one round); kW = 0 is the throughput shape.
template <int TR, int TC, int kW = 0>
struct PlaneGeo {
  static constexpr int kRows = TR * 6 + 2, kCols = TC * 6 + 2;    // padded input
  static constexpr int kCells = kRows * kCols;
  static constexpr int kInPerLane = (kCells + 31) / 32;
  static constexpr int kOutCells = 36 * TR * TC;
  static constexpr int kOutPerLane = (kOutCells + 31) / 32;
  static constexpr int kPitch = 66;                                // 64 channels + 2
#ifndef NOVA_PLANE_MAX_WARPS
#define NOVA_PLANE_MAX_WARPS 5  // throughput shape: at most 5 warps (3 blocks/SM); the 3x3-tile input transform uses 3
#endif
  static constexpr int kWarps =
      kW > 0 ? kW
             : (TR * TC < 2 ? 2 : (TR * TC > NOVA_PLANE_MAX_WARPS ? NOVA_PLANE_MAX_WARPS : TR * TC));
  // Blocks per SM the register budget is sized for (about 128 registers/thread).
  static constexpr int kMinBlocks = 65536 / (128 * 32 * kWarps) < 1 ? 1 : 65536 / (128 * 32 * kWarps);
  static constexpr size_t kInSmem = (size_t)kCells * kPitch * 2;
  static constexpr size_t kOutSmem = (size_t)kOutCells * kPitch * 2;
};

// Zeroes a plane kernel's [kCells][kPitch] staging with 16-byte stores
// (kCells = 4 (3TR + 1)(3TC + 1), so the plane is a whole number of 16-byte
// words).  The caller orders it before other warps' writes with a barrier.
template <class Pg>
__device__ __forceinline__ void plane_zero_fill(__half* xs) {
  constexpr int kWords = Pg::kCells * Pg::kPitch * 2 / 16;
  static_assert(Pg::kCells * Pg::kPitch * 2 % 16 == 0, "plane not a multiple of 16 bytes");
  uint4* z = reinterpret_cast<uint4*>(xs);
  for (int i = threadIdx.x; i < kWords; i += 32 * Pg::kWarps) z[i] = make_uint4(0u, 0u, 0u, 0u);
}

// Plane args: BP/row window semantics as Args; row0 and lrow0 are tile rows and
// are multiples of nh here (blocks own whole images).
// Untiled bulk copy global -> shared, completing on an mbarrier (no multicast):
// both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// kLand = 0: each warp loads channels cell by cell with 2-byte loads, two
// channels per round (one memory round trip per round).  kLand = 2 (W even):
// 4-byte loads of cell pairs, NOVA_PLANE_PAIR_CH channels per round.
// kLand = 32 or 64: the
// block's channels of one image are one contiguous span of x ([c][h][w]); it
// lands in shared memory by bulk copies of kLand channels (one round trip
// each) while the zero border of the padded plane is written, and is then
// transposed into [cell][channel].  Needs C % 8 == 0 and a 16-byte aligned x.
// Blocks per SM the plane input transform's register budget is sized for: as
// many as its shared memory admits, up to a budget of 96 registers per thread
// for the bulk-landed throughput shapes of at most 2 x 2 tiles (their staging
// needs no per-lane cell tables and the column pass runs in halves), 128
// registers otherwise.
template <int TR, int TC, int kW, int kLand>
constexpr int plane_it_min_blocks() {
  using Pg = PlaneGeo<TR, TC, kW>;
  constexpr size_t land = kLand >= 32 ? (size_t)kLand * Pg::kCells * 2 : 0;
  constexpr int by_smem = (int)((227 * 1024) / (Pg::kInSmem + land + 1024));
  constexpr int regs = (kW == 0 && kLand >= 32 && TR <= 2 && TC <= 2) ? 96 : 128;
  constexpr int by_regs = 65536 / (regs * 32 * Pg::kWarps);
  constexpr int n = by_smem < by_regs ? by_smem : by_regs;
  return n < 1 ? 1 : n;
}

// One tile of the plane input transform for the lane's channel pair: rows
// (columns) of the 8 x 8 window at index >= NR (NC) are known zero, so their
// loads and terms are skipped.  The column pass runs in two halves of its
// output rows ({0,1,2,7}, {3,4,5,6}): 64 live registers for the intermediate
// instead of 128 (no spills).
template <class Pg, int NR, int NC>
__device__ __forceinline__ void it_plane_tile(const __half* tile_s, __half2* const vt,
                                              const long long step) {
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {
    float2 tt[4][8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= NC) {
#pragma unroll
        for (int i = 0; i < 4; ++i) tt[i][j] = make_float2(0.f, 0.f);
        continue;
      }
      float2 v[8], f[4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[i] = i < NR ? __half22float2(*reinterpret_cast<const __half2*>(
                            tile_s + (i * Pg::kCols + j) * Pg::kPitch))
                      : make_float2(0.f, 0.f);
      if (half == 0)
        bt_1d2_za<NR>(v, f);
      else
        bt_1d2_zb<NR>(v, f);
#pragma unroll
      for (int i = 0; i < 4; ++i) tt[i][j] = f[i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = half == 0 ? (i < 3 ? i : 7) : 3 + i;
      float2 f[8];
      bt_1d2_z<NC>(tt[i], f);
      __half2* out = vt + (long long)(r * 8) * step;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        st_global_h2(out, __float22half2_rn(f[s]));
        out += step;
      }
    }
  }
}

template <int TR, int TC, int kW, int kLand>
__global__ void __launch_bounds__(32 * PlaneGeo<TR, TC, kW>::kWarps,
                                  (plane_it_min_blocks<TR, TC, kW, kLand>()))
    input_transform_plane(const __half* __restrict__ x, __half* __restrict__ V, const Args a) {
  using Pg = PlaneGeo<TR, TC, kW>;
  extern __shared__ __align__(16) __half xs[];  // [kCells][kPitch], then the landing
  __shared__ __align__(8) uint64_t land_bar;
  const int cg = blockIdx.x;
  const long long limg = a.lrow0 / TR + blockIdx.y;  // image inside the window
  const long long b = a.row0 / TR + limg;
  const int C = a.C, H = a.H, W = a.W, pad = a.pad;
  const int c0 = cg * 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();

  const long long plane_x = (long long)H * W;
  const __half* xb = x + (b * C + c0) * plane_x;
  if constexpr (kLand >= 32) {
    const int HW = H * W;
    const int nch = C - c0 < 64 ? C - c0 : 64;
    __half* land = xs + Pg::kCells * Pg::kPitch;  // [kLand][H*W]
    const uint32_t land_s = static_cast<uint32_t>(__cvta_generic_to_shared(land));
    const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(&land_bar));
    if (threadIdx.x == 0) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Padded cell of each of the lane's image cells e = lane + 32 m; only the
    // first n_m rounds hold image cells.  Row h = floor(e / W) by one
    // reciprocal: e < 2^10 and W <= 64, so (e + 1/2) / W sits at least 1/(2W)
    // from an integer, far beyond the FP32 rounding of the product.
    const int n_m = (HW + 31) >> 5;
    const float rcp_w = 1.0f / (float)W;
    int cellofs[Pg::kInPerLane];
#pragma unroll
    for (int m = 0; m < Pg::kInPerLane; ++m) {
      const int e = lane + 32 * m;
      const int h = __float2int_rz(((float)e + 0.5f) * rcp_w);
      const int w = e - h * W;
      cellofs[m] = e < HW ? ((h + pad) * Pg::kCols + w + pad) * Pg::kPitch : -1;
    }
    uint32_t phase = 0;
    for (int ch0 = 0; ch0 < nch; ch0 += kLand) {
      const int n = nch - ch0 < kLand ? nch - ch0 : kLand;
      if (threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                     "r"((uint32_t)(n * HW * 2))
                     : "memory");
        bulk_load(land_s, xb + (long long)ch0 * HW, (uint32_t)(n * HW * 2), bar);
      }
      if (ch0 == 0) {
        // Zero the whole staging plane with 16-byte stores while the copy is
        // in flight (the border is most of it: 147 of 196 cells at 7 x 7); the
        // barrier orders these stores before the interior writes below.
        plane_zero_fill<Pg>(xs);
        __syncthreads();
      }
      if (!mbar_wait_bounded(bar, phase)) return;
      phase ^= 1u;
      // Channel pairs: lanes walk cells (consecutive halves of one channel).
      for (int p2 = warp; 2 * p2 < n; p2 += Pg::kWarps) {
        const __half* s0 = land + (2 * p2) * HW;
        const __half* s1 = s0 + HW;
#pragma unroll
        for (int m = 0; m < Pg::kInPerLane; ++m) {
          if (m >= n_m) break;
          const int e = lane + 32 * m;
          if (cellofs[m] >= 0)
            *reinterpret_cast<__half2*>(xs + cellofs[m] + ch0 + 2 * p2) =
                __halves2half2(s0[e], s1[e]);
        }
      }
      __syncthreads();  // the landing is read before it is refilled
    }
  } else if constexpr (kLand == 2) {
    // W even: one 4-byte load brings cells (w, w + 1) of a row of one
    // channel, so a channel takes H*W/64 loads per lane and several channels
    // fit a round.  The zero border is written once, not loaded.
    const int HW2 = (H * W) >> 1;
    constexpr int kPairPer = (Pg::kCells / 2 + 31) / 32;
    const int n_m = (HW2 + 31) >> 5;  // rounds that hold image cell pairs
    const float rcp_w = 1.0f / (float)W;  // as in the bulk path: exact floor(e / W)
    int pofs[kPairPer];  // padded cell of the pair's first element, -1 past the plane
#pragma unroll
    for (int m = 0; m < kPairPer; ++m) {
      const int e = 2 * (lane + 32 * m);
      const int h = __float2int_rz(((float)e + 0.5f) * rcp_w);
      const int w = e - h * W;
      pofs[m] = e < 2 * HW2 ? ((h + pad) * Pg::kCols + w + pad) * Pg::kPitch : -1;
    }
    // Zero the whole plane with 16-byte stores, then the interior is written.
    plane_zero_fill<Pg>(xs);
    __syncthreads();
    const uint32_t* xb2 = reinterpret_cast<const uint32_t*>(xb);
    constexpr int kCh = NOVA_PLANE_PAIR_CH;
    for (int cl0 = warp; cl0 < 64; cl0 += Pg::kWarps * kCh) {
      uint32_t v[kCh][kPairPer];
#pragma unroll
      for (int u = 0; u < kCh; ++u) {
        const int cl = cl0 + u * Pg::kWarps;
        const bool cok = cl < 64 && c0 + cl < C;
        const uint32_t* cp = xb2 + (cok ? cl : 0) * (long long)HW2;
#pragma unroll
        for (int m = 0; m < kPairPer; ++m) {
          if (m >= n_m) break;
          v[u][m] = (cok && pofs[m] >= 0) ? __ldg(cp + lane + 32 * m) : 0u;
        }
      }
#pragma unroll
      for (int u = 0; u < kCh; ++u) {
        const int cl = cl0 + u * Pg::kWarps;
        if (cl < 64) {
#pragma unroll
          for (int m = 0; m < kPairPer; ++m) {
            if (m >= n_m) break;
            if (pofs[m] >= 0) {
              xs[pofs[m] + cl] = __ushort_as_half((unsigned short)(v[u][m] & 0xffffu));
              xs[pofs[m] + Pg::kPitch + cl] = __ushort_as_half((unsigned short)(v[u][m] >> 16));
            }
          }
        }
      }
    }
  } else {
    // Lane's padded-plane cells: global offset inside the image plane (or -1 for
    // zero padding) and shared-memory cell offset.
    int goff[Pg::kInPerLane], soff[Pg::kInPerLane];
#pragma unroll
    for (int m = 0; m < Pg::kInPerLane; ++m) {
      const int e = lane + 32 * m;
      const int r = e / Pg::kCols, col = e - (e / Pg::kCols) * Pg::kCols;
      const int h = r - pad, w = col - pad;
      soff[m] = e < Pg::kCells ? e * Pg::kPitch : -1;
      goff[m] = (e < Pg::kCells && h >= 0 && h < H && w >= 0 && w < W) ? h * W + w : -1;
    }
    // Two channels per round: their loads are all in flight before any store.
    constexpr int kCh = 2;
    for (int cl0 = warp; cl0 < 64; cl0 += Pg::kWarps * kCh) {
      __half v[kCh][Pg::kInPerLane];
#pragma unroll
      for (int u = 0; u < kCh; ++u) {
        const int cl = cl0 + u * Pg::kWarps;
        const bool cok = cl < 64 && c0 + cl < C;
        const __half* cp = xb + (cok ? cl : 0) * plane_x;
#pragma unroll
        for (int m = 0; m < Pg::kInPerLane; ++m)
          v[u][m] = (cok && goff[m] >= 0) ? cp[goff[m]] : __ushort_as_half(0);
      }
#pragma unroll
      for (int u = 0; u < kCh; ++u) {
        const int cl = cl0 + u * Pg::kWarps;
        if (cl < 64) {
#pragma unroll
          for (int m = 0; m < Pg::kInPerLane; ++m)
            if (soff[m] >= 0) xs[soff[m] + cl] = v[u][m];
        }
      }
    }
  }
  __syncthreads();

  const long long plane = a.BP * (long long)C;
  for (int t = warp; t < TR * TC; t += Pg::kWarps) {
    const int tr = t / TC, tc = t - (t / TC) * TC;
    const int cl = 2 * lane;
    const int c = c0 + cl;
    if (c >= C) continue;  // C is even: the lane's pair is wholly in or out
    const long long bp = (limg * TR + tr) * TC + tc;
    __half2* const vt = reinterpret_cast<__half2*>(V + bp * C + c);
    const long long step = plane >> 1;  // one position plane of V, in half2
    const __half* tile_s = xs + ((tr * 6) * Pg::kCols + tc * 6) * Pg::kPitch + cl;
    // Window rows (columns) at or past H + pad (W + pad) lie in the zero
    // border: a tile with at most 3 image rows (columns) takes the body that
    // drops their terms.
    const bool short_r = H + pad - 6 * tr <= 3, short_c = W + pad - 6 * tc <= 3;
    if (short_r) {
      if (short_c)
        it_plane_tile<Pg, 3, 3>(tile_s, vt, step);
      else
        it_plane_tile<Pg, 3, 8>(tile_s, vt, step);
    } else {
      if (short_c)
        it_plane_tile<Pg, 8, 3>(tile_s, vt, step);
      else
        it_plane_tile<Pg, 8, 8>(tile_s, vt, step);
    }
  }
  __syncthreads();
  pdl_trigger();  // after the whole block is done
}

template <int TR, int TC, int kW, bool kTma>
__global__ void __launch_bounds__(32 * PlaneGeo<TR, TC, kW>::kWarps, PlaneGeo<TR, TC, kW>::kMinBlocks)
    output_transform_plane(const __half* __restrict__ M, __half* __restrict__ y,
                           const __grid_constant__ CUtensorMap map_m, const Args a) {
  constexpr bool m_tma = kTma;
  using Pg = PlaneGeo<TR, TC, kW>;
  extern __shared__ __align__(16) __half ys[];  // [kOutCells][kPitch], then the M slots
  // With kTma, each warp brings its tile's M ([pos][64 channels], 8 KB) into
  // its own 128-byte aligned slot by one TMA tile load: all 64 positions arrive
  // in one round trip instead of eight.
  __half* mslot = reinterpret_cast<__half*>(
      (reinterpret_cast<uintptr_t>(ys + Pg::kOutCells * Pg::kPitch) + 127) & ~uintptr_t(127));
  __shared__ uint64_t wbar[Pg::kWarps];
  const int kg = blockIdx.x;
  const long long limg = a.lrow0 / TR + blockIdx.y;
  const long long b = a.row0 / TR + limg;
  const int K = a.C, H_out = a.H, W_out = a.W;
  const int k0 = kg * 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();
  const long long plane = a.BP * (long long)K;
  if constexpr (m_tma) {
    if (threadIdx.x == 0) {
      for (int w = 0; w < Pg::kWarps; ++w)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(
                         static_cast<uint32_t>(__cvta_generic_to_shared(&wbar[w])))
                     : "memory");
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
  }
  const __half* my_slot = mslot + warp * 64 * 64;
  const uint32_t my_bar = static_cast<uint32_t>(__cvta_generic_to_shared(&wbar[warp]));

  int round = 0;
  for (int t = warp; t < TR * TC; t += Pg::kWarps, ++round) {
    const int tr = t / TC, tc = t - (t / TC) * TC;
    const int kl = 2 * lane;
    const int k = k0 + kl;
    const bool kok = k < K;
    const long long bp = (limg * TR + tr) * TC + tc;
    const __half2* in = reinterpret_cast<const __half2*>(M + bp * K + (kok ? k : 0));
    if constexpr (m_tma) {
      __syncwarp();  // every lane is done with the slot's previous tile
      if (lane == 0) {
        tc::mbar_expect_tx(my_bar, 64 * 64 * 2);
        tc::tma_load_3d(static_cast<uint32_t>(__cvta_generic_to_shared(my_slot)), &map_m, k0,
                        (int)bp, 0, my_bar);
      }
      if (!mbar_wait_bounded(my_bar, (uint32_t)round & 1u)) return;
    }
    float2 tt[6][8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float2 m[8], g[6];
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        if constexpr (m_tma)
          m[p] = __half22float2(
              *reinterpret_cast<const __half2*>(my_slot + (p * 8 + q) * 64 + kl));
        else
          m[p] = kok ? __half22float2(in[(long long)(p * 8 + q) * (plane >> 1)])
                     : make_float2(0.f, 0.f);
      }
      a_1d2(m, g);
#pragma unroll
      for (int i = 0; i < 6; ++i) tt[i][q] = g[i];
    }
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      float2 g[6];
      a_1d2(tt[i], g);
#pragma unroll
      for (int j = 0; j < 6; ++j)
        *reinterpret_cast<__half2*>(ys + ((tr * 6 + i) * (TC * 6) + tc * 6 + j) * Pg::kPitch +
                                    kl) = __float22half2_rn(g[j]);
    }
  }
  __syncthreads();

  // Whole output planes: lane over the plane's elements.
  const int HW = H_out * W_out;
  int soff[Pg::kOutPerLane];
#pragma unroll
  for (int m = 0; m < Pg::kOutPerLane; ++m) {
    const int e = lane + 32 * m;
    const int r = e / W_out, col = e - (e / W_out) * W_out;
    soff[m] = e < HW ? (r * (TC * 6) + col) * Pg::kPitch : -1;
  }
  __half* yb = y + (b * K + k0) * (long long)HW;
  for (int kl = warp; kl < 64; kl += Pg::kWarps) {
    if (k0 + kl >= K) break;
    __half* dst = yb + (long long)kl * HW;
#pragma unroll
    for (int m = 0; m < Pg::kOutPerLane; ++m)
      if (soff[m] >= 0) dst[lane + 32 * m] = ys[soff[m] + kl];
  }
  __syncthreads();
  pdl_trigger();  // after the whole block is done
}

// Kernel addresses for the shared-memory opt-in.
template <int TR, int TC, int kW, int kLand>
const void* it_plane_fn() { return (const void*)input_transform_plane<TR, TC, kW, kLand>; }
template <int TR, int TC, int kW, bool kTma>
const void* ot_plane_fn() { return (const void*)output_transform_plane<TR, TC, kW, kTma>; }

// Blocks of the plane kernels a launch needs before the throughput shape
// (5 warps, several blocks per SM) beats one warp per tile.
static bool plane_small(long long blocks) {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  if (!sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return blocks < sms[dev];
}

// Bulk-landed plane input (kLand channels per copy) for the throughput shapes
// of fewer than 9 tiles: 7x7 images, 512 channels, batch 128 went from 27.0 to
// 21.5 us.  At 3x3 tiles the landing buffer costs a block per SM and the
// kernel is issue-bound (32.7 us with 32-channel copies, 32.8 with 64, 14x14
// images, 256 channels); there cell-pair loads take it from 31.7 to 27.6 us.
// NOVA_PLANE_LAND=0, 2 (cell-pair loads), 32 or 64 forces a choice.
static int plane_land_choice(int TRTC) {
  static const int env = [] {
    const char* e = std::getenv("NOVA_PLANE_LAND");
    return e ? std::atoi(e) : -1;
  }();
  if (env == 0 || env == 2 || env == 32 || env == 64) return env;
  return TRTC >= 9 ? 2 : 64;
}

template <int TR, int TC, int kW, int kLand>
static void launch_it_plane_k(const __half* x, __half* V, Args a, long long nimg, unsigned gx,
                              cudaStream_t s) {
  using Pg = PlaneGeo<TR, TC, kW>;
  constexpr size_t kLandCh = kLand >= 32 ? kLand : 0;  // channels of the bulk landing buffer
  const size_t smem = Pg::kInSmem + kLandCh * a.H * a.W * 2;
  if (!smem_optin_once<it_plane_fn<TR, TC, kW, kLand>>(Pg::kInSmem + kLandCh * Pg::kCells * 2))
    return;
  for (long long done = 0; done < nimg; done += kMaxGridY) {
    a.lrow0 = done * TR;
    dim3 grid(gx, (unsigned)std::min(kMaxGridY, nimg - done));
    launch_pdl(kPdlInput, input_transform_plane<TR, TC, kW, kLand>, grid, dim3(32 * Pg::kWarps),
               smem, s, x, V, a);
  }
}

template <int TR, int TC, int kW>
static void launch_it_plane_w(const __half* x, __half* V, Args a, long long nimg, unsigned gx,
                              cudaStream_t s) {
  constexpr bool kThroughput = kW != (TR * TC < 2 ? 2 : TR * TC);
  int land = (kThroughput && a.C % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0)
                 ? plane_land_choice(TR * TC)
                 : 0;
  if (land == 2 && (a.W % 2 || (reinterpret_cast<uintptr_t>(x) & 3))) land = 0;
  if (land == 64)
    launch_it_plane_k<TR, TC, kW, 64>(x, V, a, nimg, gx, s);
  else if (land == 32)
    launch_it_plane_k<TR, TC, kW, 32>(x, V, a, nimg, gx, s);
  else if (land == 2)
    launch_it_plane_k<TR, TC, kW, 2>(x, V, a, nimg, gx, s);
  else
    launch_it_plane_k<TR, TC, kW, 0>(x, V, a, nimg, gx, s);
}

template <int TR, int TC>
static void launch_it_plane(const __half* x, __half* V, Args a, long long nimg, unsigned gx,
                            cudaStream_t s) {
  constexpr int kOne = TR * TC < 2 ? 2 : TR * TC;
  // 3x3-tile images at throughput batches: 3 warps of 3 tiles each, so that
  // 4 blocks fit per SM and a batch-128 launch of 64-channel groups runs in one
  // wave (measured 25.0 -> 23.8 us at 256 channels, 14x14, batch 128).
  if (TR * TC > NOVA_PLANE_MAX_WARPS && plane_small(nimg * gx))
    launch_it_plane_w<TR, TC, kOne>(x, V, a, nimg, gx, s);
  else if (TR * TC == 9)
    launch_it_plane_w<TR, TC, 3>(x, V, a, nimg, gx, s);
  else
    launch_it_plane_w<TR, TC, 0>(x, V, a, nimg, gx, s);
}

static bool encode_v_map(CUtensorMap* map, const __half* V, int C, long long BP, int cgn);

// M by TMA tile loads into per-warp slots for the throughput shapes (conv4_x
// batch 128: 15.5 us against 21.1 with direct loads in that kernel); direct
// loads for the one-warp-per-tile small-batch shapes, where the extra round
// trip before the first position costs more than it hides.
template <int TR, int TC, int kW>
static void launch_ot_plane_w(const __half* M, __half* y, Args a, long long nimg, unsigned gx,
                              cudaStream_t s) {
  using Pg = PlaneGeo<TR, TC, kW>;
  CUtensorMap map_m{};
  const size_t tma_smem = (size_t)Pg::kOutCells * Pg::kPitch * 2 + 128 +
                          (size_t)Pg::kWarps * 64 * 64 * 2;
  const bool tma = kW == 0 && encode_v_map(&map_m, M, a.C, a.BP, 64) &&
                   smem_optin_once<ot_plane_fn<TR, TC, kW, true>>(tma_smem);
  if (!tma && !smem_optin_once<ot_plane_fn<TR, TC, kW, false>>(Pg::kOutSmem)) return;
  for (long long done = 0; done < nimg; done += kMaxGridY) {
    a.lrow0 = done * TR;
    dim3 grid(gx, (unsigned)std::min(kMaxGridY, nimg - done));
    if (tma)
      launch_pdl(kPdlOutput, output_transform_plane<TR, TC, kW, true>, grid,
                 dim3(32 * Pg::kWarps), tma_smem, s, M, y, map_m, a);
    else
      launch_pdl(kPdlOutput, output_transform_plane<TR, TC, kW, false>, grid,
                 dim3(32 * Pg::kWarps), Pg::kOutSmem, s, M, y, map_m, a);
  }
}

template <int TR, int TC>
static void launch_ot_plane(const __half* M, __half* y, Args a, long long nimg, unsigned gx,
                            cudaStream_t s) {
  constexpr int kOne = TR * TC < 2 ? 2 : TR * TC;
  if (TR * TC > NOVA_PLANE_MAX_WARPS && plane_small(nimg * gx))
    launch_ot_plane_w<TR, TC, kOne>(M, y, a, nimg, gx, s);
  else
    launch_ot_plane_w<TR, TC, 0>(M, y, a, nimg, gx, s);
}

#define NOVA_PLANE_SWITCH(TR_VAL, TC_VAL, FN, ...)  \
  switch ((TR_VAL) * 4 + (TC_VAL)) {                \
    case 1 * 4 + 1: FN<1, 1>(__VA_ARGS__); break;   \
    case 1 * 4 + 2: FN<1, 2>(__VA_ARGS__); break;   \
    case 1 * 4 + 3: FN<1, 3>(__VA_ARGS__); break;   \
    case 2 * 4 + 1: FN<2, 1>(__VA_ARGS__); break;   \
    case 2 * 4 + 2: FN<2, 2>(__VA_ARGS__); break;   \
    case 2 * 4 + 3: FN<2, 3>(__VA_ARGS__); break;   \
    case 3 * 4 + 1: FN<3, 1>(__VA_ARGS__); break;   \
    case 3 * 4 + 2: FN<3, 2>(__VA_ARGS__); break;   \
    default: FN<3, 3>(__VA_ARGS__); break;          \
  }

// Plane mode applies to whole images of at most 3x3 tiles.
static bool use_plane(int nh, int nw, long long row0, long long nrows) {
  return nh <= 3 && nw <= 3 && row0 % nh == 0 && nrows % nh == 0;
}

// ---------------------------------------------------------------------------
// Host dispatch.
// ---------------------------------------------------------------------------
struct Plan {
  int n_twc, tpc, G, n_cg;
};

static Plan make_plan(int nw, int C) {
  Plan p;
  p.n_twc = (nw + kMaxTPC - 1) / kMaxTPC;
  p.tpc = (nw + p.n_twc - 1) / p.n_twc;
  p.G = (p.tpc <= 2 && C >= 128) ? 2 : 1;
  p.n_cg = (C + 64 * p.G - 1) / (64 * p.G);
  return p;
}


using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return static_cast<EncodeTiledFn>(nullptr);
  }();
  return fn;
}

// 4-D map over x [B][C][H][W] (W fastest) with box {box_w, 8, cgn, 1}; needs
// W % 8 == 0 (16-byte row stride) and a 16-byte aligned base.
static bool encode_x_map_raw(CUtensorMap* map, const __half* x, int B, int C, int H, int W,
                         int box_w, int cgn) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (W % 8) || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)C, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)W * 2, (cuuint64_t)H * W * 2, (cuuint64_t)C * H * W * 2};
  cuuint32_t box[4] = {(cuuint32_t)box_w, 8, (cuuint32_t)cgn, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(x), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_x_map(CUtensorMap* map, const __half* x, int B, int C, int H, int W,
                         int box_w, int cgn) {
  return cached_tensor_map(map, x, ((long long)B << 32) | (unsigned)C, ((long long)H << 32) | (unsigned)W, ((long long)box_w << 32) | (unsigned)cgn, 3, [&](CUtensorMap* m) {
    return encode_x_map_raw(m, x, B, C, H, W, box_w, cgn);
  });
}

template <int TPC, int G>
const void* it_tma_fn() { return (const void*)input_transform_fast<TPC, G, 1>; }
template <int TPC, int G>
const void* it_pair_fn() { return (const void*)input_transform_fast<TPC, G, 2>; }

constexpr size_t kPairSmemMax = 100 * 1024;

// Pair-row view of x: dims {2W, H/2, C, B}, box {2W, 5, cgn, 1}.
static bool encode_x_pair_map_raw(CUtensorMap* map, const __half* x, int B, int C, int H, int W,
                              int cgn) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (W % 4) || (H % 2) || 2 * W > 256 || (reinterpret_cast<uintptr_t>(x) & 15))
    return false;
  cuuint64_t dims[4] = {(cuuint64_t)2 * W, (cuuint64_t)H / 2, (cuuint64_t)C, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)W * 4, (cuuint64_t)H * W * 2, (cuuint64_t)C * H * W * 2};
  cuuint32_t box[4] = {(cuuint32_t)(2 * W), 5, (cuuint32_t)cgn, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(x), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_x_pair_map(CUtensorMap* map, const __half* x, int B, int C, int H, int W,
                              int cgn) {
  return cached_tensor_map(map, x, ((long long)B << 32) | (unsigned)C, ((long long)H << 32) | (unsigned)W, cgn, 4, [&](CUtensorMap* m) {
    return encode_x_pair_map_raw(m, x, B, C, H, W, cgn);
  });
}

// V as [64 pos][BP][C] (C fastest), box {cgn, 1 tile, 64 pos}: one TMA store
// per staged tile.  Needs C % 8 == 0 (16-byte strides) and BP < 2^31.
static bool encode_v_map_raw(CUtensorMap* map, const __half* V, int C, long long BP, int cgn) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (C % 8) || BP <= 0 || BP >= (1ll << 31) ||
      (reinterpret_cast<uintptr_t>(V) & 15))
    return false;
  cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)BP, 64};
  cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)C * 2 * (cuuint64_t)BP};
  cuuint32_t box[3] = {(cuuint32_t)cgn, 1, 64};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(V), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_v_map(CUtensorMap* map, const __half* V, int C, long long BP, int cgn) {
  return cached_tensor_map(map, V, C, BP, cgn, 1, [&](CUtensorMap* m) {
    return encode_v_map_raw(m, V, C, BP, cgn);
  });
}

// The streaming input transform for TMA-staged rows, on unless NOVA_IT_STREAM=0.
static bool it_stream_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("NOVA_IT_STREAM");
    return !(e && e[0] == '0');
  }();
  return on;
}

// SMs of the current device (persistent grids), looked up once per device.
static int num_sms_cached() {
  static int sms[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    sms[dev] = n;
  }
  return sms[dev];
}

template <int TPC, int G>
static void launch_it(const __half* x, __half* V, Args a, long long nrows, unsigned gx,
                      cudaStream_t s) {
  using Gm = Geo<TPC, G>;
  CUtensorMap map{}, map_v{};
  int mode = 0;
  size_t smem = Gm::kInSmem + 128;
  if (encode_x_map(&map, x, a.B, a.C, a.H, a.W, Gm::kBoxW, Gm::kCGN) &&
      encode_v_map(&map_v, V, a.C, a.BP, Gm::kCGN) &&
      smem_optin_once<it_tma_fn<TPC, G>>(Gm::kInSmemTma)) {
    mode = 1;  // TMA in, TMA out
    smem = Gm::kInSmemTma;
  } else {
    const size_t pair_smem = 128 + pair_land_bytes<TPC, G>(a.W) + Gm::kInSmem;
    if (pair_smem <= kPairSmemMax &&
        encode_x_pair_map(&map, x, a.B, a.C, a.H, a.W, Gm::kCGN) &&
        encode_v_map(&map_v, V, a.C, a.BP, Gm::kCGN) &&
        smem_optin_once<it_pair_fn<TPC, G>>(kPairSmemMax)) {
      mode = 2;
      smem = pair_smem;
    }
  }
  if constexpr (G == 1 && TPC >= 4 && TPC <= 6) {
    if (mode == 1 && it_stream_enabled() &&
        smem_optin_once<it_stream_fn<TPC>>(StreamGeo<TPC>::kSmem)) {
      a.lrow0 = 0;
      const long long n_items = nrows * (long long)gx;
      const long long grid = std::min<long long>(n_items, num_sms_cached());
      launch_pdl(kPdlInput, input_transform_stream<TPC>, dim3((unsigned)grid),
                 dim3(32 * StreamGeo<TPC>::kWarps), StreamGeo<TPC>::kSmem, s, V, map, a,
                 n_items);
      return;
    }
  }
  for (long long done = 0; done < nrows; done += kMaxGridY) {
    a.lrow0 = done;
    dim3 grid(gx, (unsigned)std::min(kMaxGridY, nrows - done));
    const unsigned thr = 32 * Gm::kWarps;
    if (mode == 1)
      launch_pdl(kPdlInput, input_transform_fast<TPC, G, 1>, grid, dim3(thr), smem, s, x, V, map, map_v, a);
    else if (mode == 2)
      launch_pdl(kPdlInput, input_transform_fast<TPC, G, 2>, grid, dim3(thr), smem, s, x, V, map, map_v, a);
    else
      launch_pdl(kPdlInput, input_transform_fast<TPC, G, 0>, grid, dim3(thr), smem, s, x, V, map, map_v, a);
  }
}

template <int TPC, int G>
const void* ot_tma_fn() { return (const void*)output_transform_fast<TPC, G, true>; }
const void* ot_ytma_fn() { return (const void*)output_transform_fast<4, 1, true, true>; }

// y as [B][K][H_out][W_out] (W fastest), box {24, 6, 64, 1}: one TMA store per
// 4-tile chunk.  Needs W_out % 8 == 0 (16-byte row stride).
static bool encode_y_map_raw(CUtensorMap* map, const __half* y, int B, int K, int H_out, int W_out) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || (W_out % 8) || (reinterpret_cast<uintptr_t>(y) & 15)) return false;
  cuuint64_t dims[4] = {(cuuint64_t)W_out, (cuuint64_t)H_out, (cuuint64_t)K, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)W_out * 2, (cuuint64_t)H_out * W_out * 2,
                           (cuuint64_t)K * H_out * W_out * 2};
  cuuint32_t box[4] = {24, 6, 64, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(y), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_y_map(CUtensorMap* map, const __half* y, int B, int K, int H_out, int W_out) {
  return cached_tensor_map(map, y, ((long long)B << 32) | (unsigned)K, ((long long)H_out << 32) | (unsigned)W_out, 0, 5, [&](CUtensorMap* m) {
    return encode_y_map_raw(m, y, B, K, H_out, W_out);
  });
}

// The TMA y-store output transform, on unless NOVA_OT_YTMA=0.
static bool ot_ytma_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("NOVA_OT_YTMA");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <int TPC, int G>
static void launch_ot(const __half* M, __half* y, Args a, long long nrows, unsigned gx,
                      cudaStream_t s) {
  using Gm = Geo<TPC, G>;
  CUtensorMap map_m{};
  const size_t tma_smem = 128 + (size_t)TPC * 64 * Gm::kCGN * 2;
  const bool tma = encode_v_map(&map_m, M, a.C, a.BP, Gm::kCGN) &&
                   smem_optin_once<ot_tma_fn<TPC, G>>(tma_smem, 6 * Gm::kOutCols * Gm::kPitch * 2 + 8);
  for (long long done = 0; done < nrows; done += kMaxGridY) {
    a.lrow0 = done;
    dim3 grid(gx, (unsigned)std::min(kMaxGridY, nrows - done));
    if (tma)
      launch_pdl(kPdlOutput, output_transform_fast<TPC, G, true>, grid, dim3(32 * Gm::kWarps),
                 tma_smem, s, M, y, map_m, map_m, a);
    else
      launch_pdl(kPdlOutput, output_transform_fast<TPC, G, false>, grid, dim3(32 * Gm::kWarps),
                 0, s, M, y, map_m, map_m, a);
  }
}

#define NOVA_TPC_SWITCH(TPC_VAL, G_VAL, FN, ...)                       \
  switch ((TPC_VAL) * 4 + (G_VAL)) {                                   \
    case 1 * 4 + 1: FN<1, 1>(__VA_ARGS__); break;                      \
    case 1 * 4 + 2: FN<1, 2>(__VA_ARGS__); break;                      \
    case 2 * 4 + 1: FN<2, 1>(__VA_ARGS__); break;                      \
    case 2 * 4 + 2: FN<2, 2>(__VA_ARGS__); break;                      \
    case 3 * 4 + 1: FN<3, 1>(__VA_ARGS__); break;                      \
    case 4 * 4 + 1: FN<4, 1>(__VA_ARGS__); break;                      \
    case 5 * 4 + 1: FN<5, 1>(__VA_ARGS__); break;                      \
    default: FN<6, 1>(__VA_ARGS__); break;                             \
  }

}  // namespace fast

#ifdef NOVA_FAST_TRACE
extern "C" __attribute__((visibility("default"))) int nova_debug_fast_trace(
    unsigned long long* out, int n_blocks) {
  if (n_blocks > fast::kFtBlocks) n_blocks = fast::kFtBlocks;
  return (int)cudaMemcpyFromSymbol(out, fast::g_fast_trace,
                                   sizeof(unsigned long long) * fast::kFtSlots * (size_t)n_blocks);
}
#endif

cudaError_t launch_input_transform_fast(const __half* x, __half* V, int B, int C, int H, int W,
                                        int pad, int nh, int nw, long long row0, long long nrows,
                                        long long BP, cudaStream_t s) {
  if (nrows <= 0) return cudaSuccess;
  if (fast::use_plane(nh, nw, row0, nrows)) {
    fast::Args a{C, H, W, pad, B, nh, nw, row0, 0, BP, 1};
    NOVA_PLANE_SWITCH(nh, nw, fast::launch_it_plane, x, V, a, nrows / nh,
                      (unsigned)((C + 63) / 64), s);
    return cudaGetLastError();
  }
  const fast::Plan p = fast::make_plan(nw, C);
  fast::Args a{C, H, W, pad, B, nh, nw, row0, 0, BP, p.n_twc};
  const unsigned gx = (unsigned)(p.n_twc * p.n_cg);
  NOVA_TPC_SWITCH(p.tpc, p.G, fast::launch_it, x, V, a, nrows, gx, s);
  return cudaGetLastError();
}

cudaError_t launch_output_transform_fast(const __half* M, __half* y, int K, int H_out, int W_out,
                                         int nh, int nw, long long row0, long long nrows,
                                         long long BP, cudaStream_t s) {
  if (nrows <= 0) return cudaSuccess;
  if (fast::use_plane(nh, nw, row0, nrows)) {
    fast::Args a{K, H_out, W_out, 0, 0, nh, nw, row0, 0, BP, 1};
    NOVA_PLANE_SWITCH(nh, nw, fast::launch_ot_plane, M, y, a, nrows / nh,
                      (unsigned)((K + 63) / 64), s);
    return cudaGetLastError();
  }
  if ((W_out % 8) == 0 && nw >= 4 && fast::ot_ytma_enabled()) {
    // 4-tile chunks, 64 channels per block, y out by TMA tile stores.
    using Gm = fast::Geo<4, 1>;
    const int B_imgs = (int)((row0 + nrows + nh - 1) / nh);
    CUtensorMap map_m{}, map_y{};
    const size_t tma_smem = 128 + (size_t)4 * 64 * 64 * 2;
    if (fast::encode_v_map(&map_m, M, K, BP, 64) &&
        fast::encode_y_map(&map_y, y, B_imgs, K, H_out, W_out) &&
        fast::smem_optin_once<fast::ot_ytma_fn>(tma_smem, 6 * Gm::kOutCols * (Gm::kCGN + 8) * 2 + 8)) {
      const int n_twc = (nw + 3) / 4;
      fast::Args a{K, H_out, W_out, 0, 0, nh, nw, row0, 0, BP, n_twc};
      const unsigned gx = (unsigned)(n_twc * ((K + 63) / 64));
      for (long long done = 0; done < nrows; done += fast::kMaxGridY) {
        a.lrow0 = done;
        dim3 grid(gx, (unsigned)std::min(fast::kMaxGridY, nrows - done));
        launch_pdl(kPdlOutput, fast::output_transform_fast<4, 1, true, true>, grid,
                   dim3(32 * Gm::kWarps), tma_smem, s, M, y, map_m, map_y, a);
      }
      return cudaGetLastError();
    }
  }
  const fast::Plan p = fast::make_plan(nw, K);
  fast::Args a{K, H_out, W_out, 0, 0, nh, nw, row0, 0, BP, p.n_twc};
  const unsigned gx = (unsigned)(p.n_twc * p.n_cg);
  NOVA_TPC_SWITCH(p.tpc, p.G, fast::launch_ot, M, y, a, nrows, gx, s);
  return cudaGetLastError();
}

}  // namespace nova
