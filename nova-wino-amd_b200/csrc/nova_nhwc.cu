// Input and output transforms for channels-last (NHWC) activations.
//
// The reference takes NCHW only (Jayluci4/nova-wino-amd csrc/nova_winograd.hip:
// 141-205 / 264-328, the per-tile input and output transforms).  Models on
// B200 run FP16 convolutions channels-last, and in that layout the 8 x 8
// window of a tile is 64 cells of C contiguous channels: a warp reads one cell
// of 64 channels as one 128-byte line, so neither kernel needs the
// shared-memory transposes of the NCHW kernels.  V and M keep the NCHW path's
// layout ([pos][bp][channel]), so the tcgen05 GEMM between them is the same.
// The butterflies are the NCHW plane kernels' (the same operations in the
// same order); the NCHW row and streaming kernels order some FP32 sums
// differently, so the two layouts agree within FP32 reordering.
//
// Both transforms: one warp per (tile, 64-channel group), lane = channel
// pair; a block is TR x TC tiles of one image and one channel group.  The
// input transform lands the block's window by one TMA box load (C % 8 == 0,
// zeros outside the image from the tensor map).  The output transform lands
// each tile's M by a TMA tile load and stores the block's outputs by one TMA
// tile store (K % 8 == 0); for other even K a plain form reads M and writes y
// with 4-byte accesses, 4 warps per block.
#include "nova_common.cuh"
#include "nova_internal.h"

namespace nova {
namespace nhwc {

constexpr int kWarps = 4;  // plain output transform: warps per block
#ifndef NOVA_NHWC_OT_MIN_BLOCKS
#define NOVA_NHWC_OT_MIN_BLOCKS 3  // plain output transform: 168 registers (8 bytes spill at 128)
#endif
constexpr int kMinBlocks = NOVA_NHWC_OT_MIN_BLOCKS;

struct Args {
  int C, H, W, pad;  // input transform: input geometry; output transform: K, H_out, W_out, -
  int nh, nw;
  int n_cg;          // 64-channel groups
  long long BP;      // tiles (= B * nh * nw); V / M extent along bp
};

// One 4-byte store kept in program order (the compiler would otherwise batch
// a tile's stores with their 64-bit addresses and run out of registers).
__device__ __forceinline__ void st_b32(void* p, uint32_t v) {
  asm volatile("st.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t h2_bits(__half2 v) {
  return *reinterpret_cast<const uint32_t*>(&v);
}

constexpr int kCell = 64;                // channels per cell in shared memory

// Block geometry of the input transform: TR tile rows x TC tiles of one image
// row band, one warp per tile; the block's window is (6 TR + 2) x (6 TC + 2)
// cells of 64 channels.
template <int TR, int TC>
struct ItGeo {
  static constexpr int kWarps = TR * TC;
  static constexpr int kBoxW = 6 * TC + 2, kBoxH = 6 * TR + 2;
  static constexpr uint32_t kBoxBytes = (uint32_t)kBoxH * kBoxW * kCell * 2u;
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// Bounded wait on a TMA landing (2 s of globaltimer); false when it expired.
__device__ __forceinline__ bool wait_landing(uint32_t bar) {
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 0) {
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t0 == 0)
        t0 = t;
      else if (t - t0 > 2000000000ull)
        return false;
    }
  }
}

// One tile from the block's landed window ([8 rows][kBoxW columns][64
// channels], zeros outside the image): rows (columns) of the tile's window at
// index >= NR (NC) lie past the image's last row (column) and are known zero,
// so their reads and terms are skipped (bt_1d2_za / _zb / _z drop exactly
// those terms).  The column pass runs in two halves of its output rows
// ({0,1,2,7}, {3,4,5,6}) to keep the intermediate at 64 registers.
template <int kBoxW, int NR, int NC>
__device__ __forceinline__ void it_tile(const __half* ws, __half2* vt, long long step) {
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
                            ws + (i * kBoxW + j) * kCell))
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
        st_b32(out, h2_bits(__float22half2_rn(f[s])));
        out += step;
      }
    }
  }
}

// V[pos][bp][c] = (B^T d B)[pos] for the tile windows d of x[b][h][w][c].
// Block = TR x TC tiles (TR consecutive tile rows, TC consecutive tiles in
// each) and one 64-channel group: one TMA box load lands their window of
// 64-channel cells (out-of-image cells read as zero), then each warp
// transforms one tile from shared memory.
#ifndef NOVA_NHWC_IT_WARPS
#define NOVA_NHWC_IT_WARPS 20  // warps per SM the registers are sized for (96 per thread): conv2_x batch 128 32.5 -> 30.0 us against 16
#endif
template <int TR, int TC>
__global__ void __launch_bounds__(32 * ItGeo<TR, TC>::kWarps, NOVA_NHWC_IT_WARPS / (TR * TC))
    input_transform_nhwc(const __grid_constant__ CUtensorMap map_x, __half* __restrict__ V,
                         const Args a) {
  using Gm = ItGeo<TR, TC>;
  extern __shared__ __align__(128) __half xs[];  // [kBoxH][kBoxW][kCell]
  __shared__ __align__(8) uint64_t bar;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_twc = (a.nw + TC - 1) / TC, n_thr = (a.nh + TR - 1) / TR;
  const uint32_t seg = blockIdx.x;  // 32-bit decode (64-bit division is emulated)
  const int cg = blockIdx.y;
  const int twc = (int)(seg % (uint32_t)n_twc);
  const uint32_t band = seg / (uint32_t)n_twc;  // b * n_thr + thr
  const int thr = (int)(band % (uint32_t)n_thr);
  const long long b = band / (uint32_t)n_thr;
  const int h0 = thr * TR * 6 - a.pad, w0 = twc * TC * 6 - a.pad;
  const uint32_t bar_s = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_s) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_wait();
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_s),
                 "r"(Gm::kBoxBytes)
                 : "memory");
    tma_load_4d(static_cast<uint32_t>(__cvta_generic_to_shared(xs)), &map_x, cg * kCell, w0, h0,
                (int)b, bar_s);
  }
  const bool landed = wait_landing(bar_s);
  const int tr = warp / TC, tc = warp - (warp / TC) * TC;
  const int th = thr * TR + tr, tw = twc * TC + tc;
  const int c = cg * kCell + 2 * lane;
  if (landed && th < a.nh && tw < a.nw && c < a.C) {
    const long long bp = (b * a.nh + th) * a.nw + tw;
    __half2* const vt = reinterpret_cast<__half2*>(V + bp * a.C + c);
    const long long step = (a.BP * a.C) >> 1;  // one position plane of V, in half2
    const __half* ws = xs + ((tr * 6) * Gm::kBoxW + tc * 6) * kCell + 2 * lane;
    // Window rows th*6 - pad + i with i >= H - (th*6 - pad) (columns likewise)
    // are past the image: a tile with at most 3 inside takes the body that
    // drops the rest.
    const bool short_r = a.H - (h0 + tr * 6) <= 3, short_c = a.W - (w0 + tc * 6) <= 3;
    if (short_r) {
      if (short_c)
        it_tile<Gm::kBoxW, 3, 3>(ws, vt, step);
      else
        it_tile<Gm::kBoxW, 3, 8>(ws, vt, step);
    } else {
      if (short_c)
        it_tile<Gm::kBoxW, 8, 3>(ws, vt, step);
      else
        it_tile<Gm::kBoxW, 8, 8>(ws, vt, step);
    }
  }
  __syncthreads();
  pdl_trigger();
}

// y[b][ho][wo][k] = (A^T M A) over the tile's 64 positions, for the output
// cells inside the image.
__global__ void __launch_bounds__(32 * kWarps, kMinBlocks)
    output_transform_nhwc(const __half* __restrict__ M, __half* __restrict__ y, const Args a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * kWarps + warp;
  pdl_wait();
  if (item < a.BP * a.n_cg) {
    const long long bp = item / a.n_cg;
    const int kg = (int)(item - bp * a.n_cg);
    const int K = a.C, H_out = a.H, W_out = a.W;
    const int k = kg * 64 + 2 * lane;
    if (k < K) {
      const int tiles = a.nh * a.nw;
      const long long b = bp / tiles;
      const int t = (int)(bp - b * tiles);
      const int th = t / a.nw, tw = t - (t / a.nw) * a.nw;
      const long long plane = a.BP * K;  // one position plane of M, in halves
      const __half* in = M + bp * K + k;
      float2 tt[6][8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float2 m[8], g[6];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const uint32_t u = __ldg(reinterpret_cast<const unsigned int*>(
              in + (long long)(p * 8 + q) * plane));
          m[p] = __half22float2(*reinterpret_cast<const __half2*>(&u));
        }
        a_1d2(m, g);
#pragma unroll
        for (int i = 0; i < 6; ++i) tt[i][q] = g[i];
      }
      const int rows = min(6, H_out - th * 6), cols = min(6, W_out - tw * 6);
      __half* yt = y + ((b * H_out + th * 6) * (long long)W_out + tw * 6) * K + k;
#pragma unroll
      for (int i = 0; i < 6; ++i) {
        if (i >= rows) break;
        float2 g[6];
        a_1d2(tt[i], g);
#pragma unroll
        for (int j = 0; j < 6; ++j)
          if (j < cols)
            st_b32(yt + ((long long)i * W_out + j) * K, h2_bits(__float22half2_rn(g[j])));
      }
    }
  }
  pdl_trigger();
}

// The output transform with TMA on both sides (K % 8 == 0): block = TR x TC
// tiles (the input transform's block shapes) and one 64-channel group.  Each
// warp brings its tile's M ([64 positions][64 channels], 8 KB) into its own
// slot by one TMA tile load, transforms it and writes its 6 x 6 outputs into
// the block's [6 TR][6 TC][64] staging; one TMA tile store then writes the
// block's outputs to y, clipped at the image's edge and at K.
template <int TR, int TC>
struct OtGeo {
  static constexpr int kWarps = TR * TC;
  static constexpr uint32_t kSlotBytes = 64u * kCell * 2u;
  static constexpr uint32_t kStageBytes = 36u * TR * TC * kCell * 2u;
  static constexpr uint32_t kSmem = kWarps * kSlotBytes + kStageBytes;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

template <int TR, int TC>
__global__ void __launch_bounds__(32 * OtGeo<TR, TC>::kWarps, 16 / (TR * TC))
    output_transform_nhwc_tma(const __grid_constant__ CUtensorMap map_m,
                              const __grid_constant__ CUtensorMap map_y, const Args a) {
  using Gm = OtGeo<TR, TC>;
  extern __shared__ __align__(128) __half ot_smem[];  // slots [kWarps][64][64], staging
  __half* stage = ot_smem + Gm::kWarps * 64 * kCell;  // [6 TR][6 TC][kCell]
  __shared__ __align__(8) uint64_t bars[Gm::kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_twc = (a.nw + TC - 1) / TC, n_thr = (a.nh + TR - 1) / TR;
  const uint32_t seg = blockIdx.x;  // 32-bit decode, as in the input transform
  const int kg = blockIdx.y;
  const int twc = (int)(seg % (uint32_t)n_twc);
  const uint32_t band = seg / (uint32_t)n_twc;
  const int thr = (int)(band % (uint32_t)n_thr);
  const long long b = band / (uint32_t)n_thr;
  const int tr = warp / TC, tc = warp - (warp / TC) * TC;
  const int th = thr * TR + tr, tw = twc * TC + tc;
  const bool live = th < a.nh && tw < a.nw;
  const uint32_t bar_s = static_cast<uint32_t>(__cvta_generic_to_shared(&bars[warp]));
  __half* slot = ot_smem + warp * 64 * kCell;
  if (lane == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_s) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  pdl_wait();
  const long long bp = (b * a.nh + th) * a.nw + tw;
  if (live && lane == 0) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar_s),
                 "r"(Gm::kSlotBytes)
                 : "memory");
    tma_load_3d(static_cast<uint32_t>(__cvta_generic_to_shared(slot)), &map_m, kg * kCell,
                (int)bp, 0, bar_s);
  }
  bool ok = true;
  if (live) {
    ok = wait_landing(bar_s);
    if (ok) {
      const __half* src = slot + 2 * lane;
      float2 tt[6][8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float2 m[8], g[6];
#pragma unroll
        for (int p = 0; p < 8; ++p)
          m[p] = __half22float2(*reinterpret_cast<const __half2*>(src + (p * 8 + q) * kCell));
        a_1d2(m, g);
#pragma unroll
        for (int i = 0; i < 6; ++i) tt[i][q] = g[i];
      }
      __half* dst = stage + ((tr * 6) * (TC * 6) + tc * 6) * kCell + 2 * lane;
#pragma unroll
      for (int i = 0; i < 6; ++i) {
        float2 g[6];
        a_1d2(tt[i], g);
#pragma unroll
        for (int j = 0; j < 6; ++j)
          *reinterpret_cast<__half2*>(dst + (i * (TC * 6) + j) * kCell) = __float22half2_rn(g[j]);
      }
    }
  }
  // Every warp's outputs are staged (or its tile lies past the image, where
  // the store is clipped) before one thread stores the block's tile of y.
  const int all_ok = __syncthreads_and(ok ? 1 : 0);
  if (threadIdx.x == 0 && all_ok) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
            reinterpret_cast<uint64_t>(&map_y)),
        "r"(kg * kCell), "r"(twc * TC * 6), "r"(thr * TR * 6), "r"((int)b),
        "r"(static_cast<uint32_t>(__cvta_generic_to_shared(stage)))
        : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();
}

}  // namespace nhwc

// 4-D map over x [B][H][W][C] (C fastest), box {64 channels, box_w columns,
// box_h rows, 1 image}, no swizzle, zeros outside.
static bool encode_x_nhwc_map(CUtensorMap* map, const __half* x, int B, int C, int H, int W,
                              int box_w, int box_h) {
  return cached_tensor_map(map, x, C, W, (long long)H * 1000003ll + B, 0x100000 + box_w * 256 + box_h,
                           [&](CUtensorMap* m) {
    TensorMapEncodeFn fn = tensor_map_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2, (cuuint64_t)H * W * C * 2};
    cuuint32_t box[4] = {(cuuint32_t)nhwc::kCell, (cuuint32_t)box_w, (cuuint32_t)box_h, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(x), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
  });
}

template <int TR, int TC>
static cudaError_t launch_it_nhwc(const __half* x, __half* V, int B, const nhwc::Args& a,
                                  cudaStream_t s) {
  using Gm = nhwc::ItGeo<TR, TC>;
  CUtensorMap map;
  if (!encode_x_nhwc_map(&map, x, B, a.C, a.H, a.W, Gm::kBoxW, Gm::kBoxH))
    return cudaErrorInvalidValue;
  const long long segs = (long long)B * ((a.nh + TR - 1) / TR) * ((a.nw + TC - 1) / TC);
  return launch_pdl(kPdlInput, nhwc::input_transform_nhwc<TR, TC>,
                    dim3((unsigned)segs, (unsigned)a.n_cg), dim3(32 * Gm::kWarps), Gm::kBoxBytes,
                    s, map, V, a);
}

cudaError_t launch_input_transform_nhwc(const __half* x, __half* V, int B, int C, int H, int W,
                                        int pad, int nh, int nw, long long BP, cudaStream_t s) {
  if (BP == 0 || B == 0) return cudaSuccess;
  if (C % 8 || reinterpret_cast<uintptr_t>(x) % 16) return cudaErrorInvalidValue;
  nhwc::Args a;
  a.C = C;
  a.H = H;
  a.W = W;
  a.pad = pad;
  a.nh = nh;
  a.nw = nw;
  a.n_cg = (C + nhwc::kCell - 1) / nhwc::kCell;
  a.BP = BP;
  // Blocks of 4-5 warps with no idle tile slot where the tile row allows it:
  // 5 tiles for rows of 5 or 10, 3 for 3, 2 x 2 for rows of 2 (7 x 7 images),
  // else 4 (the last block of a row may be partial).
  if (nw % 5 == 0) return launch_it_nhwc<1, 5>(x, V, B, a, s);
  if (nw == 3) return launch_it_nhwc<1, 3>(x, V, B, a, s);
  if (nw == 2) return launch_it_nhwc<2, 2>(x, V, B, a, s);
  return launch_it_nhwc<1, 4>(x, V, B, a, s);
}

template <int TR, int TC>
static cudaError_t launch_ot_nhwc_tma(const __half* M, __half* y, int B, const nhwc::Args& a,
                                      cudaStream_t s) {
  using Gm = nhwc::OtGeo<TR, TC>;
  TensorMapEncodeFn fn = tensor_map_encode_fn();
  if (!fn) return cudaErrorInvalidValue;
  const int K = a.C, Ho = a.H, Wo = a.W;
  CUtensorMap map_m, map_y;
  const bool ok_m = cached_tensor_map(&map_m, M, K, a.BP, 64, 0x200000, [&](CUtensorMap* m) {
    cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)a.BP, 64};
    cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)a.BP * K * 2};
    cuuint32_t box[3] = {(cuuint32_t)nhwc::kCell, 1, 64};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(M), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
  });
  const bool ok_y = cached_tensor_map(
      &map_y, y, K, Wo, (long long)Ho * 1000003ll + B, 0x300000 + TR * 16 + TC,
      [&](CUtensorMap* m) {
        cuuint64_t dims[4] = {(cuuint64_t)K, (cuuint64_t)Wo, (cuuint64_t)Ho, (cuuint64_t)B};
        cuuint64_t strides[3] = {(cuuint64_t)K * 2, (cuuint64_t)Wo * K * 2,
                                 (cuuint64_t)Ho * Wo * K * 2};
        cuuint32_t box[4] = {(cuuint32_t)nhwc::kCell, 6u * TC, 6u * TR, 1};
        cuuint32_t estr[4] = {1, 1, 1, 1};
        return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, y, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
               CUDA_SUCCESS;
      });
  if (!ok_m || !ok_y) return cudaErrorInvalidValue;
  static bool opted[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !opted[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nhwc::output_transform_nhwc_tma<TR, TC>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::kSmem);
    if (e != cudaSuccess) return e;
    opted[dev] = true;
  }
  const long long segs = (long long)B * ((a.nh + TR - 1) / TR) * ((a.nw + TC - 1) / TC);
  return launch_pdl(kPdlOutput, nhwc::output_transform_nhwc_tma<TR, TC>,
                    dim3((unsigned)segs, (unsigned)a.n_cg), dim3(32 * Gm::kWarps), Gm::kSmem, s,
                    map_m, map_y, a);
}

cudaError_t launch_output_transform_nhwc(const __half* M, __half* y, int B, int K, int H_out,
                                         int W_out, int nh, int nw, long long BP, cudaStream_t s) {
  nhwc::Args a;
  a.C = K;
  a.H = H_out;
  a.W = W_out;
  a.pad = 0;
  a.nh = nh;
  a.nw = nw;
  a.n_cg = (K + 63) / 64;
  a.BP = BP;
  const long long items = BP * a.n_cg;
  if (items == 0) return cudaSuccess;
  // K % 8 == 0 and 16-byte aligned M and y: TMA on both sides, in the input
  // transform's block shapes; otherwise plain 4-byte loads and stores.
  if (K % 8 == 0 && reinterpret_cast<uintptr_t>(M) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(y) % 16 == 0) {
    if (nw % 5 == 0) return launch_ot_nhwc_tma<1, 5>(M, y, B, a, s);
    if (nw == 3) return launch_ot_nhwc_tma<1, 3>(M, y, B, a, s);
    if (nw == 2) return launch_ot_nhwc_tma<2, 2>(M, y, B, a, s);
    return launch_ot_nhwc_tma<1, 4>(M, y, B, a, s);
  }
  const long long blocks = (items + nhwc::kWarps - 1) / nhwc::kWarps;
  return launch_pdl(kPdlOutput, nhwc::output_transform_nhwc, dim3((unsigned)blocks),
                    dim3(32 * nhwc::kWarps), 0, s, M, y, a);
}

}  // namespace nova
