// The 64 per-frequency Winograd GEMMs on the 5th-generation tensor cores.
//
//   M[pos][bp][k] = sum_c V[pos][bp][c] * U[pos][k][c]       pos = 0..63
//
// This replaces the reference's rocBLAS gemm_strided_batched_ex call
// (Jayluci4/nova-wino-amd csrc/nova_winograd.hip:534-548: FP16 in, FP32
// compute, FP16 out, batch 64).  Design:
//
// * Persistent kernel, one CTA per SM, tiles enumerated pos-major, then bp tile,
//   then k tile, so CTAs running at the same time share U[pos] and V tiles in L2.
// * Tile = 128 bp rows (MMA M, TMEM lanes) x BN output channels (MMA N <= 256;
//   half of BN when BN-wide tiles would leave most SMs idle) x 64 input
//   channels per pipeline stage (one 128-byte SWIZZLE_128B row).
// * Warp 0: TMA producer (cp.async.bulk.tensor.3d, no multicast).  Warp 1: TMEM
//   allocation and the single-thread tcgen05.mma issuer.  Warps 2-9: two
//   epilogue warpgroups, one per accumulator buffer (tcgen05.ld -> FP16 ->
//   32-row x 64-column swizzled smem slabs -> TMA tile stores of M).  The
//   accumulator is double buffered in TMEM (2 x BN columns) so the epilogue of
//   tile i overlaps the MMAs of tile i+1.
// * Every mbarrier wait is bounded (globaltimer); on expiry the kernel records a
//   status code in device memory, stops issuing work and returns.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "nova_internal.h"
#include "nova_tc_ptx.cuh"

namespace nova {
namespace tc {

constexpr int kBM = 128;        // bp rows per tile
constexpr int kBK = 64;         // input channels per stage (128 B of FP16)
constexpr int kUmmaK = 16;      // K of one kind::f16 MMA
constexpr int kMaxStages = 8;
constexpr int kThreads = 320;   // 10 warps: producer, MMA, 2 epilogue warpgroups
#ifndef NOVA_GEMM_CTAS
#define NOVA_GEMM_CTAS 1
#endif
constexpr int kCtasPerSm = NOVA_GEMM_CTAS;       // co-resident CTAs per SM
constexpr int kTmemCols = 512 / kCtasPerSm;      // each CTA's TMEM share
constexpr int kMaxBN = kTmemCols / 2 > 256 ? 256 : kTmemCols / 2;  // 2 accumulators
constexpr int kSlabCols = 64;   // epilogue staging: output columns per slab fill
constexpr int kSmemLimit = (227 * 1024) / kCtasPerSm - (kCtasPerSm > 1 ? 1024 : 0);

#ifdef NOVA_GEMM_TRACE
__device__ unsigned long long g_gemm_trace[1024][8];
#define TR_T0(v) const long long v = clock64()
#define TR_ADD(slot, t0) atomicAdd(&g_gemm_trace[blockIdx.x & 1023][slot], (unsigned long long)(clock64() - (t0)))
#else
#define TR_T0(v)
#define TR_ADD(slot, t0)
#endif

struct Params {
  __half* M;
  float* Mf;       // non-null: FP32 output, one [64][BP][K] slice per split of the reduction
  long long BP;
  int C, K, BN;
  int n_bp_tiles, n_k_tiles, n_cblk;
  int n_split;     // the reduction's 64-channel blocks split into n_split ranges
  int kb_per_split;
  long long total_tiles;
  int stages;
  int tma_store;  // 1: epilogue stages 32-row slabs in smem and TMA-stores them
  int epi_split;  // 1: both epilogue warpgroups drain every tile, one half of its columns each
  int* status;
};

// Tile t -> (pos, bp tile, k tile) and its range of reduction blocks.  The
// split index runs fastest, so with one split the order is (pos, bp, k).
// 32-bit unsigned arithmetic: the host keeps total_tiles below 2^31 (64-bit
// division is a long emulated sequence, and every warp role decodes every
// tile: at conv2_x that was a measurable share of the MMA issuer's time).
__device__ __forceinline__ void tile_of(const Params& p, long long t64, int& pos, int& bpt,
                                        int& kt, int& cb0, int& cb1) {
  uint32_t t = (uint32_t)t64;
  const uint32_t split = t % (uint32_t)p.n_split;
  t /= (uint32_t)p.n_split;
  const uint32_t per_pos = (uint32_t)p.n_bp_tiles * (uint32_t)p.n_k_tiles;
  pos = (int)(t / per_pos);
  const uint32_t rem = t - (uint32_t)pos * per_pos;
  bpt = (int)(rem / (uint32_t)p.n_k_tiles);
  kt = (int)(rem - (uint32_t)bpt * (uint32_t)p.n_k_tiles);
  cb0 = (int)split * p.kb_per_split;
  cb1 = min(p.n_cblk, cb0 + p.kb_per_split);
}

// FP32 accumulator bits -> FP16, written as kVec 16-byte stores (8 columns each).
template <int kVec>
__device__ __forceinline__ void store_row_f16(__half* dst, const uint32_t* r) {
  uint4* o = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int v = 0; v < kVec; ++v) {
    uint4 w;
    w.x = pack_half2(r[8 * v + 0], r[8 * v + 1]);
    w.y = pack_half2(r[8 * v + 2], r[8 * v + 3]);
    w.z = pack_half2(r[8 * v + 4], r[8 * v + 5]);
    w.w = pack_half2(r[8 * v + 6], r[8 * v + 7]);
    o[v] = w;
  }
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmU,
                   const __grid_constant__ CUtensorMap tmM, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int S = p.stages;
  const uint32_t a_bytes = kBM * kBK * 2;
  const uint32_t b_bytes = (uint32_t)p.BN * kBK * 2;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  // Epilogue staging: one 32-row slab per epilogue warp, BN/64 chunks of
  // 32 x 128 B in the SWIZZLE_128B layout the M tensor map stores from.
  uint8_t* out_stage = base + (size_t)S * stage_bytes;
  const uint32_t slab_bytes = p.tma_store ? 32u * (uint32_t)min(p.BN, kSlabCols) * 2u : 0u;
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + 8 * (size_t)slab_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + kMaxStages;
  uint64_t* tfull = bars + 2 * kMaxStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // MMA issuer: every MMA it issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), p.epi_split ? 256 : 128);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
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
  pdl_wait();  // V (and U) come from earlier kernels in the stream
  TR_T0(tk0);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      long long issued = 0;
      for (long long t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x) {
        int pos, bpt, kt, cb0, cb1;
        tile_of(p, t, pos, bpt, kt, cb0, cb1);
        for (int cb = cb0; cb < cb1; ++cb) {
          TR_T0(tw0);
          if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1u, abort_flag, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          TR_ADD(0, tw0);
          const uint32_t sa = smem_u32(base + (size_t)s * stage_bytes);
          const uint32_t fb = smem_u32(&full[s]);
          mbar_expect_tx(fb, stage_bytes);
          tma_load_3d(sa, &tmV, cb * kBK, bpt * kBM, pos, fb);
          tma_load_3d(sa + a_bytes, &tmU, cb * kBK, kt * p.BN, pos, fb);
          ++issued;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {
        // Aborted: the last min(S, issued) stage loads may still be landing in
        // shared memory.  Wait (bounded) for each one's completion before the
        // CTA can exit and its shared memory be reused.
        const long long n = issued < S ? issued : S;
        for (long long i = 0; i < n; ++i) {
          if (--s < 0) {
            s = S - 1;
            ph ^= 1u;
          }
          mbar_wait_drain(smem_u32(&full[s]), ph);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc =
          (1u << 4) | ((uint32_t)(p.BN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
      int s = 0;
      uint32_t ph = 0;
      uint32_t it = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < p.total_tiles && ok; t += gridDim.x, ++it) {
        const uint32_t acc = it & 1u;
        const uint32_t aph = (it >> 1) & 1u;
        TR_T0(tw1);
        if (!mbar_wait(smem_u32(&tempty[acc]), aph ^ 1u, abort_flag, p.status, kDevTimeoutMma))
          break;
        TR_ADD(1, tw1);
        tc_fence_after();
        const uint32_t dcol = tmem_base + acc * (uint32_t)p.BN;
        int pos_, bpt_, kt_, cb0 = 0, cb1 = p.n_cblk;
        if (p.n_split > 1) tile_of(p, t, pos_, bpt_, kt_, cb0, cb1);
        for (int cb = cb0; cb < cb1; ++cb) {
          TR_T0(tw2);
          if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          TR_ADD(2, tw2);
          tc_fence_after();
          const uint32_t sa = smem_u32(base + (size_t)s * stage_bytes);
          const uint64_t ad = smem_desc_sw128(sa);
          const uint64_t bd = smem_desc_sw128(sa + a_bytes);
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            // +32 bytes along K inside the swizzled 128-byte row = +2 in the
            // descriptor's 16-byte address units.
            umma_f16(dcol, ad + 2ull * k, bd + 2ull * k, idesc, (cb != cb0) || (k != 0));
          }
          umma_commit(smem_u32(&empty[s]));
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) umma_commit(smem_u32(&tfull[acc]));
      }
      // Every MMA this thread issued completes before the commit below arrives.
      // On the normal path the epilogue has already waited for all of them; on
      // the abort path this keeps tcgen05.dealloc from freeing TMEM under MMAs
      // still in flight.
      umma_commit(smem_u32(drain));
      mbar_wait_drain(smem_u32(drain), 0);
    }
  } else {
    // ---------------- Epilogue: warps 2..9 ----------------
    // epi_split: warpgroup eg (warps 2-5 / 6-9) drains columns
    // [eg BN/2, (eg + 1) BN/2) of every tile, so a tile's accumulator is free
    // after half the time one warpgroup would take.  Otherwise warpgroup eg
    // drains all of accumulator buffer eg, i.e. every other tile.
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int eg = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int tstep = p.epi_split ? 1 : 2;
    const int jlo = p.epi_split ? eg * (p.BN >> 1) : 0;
    const int jhi = p.epi_split ? jlo + (p.BN >> 1) : p.BN;
    uint32_t it = p.epi_split ? 0u : (uint32_t)eg;
    for (long long t = blockIdx.x + (p.epi_split ? 0ll : (long long)eg * gridDim.x);
         t < p.total_tiles; t += (long long)tstep * gridDim.x, it += tstep) {
      int pos, bpt, kt, cb0_, cb1_;
      tile_of(p, t, pos, bpt, kt, cb0_, cb1_);
      const uint32_t acc = it & 1u;
      const uint32_t aph = (it >> 1) & 1u;
      TR_T0(tw3);
      if (!mbar_wait(smem_u32(&tfull[acc]), aph, abort_flag, p.status, kDevTimeoutEpilogue)) break;
      if (q == 0 && lane == 0) TR_ADD(3 + eg, tw3);
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * (uint32_t)p.BN;
      if (p.tma_store) {
        // The slab holds up to kSlabCols columns; wider tiles go out in
        // kSlabCols-column pieces, each piece's stores read before the next fill.
        uint8_t* slab = out_stage + (eg * 4 + q) * slab_bytes;
        uint8_t* my_row = slab + lane * 128;
        for (int h0 = jlo; h0 < jhi; h0 += kSlabCols) {
          const int h1 = min(jhi, h0 + kSlabCols);
          TR_T0(tw5);
          if (lane == 0) bulk_wait_read_all();  // earlier stores have read the slab
          __syncwarp();
          if (q == 0 && lane == 0 && eg == 0) TR_ADD(5, tw5);
          for (int j = h0; j < h1; j += 32) {
            uint32_t r[32];
            tmem_ld32(taddr + j, r);
            uint8_t* chunk_row = my_row + ((j - h0) >> 6) * 4096;
            const int c_base = (j & 63) >> 3;  // first 16-byte chunk of these 32 columns
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_half2(r[8 * v + 0], r[8 * v + 1]);
              w.y = pack_half2(r[8 * v + 2], r[8 * v + 3]);
              w.z = pack_half2(r[8 * v + 4], r[8 * v + 5]);
              w.w = pack_half2(r[8 * v + 6], r[8 * v + 7]);
              *reinterpret_cast<uint4*>(chunk_row + (((c_base + v) ^ (lane & 7)) << 4)) = w;
            }
          }
          if (h1 == jhi) {
            tc_fence_before();
            mbar_arrive(smem_u32(&tempty[acc]));  // TMEM is free once read
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int jc = 0; jc < (h1 - h0) / 64; ++jc)
              tma_store_3d(&tmM, smem_u32(slab + jc * 4096), kt * p.BN + h0 + jc * 64,
                           bpt * kBM + q * 32, pos);
            bulk_commit();
          }
        }
        continue;
      }
      const long long bp = (long long)bpt * kBM + row;
      if (p.Mf) {
        // FP32 output: each split of the reduction writes its partial sums to
        // its own slice (the caller adds the slices in a fixed order).
        const long long split = cb0_ / p.kb_per_split;
        float* outf = p.Mf + split * 64ll * p.BP * p.K + ((long long)pos * p.BP + bp) * p.K +
                      (long long)kt * p.BN;
        for (int j = jlo; j < jhi; j += 16) {
          uint32_t r[16];
          tmem_ld16(taddr + j, r);
          if (bp < p.BP) {
#pragma unroll
            for (int q = 0; q < 16; q += 4)
              *reinterpret_cast<uint4*>(outf + j + q) = make_uint4(r[q], r[q + 1], r[q + 2], r[q + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(smem_u32(&tempty[acc]));
        continue;
      }
      __half* out = p.M + ((long long)pos * p.BP + bp) * p.K + (long long)kt * p.BN;
      int j = jlo;
      for (; j + 32 <= jhi; j += 32) {
        uint32_t r[32];
        tmem_ld32(taddr + j, r);
#ifndef NOVA_GEMM_NO_STORE
        if (bp < p.BP) store_row_f16<4>(out + j, r);
#else
        if (bp < 0) store_row_f16<4>(out + j, r);
#endif
      }
      if (j < jhi) {  // BN is a multiple of 16: at most one 16-column tail
        uint32_t r[16];
        tmem_ld16(taddr + j, r);
        if (bp < p.BP) store_row_f16<2>(out + j, r);
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[acc]));
    }
    if (p.tma_store && lane == 0) bulk_wait_all();  // stores complete before smem goes away
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) TR_ADD(6, tk0);
  pdl_trigger();  // after the whole CTA, epilogue stores included, is done
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 3-D FP16 map over [64][rows][C] (C fastest), box {64, box_rows, 1}, SWIZZLE_128B.
static bool encode_operand_map_raw(CUtensorMap* map, const void* ptr, int C, long long rows,
                                   int box_rows);
static bool encode_operand_map(CUtensorMap* map, const void* ptr, int C, long long rows,
                               int box_rows) {
  return cached_tensor_map(map, ptr, C, rows, box_rows, 2, [&](CUtensorMap* m) {
    return encode_operand_map_raw(m, ptr, C, rows, box_rows);
  });
}
static bool encode_operand_map_raw(CUtensorMap* map, const void* ptr, int C, long long rows,
                                   int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)rows, 64};
  cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)C * 2 * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)kBK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int pick_bn(int K) {
  for (int bn = kMaxBN; bn >= 16; bn -= 16)
    if (K % bn == 0) return bn;
  return 0;
}

}  // namespace tc

TensorMapEncodeFn tensor_map_encode_fn() { return tc::get_encode_fn(); }

bool tc_encode_operand_map(CUtensorMap* map, const void* ptr, int C, long long rows,
                           int box_rows) {
  return tc::encode_operand_map(map, ptr, C, rows, box_rows);
}

bool tc_gemm_supported(int C, int K) {
  return C > 0 && K > 0 && (C % 8) == 0 && (K % 16) == 0 && tc::pick_bn(K) > 0;
}

cudaError_t tc_gemm_plan(TcGemmPlan* plan, const __half* U, int K, int C, const char** why) {
  plan->valid = false;
  if (!tc_gemm_supported(C, K)) {
    *why = "shape not supported by the tensor-core GEMM";
    return cudaErrorInvalidValue;
  }
  if (reinterpret_cast<uintptr_t>(U) % 16) {
    *why = "U not 16-byte aligned";
    return cudaErrorInvalidValue;
  }
  plan->BN = tc::pick_bn(K);
  plan->K = K;
  plan->C = C;
  if (!tc::encode_operand_map(&plan->tmU, U, C, K, plan->BN)) {
    *why = "cuTensorMapEncodeTiled failed for U";
    return cudaErrorInvalidValue;
  }
  // Narrower tiles for launches too small to fill the GPU with wide ones.
  plan->has_half = plan->BN > 128 && (plan->BN / 2) % 16 == 0 &&
                   tc::encode_operand_map(&plan->tmU_half, U, C, K, plan->BN / 2);
  plan->has_pair = plan->BN % 64 == 0 &&
                   tc::encode_operand_map(&plan->tmU_pair, U, C, K, plan->BN / 2);
  plan->valid = true;
  return cudaSuccess;
}

// SM-pair tiles (nova_gemm_tc2.cu) are opt-in: NOVA_GEMM_PAIR=1 uses them
// wherever eligible.  Measured on the batch-256 and batch-128 conv4_x /
// conv5_x GEMMs they are no faster than one SM per tile (conv5_x batch 256:
// 38.9 us both ways; conv4_x batch 128: 24.6 against 20.5 us), so halving the
// per-SM operand traffic does not relieve what bounds these launches.
static bool use_pair_gemm(const TcGemmPlan& plan, long long BP, int num_sms) {
  static const int mode = [] {
    const char* e = std::getenv("NOVA_GEMM_PAIR");
    return e ? std::atoi(e) : 0;
  }();
  (void)num_sms;
  return mode == 1 && tc2_gemm_eligible(plan, BP);
}

// Both epilogue warpgroups on every tile (halves of BN columns), for short
// reductions (at most 4 blocks of 64 channels), where a tile's epilogue
// outlasts the next tile's MMAs and the MMA issuer waits for a drained
// accumulator: conv3_x batch 128 22.4 -> 21.2 us, conv4_x batch 256
// 30.8 -> 30.1 us; neutral at 512 channels.  BN/2 a multiple of 16 (TMEM
// loads), and of the 64-column slab when stored by TMA.
// NOVA_GEMM_EPI_SPLIT=0 turns it off, =2 forces it wherever the shape allows.
static int epi_split_ok(int BN, int tma_store, int n_cblk) {
  static const int env = [] {
    const char* e = std::getenv("NOVA_GEMM_EPI_SPLIT");
    return e ? std::atoi(e) : 1;
  }();
  if (!env || BN < 32 || (BN / 2) % 16) return 0;
  if (tma_store && (BN / 2) % 64) return 0;
  return env == 2 || n_cblk <= 4;
}

cudaError_t tc_gemm_run(const TcGemmPlan& plan, const __half* V, __half* M, long long BP,
                        int* dev_status, int num_sms, cudaStream_t s, const char** why) {
  if (!plan.valid) {
    *why = "tensor-core GEMM plan not built";
    return cudaErrorInvalidValue;
  }
  if (BP <= 0) return cudaSuccess;
  if (reinterpret_cast<uintptr_t>(V) % 16 || reinterpret_cast<uintptr_t>(M) % 16) {
    *why = "V/M workspace not 16-byte aligned";
    return cudaErrorInvalidValue;
  }
  if (use_pair_gemm(plan, BP, num_sms))
    return tc2_gemm_run(plan, V, M, BP, dev_status, num_sms, s, why);
  CUtensorMap tmV;
  if (!tc::encode_operand_map(&tmV, V, plan.C, BP, tc::kBM)) {
    *why = "cuTensorMapEncodeTiled failed for V";
    return cudaErrorInvalidValue;
  }
  // Tile width: BN, or BN/2 when BN-wide tiles would leave more than half of
  // the SMs idle (batch-1 shapes), so the launch spreads over more CTAs.
  int BN = plan.BN;
  const CUtensorMap* tmU = &plan.tmU;
  {
    const long long n_bp = (BP + tc::kBM - 1) / tc::kBM;
    if (plan.has_half && 64ll * n_bp * (plan.K / plan.BN) * 2 <= num_sms) {
      BN = plan.BN / 2;
      tmU = &plan.tmU_half;
    }
  }
  tc::Params p;
  CUtensorMap tmM;
  p.tma_store = (BN % 64) == 0 &&
                tc::encode_operand_map(&tmM, M, plan.K, BP, 32);
  p.M = M;
  p.Mf = nullptr;
  p.BP = BP;
  p.C = plan.C;
  p.K = plan.K;
  p.BN = BN;
  p.n_bp_tiles = (int)((BP + tc::kBM - 1) / tc::kBM);
  p.n_k_tiles = plan.K / BN;
  p.n_cblk = (plan.C + tc::kBK - 1) / tc::kBK;
  p.n_split = 1;
  p.kb_per_split = p.n_cblk;
  p.total_tiles = 64ll * p.n_bp_tiles * p.n_k_tiles;
  if (p.total_tiles >= (1ll << 31)) {
    *why = "tensor-core GEMM: too many tiles for one launch";
    return cudaErrorInvalidValue;
  }
  p.epi_split = epi_split_ok(BN, p.tma_store, (plan.C + tc::kBK - 1) / tc::kBK);
  p.status = dev_status;
  const int stage_bytes = tc::kBM * tc::kBK * 2 + BN * tc::kBK * 2;
  const int out_bytes = p.tma_store ? 8 * 32 * std::min(BN, tc::kSlabCols) * 2 : 0;
  const int overhead = 1024 + 256 + out_bytes;
  p.stages = (tc::kSmemLimit - overhead) / stage_bytes;
  if (p.stages > tc::kMaxStages) p.stages = tc::kMaxStages;
#ifdef NOVA_GEMM_STAGES
  if (p.stages > NOVA_GEMM_STAGES) p.stages = NOVA_GEMM_STAGES;
#endif
  const int smem = overhead + p.stages * stage_bytes;
  // The shared-memory opt-in is a per-device function attribute.
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tc::gemm_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tc::kSmemLimit);
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed";
      return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const long long slots = (long long)num_sms * tc::kCtasPerSm;
  long long grid = p.total_tiles < slots ? p.total_tiles : slots;
  cudaError_t e = launch_pdl(kPdlGemm, tc::gemm_tc_kernel, dim3((unsigned)grid), dim3(tc::kThreads), smem, s,
                             tmV, *tmU, tmM, p);
  if (e != cudaSuccess) *why = "tensor-core GEMM launch failed";
  return e;
}

// Weight-gradient GEMM (nova_wgrad.cu): Ug[pos][K][C] += sum over bp of
// A[pos][K][bp] * Bop[pos][C][bp], both operands with the reduction (bp)
// contiguous at a row pitch of `pitch` halves, FP32 output by atomic adds.
// The reduction is split over enough CTAs to fill the GPU; Ug must be zeroed.
static bool encode_pitched_map(CUtensorMap* map, const void* ptr, long long inner,
                               long long pitch, long long rows, int box_rows) {
  tc::EncodeTiledFn fn = tc::get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)rows, 64};
  cuuint64_t strides[2] = {(cuuint64_t)pitch * 2, (cuuint64_t)pitch * 2 * (cuuint64_t)rows};
  cuuint32_t box[3] = {(cuuint32_t)tc::kBK, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Splits of the reduction: only when the output tiles alone would leave most
// SMs idle; enough for about two tiles per SM, at least two 64-tile blocks of
// reduction per split, at most kWgradMaxSplits.
int tc_gemm_wgrad_splits(int K, int C, long long BP, int num_sms) {
  const int BN = tc::pick_bn(C);
  if (BN == 0) return 1;
  const long long base = 64ll * ((K + tc::kBM - 1) / tc::kBM) * (C / BN);
  if (2 * base >= num_sms) return 1;
  const long long n_cblk = (BP + tc::kBK - 1) / tc::kBK;
  long long n = std::min<long long>(n_cblk / 2, (2ll * num_sms + base - 1) / base);
  n = std::min<long long>(n, kWgradMaxSplits);
  if (n < 1) n = 1;
  const long long per = (n_cblk + n - 1) / n;
  return (int)((n_cblk + per - 1) / per);
}

cudaError_t tc_gemm_wgrad_run(const __half* A, const __half* Bop, float* Ug, int K, int C,
                              long long BP, long long pitch, int* dev_status, int num_sms,
                              cudaStream_t s, const char** why) {
  const int BN = tc::pick_bn(C);
  if (BN == 0 || K <= 0 || BP <= 0 || pitch % 8 || pitch < BP) {
    *why = "weight-gradient GEMM: unsupported shape";
    return cudaErrorInvalidValue;
  }
  if (reinterpret_cast<uintptr_t>(A) % 16 || reinterpret_cast<uintptr_t>(Bop) % 16) {
    *why = "weight-gradient GEMM: operands not 16-byte aligned";
    return cudaErrorInvalidValue;
  }
  CUtensorMap tmA, tmB, tmNone;
  std::memset(&tmNone, 0, sizeof(tmNone));
  if (!encode_pitched_map(&tmA, A, BP, pitch, K, tc::kBM) ||
      !encode_pitched_map(&tmB, Bop, BP, pitch, C, BN)) {
    *why = "cuTensorMapEncodeTiled failed for the weight-gradient operands";
    return cudaErrorInvalidValue;
  }
  tc::Params p;
  p.M = nullptr;
  p.Mf = Ug;
  p.BP = K;  // rows of the output
  p.C = (int)std::min<long long>(BP, 1ll << 30);
  p.K = C;   // columns of the output
  p.BN = BN;
  p.n_bp_tiles = (K + tc::kBM - 1) / tc::kBM;
  p.n_k_tiles = C / BN;
  p.n_cblk = (int)((BP + tc::kBK - 1) / tc::kBK);
  const long long base = 64ll * p.n_bp_tiles * p.n_k_tiles;
  p.n_split = tc_gemm_wgrad_splits(K, C, BP, num_sms);
  p.kb_per_split = (p.n_cblk + p.n_split - 1) / p.n_split;
  p.total_tiles = base * p.n_split;
  if (p.total_tiles >= (1ll << 31)) {
    *why = "weight-gradient GEMM: too many tiles for one launch";
    return cudaErrorInvalidValue;
  }
  p.tma_store = 0;
  p.epi_split = epi_split_ok(BN, 0, p.n_cblk);
  p.status = dev_status;
  const int stage_bytes = tc::kBM * tc::kBK * 2 + BN * tc::kBK * 2;
  const int overhead = 1024 + 256;
  p.stages = std::min(tc::kMaxStages, (tc::kSmemLimit - overhead) / stage_bytes);
  const int smem = overhead + p.stages * stage_bytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tc::gemm_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tc::kSmemLimit);
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed";
      return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const long long grid = std::min<long long>(p.total_tiles, (long long)num_sms * tc::kCtasPerSm);
  cudaError_t e = launch_pdl(kPdlGemm, tc::gemm_tc_kernel, dim3((unsigned)grid),
                             dim3(tc::kThreads), smem, s, tmA, tmB, tmNone, p);
  if (e != cudaSuccess) *why = "weight-gradient GEMM launch failed";
  return e;
}

#ifdef NOVA_GEMM_TRACE
extern "C" __attribute__((visibility("default"))) int nova_debug_gemm_trace(unsigned long long* out, int reset) {
  if (reset) {
    static unsigned long long z[1024][8];
    return (int)cudaMemcpyToSymbol(tc::g_gemm_trace, z, sizeof(z));
  }
  return (int)cudaMemcpyFromSymbol(out, tc::g_gemm_trace, sizeof(unsigned long long) * 1024 * 8);
}
#endif
}  // namespace nova
