// The 64 per-frequency Winograd GEMMs on SM pairs (tcgen05 cta_group::2).
//
//   M[pos][bp][k] = sum_c V[pos][bp][c] * U[pos][k][c]
//
// Same contract as gemm_tc_kernel (nova_gemm_tc.cu; the reference's rocBLAS
// gemm_strided_batched_ex at Jayluci4/nova-wino-amd csrc/nova_winograd.hip:
// 534-548), for the launches whose operands stream from L2 faster than one SM
// can consume them: at 256 and 512 channels the 1-SM kernel moves 48 KB of
// operands per 64-channel k-step for a 128 x 256 tile, and its tensor pipe
// waits on those loads.
//
// Design:
// * Clusters of 2 CTAs on an SM pair.  A pair tile is 256 bp rows x BN output
//   channels.  Each CTA lands its own 128 bp rows of V and its own BN/2 rows of
//   U per k-step (TMA tile loads into its own shared memory, no multicast);
//   the leader CTA (rank 0) issues one tcgen05.mma.cta_group::2 (M = 256,
//   N = BN) that reads both CTAs' operands, and each CTA's TMEM receives its
//   128 rows x BN columns.  Operand traffic per CTA and k-step: 16 KB of V +
//   BN/2 x 128 B of U (32 KB at BN = 256, against 48 KB on one SM).
// * Both CTAs' TMA loads complete on the leader's "full" barrier (the
//   .cta_group::2 form of the tile load may signal the peer CTA's barrier).
//   The leader's commits arrive on both CTAs' "empty" / "tfull" barriers
//   (tcgen05.commit multicast to the pair); both CTAs' epilogue warps arrive on
//   the leader's "tempty" barrier.
// * Warp roles per CTA as in the 1-SM kernel: warp 0 TMA producer, warp 1 TMEM
//   allocation (both CTAs, collectively) and, in the leader, the MMA issuer;
//   warps 2-9 two epilogue warpgroups over a double-buffered accumulator,
//   writing M through swizzled shared-memory slabs and TMA tile stores.
// * Every mbarrier wait is bounded; on expiry the kernel records a status code,
//   stops issuing work and falls through to the common exit, where the leader
//   first drains the MMAs it issued and the pair meets at a cluster barrier
//   before TMEM is released.
#include <algorithm>
#include <cstdlib>

#include "nova_internal.h"
#include "nova_tc_ptx.cuh"

namespace nova {
namespace tc2 {

using namespace nova::tc;

constexpr int kBM = 128;        // bp rows per CTA (256 per pair)
constexpr int kBK = 64;         // input channels per stage
constexpr int kUmmaK = 16;
constexpr int kMaxStages = 8;
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr int kSlabCols = 64;
constexpr int kSmemLimit = 227 * 1024;

#ifdef NOVA_GEMM_TRACE
__device__ unsigned long long g_gemm2_trace[1024][8];
#define TR_T0(v) const long long v = clock64()
#define TR_ADD(slot, t0) atomicAdd(&g_gemm2_trace[blockIdx.x & 1023][slot], (unsigned long long)(clock64() - (t0)))
#else
#define TR_T0(v)
#define TR_ADD(slot, t0)
#endif

struct Params {
  long long BP;
  int C, K, BN;
  int n_bp_tiles;   // pair tiles along bp (256 rows each)
  int n_k_tiles;
  int n_cblk;
  long long total_tiles;
  int stages;
  int epi_split;  // 1: both epilogue warpgroups drain every tile, one half of its columns each
  int* status;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t n_clusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Tile load whose completion is signalled on a barrier that may live in the
// peer CTA of the pair (cluster address); destination in this CTA.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int c0,
                                                 int c1, int c2, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this shared-memory offset in every CTA of `mask`
// once all MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmU,
                    const __grid_constant__ CUtensorMap tmM, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int S = p.stages;
  const int half_n = p.BN / 2;
  const uint32_t a_bytes = kBM * kBK * 2;
  const uint32_t b_bytes = (uint32_t)half_n * kBK * 2;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  uint8_t* out_stage = base + (size_t)S * stage_bytes;
  const uint32_t slab_bytes = 32u * (uint32_t)min(p.BN, kSlabCols) * 2u;
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + 8 * (size_t)slab_bytes);
  uint64_t* full = bars;                 // leader: operands of both CTAs landed
  uint64_t* empty = bars + kMaxStages;   // both: stage free (leader's MMAs read it)
  uint64_t* tfull = bars + 2 * kMaxStages;
  uint64_t* tempty = tfull + 2;          // leader: both CTAs' epilogues drained
  uint64_t* drain = tempty + 2;          // leader: every MMA it issued completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      // 4 epilogue warps x 2 CTAs, or 8 x 2 when both warpgroups drain every tile
      mbar_init(smem_u32(&tempty[a]), p.epi_split ? 16 : 8);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    // One warp of each CTA of the pair allocates collectively.
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // 32-bit tile arithmetic (the host keeps total_tiles below 2^31).
  const uint32_t tiles_per_pos = (uint32_t)p.n_bp_tiles * (uint32_t)p.n_k_tiles;
  const long long t0 = cluster_id_x(), dt = n_clusters_x();
  pdl_wait();
  TR_T0(tk0);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs) ----------------
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      long long issued = 0;
      for (long long t = t0; t < p.total_tiles && ok; t += dt) {
        const uint32_t tu = (uint32_t)t;
        const int pos = (int)(tu / tiles_per_pos);
        const uint32_t rem = tu - (uint32_t)pos * tiles_per_pos;
        const int bpt = (int)(rem / (uint32_t)p.n_k_tiles);
        const int kt = (int)(rem - (uint32_t)bpt * (uint32_t)p.n_k_tiles);
        const int bp_row = bpt * 2 * kBM + (int)rank * kBM;
        const int k_row = kt * p.BN + (int)rank * half_n;
        for (int cb = 0; cb < p.n_cblk; ++cb) {
          TR_T0(tw0);
          if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1u, abort_flag, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          TR_ADD(0, tw0);
          const uint32_t sa = smem_u32(base + (size_t)s * stage_bytes);
          const uint32_t fb = map_to_rank(smem_u32(&full[s]), 0);
          if (leader) mbar_expect_tx(smem_u32(&full[s]), 2u * stage_bytes);
          tma_load_3d_pair(sa, &tmV, cb * kBK, bp_row, pos, fb);
          tma_load_3d_pair(sa + a_bytes, &tmU, cb * kBK, k_row, pos, fb);
          ++issued;
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // Aborted: let the loads already issued into this CTA land before its
        // shared memory can be released (the peer's loads complete on the
        // leader's barriers too, so only the leader can wait for them).
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
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader only) ----------------
      const uint32_t idesc =
          (1u << 4) | ((uint32_t)(p.BN >> 3) << 17) | ((uint32_t)((2 * kBM) >> 4) << 24);
      int s = 0;
      uint32_t ph = 0;
      uint32_t it = 0;
      bool ok = true;
      for (long long t = t0; t < p.total_tiles && ok; t += dt, ++it) {
        const uint32_t acc = it & 1u;
        const uint32_t aph = (it >> 1) & 1u;
        TR_T0(tw1);
        if (!mbar_wait(smem_u32(&tempty[acc]), aph ^ 1u, abort_flag, p.status, kDevTimeoutMma))
          break;
        TR_ADD(1, tw1);
        tc_fence_after();
        const uint32_t dcol = tmem_base + acc * (uint32_t)p.BN;
        for (int cb = 0; cb < p.n_cblk; ++cb) {
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
          for (int k = 0; k < kBK / kUmmaK; ++k)
            umma_f16_pair(dcol, ad + 2ull * k, bd + 2ull * k, idesc, (cb | k) != 0);
          umma_commit_pair(smem_u32(&empty[s]), 0x3);
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) umma_commit_pair(smem_u32(&tfull[acc]), 0x3);
      }
      umma_commit_pair(smem_u32(drain), 0x1);
      mbar_wait_drain(smem_u32(drain), 0);
    }
  } else {
    // ---------------- Epilogue: warps 2..9 of both CTAs ----------------
    const int q = warp & 3;
    const int eg = (warp - 2) >> 2;
    const uint32_t tempty_leader[2] = {map_to_rank(smem_u32(&tempty[0]), 0),
                                       map_to_rank(smem_u32(&tempty[1]), 0)};
    const int tstep = p.epi_split ? 1 : 2;
    const int jlo = p.epi_split ? eg * (p.BN >> 1) : 0;
    const int jhi = p.epi_split ? jlo + (p.BN >> 1) : p.BN;
    uint32_t it = p.epi_split ? 0u : (uint32_t)eg;
    for (long long t = t0 + (p.epi_split ? 0ll : (long long)eg * dt); t < p.total_tiles;
         t += (long long)tstep * dt, it += tstep) {
      const uint32_t tu = (uint32_t)t;
      const int pos = (int)(tu / tiles_per_pos);
      const uint32_t rem = tu - (uint32_t)pos * tiles_per_pos;
      const int bpt = (int)(rem / (uint32_t)p.n_k_tiles);
      const int kt = (int)(rem - (uint32_t)bpt * (uint32_t)p.n_k_tiles);
      const uint32_t acc = it & 1u;
      const uint32_t aph = (it >> 1) & 1u;
      TR_T0(tw3);
      if (!mbar_wait(smem_u32(&tfull[acc]), aph, abort_flag, p.status, kDevTimeoutEpilogue)) break;
      if (q == 0 && lane == 0) TR_ADD(3 + eg, tw3);
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + acc * (uint32_t)p.BN;
      uint8_t* slab = out_stage + (eg * 4 + q) * slab_bytes;
      uint8_t* my_row = slab + lane * 128;
      const int row0 = bpt * 2 * kBM + (int)rank * kBM + q * 32;
      for (int h0 = jlo; h0 < jhi; h0 += kSlabCols) {
        TR_T0(tw5);
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        if (q == 0 && lane == 0 && eg == 0) TR_ADD(5, tw5);
        for (int j = h0; j < h0 + kSlabCols; j += 32) {
          uint32_t r[32];
          tmem_ld32(taddr + j, r);
          const int c_base = (j & 63) >> 3;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_half2(r[8 * v + 0], r[8 * v + 1]);
            w.y = pack_half2(r[8 * v + 2], r[8 * v + 3]);
            w.z = pack_half2(r[8 * v + 4], r[8 * v + 5]);
            w.w = pack_half2(r[8 * v + 6], r[8 * v + 7]);
            *reinterpret_cast<uint4*>(my_row + (((c_base + v) ^ (lane & 7)) << 4)) = w;
          }
        }
        if (h0 + kSlabCols >= jhi) {
          // This warp's TMEM quarter of the accumulator has been read.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmM, smem_u32(slab), kt * p.BN + h0, row0, pos);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) TR_ADD(6, tk0);
  cluster_sync();  // the leader's MMAs (reading both CTAs) have drained
  pdl_trigger();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc2

#ifdef NOVA_GEMM_TRACE
extern "C" __attribute__((visibility("default"))) int nova_debug_gemm2_trace(unsigned long long* out, int reset) {
  if (reset) {
    static unsigned long long z[1024][8];
    return (int)cudaMemcpyToSymbol(tc2::g_gemm2_trace, z, sizeof(z));
  }
  return (int)cudaMemcpyFromSymbol(out, tc2::g_gemm2_trace, sizeof(unsigned long long) * 1024 * 8);
}
#endif

bool tc2_gemm_eligible(const TcGemmPlan& plan, long long BP) {
  // TMA-store epilogue needs BN % 64 == 0; U halves of BN/2 rows.
  return plan.valid && plan.has_pair && plan.BN % 64 == 0 && BP >= 2 * tc2::kBM;
}

cudaError_t tc2_gemm_run(const TcGemmPlan& plan, const __half* V, __half* M, long long BP,
                         int* dev_status, int num_sms, cudaStream_t s, const char** why) {
  CUtensorMap tmV, tmM;
  if (!tc_encode_operand_map(&tmV, V, plan.C, BP, tc2::kBM) ||
      !tc_encode_operand_map(&tmM, M, plan.K, BP, 32)) {
    *why = "cuTensorMapEncodeTiled failed for V / M";
    return cudaErrorInvalidValue;
  }
  tc2::Params p;
  p.BP = BP;
  p.C = plan.C;
  p.K = plan.K;
  p.BN = plan.BN;
  p.n_bp_tiles = (int)((BP + 2 * tc2::kBM - 1) / (2 * tc2::kBM));
  p.n_k_tiles = plan.K / plan.BN;
  p.n_cblk = (plan.C + tc2::kBK - 1) / tc2::kBK;
  p.total_tiles = 64ll * p.n_bp_tiles * p.n_k_tiles;
  if (p.total_tiles >= (1ll << 31)) {
    *why = "SM-pair GEMM: too many tiles for one launch";
    return cudaErrorInvalidValue;
  }
  {
    // The 1-SM kernel's rule: short reductions only; NOVA_GEMM_EPI_SPLIT=0
    // turns it off, =2 forces it wherever the shape allows.
    const char* e = std::getenv("NOVA_GEMM_EPI_SPLIT");
    const int env = e ? std::atoi(e) : 1;
    p.epi_split = env && (plan.BN / 2) % 64 == 0 && (env == 2 || p.n_cblk <= 4);
  }
  p.status = dev_status;
  const int stage_bytes = tc2::kBM * tc2::kBK * 2 + (plan.BN / 2) * tc2::kBK * 2;
  const int out_bytes = 8 * 32 * std::min(plan.BN, tc2::kSlabCols) * 2;
  const int overhead = 1024 + 256 + out_bytes;
  p.stages = std::min(tc2::kMaxStages, (tc2::kSmemLimit - overhead) / stage_bytes);
  const int smem = overhead + p.stages * stage_bytes;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tc2::gemm_tc2_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         tc2::kSmemLimit);
    if (e != cudaSuccess) {
      *why = "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed (pair GEMM)";
      return e;
    }
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  // Persistent grid: as many pairs as can be resident at once (an SM whose
  // GPC has no free partner cannot host a pair, so this can be below
  // num_sms / 2); later clusters would otherwise run as a second wave.
  static int resident[64] = {};
  if (dev >= 0 && dev < 64 && resident[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms / 2));
    cfg.blockDim = dim3(tc2::kThreads);
    cfg.dynamicSmemBytes = tc2::kSmemLimit;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc2::gemm_tc2_kernel, &cfg) != cudaSuccess || n <= 0)
      n = num_sms / 2;
    resident[dev] = n;
  }
  const int max_pairs = (dev >= 0 && dev < 64) ? resident[dev] : num_sms / 2;
  const long long pairs = std::min<long long>(p.total_tiles, max_pairs);
  cudaError_t e = launch_pdl(kPdlGemm, tc2::gemm_tc2_kernel, dim3((unsigned)(2 * pairs)),
                             dim3(tc2::kThreads), smem, s, tmV, plan.tmU_pair, tmM, p);
  if (e != cudaSuccess) *why = "pair GEMM launch failed";
  return e;
}

}  // namespace nova
