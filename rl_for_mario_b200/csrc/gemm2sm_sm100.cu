// Residual GEMM y += x W^T (in place, fp32 accumulation, one rounding of the
// sum) on CTA pairs, sm_100a: the DT block's o_proj + residual
// (model/model_decision_transformer.py:247-248, :300) and down_proj + residual
// (:271, :303).
//
// A cluster of two CTAs computes 256 x 256 output tiles with tcgen05.mma
// .cta_group::2 (M = 256): CTA r of the pair stages rows 128 r .. 128 r + 127
// of the tile's x block and rows 128 r .. 128 r + 127 of its W block (half of
// the tile's N) for every 64-wide K chunk, so each SM brings in 32 KB per chunk
// instead of the 48 KB a 128 x 256 tile of one CTA needs for the same FLOPs;
// both halves' copies complete on the first CTA's barrier, whose one thread
// issues the MMAs for the pair.  Each CTA's TMEM holds its 128 rows of the
// accumulator (two 256-column buffers, so a tile's epilogue overlaps the next
// tile's MMAs).  No copy is multicast: each CTA loads only what it stages.
//
// Warps (per CTA): 0 TMA producer, 1 TMEM owner (both CTAs) and MMA issuer
// (first CTA only), 2-17 epilogue (lane quarter = warp % 4, 64-column quarter
// = (warp - 2) / 4): each warp's 32 x 64 residual slice is brought into its own
// 4 KB of shared memory by TMA (requested before the accumulator wait), the
// sum is rounded once into the same slice and stored back by TMA: whole rows
// per copy instead of one scattered 16-byte access per thread and row.
//
// Every mbarrier wait is bounded (dt_common.cuh); the only unbounded waits are
// the two cluster barriers at the start and the end, which every thread of
// both CTAs reaches whatever happened in between.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int k2Threads = 576;
constexpr int k2EpiWarps = 16;
constexpr int k2Stages = 5;
constexpr int k2A = 128 * 128;  // 128 rows x 64 K values, 16-bit
constexpr int k2Stage = 2 * k2A;  // A half + B half
struct G2Shape {
  static constexpr int OFF_EPI = k2Stages * k2Stage;          // [16 warps][32 rows][128 B]
  static constexpr int OFF_BAR = OFF_EPI + k2EpiWarps * 4096;
  // full[S] (first CTA's counts), empty[S], acc_full[2], acc_empty[2] (first CTA's counts), drain,
  // res_full[16]
  static constexpr int NBAR = 2 * k2Stages + 5 + k2EpiWarps;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs (the warp reconverged first; the non-aligned form
// does not require it, the __syncwarp keeps the warp's lanes together anyway).
__device__ __forceinline__ void cluster_sync() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Shared::cluster address of this CTA's shared variable at `saddr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
// Bounded wait with cluster-scope acquire (arrivals that come from the other CTA).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, int* status) {
  const uint32_t a = smem_u32(bar);
  auto try_once = [&](uint32_t hint) -> bool {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity), "r"(hint)
        : "memory");
    return ok != 0;
  };
  if (try_once(0u)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (try_once(20000u)) return true;
    if (abort && *abort) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (abort) *abort = 1;
      if (status) atomicExch(status, (int)kDevWaitTimeout);
      return false;
    }
  }
}
// 2-D tensor load for a CTA pair: lands in this CTA's shared memory, completes
// on the mbarrier at shared::cluster address `cbar` (the first CTA's).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t cbar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cbar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_pair_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at shared::cluster address `cbar` once every pair MMA
// issued so far by this thread completes.
__device__ __forceinline__ void umma_pair_commit(uint32_t cbar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cbar)
               : "memory");
}

template <bool BF16>
__global__ void __launch_bounds__(k2Threads, 1)
    gemm_residual_pair_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                              const __grid_constant__ CUtensorMap tmY, int M, int N, int K, int* status) {
  using SH = G2Shape;
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* empty = full + k2Stages;
  uint64_t* acc_full = empty + k2Stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* res_full = drain + 1;  // [epilogue warp]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_full + k2EpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;
  const int nk = (K + 63) / 64;
  const int nmb = (M + 255) / 256;
  const int nt = N / 256;
  // This pair's tiles: its row blocks (pair, pair + npairs, ...), each with all of
  // its column tiles back to back, so a 256-row block of x is read from HBM once
  // and re-read by the block's other column tiles from L2.
  const int my_items = (nmb > pair ? (nmb - pair + npairs - 1) / npairs : 0) * nt;

  if (tid == 0) {
    for (int s = 0; s < k2Stages; ++s) {
      mbar_init(&full[s], 1);   // the first CTA's producer arms it with both CTAs' bytes
      mbar_init(&empty[s], 1);  // the pair's MMA commit
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], 2 * k2EpiWarps);  // the epilogue warps of both CTAs
    }
    mbar_init(drain, 1);
    for (int j = 0; j < k2EpiWarps; ++j) mbar_init(&res_full[j], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmW);
      int cnt = 0;
      bool ok = true;
      for (int j = 0; j < my_items && ok; ++j) {
        const int mb = pair + (j / nt) * npairs, ct = j % nt;
        for (int kc = 0; kc < nk; ++kc, ++cnt) {
          const int s = cnt % k2Stages;
          if (!(ok = mbar_wait_cluster(&empty[s], ((cnt / k2Stages) & 1) ^ 1, abort_flag, status))) break;
          uint8_t* st = smem + s * k2Stage;
          const uint32_t cbar = mapa_rank(smem_u32(&full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(2 * k2Stage));
          tma_load_2d_pair(st, &tmX, cbar, kc * 64, mb * 256 + (int)rank * 128);
          tma_load_2d_pair(st + k2A, &tmW, cbar, kc * 64, ct * 256 + (int)rank * 128);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (first CTA)
    if (rank == 0 && lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BF16, 256, 256, 0, 0);
      int cnt = 0, tc = 0;
      bool ok = true;
      for (int j = 0; j < my_items && ok; ++j, ++tc) {
        const int buf = tc & 1;
        if (!(ok = mbar_wait_cluster(&acc_empty[buf], ((tc >> 1) & 1) ^ 1, abort_flag, status))) break;
        tc_fence_after();
        for (int kc = 0; kc < nk; ++kc, ++cnt) {
          const int s = cnt % k2Stages;
          if (!(ok = mbar_wait_cluster(&full[s], (cnt / k2Stages) & 1, abort_flag, status))) break;
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * k2Stage);
          const uint64_t ad = umma_smem_desc(a, 16, 1024, kSw128);
          const uint64_t bd = umma_smem_desc(a + k2A, 16, 1024, kSw128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 32 bytes per K step inside the 128-byte rows
            umma_pair_ss(tmem + (uint32_t)(buf * 256), ad + 2 * kk, bd + 2 * kk, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
          // The stage is free in both CTAs once these MMAs have read it.
          umma_pair_commit(mapa_rank(smem_u32(&empty[s]), 0));
          umma_pair_commit(mapa_rank(smem_u32(&empty[s]), 1));
        }
        if (!ok) break;
        umma_pair_commit(mapa_rank(smem_u32(&acc_full[buf]), 0));
        umma_pair_commit(mapa_rank(smem_u32(&acc_full[buf]), 1));
      }
      umma_pair_commit(mapa_rank(smem_u32(drain), 0));
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-17, both CTAs)
    const int wq = warp & 3;
    const int ew = warp - 2;
    const int cq = ew >> 2;  // 64-column quarter of the tile
    const uint32_t t_row = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(cq * 64);
    const uint32_t empty_c = mapa_rank(smem_u32(&acc_empty[0]), 0);  // acc_empty[j] at + 8 j
    uint8_t* slice = smem + SH::OFF_EPI + ew * 4096;  // 32 rows x 128 B, 128-byte swizzle
    if (lane == 0) prefetch_tmap(&tmY);
    int tc = 0;
    bool ok = true;
    for (int j = 0; j < my_items && ok; ++j, ++tc) {
      const int buf = tc & 1;
      const int mb = pair + (j / nt) * npairs, ct = j % nt;
      const int r0 = mb * 256 + (int)rank * 128 + wq * 32, c0 = ct * 256 + cq * 64;
      if (lane == 0) {
        bulk_wait_read<0>();  // the previous tile's store has read this slice
        mbar_arrive_expect_tx(&res_full[ew], 4096u);
        tma_load_2d(slice, &tmY, &res_full[ew], c0, r0);
      }
      __syncwarp();
      if (!(ok = __all_sync(0xffffffffu, mbar_wait_cluster(&acc_full[buf], (tc >> 1) & 1, abort_flag, status))))
        break;
      tc_fence_after();
      float v[64];
      tmem_ld32(t_row + (uint32_t)(buf * 256), *reinterpret_cast<float(*)[32]>(&v[0]));
      tmem_ld32(t_row + (uint32_t)(buf * 256 + 32), *reinterpret_cast<float(*)[32]>(&v[32]));
      // Every TMEM read of this buffer is done: release it to the pair's MMA.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty_c + 8u * (uint32_t)buf);
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&res_full[ew], tc & 1, abort_flag, status)))) break;
      // Row `lane` of the slice: 8 pieces of 16 bytes at swizzled positions.
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint4* pc = reinterpret_cast<uint4*>(slice + lane * 128 + ((q ^ (lane & 7)) << 4));
        const uint4 rq = *pc;
        const uint32_t w4[4] = {rq.x, rq.y, rq.z, rq.w};
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = E::to_f2(w4[e]);
          o4[e] = E::from_f2(v[q * 8 + 2 * e] + f.x, v[q * 8 + 2 * e + 1] + f.y);
        }
        *pc = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmY, slice, c0, r0);  // rows past M are clipped by the copy
        bulk_commit();
      }
    }
    if (lane == 0) {
      bulk_wait<0>();  // stores complete before the CTA exits
      // A residual load issued before an abort lands before the CTA exits.
      if (!ok) mbar_wait(&res_full[ew], tc & 1, nullptr, nullptr);
    }
  }
  // Both CTAs meet here before TMEM goes back: no remote arrival or MMA of the
  // pair is still pending on either CTA's memory.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace

cudaError_t launch_gemm_residual_pair_sm100(const CUtensorMap& x, const CUtensorMap& w, const CUtensorMap& y, int M,
                                            int N, int K, bool bf16, int num_sms, int* status, cudaStream_t st) {
  const long long blocks = (M + 255) / 256;  // 256-row blocks, dealt to the pairs whole
  long long pairs = num_sms / 2;
  if (pairs > blocks) pairs = blocks;
  if (pairs < 1) pairs = 1;
  const void* fn = bf16 ? reinterpret_cast<const void*>(gemm_residual_pair_kernel<true>)
                        : reinterpret_cast<const void*>(gemm_residual_pair_kernel<false>);
  cudaError_t e = smem_limit_once(fn, G2Shape::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  cfg.blockDim = dim3(k2Threads, 1, 1);
  cfg.dynamicSmemBytes = G2Shape::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (bf16)
    e = cudaLaunchKernelEx(&cfg, gemm_residual_pair_kernel<true>, x, w, y, M, N, K, status);
  else
    e = cudaLaunchKernelEx(&cfg, gemm_residual_pair_kernel<false>, x, w, y, M, N, K, status);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace dtk
