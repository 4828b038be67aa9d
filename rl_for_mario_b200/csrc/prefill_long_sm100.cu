// Long-context fused prefill, sm_100a, head_dim 64.
//
// Replaces the prefill branch of DecisionTransformerAttention.forward
// (model/model_decision_transformer.py:198-224: SDPA under the causal and
// left-padding masks, GQA via repeat_kv :121-130) for sequences longer than
// the 192-token context that the resident-K/V kernel covers.
//
// Work item = two neighbouring 128-row query tiles ("slots") of one
// (sample, KV head) unit.  A tile packs PT = 128 / R positions x R query
// heads of one KV group, so every key block is loaded once for the whole
// group and once for both slots.  Key blocks of 64 stream through a TMA
// ring; per block and slot:
//   S  = Q K^T          tcgen05.mma, fp32 in TMEM (64 columns, three
//                       buffers per slot: the P V of a block is issued two
//                       blocks after its S, so S stays two blocks ahead of
//                       the softmax instead of waiting on the previous P)
//   P  = exp2(S c2 - m) softmax warpgroup of the slot, one thread per row;
//                       P is written back over its S columns as packed
//                       16-bit pairs
//   O += P V            tcgen05.mma with A = P from TMEM, fp32 in TMEM
// The softmax never waits for a P V: the running maximum m only moves when a
// block's maximum exceeds it by more than 2^8 (P <= 256 otherwise, exact in
// 16 bits); then (rarely) it waits for the slot's previous P V and scales the
// O row in TMEM and the row sum by the exact power of two.  A slot's
// epilogue (O / l -> HBM) runs after the next item's first softmax block; the
// next item's first P V waits for it (one O buffer per slot).
//
// Warp roles (384 threads): warp 0 TMA producer, warp 1 TMEM owner and MMA
// issuer of slot 0, warp 2 MMA issuer of slot 1, warp 3 RoPE (rotates each
// Q tile and K block in shared memory when the inputs are not yet rotated);
// warps 4-7 softmax of slot 0, warps 8-11 of slot 1.
// setmaxnreg moves registers from the first warpgroup (152) to the softmax
// warpgroups (176): 128 x 152 + 256 x 176 = 384 x 168, the launch allocation.
//
// Mask semantics are those of the other prefill kernels: a valid row q >= pad
// attends keys pad..q; a fully padded row q < pad weighs keys 0..q in the
// reference's 64-wide -1e9 bands (RowScore).
#include "dt_common.cuh"
#include "dt_internal.h"
#include "prefill_common.cuh"

namespace dtk {

namespace {

constexpr int kLongThreads = 384;
constexpr int kBK = 64;  // keys per block
constexpr uint32_t kRegsCtl = 152;
constexpr uint32_t kRegsSoftmax = 176;
static_assert(128 * kRegsCtl + 256 * kRegsSoftmax == kLongThreads * 168, "register split must match the launch");

template <int D>
struct LongShape {
  static_assert(D == 64, "the long-context kernel is written for head_dim 64");
  static constexpr int ROWB = D * 2;
  static constexpr uint32_t LAYOUT = D == 64 ? kSw128 : kSw64;
  static constexpr int SBO = 8 * ROWB;
  static constexpr int Q_BYTES = 128 * ROWB;
  static constexpr int KV_BYTES = kBK * ROWB;
  static constexpr int NQB = 2;  // Q buffers per slot
  static constexpr int NKV = 8;  // K/V stages
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * NQB * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NKV * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NKV * KV_BYTES;
  static constexpr int NSB = 3;  // S buffers per slot (P V lags its S by two blocks)
  // q_full[2][NQB], q_empty[2][NQB], q_ready[2][NQB], kv_full[NKV], kv_empty[NKV],
  // kv_ready[NKV], s_full[2][NSB], p_full[2][NSB], pv_done[2][NSB], o_full[2],
  // o_empty[2], drain[2]
  static constexpr int NBAR = 6 * NQB + 3 * NKV + 3 * 2 * NSB + 2 + 2 + 2;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr uint32_t TMEM_S = 0;    // slot s, buffer b: TMEM_S + (NSB s + b) kBK
  static constexpr uint32_t TMEM_O = 384;  // slot s: TMEM_O + s D (one O per slot)
  static_assert(TMEM_S + 2 * NSB * kBK <= TMEM_O && TMEM_O + 2 * D <= 512, "TMEM budget");
};

// Geometry of one work item; every role derives it from the item index.
constexpr int kLongGroupUnits = 128;  // units whose pairs are scheduled together (L2 reuse of K/V)

struct LongItem {
  int b, g, pad, kstart, nblocks;
  int tile[2], first[2], last[2];
};

__device__ __forceinline__ LongItem long_item(int i, const PrefillParams& prm, int n_units, int npairs,
                                              int ntiles) {
  LongItem it;
  // Units in groups of kLongGroupUnits: within a group the heaviest pairs
  // (latest positions) go first, units innermost, so the end of the grid runs
  // the lightest items; a group's K/V (128 units x 196 KB at cfg4, 25 MB) stays
  // in L2 while its pairs are worked through, so each K/V block crosses HBM
  // about once instead of once per pair.  With an odd tile count the lone tile
  // is tile 0, the lightest.
  const int per = kLongGroupUnits * npairs;
  const int grp = i / per;
  const int j = i - grp * per;
  const int gu = min(kLongGroupUnits, n_units - grp * kLongGroupUnits);  // units in this group
  const int p = npairs - 1 - j / gu;
  const int unit = grp * kLongGroupUnits + (j - (j / gu) * gu);
  it.b = unit / prm.Hkv;
  it.g = unit - it.b * prm.Hkv;
  const int S = prm.S, PT = prm.PT;
  it.pad = prm.pad_len ? min(max(__ldg(prm.pad_len + it.b), 0), S) : 0;
  const int t0 = 2 * p - (ntiles & 1);
  int lo[2], hi[2];
  it.kstart = S;
  int hmax = 0;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int t = t0 + s;
    it.tile[s] = t >= 0 ? t : -1;
    const int pos0 = t * PT;
    lo[s] = pos0 >= it.pad ? it.pad : 0;
    hi[s] = min(pos0 + PT, S) - 1;
    if (t >= 0) {
      it.kstart = min(it.kstart, lo[s]);
      hmax = max(hmax, hi[s]);
    }
  }
  it.nblocks = (hmax - it.kstart) / kBK + 1;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    it.first[s] = (lo[s] - it.kstart) / kBK;
    it.last[s] = (hi[s] - it.kstart) / kBK;
  }
  return it;
}

template <uint32_t N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Allowed keys of a row inside 32 keys starting at k0: bit j = key k0 + j in [lo, hi].
__device__ __forceinline__ uint32_t key_mask32(int k0, int lo, int hi) {
  const int jlo = lo - k0, jhi = hi - k0;
  const uint32_t hm = jhi < 0 ? 0u : (jhi >= 31 ? 0xffffffffu : ((2u << jhi) - 1u));
  const uint32_t lm = jlo <= 0 ? 0xffffffffu : (jlo >= 32 ? 0u : (0xffffffffu << jlo));
  return hm & lm;
}

}  // namespace

template <int D, bool BF16>
__global__ void __launch_bounds__(kLongThreads, 1)
    dt_prefill_long_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const PrefillParams prm, int n_units) {
  using SH = LongShape<D>;
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem + SH::OFF_Q;
  uint8_t* k_s = smem + SH::OFF_K;
  uint8_t* v_s = smem + SH::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* q_full = bars;                      // [slot * NQB + buf]
  uint64_t* q_empty = q_full + 2 * SH::NQB;
  uint64_t* q_ready = q_empty + 2 * SH::NQB;   // Q tile rotated (RoPE inputs only)
  uint64_t* kv_full = q_ready + 2 * SH::NQB;
  uint64_t* kv_empty = kv_full + SH::NKV;
  uint64_t* kv_ready = kv_empty + SH::NKV;      // K block rotated (RoPE inputs only)
  uint64_t* s_full = kv_ready + SH::NKV;        // [slot * NSB + buf]: S of a block is in TMEM
  uint64_t* p_full = s_full + 2 * SH::NSB;      // [slot * NSB + buf]: P of a block is in TMEM
  uint64_t* pv_done = p_full + 2 * SH::NSB;     // [slot * NSB + buf]: the P V reading buf completed
  uint64_t* o_full = pv_done + 2 * SH::NSB;     // [slot]
  uint64_t* o_empty = o_full + 2;
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = prm.S, R = prm.R, PT = prm.PT;
  const int ntiles = (S + PT - 1) / PT;
  const int npairs = (ntiles + 1) / 2;
  const int n_items = n_units * npairs;
  const int q_rows = R * PT;

  if (tid == 0) {
    for (int j = 0; j < 2 * SH::NQB; ++j) {
      mbar_init(&q_full[j], 1);
      mbar_init(&q_empty[j], 1);
      mbar_init(&q_ready[j], 1);
    }
    for (int j = 0; j < SH::NKV; ++j) {
      mbar_init(&kv_full[j], 1);
      mbar_init(&kv_empty[j], 2);  // both MMA issuers release every block
      mbar_init(&kv_ready[j], 1);
    }
    for (int j = 0; j < 2 * SH::NSB; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&p_full[j], 4);  // one arrival per softmax warp
      mbar_init(&pv_done[j], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&o_full[j], 1);
      mbar_init(&o_empty[j], 4);
    }
    mbar_init(drain, 1);
    mbar_init(drain + 1, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  // Rows q_rows..127 of the Q buffers are never loaded (R * PT < 128 when R
  // does not divide 128): zero them once so their scores stay finite.
  for (int e = tid; e < 2 * SH::NQB * (128 - q_rows) * (SH::ROWB / 16); e += kLongThreads) {
    const int per = (128 - q_rows) * (SH::ROWB / 16);
    const int buf = e / per, rem = e - buf * per;
    *reinterpret_cast<uint4*>(q_s + buf * SH::Q_BYTES + (q_rows + rem / (SH::ROWB / 16)) * SH::ROWB +
                              (rem % (SH::ROWB / 16)) * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp < 4) {
    regs_dec<kRegsCtl>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ TMA producer
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      int qc0 = 0, qc1 = 0;
      int kvc = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
        const LongItem it = long_item(i, prm, n_units, npairs, ntiles);
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          int& qc = s ? qc1 : qc0;
          if (!ok || it.tile[s] < 0) continue;
          const int qb = qc % SH::NQB;
          uint64_t* fb = &q_full[s * SH::NQB + qb];
          if (!(ok = mbar_wait(&q_empty[s * SH::NQB + qb], ((qc / SH::NQB) & 1) ^ 1, abort_flag, prm.status)))
            continue;
          mbar_arrive_expect_tx(fb, (uint32_t)(q_rows * SH::ROWB));
          tma_load_4d(q_s + (s * SH::NQB + qb) * SH::Q_BYTES, &tmQ, fb, 0, it.g * R, it.tile[s] * PT, it.b);
          ++qc;
        }
        for (int j = 0; j < it.nblocks && ok; ++j, ++kvc) {
          const int st = kvc % SH::NKV;
          if (!(ok = mbar_wait(&kv_empty[st], ((kvc / SH::NKV) & 1) ^ 1, abort_flag, prm.status))) break;
          mbar_arrive_expect_tx(&kv_full[st], 2u * SH::KV_BYTES);
          tma_load_4d(k_s + st * SH::KV_BYTES, &tmK, &kv_full[st], 0, it.g, it.kstart + j * kBK, it.b);
          tma_load_4d(v_s + st * SH::KV_BYTES, &tmV, &kv_full[st], 0, it.g, it.kstart + j * kBK, it.b);
        }
      }
      if (!ok) {
        // Let the copies already issued land before the CTA can exit.
#pragma unroll
        for (int j = 0; j < SH::NKV; ++j) {
          const int uses = kvc / SH::NKV + (j < kvc % SH::NKV ? 1 : 0);
          if (uses > 0) mbar_wait(&kv_full[j], (uses - 1) & 1, nullptr, nullptr);
        }
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int j = 0; j < SH::NQB; ++j) {
            const int qc = s ? qc1 : qc0;
            const int uses = qc / SH::NQB + (j < qc % SH::NQB ? 1 : 0);
            if (uses > 0) mbar_wait(&q_full[s * SH::NQB + j], (uses - 1) & 1, nullptr, nullptr);
          }
      }
    } else if (warp == 1 || warp == 2) {
      // ------------------------------------------------------------ MMA issuers
      // One warp per slot (warps 1 and 2 sit on different SM sub-partitions,
      // so the two slots' MMAs issue in parallel).  The whole warp runs the
      // loop with warp-uniform values, lane 0 waits and issues.  The issuers
      // share only the K/V ring: kv_empty completes when both have released a
      // block, by an MMA commit after their last use of it or by a plain
      // arrive when their slot does not use it.
      const int s = __shfl_sync(0xffffffffu, warp - 1, 0);
      const bool leader = lane == 0;
      auto wait1 = [&](uint64_t* bar, uint32_t parity) -> bool {
        int w = 1;
        if (leader) w = mbar_wait(bar, parity, abort_flag, prm.status) ? 1 : 0;
        return __shfl_sync(0xffffffffu, w, 0) != 0;
      };
      // With RoPE inputs the MMAs wait for the rotated tiles.
      uint64_t* const q_avail = prm.rope ? q_ready : q_full;
      uint64_t* const kv_avail = prm.rope ? kv_ready : kv_full;
      const uint32_t idesc_s = umma_idesc_f16(BF16, 128, kBK, 0, 0);
      const uint32_t idesc_pv = umma_idesc_f16(BF16, 128, D, 0, 1);
      // Descriptors of stage 0 / buffer 0; others differ only in the address field.
      const uint64_t q_desc0 = umma_smem_desc(smem_u32(q_s + s * SH::NQB * SH::Q_BYTES), 16, SH::SBO, SH::LAYOUT);
      const uint64_t k_desc0 = umma_smem_desc(smem_u32(k_s), 16, SH::SBO, SH::LAYOUT);
      const uint64_t v_desc0 = umma_smem_desc(smem_u32(v_s), SH::KV_BYTES, SH::SBO, SH::LAYOUT);
      const uint32_t t_s0 = tmem + SH::TMEM_S + (uint32_t)(SH::NSB * s * kBK);
      const uint32_t t_o = tmem + SH::TMEM_O + (uint32_t)(s * D);
      int qc = 0, oc = 0, sc = 0, pc = 0;  // Q loads consumed, items, S issued, P consumed
      int kvc = 0;
      bool ok = true;
      // Blocks ("events") in the producer's order; the P V of an event is
      // issued two events after its S, so S runs two blocks ahead of the
      // softmax (three S buffers per slot) and an item's first S goes out
      // before the previous item's last two P V.
      struct Ev {
        int st, act, first, last;
      };
      Ev pq0{0, 0, 0, 0}, pq1{0, 0, 0, 0};
      int npend = 0;
      auto do_pv = [&](const Ev& e) -> bool {
        if (e.act) {
          // O += P V; the P sits in the S buffer its S used (PV k reads buffer k % NSB).
          const int pb = pc % SH::NSB;
          if (!wait1(&p_full[s * SH::NSB + pb], (pc / SH::NSB) & 1)) return false;
          if (e.first && !wait1(&o_empty[s], (oc & 1) ^ 1)) return false;
          const uint64_t vd = v_desc0 + (uint64_t)((e.st * SH::KV_BYTES) >> 4);
          const uint32_t t_p = t_s0 + (uint32_t)(pb * kBK);
          if (leader) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)  // 16 keys = 16 rows of 128 bytes per K step
              umma_f16_ts(t_o, t_p + kk * 8, vd + (uint64_t)(kk * 16 * SH::ROWB >> 4), idesc_pv,
                          (kk > 0 || !e.first) ? 1u : 0u);
            umma_commit(&pv_done[s * SH::NSB + pb]);
            if (e.last) umma_commit(&o_full[s]);
            umma_commit(&kv_empty[e.st]);  // the block is released once this P V has read it
          }
          ++pc;
          if (e.last) ++oc;
        } else if (leader) {
          mbar_arrive(&kv_empty[e.st]);  // a block this slot does not use
        }
        return true;
      };
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
        const LongItem it = long_item(i, prm, n_units, npairs, ntiles);
        const bool act = (s ? it.tile[1] : it.tile[0]) >= 0;
        const int first = s ? it.first[1] : it.first[0], last = s ? it.last[1] : it.last[0];
        const int qb = qc % SH::NQB;
        if (act && !(ok = wait1(&q_avail[s * SH::NQB + qb], (qc / SH::NQB) & 1))) break;
        const uint64_t qd = q_desc0 + (uint64_t)((qb * SH::Q_BYTES) >> 4);
        for (int j = 0; j < it.nblocks && ok; ++j) {
          const int st = (kvc + j) % SH::NKV;
          if (!(ok = wait1(&kv_avail[st], ((kvc + j) / SH::NKV) & 1))) break;
          const bool a = act && j >= first && j <= last;
          if (a) {
            // S = Q K^T of block j into the slot's next S buffer; the P V that
            // last read it (three S back) was issued before the previous S.
            const int sb = sc % SH::NSB;
            const uint64_t kd = k_desc0 + (uint64_t)((st * SH::KV_BYTES) >> 4);
            if (leader) {
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < D / 16; ++kk)
                umma_f16_ss(t_s0 + (uint32_t)(sb * kBK), qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
              umma_commit(&s_full[s * SH::NSB + sb]);
              if (j == last) umma_commit(&q_empty[s * SH::NQB + qb]);
            }
            ++sc;
            if (j == last) ++qc;
          }
          const Ev e{st, a ? 1 : 0, j == first ? 1 : 0, j == last ? 1 : 0};
          if (npend == 2) {
            if (!(ok = do_pv(pq0))) break;
            pq0 = pq1;
            pq1 = e;
          } else if (npend == 1) {
            pq1 = e;
            npend = 2;
          } else {
            pq0 = e;
            npend = 1;
          }
        }
        kvc += it.nblocks;
      }
      if (ok && npend >= 1) ok = do_pv(pq0);
      if (ok && npend == 2) ok = do_pv(pq1);
      if (leader) {
        umma_commit(drain + s);
        mbar_wait(drain + s, 0, nullptr, nullptr);
      }
      __syncwarp();
    } else if (warp == 3 && prm.rope) {
      // ------------------------------------------------------------ RoPE
      // Follows the producer's order: each item's Q tiles, then its K blocks.
      // Rows past the sequence end (zero-filled by TMA) stay as they are.
      int qc0 = 0, qc1 = 0;
      int kvc = 0;
      bool ok = true;
      for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
        const LongItem it = long_item(i, prm, n_units, npairs, ntiles);
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          int& qc = s ? qc1 : qc0;
          const int tile = s ? it.tile[1] : it.tile[0];
          if (!ok || tile < 0) continue;
          const int qb = qc % SH::NQB;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&q_full[s * SH::NQB + qb], (qc / SH::NQB) & 1, abort_flag,
                                                       prm.status))))
            continue;
          uint8_t* tq = q_s + (s * SH::NQB + qb) * SH::Q_BYTES;
          for (int rr = lane; rr < q_rows; rr += 32) {
            const int pos = tile * PT + rr / R;
            if (pos < S)
              rope_row_inplace<D, BF16>(tq, rr, prm.cos + (size_t)pos * prm.cs_stride,
                                        prm.sin + (size_t)pos * prm.cs_stride, prm.rope == kRopeRefRound);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&q_ready[s * SH::NQB + qb]);
          ++qc;
        }
        for (int j = 0; j < it.nblocks && ok; ++j, ++kvc) {
          const int st = kvc % SH::NKV;
          if (!(ok = __all_sync(0xffffffffu,
                                mbar_wait(&kv_full[st], (kvc / SH::NKV) & 1, abort_flag, prm.status))))
            break;
          uint8_t* tk = k_s + st * SH::KV_BYTES;
          for (int rr = lane; rr < kBK; rr += 32) {
            const int key = it.kstart + j * kBK + rr;
            if (key < S)
              rope_row_inplace<D, BF16>(tk, rr, prm.cos + (size_t)key * prm.cs_stride,
                                        prm.sin + (size_t)key * prm.cs_stride, prm.rope == kRopeRefRound);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&kv_ready[st]);
        }
      }
    }
  } else {
    // -------------------------------------------------------------- softmax
    regs_inc<kRegsSoftmax>();
    const int s = (warp - 4) >> 2;      // slot
    const int wq = warp & 3;            // TMEM lane quadrant
    const int r = wq * 32 + lane;       // tile row
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = prm.scale_log2;
    const float sd64 = prm.scale_div64;
    const int h = r % R, rowpos = r / R;
    int sc = 0, oc = 0;  // blocks and items this slot has processed
    bool ok = true;

    // Deferred epilogue of a finished item: O / l -> HBM.
    struct Pending {
      int valid, b, g, pos, k;
      float l;
    } pend{0, 0, 0, 0, 0, 0.f};
    auto epilogue = [&](const Pending& pe) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(&o_full[s], pe.k & 1, abort_flag, prm.status)))
        return false;
      tc_fence_after();
      const uint32_t t_o = t_lane + SH::TMEM_O + (uint32_t)(s * D);
      uint32_t o0[32], o1[32];
      tmem_ld32_async(t_o, o0);
      tmem_ld32_async(t_o + 32, o1);
      tmem_wait_ld(o0);
      tmem_wait_ld(o1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[s]);
      if (r < q_rows && pe.pos < S) {
        const float inv = 1.f / pe.l;
        typename E::T* orow = reinterpret_cast<typename E::T*>(prm.o) + (size_t)pe.b * prm.o_sb +
                              (size_t)pe.pos * prm.o_ss + (size_t)(pe.g * R + h) * prm.o_sh;
        auto put8 = [&](const uint32_t* v, int c) {
          uint4 w;
          w.x = E::from_f2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv);
          w.y = E::from_f2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv);
          w.z = E::from_f2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv);
          w.w = E::from_f2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv);
          *reinterpret_cast<uint4*>(orow + c) = w;
        };
#pragma unroll
        for (int c = 0; c < 32; c += 8) put8(o0 + c, c);
#pragma unroll
        for (int c = 0; c < 32; c += 8) put8(o1 + c, 32 + c);
      }
      return true;
    };

    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
      const LongItem it = long_item(i, prm, n_units, npairs, ntiles);
      const int tile = s ? it.tile[1] : it.tile[0];
      if (tile < 0) continue;
      const int first = s ? it.first[1] : it.first[0], last = s ? it.last[1] : it.last[0];
      const int pos = tile * PT + rowpos;
      const bool valid_row = r < q_rows && pos < S;
      const bool padded = valid_row && pos < it.pad;
      // Rows without a query (past the packed heads or the sequence end) are
      // never stored: they take every key so that they never force the
      // masked path on their warp.
      const int lo = !valid_row ? -(1 << 30) : (padded ? 0 : it.pad);
      const int hi = valid_row ? pos : (1 << 30);
      const bool warp_band = __any_sync(0xffffffffu, padded);
      const RowScore rs(padded, c2, sd64);
      float m = -INFINITY, l0 = 0.f, l1 = 0.f;
      for (int j = first; j <= last; ++j) {
        const int sb = sc % SH::NSB;
        if (!(ok = __all_sync(0xffffffffu,
                              mbar_wait(&s_full[s * SH::NSB + sb], (sc / SH::NSB) & 1, abort_flag, prm.status))))
          break;
        tc_fence_after();
        const uint32_t t_sb = t_lane + SH::TMEM_S + (uint32_t)((SH::NSB * s + sb) * kBK);
        const int kb = it.kstart + j * kBK;
        uint32_t u[2][32];
        tmem_ld32_async(t_sb, u[0]);
        tmem_ld32_async(t_sb + 32, u[1]);
        // Rows needing a mask anywhere in this block (warp-uniform).
        const bool masked = warp_band || __any_sync(0xffffffffu, lo > kb || hi < kb + kBK - 1);
        uint32_t mk[2];
#pragma unroll
        for (int c = 0; c < 2; ++c) mk[c] = masked ? key_mask32(kb + 32 * c, lo, hi) : 0xffffffffu;
        tmem_wait_ld(u[0]);
        tmem_wait_ld(u[1]);
        if (masked) {
          // A disallowed key's score becomes -inf, after which the row max and
          // P need no mask (P = 0 for it): one test and select per score
          // instead of separate, slower masked paths.
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              if (!((mk[c] >> jj) & 1u)) u[c][jj] = 0xff800000u;
        }

        // Block maximum over the allowed keys, in log2 units.
        // (the row score is monotonic in s, so the max of the raw scores gives it)
        float x0 = -INFINITY, x1 = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int jj = 0; jj < 32; jj += 4) {
            x0 = fmax3(x0, __uint_as_float(u[c][jj]), __uint_as_float(u[c][jj + 1]));
            x1 = fmax3(x1, __uint_as_float(u[c][jj + 2]), __uint_as_float(u[c][jj + 3]));
          }
        const float bmax = rs(fmaxf(x0, x1));
        // Move the reference only when P would exceed 2^8; then scale what
        // this row has accumulated (O in TMEM, the row sum) exactly.
        float f = 1.f;
        if (bmax != -INFINITY) {
          if (m == -INFINITY) {
            m = bmax;
          } else if (bmax > m + 8.f) {
            const float k = ceilf(bmax - m);
            m += k;
            f = exp2f(-k);
            l0 *= f;
            l1 *= f;
          }
        }
        if (__any_sync(0xffffffffu, f != 1.f)) {
          // f != 1 only after an earlier block of this item.  Wait for the
          // slot's latest P V (the completed S of this block implies every
          // earlier one is done), then scale the O rows.
          const int pvb = (sc - 1) % SH::NSB;  // P V of the previous block read S buffer pvb
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&pv_done[s * SH::NSB + pvb], ((sc - 1) / SH::NSB) & 1,
                                                       abort_flag, prm.status))))
            break;
          tc_fence_after();
          const uint32_t t_o = t_lane + SH::TMEM_O + (uint32_t)(s * D);
#pragma unroll 1
          for (int c = 0; c < D; c += 16) {
            uint32_t ov[16];
            tmem_ld16_u(t_o + c, ov);
#pragma unroll
            for (int z = 0; z < 16; ++z) ov[z] = __float_as_uint(__uint_as_float(ov[z]) * f);
            tmem_st16(t_o + c, ov);
          }
        }
        const float mm = m == -INFINITY ? 0.f : m;  // no allowed key yet: every t below is -inf
        // P = exp2(score - m), packed pairs over the first 32 columns of the S buffer.
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
          if (!warp_band) {
            const float2 c2v = make_float2(c2, c2), nmv = make_float2(-mm, -mm);
            float2 lv = make_float2(0.f, 0.f);
#pragma unroll
            for (int jj = 0; jj < 32; jj += 2) {
              // two lanes of scale-and-shift / row-sum work per f32x2 instruction
              const float2 t = ffma2(make_float2(__uint_as_float(u[c][jj]), __uint_as_float(u[c][jj + 1])), c2v, nmv);
              const float2 pp = make_float2(ex2_approx(t.x), ex2_approx(t.y));
              lv = fadd2(lv, pp);
              pk[jj >> 1] = E::from_f2(pp.x, pp.y);
            }
            l0 += lv.x;
            l1 += lv.y;
          } else {
            // warps holding fully padded rows: the row score rs(s) - m as
            // ((s mul + add) - add) out - m, two lanes per f32x2 instruction with
            // the same roundings as the scalar form (disallowed keys are -inf)
            const float2 mul2 = make_float2(rs.mul, rs.mul), add2 = make_float2(rs.add, rs.add);
            const float2 nadd2 = make_float2(-rs.add, -rs.add), out2 = make_float2(rs.out, rs.out);
            const float2 nmv = make_float2(-mm, -mm);
            float2 lv = make_float2(0.f, 0.f);
#pragma unroll
            for (int jj = 0; jj < 32; jj += 2) {
              const float2 sv = make_float2(__uint_as_float(u[c][jj]), __uint_as_float(u[c][jj + 1]));
              const float2 t = fadd2(fmul2(fadd2(ffma2(sv, mul2, add2), nadd2), out2), nmv);
              const float2 pp = make_float2(ex2_approx(t.x), ex2_approx(t.y));
              lv = fadd2(lv, pp);
              pk[jj >> 1] = E::from_f2(pp.x, pp.y);
            }
            l0 += lv.x;
            l1 += lv.y;
          }
          tmem_st16(t_sb + 16 * c, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s * SH::NSB + sb]);
        ++sc;
        if (j == first && pend.valid) {
          if (!(ok = epilogue(pend))) break;
          pend.valid = 0;
        }
      }
      if (!ok) break;
      pend = Pending{1, it.b, it.g, pos, oc, l0 + l1};
      ++oc;
    }
    if (ok && pend.valid) epilogue(pend);
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool BF16>
static cudaError_t launch_long(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                               const PrefillParams& prm, int n_units, int grid, cudaStream_t st) {
  using SH = LongShape<D>;
  auto kern = dt_prefill_long_kernel<D, BF16>;
  cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(kern), SH::SMEM);
  if (e != cudaSuccess) return e;
  kern<<<grid, kLongThreads, SH::SMEM, st>>>(q, k, v, prm, n_units);
  return cudaGetLastError();
}

cudaError_t launch_prefill_long_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                      const PrefillParams& prm, bool bf16, int n_units, int grid,
                                      cudaStream_t stream) {
  return bf16 ? launch_long<64, true>(q, k, v, prm, n_units, grid, stream)
              : launch_long<64, false>(q, k, v, prm, n_units, grid, stream);
}

}  // namespace dtk
