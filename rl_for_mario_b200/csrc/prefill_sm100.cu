// Fused causal GQA prefill attention for the Decision Transformer, sm_100a.
//
// Replaces the prefill branch of DecisionTransformerAttention.forward
// (model/model_decision_transformer.py:179-224 and :247): RoPE on Q/K
// (:103-117, :180), repeat_kv (:121-130, :194-195) and the masked SDPA
// (:198-224).  One CTA owns one (sample b, KV head g) unit; the R = Hq/Hkv
// query heads of that group are packed into the 128-row M tiles as rows
// (position, head), so K/V are read once per group and never repeated.
//
// Pipeline inside a CTA (8 warps):
//   warp 0      TMA producer: Q tiles (2-stage ring), K/V key blocks (ring)
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//   warps 2-3   RoPE workers: rotate the landed Q tile / K block in place
//   warps 4-7   softmax + epilogue warpgroup, one thread per TMEM lane (row)
// S = Q K^T and O = P V run on the tensor cores (kind::f16, fp32 accumulate
// in TMEM).  The softmax is online over key blocks of 128.
//
// Mask semantics (reference :206-224, left padding of `pad` tokens):
//   valid row q >= pad : softmax over keys pad..q (keys < pad get -1e9, whose
//                        weight underflows to exactly 0 in fp32);
//   padded row q < pad : every key 0..q carries -1e9; the fp32 sum rounds the
//                        scaled scores to 64-wide bands (padded_score_log2),
//                        a plain mean of V[0..q] while |score| < 32.
#include <cstdio>

#include "dt_common.cuh"
#include "dt_internal.h"
#include "prefill_common.cuh"

namespace dtk {

template <int D>
struct PrefillShape {
  static constexpr int KB = 128;  // keys per block (max N of the S MMA used here)
  static constexpr int ROWB = D * 2;
  static constexpr int Q_BYTES = 128 * ROWB;
  static constexpr int KV_BYTES = KB * ROWB;
  static constexpr int NQ = 2;
  static constexpr int NKV = (D == 32) ? 3 : 2;
  static constexpr int P_BYTES = 128 * KB * 2;
  static constexpr uint32_t LAYOUT = (D == 32) ? kSw64 : kSw128;
  static constexpr uint32_t SBO = 8 * ROWB;  // byte distance between 8-row core groups
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NQ * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NKV * KV_BYTES;
  static constexpr int OFF_P = OFF_V + NKV * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // q_full, q_ready, q_empty [NQ]; kv_full, k_ready, kv_empty [NKV]; s_full, p_full, o_full, drain
  static constexpr int NBAR = 3 * NQ + 3 * NKV + 4;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;  // + slack to align the base to 1024
  static constexpr uint32_t TMEM_COLS = 256;
  static constexpr uint32_t TMEM_S = 0;
  static constexpr uint32_t TMEM_O = 128;
  static constexpr int MIN_BLOCKS = (D == 32) ? 2 : 1;
};

template <int D, bool BF16>
__global__ void __launch_bounds__(256, PrefillShape<D>::MIN_BLOCKS)
    dt_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const PrefillParams prm) {
  using SH = PrefillShape<D>;
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_ready = bars + SH::NQ;
  uint64_t* q_empty = bars + 2 * SH::NQ;
  uint64_t* kv_full = bars + 3 * SH::NQ;
  uint64_t* k_ready = kv_full + SH::NKV;
  uint64_t* kv_empty = kv_full + 2 * SH::NKV;
  uint64_t* s_full = kv_full + 3 * SH::NKV;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_full = s_full + 2;
  uint64_t* drain = s_full + 3;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SH::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SH::OFF_MISC + 4);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int b = blockIdx.x / prm.Hkv;
  const int g = blockIdx.x % prm.Hkv;
  const int S = prm.S;
  const int R = prm.R;
  const int PT = prm.PT;
  int pad = prm.pad_len ? prm.pad_len[b] : 0;
  pad = max(0, min(pad, S));
  const int ntiles = (S + PT - 1) / PT;

  if (tid == 0) {
    for (int i = 0; i < SH::NQ; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_ready[i], 64);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < SH::NKV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&k_ready[i], 64);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, SH::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  uint8_t* q_s = smem + SH::OFF_Q;
  uint8_t* k_s = smem + SH::OFF_K;
  uint8_t* v_s = smem + SH::OFF_V;
  uint8_t* p_s = smem + SH::OFF_P;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      int qi = 0, kvi = 0;
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        const TilePlan tp = plan_tile(t, PT, S, pad);
        const int qs = qi % SH::NQ;
        if (!(ok = mbar_wait(&q_empty[qs], ((qi / SH::NQ) & 1) ^ 1, abort_flag, prm.status))) break;
        mbar_arrive_expect_tx(&q_full[qs], (uint32_t)(PT * R * SH::ROWB));
        tma_load_4d(q_s + qs * SH::Q_BYTES, &tmQ, &q_full[qs], 0, g * R, tp.pos0, b);
        ++qi;
        for (int j = 0; j < tp.nblocks; ++j) {
          const int ks = kvi % SH::NKV;
          if (!(ok = mbar_wait(&kv_empty[ks], ((kvi / SH::NKV) & 1) ^ 1, abort_flag, prm.status))) break;
          const int kb0 = tp.kstart + j * 128;
          mbar_arrive_expect_tx(&kv_full[ks], (uint32_t)(2 * SH::KV_BYTES));
          tma_load_4d(k_s + ks * SH::KV_BYTES, &tmK, &kv_full[ks], 0, g, kb0, b);
          tma_load_4d(v_s + ks * SH::KV_BYTES, &tmV, &kv_full[ks], 0, g, kb0, b);
          ++kvi;
        }
      }
      if (*abort_flag) {
        // Let every load already issued land before the CTA can exit.
        for (int i = 0; i < SH::NQ; ++i) {
          const int uses = qi / SH::NQ + (i < qi % SH::NQ ? 1 : 0);
          if (uses > 0) mbar_wait(&q_full[i], (uses - 1) & 1, nullptr, nullptr);
        }
        for (int i = 0; i < SH::NKV; ++i) {
          const int uses = kvi / SH::NKV + (i < kvi % SH::NKV ? 1 : 0);
          if (uses > 0) mbar_wait(&kv_full[i], (uses - 1) & 1, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_pv = umma_idesc_f16(BF16, 128, D, 0, 1);
      int qi = 0, kvi = 0;
      uint32_t p_ph = 0;
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        const TilePlan tp = plan_tile(t, PT, S, pad);
        const int qs = qi % SH::NQ;
        if (!(ok = mbar_wait(&q_ready[qs], (qi / SH::NQ) & 1, abort_flag, prm.status))) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(q_s + qs * SH::Q_BYTES);
        for (int j = 0; j < tp.nblocks; ++j) {
          const int ks = kvi % SH::NKV;
          if (!(ok = mbar_wait(&k_ready[ks], (kvi / SH::NKV) & 1, abort_flag, prm.status))) break;
          tc_fence_after();
          const int n = block_cols(tp, j);
          const uint32_t ka = smem_u32(k_s + ks * SH::KV_BYTES);
          const uint32_t va = smem_u32(v_s + ks * SH::KV_BYTES);
          const uint32_t idesc_s = umma_idesc_f16(BF16, 128, (uint32_t)n, 0, 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ad = umma_smem_desc(qa + kk * 32, 16, SH::SBO, SH::LAYOUT);
            const uint64_t bd = umma_smem_desc(ka + kk * 32, 16, SH::SBO, SH::LAYOUT);
            umma_f16_ss(tmem + SH::TMEM_S, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(s_full);
          if (j == tp.nblocks - 1) umma_commit(&q_empty[qs]);
          if (!(ok = mbar_wait(p_full, p_ph, abort_flag, prm.status))) break;
          p_ph ^= 1;
          tc_fence_after();
          const uint32_t pa = smem_u32(p_s);
          for (int kk = 0; kk < n / 16; ++kk) {
            const uint64_t ad = umma_smem_desc(pa + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024, kSw128);
            const uint64_t bd = umma_smem_desc(va + kk * 16 * SH::ROWB, SH::KV_BYTES, SH::SBO, SH::LAYOUT);
            umma_f16_ss(tmem + SH::TMEM_O, ad, bd, idesc_pv, kk > 0 ? 1u : 0u);
          }
          umma_commit(o_full);
          umma_commit(&kv_empty[ks]);
          ++kvi;
        }
        ++qi;
      }
      // Drain: every MMA issued above has completed once this arrives.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ RoPE workers
    const int rt = tid - 64;  // 0..63
    int qi = 0, kvi = 0;
    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      const TilePlan tp = plan_tile(t, PT, S, pad);
      const int qs = qi % SH::NQ;
      if (!(ok = mbar_wait(&q_full[qs], (qi / SH::NQ) & 1, abort_flag, prm.status))) break;
      if (prm.rope) {
        uint8_t* tile = q_s + qs * SH::Q_BYTES;
        for (int row = rt; row < PT * R; row += 64) {
          const int pos = tp.pos0 + row / R;
          if (pos < S)
            rope_row_inplace<D, BF16>(tile, row, prm.cos + (size_t)pos * prm.cs_stride,
                                      prm.sin + (size_t)pos * prm.cs_stride, prm.rope == kRopeRefRound);
        }
        fence_proxy_async_smem();
      }
      mbar_arrive(&q_ready[qs]);
      ++qi;
      for (int j = 0; j < tp.nblocks; ++j) {
        const int ks = kvi % SH::NKV;
        if (!(ok = mbar_wait(&kv_full[ks], (kvi / SH::NKV) & 1, abort_flag, prm.status))) break;
        if (prm.rope) {
          uint8_t* tile = k_s + ks * SH::KV_BYTES;
          const int kb0 = tp.kstart + j * 128;
          const int n = block_cols(tp, j);
          for (int row = rt; row < n; row += 64) {
            const int key = kb0 + row;
            if (key < S)
              rope_row_inplace<D, BF16>(tile, row, prm.cos + (size_t)key * prm.cs_stride,
                                        prm.sin + (size_t)key * prm.cs_stride, prm.rope == kRopeRefRound);
          }
          fence_proxy_async_smem();
        }
        mbar_arrive(&k_ready[ks]);
        ++kvi;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int wq = warp & 3;  // TMEM lane quarter this warp may access
    const int r = wq * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const float c2 = prm.scale_log2;
    const float sd64 = prm.scale_div64;
    uint32_t s_ph = 0, o_ph = 0;
    bool ok = true;
    const int h = r % R;
    const int rowpos = r / R;
    for (int t = 0; t < ntiles && ok; ++t) {
      const TilePlan tp = plan_tile(t, PT, S, pad);
      const int pos = tp.pos0 + rowpos;
      const bool valid_row = (r < PT * R) && (pos < S);
      const bool padded = pos < pad;
      // Allowed key range [lo, hi] for this row.
      const int lo = padded ? 0 : pad;
      const int hi = valid_row ? pos : -1;
      float m = -INFINITY, l = 0.f;
      float acc[D];
#pragma unroll
      for (int d = 0; d < D; ++d) acc[d] = 0.f;
      for (int j = 0; j < tp.nblocks; ++j) {
        const int kb0 = tp.kstart + j * 128;
        const int n = block_cols(tp, j);
        // Warp-uniform outcome, so the TMEM loads below stay convergent.
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(s_full, s_ph, abort_flag, prm.status)))) break;
        s_ph ^= 1;
        tc_fence_after();
        float m_use = 0.f, alpha = 1.f;
        {
          // tcgen05.ld is .sync.aligned: every lane of the warp loads, whatever
          // its row needs, so the warp never executes it divergently.
          float bmax = -INFINITY;
          for (int c = 0; c < n; c += 16) {
            float s[16];
            tmem_ld16(t_lane + SH::TMEM_S + c, s);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int key = kb0 + c + i;
              if (key >= lo && key <= hi) bmax = fmaxf(bmax, s[i]);
            }
          }
          const float m_new = fmaxf(m, padded ? padded_score_log2(bmax, sd64) : bmax * c2);
          m_use = (m_new == -INFINITY) ? 0.f : m_new;
          alpha = ex2_approx(m - m_use);  // m = -inf -> 0
          m = m_new;
        }
        float bsum = 0.f;
        for (int c = 0; c < n; c += 16) {
          float s[16];
          tmem_ld16(t_lane + SH::TMEM_S + c, s);
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const int key = kb0 + c + i;
            const bool a0 = key >= lo && key <= hi;
            const bool a1 = key + 1 >= lo && key + 1 <= hi;
            float p0, p1;
            if (padded) {
              p0 = a0 ? ex2_approx(padded_score_log2(s[i], sd64) - m_use) : 0.f;
              p1 = a1 ? ex2_approx(padded_score_log2(s[i + 1], sd64) - m_use) : 0.f;
            } else {
              p0 = a0 ? ex2_approx(fmaf(s[i], c2, -m_use)) : 0.f;
              p1 = a1 ? ex2_approx(fmaf(s[i + 1], c2, -m_use)) : 0.f;
            }
            bsum += p0 + p1;
            pk[i >> 1] = E::from_f2(p0, p1);
          }
          // P tile: K-major, 128B swizzle, 64 keys per 16 KB column block.
          const int kc = c >> 6;           // 64-key column block
          const int ch = (c & 63) >> 3;    // first 16-byte chunk of these 16 keys
          uint8_t* prow = p_s + kc * (128 * 128);
          *reinterpret_cast<uint4*>(prow + swz<128>(r, ch)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<uint4*>(prow + swz<128>(r, ch + 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        l = l * alpha + bsum;
        tc_fence_before();
        fence_proxy_async_smem();
        mbar_arrive(p_full);
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(o_full, o_ph, abort_flag, prm.status)))) break;
        o_ph ^= 1;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D; c += 16) {
          float o[16];
          tmem_ld16(t_lane + SH::TMEM_O + c, o);
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[c + i] = fmaf(acc[c + i], alpha, o[i]);
        }
      }
      if (ok && valid_row) {
        const float inv = 1.f / l;
        typename E::T* orow = reinterpret_cast<typename E::T*>(prm.o) + (size_t)b * prm.o_sb +
                              (size_t)pos * prm.o_ss + (size_t)(g * R + h) * prm.o_sh;
#pragma unroll
        for (int c = 0; c < D; c += 8) {
          uint4 w;
          w.x = E::from_f2(acc[c + 0] * inv, acc[c + 1] * inv);
          w.y = E::from_f2(acc[c + 2] * inv, acc[c + 3] * inv);
          w.z = E::from_f2(acc[c + 4] * inv, acc[c + 5] * inv);
          w.w = E::from_f2(acc[c + 6] * inv, acc[c + 7] * inv);
          *reinterpret_cast<uint4*>(orow + c) = w;
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, SH::TMEM_COLS);
  }
}

template <int D, bool BF16>
static cudaError_t launch_t(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                            const PrefillParams& prm, int grid, cudaStream_t stream) {
  using SH = PrefillShape<D>;
  auto kfn = dt_prefill_kernel<D, BF16>;
  cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(kfn), SH::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  kfn<<<grid, 256, SH::SMEM_BYTES, stream>>>(q, k, v, prm);
  return cudaGetLastError();
}

cudaError_t launch_prefill_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                 const PrefillParams& prm, int D, bool bf16, int grid, cudaStream_t stream) {
  if (D == 32) return bf16 ? launch_t<32, true>(q, k, v, prm, grid, stream)
                           : launch_t<32, false>(q, k, v, prm, grid, stream);
  if (D == 64) return bf16 ? launch_t<64, true>(q, k, v, prm, grid, stream)
                           : launch_t<64, false>(q, k, v, prm, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace dtk
