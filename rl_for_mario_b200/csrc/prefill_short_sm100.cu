// Persistent fused causal GQA prefill for short sequences (S <= 192,
// head_dim 32): the Decision Transformer's own context (64 timesteps x 3
// tokens).  Same mathematics as prefill_sm100.cu (reference
// model/model_decision_transformer.py:179-224); different schedule:
//
//  * one CTA per SM loops over (sample b, KV head g) units; the M tiles of a
//    unit pack 128 rows (position, head) of the R query heads sharing KV head g;
//  * K and V of a unit (S x 32 each) stay resident in shared memory for all
//    of the unit's tiles; K is rotated once per unit; the cos/sin tables are
//    staged in shared memory once per CTA;
//  * two softmax warpgroups take alternate M tiles (one thread per row), each
//    with its own S columns and two O slots in TMEM, so one warpgroup's
//    exponentials overlap the other's row-max pass and epilogue while the
//    tensor core prepares the next tiles;
//  * a warpgroup reads S from TMEM twice (row max, then P = exp2), each
//    time with the next 32-column load in flight; P (bf16) is written back
//    into TMEM over the S columns it came from and O = P V reads it from there
//    (tcgen05 MMA with A in TMEM);
//  * the epilogue (O / rowsum -> bf16 -> HBM) of a tile runs after the
//    warpgroup's next tile is in softmax, from the other O slot;
//  * the TMA producer runs an 8-deep ring of Q tiles and a 3-deep ring of K/V.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer of warpgroup 0's tiles,
// 2 MMA issuer of warpgroup 1's tiles, 3-5 RoPE workers, 6-9 softmax
// warpgroup 0, 10-13 softmax warpgroup 1.  A tcgen05.mma costs the issuing
// thread tens of cycles and shares its SMSP with busy softmax warps, so each
// warpgroup has its own issuer on its own SMSP.
#include "dt_common.cuh"
#include "dt_internal.h"
#include "prefill_common.cuh"

namespace dtk {

namespace {

struct SS {
  static constexpr int D = 32;
  static constexpr int ROWB = 64;
  static constexpr int SMAX = 192;
  static constexpr int Q_BYTES = 128 * ROWB;   // one 128-row Q tile
  static constexpr int NQ = 8;
  static constexpr int KV_BYTES = SMAX * ROWB; // K (or V) of one unit
  static constexpr int NKV = 3;
  static constexpr int CS_STRIDE = D + 4;      // floats per staged cos/sin row (bank spread)
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NQ * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NKV * KV_BYTES;
  static constexpr int OFF_COS = OFF_V + NKV * KV_BYTES;
  static constexpr int OFF_SIN = OFF_COS + SMAX * CS_STRIDE * 4;
  static constexpr int OFF_PAD = OFF_SIN + SMAX * CS_STRIDE * 4;
  static constexpr int MAX_UNITS = kShortMaxUnitsPerCta;  // units per CTA (per-unit pads staged in smem)
  static constexpr int OFF_BAR = OFF_PAD + MAX_UNITS * 4;
  // q_full, q_ready, q_empty [NQ]; kv_full, kv_ready, kv_empty [NKV]; s_full, p_full [2 warpgroups];
  // o_full [2 warpgroups x 2 slots]; drain [2 issuers]
  static constexpr int NBAR = 3 * NQ + 3 * NKV + 4 + 4 + 2;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t TMEM_S = 0;    // + 192 * warpgroup (P aliases the first half)
  static constexpr uint32_t TMEM_O = 384;  // + 64 * warpgroup + 32 * slot
  static constexpr int NTHREADS = 448;
  static constexpr int NROPE = 96;
};
static_assert(SS::SMEM_BYTES <= 232448, "shared memory budget");

// Work cursor: local unit lu, tile t within the unit, local tile index i.
struct Cursor {
  int lu, t, i;
  __device__ __forceinline__ void next(int ntiles) {
    ++i;
    if (++t == ntiles) {
      t = 0;
      ++lu;
    }
  }
};

// Alternate warpgroups; (t + lu) flips the parity per unit when the tile
// count is even, so both warpgroups see the same mix of causal tile lengths.
__device__ __forceinline__ int tile_wg(const Cursor& c) { return (c.t + c.lu) & 1; }

// Key window of a tile: S columns [kb0, kb0 + n), processed in 32-column
// chunks from kb0.  kb0 is placed so that the last chunk ends at the tile's
// causal edge (the diagonal block is one chunk), rounded down to 16, >= 0.
struct TileInfo {
  int pad, pos0, kb0, n, nc;
};

__device__ __forceinline__ TileInfo tile_info(const Cursor& c, const int* pads_s, int PT, int S) {
  TileInfo T;
  T.pad = pads_s[c.lu];
  const TilePlan p = plan_tile(c.t, PT, S, T.pad);
  T.pos0 = p.pos0;
  int kb0 = p.kend - 32 * ((p.kend - p.kstart + 31) >> 5);
  kb0 = max(kb0, 0) & ~15;
  T.kb0 = kb0;
  T.n = (p.kend - kb0 + 15) & ~15;
  T.nc = (T.n + 31) >> 5;
  return T;
}

}  // namespace

template <bool BF16>
__global__ void __launch_bounds__(SS::NTHREADS, 1)
    dt_prefill_short_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const PrefillParams prm, int n_units) {
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SS::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* q_ready = bars + SS::NQ;
  uint64_t* q_empty = bars + 2 * SS::NQ;
  uint64_t* kv_full = bars + 3 * SS::NQ;
  uint64_t* kv_ready = kv_full + SS::NKV;
  uint64_t* kv_empty = kv_full + 2 * SS::NKV;
  uint64_t* s_full = kv_full + 3 * SS::NKV;  // [warpgroup]
  uint64_t* p_full = s_full + 2;             // [warpgroup]
  uint64_t* o_full = s_full + 4;             // [warpgroup * 2 + slot]
  uint64_t* drain = s_full + 8;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SS::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SS::OFF_MISC + 4);
  float* cos_s = reinterpret_cast<float*>(smem + SS::OFF_COS);
  float* sin_s = reinterpret_cast<float*>(smem + SS::OFF_SIN);
  int* pads_s = reinterpret_cast<int*>(smem + SS::OFF_PAD);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = prm.S;
  const int R = prm.R;
  const int PT = prm.PT;
  const int ntiles = (S + PT - 1) / PT;
  const int my_units = (n_units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int ntotal = my_units * ntiles;
  const int SB = (S + 15) & ~15;  // K/V rows loaded per unit (TMA box height)

  if (tid == 0) {
    for (int i = 0; i < SS::NQ; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_ready[i], SS::NROPE);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < SS::NKV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_ready[i], SS::NROPE);
      mbar_init(&kv_empty[i], 2);  // both MMA issuers release a unit's K/V
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&o_full[i], 1);
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Stage this CTA's per-unit padding and (when rotating) the cos/sin rows.
  for (int j = tid; j < my_units; j += SS::NTHREADS) {
    const int unit = blockIdx.x + j * gridDim.x;
    const int pad = prm.pad_len ? prm.pad_len[unit / prm.Hkv] : 0;
    pads_s[j] = max(0, min(pad, S));
  }
  if (prm.rope) {
    // The first half of each sin row is stored negated (rope_row_inplace_f2).
    for (int j = tid; j < S * (SS::D / 4); j += SS::NTHREADS) {
      const int row = j / (SS::D / 4), c4 = j % (SS::D / 4);
      *reinterpret_cast<float4*>(cos_s + row * SS::CS_STRIDE + c4 * 4) =
          __ldg(reinterpret_cast<const float4*>(prm.cos + (size_t)row * prm.cs_stride) + c4);
      float4 sv = __ldg(reinterpret_cast<const float4*>(prm.sin + (size_t)row * prm.cs_stride) + c4);
      if (c4 * 4 < SS::D / 2) sv = make_float4(-sv.x, -sv.y, -sv.z, -sv.w);
      *reinterpret_cast<float4*>(sin_s + row * SS::CS_STRIDE + c4 * 4) = sv;
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, SS::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  uint8_t* q_s = smem + SS::OFF_Q;
  uint8_t* k_s = smem + SS::OFF_K;
  uint8_t* v_s = smem + SS::OFF_V;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      int qi = 0, lu = 0;
      bool ok = true;
      for (; lu < my_units && ok; ++lu) {
        const int unit = blockIdx.x + lu * gridDim.x;
        const int b = unit / prm.Hkv;
        const int g = unit - b * prm.Hkv;
        const int kvb = lu % SS::NKV;
        if (!(ok = mbar_wait(&kv_empty[kvb], ((lu / SS::NKV) & 1) ^ 1, abort_flag, prm.status))) break;
        mbar_arrive_expect_tx(&kv_full[kvb], (uint32_t)(2 * SB * SS::ROWB));
        tma_load_4d(k_s + kvb * SS::KV_BYTES, &tmK, &kv_full[kvb], 0, g, 0, b);
        tma_load_4d(v_s + kvb * SS::KV_BYTES, &tmV, &kv_full[kvb], 0, g, 0, b);
        for (int t = 0; t < ntiles; ++t) {
          const int qs = qi % SS::NQ;
          if (!(ok = mbar_wait(&q_empty[qs], ((qi / SS::NQ) & 1) ^ 1, abort_flag, prm.status))) break;
          mbar_arrive_expect_tx(&q_full[qs], (uint32_t)(PT * R * SS::ROWB));
          tma_load_4d(q_s + qs * SS::Q_BYTES, &tmQ, &q_full[qs], 0, g * R, t * PT, b);
          ++qi;
        }
      }
      if (*abort_flag) {
        // Let every load already issued land before the CTA can exit.
        for (int i = 0; i < SS::NQ; ++i) {
          const int uses = qi / SS::NQ + (i < qi % SS::NQ ? 1 : 0);
          if (uses > 0) mbar_wait(&q_full[i], (uses - 1) & 1, nullptr, nullptr);
        }
        for (int i = 0; i < SS::NKV; ++i) {
          const int uses = lu / SS::NKV + (i < lu % SS::NKV ? 1 : 0);
          if (uses > 0) mbar_wait(&kv_full[i], (uses - 1) & 1, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers (one per warpgroup)
    if (lane == 0) {
      const int w = warp - 1;  // this thread issues the tiles of warpgroup w
      const uint32_t idesc_pv = umma_idesc_f16(BF16, 128, SS::D, 0, 1);
      uint32_t p_ph = 0u;   // phase of p_full[w]
      uint32_t slot = 0u;   // O slot of the next P V
      // S for tile c into warpgroup w's S columns.
      auto issue_s = [&](const Cursor& c) -> bool {
        const TileInfo T = tile_info(c, pads_s, PT, S);
        const int qs = c.i % SS::NQ;
        const int kvb = c.lu % SS::NKV;
        if (!mbar_wait(&q_ready[qs], (c.i / SS::NQ) & 1, abort_flag, prm.status)) return false;
        if (!mbar_wait(&kv_ready[kvb], (c.lu / SS::NKV) & 1, abort_flag, prm.status)) return false;
        tc_fence_after();
        // K-major 64B-swizzled operands; the second K step starts 32 bytes in.
        const uint64_t ad = umma_smem_desc(smem_u32(q_s + qs * SS::Q_BYTES), 16, 8 * SS::ROWB, kSw64);
        const uint64_t bd = umma_smem_desc(smem_u32(k_s + kvb * SS::KV_BYTES) + (uint32_t)T.kb0 * SS::ROWB, 16,
                                           8 * SS::ROWB, kSw64);
        const uint32_t idesc_s = umma_idesc_f16(BF16, 128, (uint32_t)T.n, 0, 0);
        const uint32_t td = tmem + SS::TMEM_S + 192u * w;
        umma_f16_ss(td, ad, bd, idesc_s, 0u);
        umma_f16_ss(td, ad + 2, bd + 2, idesc_s, 1u);
        umma_commit(&s_full[w]);
        umma_commit(&q_empty[qs]);
        return true;
      };
      // O = P V for tile c into the next O slot, P read from warpgroup w's S columns.
      auto issue_pv = [&](const Cursor& c) -> bool {
        const TileInfo T = tile_info(c, pads_s, PT, S);
        const int kvb = c.lu % SS::NKV;
        if (!mbar_wait(&p_full[w], p_ph, abort_flag, prm.status)) return false;
        p_ph ^= 1u;
        tc_fence_after();
        const uint32_t pa = tmem + SS::TMEM_S + 192u * w;  // packed bf16 P, 2 keys per column
        const uint32_t td = tmem + SS::TMEM_O + 64u * w + 32u * slot;
        // MN-major V rows: 16 keys per K step = 1024 bytes = 64 descriptor units.
        const uint64_t bd = umma_smem_desc(smem_u32(v_s + kvb * SS::KV_BYTES) + (uint32_t)T.kb0 * SS::ROWB,
                                           SS::KV_BYTES, 8 * SS::ROWB, kSw64);
        const int ksteps = T.n / 16;
        umma_f16_ts(td, pa, bd, idesc_pv, 0u);
        // Exactly ksteps MMAs: a predicated-off tcgen05.mma still costs its issue slot time.
#pragma unroll 1
        for (int kk = 1; kk < ksteps; ++kk) umma_f16_ts(td, pa + kk * 8, bd + (uint64_t)(kk * 64), idesc_pv, 1u);
        umma_commit(&o_full[w * 2 + slot]);
        slot ^= 1u;
        return true;
      };
      // This warpgroup's tiles in order; S of the next one goes after the
      // current P V (same S columns; the in-order tensor pipe runs P V first).
      // After the last tile of a unit that this issuer touches, it releases
      // the unit's K/V buffer (the other issuer does the same).
      Cursor cur{0, 0, 0};
      while (cur.i < ntotal && tile_wg(cur) != w) cur.next(ntiles);
      bool ok = true;
      int lu_done = 0;  // units whose K/V this issuer has released
      if (cur.i < ntotal) ok = issue_s(cur);
      while (ok && cur.i < ntotal) {
        Cursor nxt = cur;
        nxt.next(ntiles);
        while (nxt.i < ntotal && tile_wg(nxt) != w) nxt.next(ntiles);
        if (!(ok = issue_pv(cur))) break;
        // Release K/V of every unit that no later tile of this issuer uses
        // (including units none of its tiles touch).
        const int lu_next = nxt.i < ntotal ? nxt.lu : my_units;
        for (; lu_done < lu_next; ++lu_done) umma_commit(&kv_empty[lu_done % SS::NKV]);
        if (nxt.i < ntotal && !(ok = issue_s(nxt))) break;
        cur = nxt;
      }
      if (ok) {
        // Units this issuer never touched (no tile of its warpgroup) still need its release.
        for (; lu_done < my_units; ++lu_done) umma_commit(&kv_empty[lu_done % SS::NKV]);
      }
      umma_commit(&drain[w]);
      mbar_wait(&drain[w], 0, nullptr, nullptr);
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ RoPE workers
    const int rt = tid - 96;  // 0..95
    int qi = 0;
    bool ok = true;
    for (int lu = 0; lu < my_units && ok; ++lu) {
      const int kvb = lu % SS::NKV;
      if (!(ok = mbar_wait(&kv_full[kvb], (lu / SS::NKV) & 1, abort_flag, prm.status))) break;
      if (prm.rope) {
        uint8_t* kt = k_s + kvb * SS::KV_BYTES;
        for (int row = rt; row < S; row += SS::NROPE)
          rope_row_inplace_f2<32, BF16>(kt, row, cos_s + row * SS::CS_STRIDE, sin_s + row * SS::CS_STRIDE,
                                        prm.rope == kRopeRefRound);
        fence_proxy_async_smem();
      }
      mbar_arrive(&kv_ready[kvb]);
      for (int t = 0; t < ntiles; ++t) {
        const int qs = qi % SS::NQ;
        if (!(ok = mbar_wait(&q_full[qs], (qi / SS::NQ) & 1, abort_flag, prm.status))) break;
        if (prm.rope) {
          for (int row = rt; row < PT * R; row += SS::NROPE) {
            const int pos = t * PT + row / R;
            if (pos < S)
              rope_row_inplace_f2<32, BF16>(q_s + qs * SS::Q_BYTES, row, cos_s + pos * SS::CS_STRIDE,
                                            sin_s + pos * SS::CS_STRIDE, prm.rope == kRopeRefRound);
          }
          fence_proxy_async_smem();
        }
        mbar_arrive(&q_ready[qs]);
        ++qi;
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int w = (warp - 6) >> 2;  // warpgroup 0: warps 6-9, 1: warps 10-13
    const int wq = warp & 3;        // TMEM lane quarter this warp may access
    const int r = wq * 32 + lane;   // tile row = TMEM lane
    const uint32_t t_lane = tmem + ((uint32_t)(wq * 32) << 16);
    const uint32_t t_s = t_lane + SS::TMEM_S + 192u * w;
    const uint32_t t_o = t_lane + SS::TMEM_O + 64u * w;
    const float c2 = prm.scale_log2;
    const float sd64 = prm.scale_div64;
    const int h = r % R;
    const int rowpos = r / R;
    uint32_t sph = 0;
    uint32_t done = 0;  // tiles of this warpgroup finished (selects O slot and phase)
    bool ok = true;

    // Epilogue of this warpgroup's k-th tile: O from its slot / row sum -> bf16 -> HBM.
    auto epilogue = [&](const Cursor& c, uint32_t k, float l) -> bool {
      const uint32_t slot = k & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&o_full[w * 2 + slot], (k >> 1) & 1u, abort_flag, prm.status)))
        return false;
      tc_fence_after();
      float o[32];
      tmem_ld32(t_o + 32u * slot, o);
      tc_fence_before();
      const int pos = c.t * PT + rowpos;
      if (r < PT * R && pos < S) {
        const int unit = blockIdx.x + c.lu * gridDim.x;
        const int b = unit / prm.Hkv;
        const int g = unit - b * prm.Hkv;
        const float inv = rcp_newton(l);
        typename E::T* orow = reinterpret_cast<typename E::T*>(prm.o) + (size_t)b * prm.o_sb +
                              (size_t)pos * prm.o_ss + (size_t)(g * R + h) * prm.o_sh;
#pragma unroll
        for (int cc = 0; cc < 32; cc += 8) {
          uint4 v;
          v.x = E::from_f2(o[cc + 0] * inv, o[cc + 1] * inv);
          v.y = E::from_f2(o[cc + 2] * inv, o[cc + 3] * inv);
          v.z = E::from_f2(o[cc + 4] * inv, o[cc + 5] * inv);
          v.w = E::from_f2(o[cc + 6] * inv, o[cc + 7] * inv);
          *reinterpret_cast<uint4*>(orow + cc) = v;
        }
      }
      return true;
    };

    Cursor prev{0, 0, -1};
    float l_prev = 0.f;
    for (Cursor cur{0, 0, 0}; cur.i < ntotal && ok; cur.next(ntiles)) {
      if (tile_wg(cur) != w) continue;
      const TileInfo T = tile_info(cur, pads_s, PT, S);
      const int pos = T.pos0 + rowpos;
      const bool valid_row = (r < PT * R) && (pos < S);
      const bool padded = pos < T.pad;
      const int lo = padded ? 0 : T.pad;
      const int hi = valid_row ? pos : -1;
      const bool tile_clean = T.pos0 >= T.pad;
      const int nc = T.nc;
      // Allowed keys of this row inside chunk ci as a 32-bit mask (bit j = key
      // kb0 + 32 ci + j): [lo, hi] clipped to the chunk.
      auto chunk_mask = [&](int ci) -> uint32_t {
        const int k0 = T.kb0 + 32 * ci;
        const int jlo = lo - k0, jhi = hi - k0;
        const uint32_t hm = jhi < 0 ? 0u : (jhi >= 31 ? 0xffffffffu : ((2u << jhi) - 1u));
        const uint32_t lm = jlo <= 0 ? 0xffffffffu : (jlo >= 32 ? 0u : (0xffffffffu << jlo));
        return hm & lm;
      };
      // Chunks inside [pad, pos0] of a tile without padded rows need no mask
      // for any row (warp-uniform test).
      auto chunk_clean = [&](int ci) -> bool {
        const int k0 = T.kb0 + 32 * ci;
        return tile_clean && k0 >= T.pad && k0 + 31 <= T.pos0;
      };

      // Warp-uniform wait outcome keeps the .sync.aligned TMEM accesses convergent.
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[w], sph, abort_flag, prm.status)))) break;
      sph ^= 1u;
      tc_fence_after();

      uint32_t ra[32], rb[32];
      // Pass 1: row maximum over the allowed keys; the next chunk's load is in
      // flight while a chunk is reduced.
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
      auto chunk_max = [&](const uint32_t (&u)[32], int ci) {
        if (chunk_clean(ci)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            mx0 = fmax3(mx0, __uint_as_float(u[j]), __uint_as_float(u[j + 1]));
            mx1 = fmax3(mx1, __uint_as_float(u[j + 2]), __uint_as_float(u[j + 3]));
          }
        } else {
          const uint32_t mk = chunk_mask(ci);
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            mx0 = fmaxf(mx0, ((mk >> j) & 1u) ? __uint_as_float(u[j]) : -INFINITY);
            mx1 = fmaxf(mx1, ((mk >> (j + 1)) & 1u) ? __uint_as_float(u[j + 1]) : -INFINITY);
            mx2 = fmaxf(mx2, ((mk >> (j + 2)) & 1u) ? __uint_as_float(u[j + 2]) : -INFINITY);
            mx3 = fmaxf(mx3, ((mk >> (j + 3)) & 1u) ? __uint_as_float(u[j + 3]) : -INFINITY);
          }
        }
      };
      tmem_ld32_async(t_s, ra);
      for (int ci = 0; ci < nc; ci += 2) {
        tmem_wait_ld(ra);
        if (ci + 1 < nc) tmem_ld32_async(t_s + 32 * (ci + 1), rb);
        chunk_max(ra, ci);
        if (ci + 1 < nc) {
          tmem_wait_ld(rb);
          if (ci + 2 < nc) tmem_ld32_async(t_s + 32 * (ci + 2), ra);
          chunk_max(rb, ci + 1);
        }
      }
      const float bmax = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
      // t = s * c2 - m; masked keys get -inf.  Fully padded rows use c2 = m = 0
      // (weight 1) on the keys of the reference's top 64-wide -1e9 band
      // (s >= thr) and drop the rest (weights <= e^-64 there); only warps
      // holding such rows pay for the threshold test.
      const float m = (padded || bmax == -INFINITY) ? 0.f : bmax * c2;
      const float cr = padded ? 0.f : c2;
      const float thr = padded ? padded_band_floor(bmax, sd64) : -INFINITY;
      const bool warp_padded = __any_sync(0xffffffffu, padded);

      // Pass 2: P = exp2(t), packed bf16 pairs stored over the S columns just
      // read; row sum in fp32.
      float l0 = 0.f, l1 = 0.f, l2 = 0.f, l3 = 0.f;
      float2 l01 = make_float2(0.f, 0.f), l23 = make_float2(0.f, 0.f);  // clean chunks
      const float2 c2v = make_float2(c2, c2), nmv = make_float2(-m, -m);
      auto chunk_p = [&](const uint32_t (&u)[32], int ci) {
        uint32_t pk[16];
        if (chunk_clean(ci)) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            // two lanes of scale-and-shift / row-sum work per f32x2 instruction
            const float2 t01 = ffma2(make_float2(__uint_as_float(u[j]), __uint_as_float(u[j + 1])), c2v, nmv);
            const float2 t23 = ffma2(make_float2(__uint_as_float(u[j + 2]), __uint_as_float(u[j + 3])), c2v, nmv);
            const float2 p01 = make_float2(ex2_approx(t01.x), ex2_approx(t01.y));
            const float2 p23 = make_float2(ex2_approx(t23.x), ex2_approx(t23.y));
            l01 = fadd2(l01, p01);
            l23 = fadd2(l23, p23);
            pk[j >> 1] = E::from_f2(p01.x, p01.y);
            pk[(j >> 1) + 1] = E::from_f2(p23.x, p23.y);
          }
        } else if (warp_padded) {
          const uint32_t mk = chunk_mask(ci);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float s0 = __uint_as_float(u[j]), s1 = __uint_as_float(u[j + 1]);
            const float t0 = (((mk >> j) & 1u) && s0 >= thr) ? fmaf(s0, cr, -m) : -INFINITY;
            const float t1 = (((mk >> (j + 1)) & 1u) && s1 >= thr) ? fmaf(s1, cr, -m) : -INFINITY;
            const float p0 = ex2_approx(t0), p1 = ex2_approx(t1);
            if (j & 2) {
              l2 += p0;
              l3 += p1;
            } else {
              l0 += p0;
              l1 += p1;
            }
            pk[j >> 1] = E::from_f2(p0, p1);
          }
        } else {
          const uint32_t mk = chunk_mask(ci);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float s0 = __uint_as_float(u[j]), s1 = __uint_as_float(u[j + 1]);
            const float t0 = ((mk >> j) & 1u) ? fmaf(s0, cr, -m) : -INFINITY;
            const float t1 = ((mk >> (j + 1)) & 1u) ? fmaf(s1, cr, -m) : -INFINITY;
            const float p0 = ex2_approx(t0), p1 = ex2_approx(t1);
            if (j & 2) {
              l2 += p0;
              l3 += p1;
            } else {
              l0 += p0;
              l1 += p1;
            }
            pk[j >> 1] = E::from_f2(p0, p1);
          }
        }
        tmem_st16(t_s + 16 * ci, pk);
      };
      tmem_ld32_async(t_s, ra);
      for (int ci = 0; ci < nc; ci += 2) {
        tmem_wait_ld(ra);
        if (ci + 1 < nc) tmem_ld32_async(t_s + 32 * (ci + 1), rb);
        chunk_p(ra, ci);
        if (ci + 1 < nc) {
          tmem_wait_ld(rb);
          if (ci + 2 < nc) tmem_ld32_async(t_s + 32 * (ci + 2), ra);
          chunk_p(rb, ci + 1);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[w]);
      // While the tensor core runs this tile's P V and the next S, finish the
      // previous tile of this warpgroup (other O slot).
      if (prev.i >= 0 && !(ok = epilogue(prev, done - 1, l_prev))) break;
      prev = cur;
      l_prev = ((l0 + l1) + (l2 + l3)) + ((l01.x + l01.y) + (l23.x + l23.y));
      ++done;
    }
    if (ok && prev.i >= 0) epilogue(prev, done - 1, l_prev);
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, SS::TMEM_COLS);
  }
}

cudaError_t launch_prefill_short_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                       const PrefillParams& prm, bool bf16, int n_units, int grid,
                                       cudaStream_t stream) {
  if ((n_units + grid - 1) / grid > SS::MAX_UNITS) return cudaErrorInvalidValue;
  auto kfn = bf16 ? dt_prefill_short_kernel<true> : dt_prefill_short_kernel<false>;
  cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(kfn), SS::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  kfn<<<grid, SS::NTHREADS, SS::SMEM_BYTES, stream>>>(q, k, v, prm, n_units);
  return cudaGetLastError();
}

}  // namespace dtk
