// Fused RMSNorm + Q/K/V projection, sm_100a.
//
// Replaces the block's input_layernorm feeding the attention's projections
// (model/model_decision_transformer.py:76-86 RMSNorm, :296 call site,
// :175-177 q_proj / k_proj / v_proj):
//
//   y = RMSNorm(x) = w_norm * x * rsqrt(mean(x^2) + eps)
//   [q | k | v] = y @ [Wq; Wk; Wv]^T
//               = rsqrt(mean(x^2) + eps) * (x @ W'^T),  W' = [Wq; Wk; Wv] * diag(w_norm)
//
// so the GEMM runs on the raw residual stream x and the per-row scale is
// applied in the epilogue.  One CTA computes a 128-row x NCTA-column output
// tile: warp 0 streams 64-wide K chunks of x and W' with TMA (128B swizzle),
// warp 1 issues tcgen05.mma into TMEM (fp32), warps 2-5 accumulate each row's
// sum of squares from the same shared-memory x tiles during the main loop
// and run the epilogue (TMEM -> scale -> bf16 -> HBM).  Output row layout is
// the fused [q | k | v] of the projections: a [tokens, (Hq + 2 Hkv) * D] row
// is the [B, S, Hq + 2 Hkv, D] view the attention kernels take directly.
// With rope_cols > 0 the epilogue also applies the rotate-half RoPE to the q
// and k heads (apply_rotary_pos_emb, :103-117), so the attention kernels can
// take them pre-rotated.  The persistent kernel also runs the block's two
// residual GEMMs without a norm (resid mode): y += x @ W^T in place, the
// residual read in the epilogue and the sum rounded once (o_proj + residual,
// :247-248 and :300; down_proj + residual, :271 and :303).
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kGemmThreads = 192;
constexpr int kKC = 64;  // K elements per pipeline stage (one 128-byte swizzle atom)

template <int NCTA>
struct GemmShape {
  static constexpr int NSUB = NCTA <= 256 ? NCTA : NCTA / 2;  // columns per MMA instruction
  static constexpr int NMMA = NCTA / NSUB;
  static constexpr int A_BYTES = 128 * kKC * 2;
  static constexpr int B_BYTES = NCTA * kKC * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int NSTAGE = (200 * 1024) / STAGE < 6 ? (200 * 1024) / STAGE : 6;
  static constexpr int OFF_BAR = NSTAGE * STAGE;
  static constexpr int SMEM = OFF_BAR + (2 * NSTAGE + 2) * 8 + 16 + 1024;
  static constexpr uint32_t TMEM_COLS = NCTA <= 256 ? 256 : 512;
  static_assert(NSUB % 16 == 0 && NSUB <= 256, "MMA N");
};

}  // namespace

// Rotate-half RoPE of one head held in v[lo0, lo0 + 2 HALF):
//   y[d] = x[d] cos[d] - x[d + HALF] sin[d],  y[d + HALF] = x[d + HALF] cos[d + HALF] + x[d] sin[d + HALF]
template <int HALF>
__device__ __forceinline__ void rope_pairs(float (&v)[64], int lo0, const float* crow, const float* srow) {
#pragma unroll
  for (int d = 0; d < HALF; d += 4) {
    const float4 ca = *reinterpret_cast<const float4*>(crow + d);
    const float4 cb = *reinterpret_cast<const float4*>(crow + d + HALF);
    const float4 sa = *reinterpret_cast<const float4*>(srow + d);
    const float4 sb = *reinterpret_cast<const float4*>(srow + d + HALF);
    const float cav[4] = {ca.x, ca.y, ca.z, ca.w}, cbv[4] = {cb.x, cb.y, cb.z, cb.w};
    const float sav[4] = {sa.x, sa.y, sa.z, sa.w}, sbv[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float x0 = v[lo0 + d + e], x1 = v[lo0 + d + e + HALF];
      v[lo0 + d + e] = x0 * cav[e] - x1 * sav[e];
      v[lo0 + d + e + HALF] = x1 * cbv[e] + x0 * sbv[e];
    }
  }
}

// The same rotation with duplicated-half tables (cos[d] == cos[d + HALF], the
// rotate-half layout) staged as fp16 in shared memory: a 128-byte row holds
// cos[0, HALF) at halves [0, HALF) and sin[0, HALF) at halves [32, 32 + HALF),
// its 16-byte pieces XOR-swizzled by (row & 7) so the 32 rows of a warp read
// without bank conflicts.
template <int HALF>
__device__ __forceinline__ void rope_pairs_tab(float (&v)[64], int lo0, const uint8_t* trow, int sw) {
  constexpr int NP = HALF / 8;  // 16-byte pieces per half table
  uint4 cp[NP], sp[NP];
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    cp[q] = *reinterpret_cast<const uint4*>(trow + ((q ^ sw) << 4));
    sp[q] = *reinterpret_cast<const uint4*>(trow + (((4 + q) ^ sw) << 4));
  }
#pragma unroll
  for (int q = 0; q < NP; ++q) {
    const uint32_t cw[4] = {cp[q].x, cp[q].y, cp[q].z, cp[q].w};
    const uint32_t sw4[4] = {sp[q].x, sp[q].y, sp[q].z, sp[q].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 c2 = __half22float2(*reinterpret_cast<const __half2*>(&cw[e]));
      const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(&sw4[e]));
      const int d = lo0 + q * 8 + 2 * e;
      const float x0 = v[d], x1 = v[d + HALF], y0 = v[d + 1], y1 = v[d + 1 + HALF];
      v[d] = x0 * c2.x - x1 * s2.x;
      v[d + HALF] = x1 * c2.x + x0 * s2.x;
      v[d + 1] = y0 * c2.y - y1 * s2.y;
      v[d + 1 + HALF] = y1 * c2.y + y0 * s2.y;
    }
  }
}

template <int NCTA>
__global__ void __launch_bounds__(kGemmThreads, 1)
    dt_rmsnorm_qkv_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                          const RmsQkvParams p) {
  using SH = GemmShape<NCTA>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* empty = full + SH::NSTAGE;
  uint64_t* acc_full = empty + SH::NSTAGE;
  uint64_t* drain = acc_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.x * 128;
  const int n0 = blockIdx.y * NCTA;
  const int nk = (p.K + kKC - 1) / kKC;

  if (tid == 0) {
    for (int s = 0; s < SH::NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 128);  // the MMA commit + the 128 sum-of-squares threads
    }
    mbar_init(acc_full, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmW);
      int issued = 0;
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % SH::NSTAGE;
        if (!mbar_wait(&empty[s], ((kc / SH::NSTAGE) & 1) ^ 1, abort_flag, p.status)) break;
        uint8_t* st = smem + s * SH::STAGE;
        mbar_arrive_expect_tx(&full[s], (uint32_t)SH::STAGE);
        tma_load_2d(st, &tmX, &full[s], kc * kKC, m0);
#pragma unroll
        for (int j = 0; j < SH::NMMA; ++j)
          tma_load_2d(st + SH::A_BYTES + j * SH::NSUB * 128, &tmW, &full[s], kc * kKC, n0 + j * SH::NSUB);
        ++issued;
      }
      if (*abort_flag) {
        for (int s = 0; s < SH::NSTAGE; ++s) {
          const int uses = issued / SH::NSTAGE + (s < issued % SH::NSTAGE ? 1 : 0);
          if (uses > 0) mbar_wait(&full[s], (uses - 1) & 1, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(p.bf16 != 0, 128, SH::NSUB, 0, 0);
      for (int kc = 0; kc < nk; ++kc) {
        const int s = kc % SH::NSTAGE;
        if (!mbar_wait(&full[s], (kc / SH::NSTAGE) & 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + s * SH::STAGE);
        const uint64_t ad = umma_smem_desc(a, 16, 1024, kSw128);
#pragma unroll
        for (int j = 0; j < SH::NMMA; ++j) {
          const uint64_t bd = umma_smem_desc(a + SH::A_BYTES + j * SH::NSUB * 128, 16, 1024, kSw128);
#pragma unroll
          for (int kk = 0; kk < kKC / 16; ++kk)  // 32 bytes per K step inside the 128-byte atom
            umma_f16_ss(tmem + j * SH::NSUB, ad + 2 * kk, bd + 2 * kk, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(acc_full);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else {
    // Warps 2-5: row sums of squares during the main loop, then the epilogue.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // tile row = TMEM lane
    float ss[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    for (int kc = 0; kc < nk && ok; ++kc) {
      const int s = kc % SH::NSTAGE;
      if (!(ok = mbar_wait(&full[s], (kc / SH::NSTAGE) & 1, abort_flag, p.status))) break;
      // The 128-byte row r of the swizzled x tile holds 64 elements in permuted
      // 16-byte chunks; a sum of squares does not care about the order.
      const uint4* row = reinterpret_cast<const uint4*>(smem + s * SH::STAGE + r * 128);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 u = row[c];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = p.bf16 ? Elem<true>::to_f2(w[i]) : Elem<false>::to_f2(w[i]);
          ss[i] = fmaf(f.x, f.x, fmaf(f.y, f.y, ss[i]));
        }
      }
      mbar_arrive(&empty[s]);
    }
    ok = __all_sync(0xffffffffu, ok && mbar_wait(acc_full, 0, abort_flag, p.status));
    if (ok) {
      tc_fence_after();
      const float rs = p.nonorm ? 1.f : rsqrtf(((ss[0] + ss[1]) + (ss[2] + ss[3])) / (float)p.K + p.eps);
      const int row_g = m0 + r;
      // RoPE table row of this token (rows are [batch, seq_len] flattened).
      const int pos = p.rope_cols > 0 ? row_g % p.seq_len : 0;
      const float* crow = p.cos + (size_t)pos * p.cs_stride;
      const float* srow = p.sin + (size_t)pos * p.cs_stride;
      // 64 columns at a time: one head of 64 or two of 32, both halves of
      // every rotate-half pair in registers.
      for (int c = 0; c < NCTA; c += 64) {
        float v[64];
        tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + c, *reinterpret_cast<float(*)[32]>(&v[0]));
        tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + c + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] *= rs;
        if (n0 + c < p.rope_cols && row_g < p.M) {
          if (p.head_dim == 64)
            rope_pairs<32>(v, 0, crow, srow);
          else {
            rope_pairs<16>(v, 0, crow, srow);
            if (n0 + c + 32 < p.rope_cols) rope_pairs<16>(v, 32, crow, srow);  // second head may be a v head
          }
        }
        if (row_g < p.M) {
          uint8_t* yrow = reinterpret_cast<uint8_t*>(p.y) + ((size_t)row_g * p.y_stride + n0 + c) * 2;
#pragma unroll
          for (int c8 = 0; c8 < 64; c8 += 8) {
            if (n0 + c + c8 + 8 > p.N) break;
            uint4 o;
            if (p.bf16) {
              o.x = Elem<true>::from_f2(v[c8], v[c8 + 1]);
              o.y = Elem<true>::from_f2(v[c8 + 2], v[c8 + 3]);
              o.z = Elem<true>::from_f2(v[c8 + 4], v[c8 + 5]);
              o.w = Elem<true>::from_f2(v[c8 + 6], v[c8 + 7]);
            } else {
              o.x = Elem<false>::from_f2(v[c8], v[c8 + 1]);
              o.y = Elem<false>::from_f2(v[c8 + 2], v[c8 + 3]);
              o.z = Elem<false>::from_f2(v[c8 + 4], v[c8 + 5]);
              o.w = Elem<false>::from_f2(v[c8 + 6], v[c8 + 7]);
            }
            *reinterpret_cast<uint4*>(yrow + c8 * 2) = o;
          }
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

// Persistent variant for wide outputs (N > 512, e.g. hidden 768 with 12/4
// heads: N = 1280): a CTA owns 128-row blocks of x and runs all of a block's
// 256-column tiles back to back, so the block's x rows stay hot in L2 and its
// row scale is computed once.  The accumulator is double-buffered in TMEM (2 x
// 256 columns): the epilogue of one tile overlaps the main loop of the next.
// Warps: 0 TMA producer (also prefetches the next row block of x into L2),
// 1 TMEM owner + MMA issuer, 2-5 epilogue (row scale, RoPE or SwiGLU, 16-bit
// slices stored by TMA), 6-9 row sums of squares from the staged x slices of
// each block's first tile (they take part in the ring's stage release).
namespace {
constexpr int kPersistThreads = 320;
constexpr int kPN = 256;        // columns per tile
// 64 K elements per stage (128-byte rows, 128-byte swizzle), 4 stages.  (32-wide
// stages x 8 keep the same bytes in flight with twice the TMA requests; they
// measured slower.)
constexpr int kPKC = kPersistKChunk;
constexpr int kPStages = kPKC == 64 ? 4 : 8;
static_assert(kPKC == 32 || kPKC == 64, "persistent K chunk");
struct PShape {
  static constexpr int RB = kPKC * 2;  // bytes per staged row
  static constexpr uint32_t LAYOUT = kPKC == 64 ? kSw128 : kSw64;
  static constexpr int A_BYTES = 128 * kPKC * 2;
  static constexpr int B_BYTES = kPN * kPKC * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int OFF_ST = kPStages * STAGE;            // output staging: [4 warps][32 rows][64 cols]
  static constexpr int ST_WARP = 32 * 64 * 2;                // one warp's slice (4 swizzle atoms)
  static constexpr int OFF_TAB = OFF_ST + 4 * ST_WARP;       // RoPE tables: [4 warps][32 rows][128 B]
  static constexpr int TAB_WARP = 32 * 128;
  static constexpr int OFF_SS = OFF_TAB + 4 * TAB_WARP;      // [2][128] floats
  static constexpr int OFF_BAR = OFF_SS + 2 * 128 * 4;
  // full[S], empty[S], acc_full[2], acc_empty[2], ss_full[2], ss_empty[2], drain, res_full[4]
  static constexpr int NBAR = 2 * kPStages + 9 + 4;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
};
}  // namespace

__global__ void __launch_bounds__(kPersistThreads, 1)
    dt_rmsnorm_qkv_persist_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                                  const __grid_constant__ CUtensorMap tmY, const RmsQkvParams p) {
  using SH = PShape;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* ss_s = reinterpret_cast<float*>(smem + SH::OFF_SS);
  uint8_t* st_s = smem + SH::OFF_ST;
  uint8_t* tab_s = smem + SH::OFF_TAB;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* empty = full + kPStages;
  uint64_t* acc_full = empty + kPStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* ss_full = acc_empty + 2;
  uint64_t* ss_empty = ss_full + 2;
  uint64_t* drain = ss_empty + 2;
  uint64_t* res_full = drain + 1;  // [epilogue warp]: residual slice landed (resid mode)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(res_full + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nk = (p.K + kPKC - 1) / kPKC;
  const int nrb = (p.M + 127) / 128;
  const int nt = (p.N + kPN - 1) / kPN;

  if (tid == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      // MMA commit + one arrival per sum-of-squares warp; without a norm (resid /
      // nonorm) those warps read no stage, so the commit alone frees it.
      mbar_init(&empty[s], (p.resid || p.nonorm) ? 1 : 5);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], 4);  // one arrival per epilogue warp
      mbar_init(&ss_full[j], 4);    // one per sum-of-squares warp
      mbar_init(&ss_empty[j], 4);   // one per epilogue warp
    }
    mbar_init(drain, 1);
    for (int j = 0; j < 4; ++j) mbar_init(&res_full[j], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmW);
      if (p.resid) prefetch_tmap(&tmY);
      int cnt = 0;
      bool ok = true;
      for (int rb = blockIdx.x; rb < nrb && ok; rb += gridDim.x)
        for (int ct = 0; ct < nt && ok; ++ct)
          for (int kc = 0; kc < nk; ++kc, ++cnt) {
            const int s = cnt % kPStages;
            // Residual mode: this tile's residual into L2 while its K chunks
            // stream, ahead of the epilogue's TMA loads of it.
            if (p.resid && kc == 0)
              for (int q = 0; q < 16; ++q) tma_prefetch_l2_2d(&tmY, ct * kPN + (q & 3) * 64, rb * 128 + (q >> 2) * 32);
            // While the second column tile of a row block streams, pull this
            // CTA's next row block of x from HBM into L2, so that its first
            // tile (which reads x) runs at the L2 rate of the others.
            if (ct == (nt > 1 ? 1 : 0) && rb + (int)gridDim.x < nrb) {
              tma_prefetch_l2_2d(&tmX, kc * kPKC, (rb + (int)gridDim.x) * 128);
              if (kc == 0 && p.rope_cols > 0) {
                // and the RoPE table rows the next block's epilogue stages
                const int rows = p.seq_len < 128 ? p.seq_len : 128;
                const int p0 = p.seq_len < 128 ? 0 : ((rb + (int)gridDim.x) * 128) % p.seq_len;
                const int n1 = rows < p.seq_len - p0 ? rows : p.seq_len - p0;
                // (n rows end at the last row's head_dim entries: never past the table)
                const uint32_t rowb = (uint32_t)p.cs_stride * 4u, tail = (uint32_t)p.head_dim * 4u;
                bulk_prefetch_l2(p.cos + (size_t)p0 * p.cs_stride, (uint32_t)(n1 - 1) * rowb + tail);
                bulk_prefetch_l2(p.sin + (size_t)p0 * p.cs_stride, (uint32_t)(n1 - 1) * rowb + tail);
                if (n1 < rows) {
                  bulk_prefetch_l2(p.cos, (uint32_t)(rows - n1 - 1) * rowb + tail);
                  bulk_prefetch_l2(p.sin, (uint32_t)(rows - n1 - 1) * rowb + tail);
                }
              }
            }
            if (!(ok = mbar_wait(&empty[s], ((cnt / kPStages) & 1) ^ 1, abort_flag, p.status))) break;
            uint8_t* st = smem + s * SH::STAGE;
            mbar_arrive_expect_tx(&full[s], (uint32_t)SH::STAGE);
            tma_load_2d(st, &tmX, &full[s], kc * kPKC, rb * 128);
            tma_load_2d(st + SH::A_BYTES, &tmW, &full[s], kc * kPKC, ct * kPN);
          }
      if (!ok) {
        for (int s = 0; s < kPStages; ++s) {
          const int uses = cnt / kPStages + (s < cnt % kPStages ? 1 : 0);
          if (uses > 0) mbar_wait(&full[s], (uses - 1) & 1, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(p.bf16 != 0, 128, kPN, 0, 0);
      int cnt = 0, tc = 0;
      bool ok = true;
      for (int rb = blockIdx.x; rb < nrb && ok; rb += gridDim.x)
        for (int ct = 0; ct < nt && ok; ++ct, ++tc) {
          const int buf = tc & 1;
          if (!(ok = mbar_wait(&acc_empty[buf], ((tc >> 1) & 1) ^ 1, abort_flag, p.status))) break;
          for (int kc = 0; kc < nk; ++kc, ++cnt) {
            const int s = cnt % kPStages;
            if (!(ok = mbar_wait(&full[s], (cnt / kPStages) & 1, abort_flag, p.status))) break;
            tc_fence_after();
            const uint32_t a = smem_u32(smem + s * SH::STAGE);
            const uint64_t ad = umma_smem_desc(a, 16, 8 * SH::RB, SH::LAYOUT);
            const uint64_t bd = umma_smem_desc(a + SH::A_BYTES, 16, 8 * SH::RB, SH::LAYOUT);
#pragma unroll
            for (int kk = 0; kk < kPKC / 16; ++kk)  // 32 bytes per K step inside the swizzle atom
              umma_f16_ss(tmem + buf * kPN, ad + 2 * kk, bd + 2 * kk, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&empty[s]);
          }
          if (ok) umma_commit(&acc_full[buf]);
        }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else if (warp < 6) {
    // Epilogue: TMEM -> row scale -> (RoPE) -> 16-bit -> HBM.
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // tile row = TMEM lane
    const uint32_t t_row = tmem + ((uint32_t)(wq * 32) << 16);
    int tc = 0, bc = 0, sc = 0;  // tiles, row blocks, staged output chunks
    uint32_t rph = 0;            // residual slices loaded (resid mode)
    bool ok = true;
    for (int rb = blockIdx.x; rb < nrb && ok; rb += gridDim.x, ++bc) {
      const int sb = bc & 1;
      // Stage this warp's 32 table rows once per row block (coalesced reads,
      // fp16), before waiting for the block's row sums: the tables do not
      // depend on them, so this overlaps the block's first tile in the MMA.
      // Tables whose halves are not duplicated keep the direct path.
      // 16-byte loads: lane = (row of a group, float4 of a half row), 4 or 8
      // rows per warp instruction, 4 rows per lane in flight per batch; the
      // pieces go to shared memory as 8-byte stores.
      bool tab_ok = false;
      if (p.rope_cols > 0) {
        const int half = p.head_dim >> 1;   // 16 or 32
        const int qb = half == 32 ? 3 : 2;  // log2(float4s per half row)
        const int q = lane & ((1 << qb) - 1), rsub = lane >> qb, rstep = 32 >> qb;
        const int pos0 = (rb * 128 + wq * 32) % p.seq_len;
        bool dup = true;
        for (int j0 = 0; j0 < 32 / rstep; j0 += 4) {
          float4 cl[4], ch[4], sl[4], sh[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            int pi = pos0 + (j0 + u) * rstep + rsub;
            while (pi >= p.seq_len) pi -= p.seq_len;
            const float4* cr = reinterpret_cast<const float4*>(p.cos + (size_t)pi * p.cs_stride) + q;
            const float4* sr = reinterpret_cast<const float4*>(p.sin + (size_t)pi * p.cs_stride) + q;
            cl[u] = __ldg(cr);
            ch[u] = __ldg(cr + (half >> 2));
            sl[u] = __ldg(sr);
            sh[u] = __ldg(sr + (half >> 2));
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int i = (j0 + u) * rstep + rsub;  // row of the warp slice
            dup = dup && cl[u].x == ch[u].x && cl[u].y == ch[u].y && cl[u].z == ch[u].z && cl[u].w == ch[u].w &&
                  sl[u].x == sh[u].x && sl[u].y == sh[u].y && sl[u].z == sh[u].z && sl[u].w == sh[u].w;
            uint8_t* trow = tab_s + wq * SH::TAB_WARP + i * 128;
            const int sw = i & 7, off = (q & 1) * 8;
            const __half2 c01 = __floats2half2_rn(cl[u].x, cl[u].y), c23 = __floats2half2_rn(cl[u].z, cl[u].w);
            const __half2 s01 = __floats2half2_rn(sl[u].x, sl[u].y), s23 = __floats2half2_rn(sl[u].z, sl[u].w);
            // halves 4q..4q+3 of the cos table (pieces 0..3) and of the sin table (4..7)
            *reinterpret_cast<uint2*>(trow + (((q >> 1) ^ sw) << 4) + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&c01), *reinterpret_cast<const uint32_t*>(&c23));
            *reinterpret_cast<uint2*>(trow + (((4 + (q >> 1)) ^ sw) << 4) + off) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&s01), *reinterpret_cast<const uint32_t*>(&s23));
          }
        }
        tab_ok = __all_sync(0xffffffffu, dup);
        __syncwarp();
      }
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&ss_full[sb], (bc >> 1) & 1, abort_flag, p.status)))) break;
      const float rs = (p.resid || p.nonorm) ? 1.f : rsqrtf(ss_s[sb * 128 + r] / (float)p.K + p.eps);
      const int row_g = rb * 128 + r;
      const int pos = p.rope_cols > 0 ? row_g % p.seq_len : 0;
      const float* crow = p.cos + (size_t)pos * p.cs_stride;
      const float* srow = p.sin + (size_t)pos * p.cs_stride;
      const uint8_t* my_tab = tab_s + wq * SH::TAB_WARP + lane * 128;
      for (int ct = 0; ct < nt && ok; ++ct, ++tc) {
        const int buf = tc & 1;
        // (resid mode waits for the accumulator after requesting its first residual slice)
        if (!p.resid) {
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (tc >> 1) & 1, abort_flag, p.status))))
            break;
          tc_fence_after();
        }
        const int n0 = ct * kPN;
        if (p.swiglu) {
          // Column pairs (gate block, up block) of 64: one 64-column output
          // slice per pair, at output column (n0 + c) / 2.
          for (int c = 0; c < kPN && n0 + c < p.N; c += 128) {
            uint8_t* stb = st_s + wq * SH::ST_WARP;
            if (lane == 0 && sc >= 1) bulk_wait_read<0>();
            __syncwarp();
#pragma unroll
            for (int hh = 0; hh < 64; hh += 32) {
              float gv[32], uv[32];
              tmem_ld32(t_row + buf * kPN + c + hh, gv);
              tmem_ld32(t_row + buf * kPN + c + 64 + hh, uv);
              // silu(rs g) * (rs u) = rs^2 g u / (1 + 2^(-rs log2(e) g)), two
              // lanes per f32x2 instruction, exp2 and the quotient approximate
              // (the result is rounded to 16 bits).
              const float2 na2 = make_float2(-rs * 1.4426950408889634f, -rs * 1.4426950408889634f);
              const float2 rs2 = make_float2(rs * rs, rs * rs), one2 = make_float2(1.f, 1.f);
#pragma unroll
              for (int i = 0; i < 32; i += 2) {
                const float2 g2 = make_float2(gv[i], gv[i + 1]);
                const float2 t = fmul2(g2, na2);
                const float2 d = fadd2(make_float2(ex2_approx(t.x), ex2_approx(t.y)), one2);
                const float2 gu = fmul2(fmul2(g2, make_float2(uv[i], uv[i + 1])), rs2);
                gv[i] = __fdividef(gu.x, d.x);
                gv[i + 1] = __fdividef(gu.y, d.y);
              }
#pragma unroll
              for (int c8 = 0; c8 < 32; c8 += 8) {
                uint4 o;
                if (p.bf16) {
                  o.x = Elem<true>::from_f2(gv[c8], gv[c8 + 1]);
                  o.y = Elem<true>::from_f2(gv[c8 + 2], gv[c8 + 3]);
                  o.z = Elem<true>::from_f2(gv[c8 + 4], gv[c8 + 5]);
                  o.w = Elem<true>::from_f2(gv[c8 + 6], gv[c8 + 7]);
                } else {
                  o.x = Elem<false>::from_f2(gv[c8], gv[c8 + 1]);
                  o.y = Elem<false>::from_f2(gv[c8 + 2], gv[c8 + 3]);
                  o.z = Elem<false>::from_f2(gv[c8 + 4], gv[c8 + 5]);
                  o.w = Elem<false>::from_f2(gv[c8 + 6], gv[c8 + 7]);
                }
                *reinterpret_cast<uint4*>(stb + lane * 128 + ((((hh + c8) >> 3) ^ (lane & 7)) << 4)) = o;
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmY, stb, (n0 + c) >> 1, rb * 128 + wq * 32);
              bulk_commit();
            }
            ++sc;
          }
        } else
        if (p.resid) {
          // y = residual + x W^T in fp32, rounded once (a GEMM with the residual
          // as its accumulator input), in place.  Each 32 x 64 residual slice is
          // brought into this warp's 4 KB buffer (the RoPE-table region, unused
          // here) by TMA one slice ahead: the first before the accumulator wait,
          // the next as soon as the current one is in registers.
          uint8_t* resb = tab_s + wq * SH::TAB_WARP;
          const int ncs = (p.N - n0) < kPN ? (p.N - n0) / 64 : kPN / 64;  // 64-column slices of this tile
          for (int c = 0; c < ncs && ok; ++c) {
            if (c == 0 && lane == 0) {
              mbar_arrive_expect_tx(&res_full[wq], 32 * 128);
              tma_load_2d(resb, &tmY, &res_full[wq], n0, rb * 128 + wq * 32);
            }
            if (c == 0 && !(ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (tc >> 1) & 1, abort_flag,
                                                                   p.status))))
              break;
            if (c == 0) tc_fence_after();
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(&res_full[wq], rph & 1u, abort_flag, p.status)))) break;
            ++rph;
            uint4 res[8];
#pragma unroll
            for (int q8 = 0; q8 < 8; ++q8)
              res[q8] = *reinterpret_cast<const uint4*>(resb + lane * 128 + ((q8 ^ (lane & 7)) << 4));
            fence_proxy_async_smem();
            __syncwarp();
            if (c + 1 < ncs && lane == 0) {
              mbar_arrive_expect_tx(&res_full[wq], 32 * 128);
              tma_load_2d(resb, &tmY, &res_full[wq], n0 + (c + 1) * 64, rb * 128 + wq * 32);
            }
            uint8_t* stb = st_s + wq * SH::ST_WARP;
            if (lane == 0 && sc >= 1) bulk_wait_read<0>();  // the previous copy has read the slice
            __syncwarp();
#pragma unroll
            for (int hh = 0; hh < 64; hh += 32) {
              float v[32];
              tmem_ld32(t_row + buf * kPN + c * 64 + hh, v);
#pragma unroll
              for (int q8 = 0; q8 < 4; ++q8) {
                const uint4 rq = res[(hh >> 3) + q8];
                const uint32_t w4[4] = {rq.x, rq.y, rq.z, rq.w};
                uint32_t o4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int i = q8 * 8 + 2 * e;
                  if (p.bf16) {
                    const float2 f = Elem<true>::to_f2(w4[e]);
                    o4[e] = Elem<true>::from_f2(v[i] + f.x, v[i + 1] + f.y);
                  } else {
                    const float2 f = Elem<false>::to_f2(w4[e]);
                    o4[e] = Elem<false>::from_f2(v[i] + f.x, v[i + 1] + f.y);
                  }
                }
                *reinterpret_cast<uint4*>(stb + lane * 128 + ((((hh >> 3) + q8) ^ (lane & 7)) << 4)) =
                    make_uint4(o4[0], o4[1], o4[2], o4[3]);
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmY, stb, n0 + c * 64, rb * 128 + wq * 32);
              bulk_commit();
            }
            ++sc;
          }
        } else
        for (int c = 0; c < kPN; c += 64) {
          float v[64];
          tmem_ld32(t_row + buf * kPN + c, *reinterpret_cast<float(*)[32]>(&v[0]));
          tmem_ld32(t_row + buf * kPN + c + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
#pragma unroll
          for (int i = 0; i < 64; ++i) v[i] *= rs;
          if (n0 + c < p.rope_cols && row_g < p.M) {
            if (tab_ok) {
              if (p.head_dim == 64)
                rope_pairs_tab<32>(v, 0, my_tab, lane & 7);
              else {
                rope_pairs_tab<16>(v, 0, my_tab, lane & 7);
                if (n0 + c + 32 < p.rope_cols) rope_pairs_tab<16>(v, 32, my_tab, lane & 7);
              }
            } else if (p.head_dim == 64) {
              rope_pairs<32>(v, 0, crow, srow);
            } else {
              rope_pairs<16>(v, 0, crow, srow);
              if (n0 + c + 32 < p.rope_cols) rope_pairs<16>(v, 32, crow, srow);  // second head may be a v head
            }
          }
          // Each warp stages its 32 x 64 slice in shared memory (128-byte
          // swizzle) and stores it with one TMA copy: whole rows per copy
          // instead of one line per thread.  Rows past M and columns past N
          // are clipped by the copy.
          uint8_t* stb = st_s + wq * SH::ST_WARP;
          if (lane == 0 && sc >= 1) bulk_wait_read<0>();  // the previous copy has read the slice
          __syncwarp();
#pragma unroll
          for (int c8 = 0; c8 < 64; c8 += 8) {
            uint4 o;
            if (p.bf16) {
              o.x = Elem<true>::from_f2(v[c8], v[c8 + 1]);
              o.y = Elem<true>::from_f2(v[c8 + 2], v[c8 + 3]);
              o.z = Elem<true>::from_f2(v[c8 + 4], v[c8 + 5]);
              o.w = Elem<true>::from_f2(v[c8 + 6], v[c8 + 7]);
            } else {
              o.x = Elem<false>::from_f2(v[c8], v[c8 + 1]);
              o.y = Elem<false>::from_f2(v[c8 + 2], v[c8 + 3]);
              o.z = Elem<false>::from_f2(v[c8 + 4], v[c8 + 5]);
              o.w = Elem<false>::from_f2(v[c8 + 6], v[c8 + 7]);
            }
            *reinterpret_cast<uint4*>(stb + lane * 128 + (((c8 >> 3) ^ (lane & 7)) << 4)) = o;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && n0 + c < p.N) {
            tma_store_2d(&tmY, stb, n0 + c, rb * 128 + wq * 32);
            bulk_commit();
          }
          ++sc;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ss_empty[sb]);
    }
    if (lane == 0) bulk_wait<0>();  // output copies complete before the CTA exits
    // A residual load issued before an abort lands before the CTA exits.
    if (p.resid && !ok && lane == 0) mbar_wait(&res_full[wq], rph & 1u, nullptr, nullptr);
  } else {
    // Row sums of squares of a 128-row block, read from the x chunks that the
    // ring stages for the block's first column tile (no extra pass over x).
    // These warps take part in every stage's release: empty[s] completes on
    // the MMA commit plus one arrival per warp.
    const int rr = (warp - 6) * 32 + lane;  // row of the block
    int cnt = 0, bc = 0;
    bool ok = true;
    if (p.resid || p.nonorm) {
      // No norm: only the per-block handshake the epilogue waits on (the value is unused).
      for (int rb = blockIdx.x; rb < nrb && ok; rb += gridDim.x, ++bc) {
        const int sb = bc & 1;
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&ss_empty[sb], ((bc >> 1) & 1) ^ 1, abort_flag, p.status))))
          break;
        ss_s[sb * 128 + rr] = 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ss_full[sb]);
      }
    } else
    for (int rb = blockIdx.x; rb < nrb && ok; rb += gridDim.x, ++bc) {
      const int sb = bc & 1;
      float ss0 = 0.f, ss1 = 0.f;
      for (int ct = 0; ct < nt && ok; ++ct) {
        for (int kc = 0; kc < nk; ++kc, ++cnt) {
          const int s = cnt % kPStages;
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(&full[s], (cnt / kPStages) & 1, abort_flag, p.status))))
            break;
          if (ct == 0) {
            // Row rr of the chunk is the RB bytes at rr * RB (the swizzle
            // permutes 16-byte pieces inside the row); start each lane at a
            // different piece to spread a quarter warp over the banks.
            constexpr int NPc = SH::RB / 16;
            const uint8_t* row = smem + s * SH::STAGE + rr * SH::RB;
#pragma unroll
            for (int q = 0; q < NPc; ++q) {
              const uint4 u = *reinterpret_cast<const uint4*>(row + (((q + lane) & (NPc - 1)) << 4));
              const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = p.bf16 ? Elem<true>::to_f2(w4[e]) : Elem<false>::to_f2(w4[e]);
                ss0 = fmaf(f.x, f.x, ss0);
                ss1 = fmaf(f.y, f.y, ss1);
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (ok && ct == 0) {
          // Publish once the epilogue has released this buffer (row block bc - 2).
          if (!(ok = __all_sync(0xffffffffu,
                                mbar_wait(&ss_empty[sb], ((bc >> 1) & 1) ^ 1, abort_flag, p.status))))
            break;
          ss_s[sb * 128 + rr] = ss0 + ss1;
          __syncwarp();
          if (lane == 0) mbar_arrive(&ss_full[sb]);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NCTA>
static cudaError_t launch_rq(const CUtensorMap& x, const CUtensorMap& w, const RmsQkvParams& p, cudaStream_t st) {
  using SH = GemmShape<NCTA>;
  auto k = dt_rmsnorm_qkv_kernel<NCTA>;
  cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(k), SH::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((p.M + 127) / 128, (p.N + NCTA - 1) / NCTA);
  k<<<grid, kGemmThreads, SH::SMEM, st>>>(x, w, p);
  return cudaGetLastError();
}

int rmsnorm_qkv_ncta(int N) {
  // Widest accumulator that covers N in one pass when possible (x read once);
  // wider outputs use the persistent kernel (0) with 256-column tiles.
  if (N <= 128) return 128;
  if (N <= 256) return 256;
  if (N <= 384) return 384;
  if (N <= 512) return 512;
  return 0;
}

cudaError_t launch_rmsnorm_qkv_sm100(const CUtensorMap& x, const CUtensorMap& w, const CUtensorMap& y,
                                     const RmsQkvParams& p, int ncta, int num_sms, cudaStream_t st) {
  if (ncta == 0) {
    auto k = dt_rmsnorm_qkv_persist_kernel;
    cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(k), PShape::SMEM);
    if (e != cudaSuccess) return e;
    const int nrb = (p.M + 127) / 128;
    const int grid = nrb < num_sms ? nrb : num_sms;
    k<<<grid, kPersistThreads, PShape::SMEM, st>>>(x, w, y, p);
    return cudaGetLastError();
  }
  switch (ncta) {
    case 128: return launch_rq<128>(x, w, p, st);
    case 256: return launch_rq<256>(x, w, p, st);
    case 384: return launch_rq<384>(x, w, p, st);
    case 512: return launch_rq<512>(x, w, p, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dtk
