// KV-cached decode attention for the Decision Transformer rollout, sm_100a.
//
// Replaces the cached ("slow") branch of DecisionTransformerAttention.forward
// (model/model_decision_transformer.py:179-191 and :225-245): the new tokens'
// K/V are rotated (RoPE, :180) and appended to the cache (the reference's
// torch.cat, :188-190; here an in-place write into a paged cache), then the
// new queries attend over all cached keys with the causal rule on the new
// columns (:230-237), the optional padding mask (:238-242) and an fp32
// softmax (:243).
//
// One CTA per (sample b, KV head g), 2 warps (small CTAs: ~21 KB of shared
// memory, so many units' copies are in flight per SM).  The cached K/V of the
// unit are staged into shared memory (swizzled) in blocks of up to KMAX keys;
// each warp takes half of the keys of a block and runs the
// R x Sn query rows (<= 16 per row group) against them with mma.sync
// m16n8k16 (bf16/fp16 in, fp32 accumulate) and an online softmax; the
// partial (max, sum, O) are merged through shared memory (split-K).  The
// copies of the cached prefix of the first block are issued before the new
// tokens are rotated and appended, and (for up to 16 new tokens) the new rows
// reach shared memory straight from registers, so a CTA waits for one round
// trip to HBM after reading its block table.
//
// Cache layout: k_pages / v_pages [num_pages, Hkv, page_size, D], a page
// holding page_size consecutive positions of one KV head contiguously;
// block_table [B, max_pages] maps position p of sample b to page
// block_table[b][p / page_size], slot p % page_size.  seq_lens[b] is the
// number of cached positions before this call; the kernel writes the new
// tokens at seq_lens[b] .. seq_lens[b] + Sn - 1 and leaves seq_lens alone.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kDecThreads = kDecodeThreads;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kKMax = kDecodeKeyBlock;  // keys staged per block
// New tokens staged from registers (more: re-read from the cache).  8 covers
// the rollout's 3 tokens per step and keeps a D = 32 CTA under 19 KB of shared
// memory: 12 CTAs per SM, as many as the registers allow.
constexpr int kSnSmem = 8;

template <int D>
struct DecShape {
  static constexpr int ROWB = D * 2;
  static constexpr int CH = D / 8;  // 16-byte chunks per row
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + kKMax * ROWB;
  static constexpr int OFF_Q = OFF_V + kKMax * ROWB;  // 16 rows
  static constexpr int OFF_KN = OFF_Q + 16 * ROWB;    // new keys (rotated), kSnSmem rows
  static constexpr int OFF_VN = OFF_KN + kSnSmem * ROWB;
  static constexpr int OFF_BT = OFF_VN + kSnSmem * ROWB;  // block-table row (vectorised front, <= one page per thread)
  static constexpr int OFF_BAR = OFF_BT + kDecThreads * 4;  // page-copy barrier
  // Base alignment of the K/V rows: one period of the TMA swizzle pattern
  // (64-byte rows: 512 B; 128-byte rows: 1024 B).
  static constexpr int ALIGN = ROWB == 64 ? 512 : 1024;
  static constexpr int SMEM = OFF_BAR + 16 + ALIGN;
  // Split-K partials [warps][16][D + 2] floats, over the K / V rows once a row
  // group's blocks are consumed.
  static constexpr int OFF_RED = OFF_K;
  static constexpr int RED_STRIDE = D + 2;
  static_assert((kDecWarps * 16 * RED_STRIDE + kDecWarps * 16) * 4 <= 2 * kKMax * ROWB, "partials fit over the K and V rows");
};

// Swizzled byte offset of 16-byte chunk c of row r (64-byte rows: XOR with
// (r >> 1) & 3; 128-byte rows: XOR with r & 7) -- conflict-free ldmatrix.
template <int D>
__device__ __forceinline__ uint32_t dswz(int r, int c) {
  if constexpr (D == 32) return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
  else return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Rotate-half RoPE of element pair (d, d + D/2) given fp32 inputs.
__device__ __forceinline__ void rope_pair(float x0, float x1, float c0, float s0, float c1, float s1, float& y0,
                                          float& y1) {
  y0 = x0 * c0 - x1 * s0;
  y1 = x1 * c1 + x0 * s1;
}

}  // namespace

template <int D, bool BF16>
__global__ void __launch_bounds__(kDecThreads) dt_decode_kernel(const __grid_constant__ CUtensorMap tmKp,
                                                                const __grid_constant__ CUtensorMap tmVp,
                                                                const DecodeParams p) {
  using SH = DecShape<D>;
  using E = Elem<BF16>;
  using T = typename E::T;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + SH::ALIGN - 1) &
                                             ~uintptr_t(SH::ALIGN - 1));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x / p.Hkv;
  const int g = blockIdx.x - b * p.Hkv;
  const int R = p.R, Sn = p.Sn;
  constexpr int HC = D / 16;  // 16-byte chunk pairs (d, d + D/2) per row
  uint8_t* ks = smem + SH::OFF_K;
  uint8_t* vs = smem + SH::OFF_V;
  uint8_t* qs = smem + SH::OFF_Q;
  uint8_t* kns = smem + SH::OFF_KN;
  uint8_t* vns = smem + SH::OFF_VN;
  int* bt_s = reinterpret_cast<int*>(smem + SH::OFF_BT);
  uint64_t* pbar = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  // Page copies by TMA (flag set by the host for page sizes 16..256 that
  // divide the key block): one bulk tensor copy per page and tensor.
  const bool tma = p.tma_pages != 0;
  if (tma && tid == 0) {
    mbar_init(pbar, 1);
    fence_mbar_init();
  }
  float* red = reinterpret_cast<float*>(smem + SH::OFF_RED);

  // Vectorised front (flag set by the host when the inputs allow it): every
  // input that does not depend on the cache length -- the length itself,
  // the block-table row, the new q / k / v rows and their RoPE table rows --
  // is requested in one round trip, 16 bytes per load.  Roles: threads
  // [0, 16 HC) one q chunk pair of the 16-row tile, then Sn HC k chunk pairs,
  // then Sn HC v chunk pairs.
  const bool vec = p.vec_front != 0;
  uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
  float4 cra[2], crb[2], sra[2], srb[2];
  bool have = false;  // this thread loaded a row chunk pair
  int role = 3, rrow = 0, rch = 0;  // 0 q, 1 k, 2 v, 3 none
  int btv = 0;
  if (vec) {
    const int e = tid;
    if (e < 16 * HC) {
      role = 0; rrow = e / HC; rch = e % HC;
    } else if (e < 16 * HC + Sn * HC) {
      role = 1; rrow = (e - 16 * HC) / HC; rch = (e - 16 * HC) % HC;
    } else if (e < 16 * HC + 2 * Sn * HC) {
      role = 2; rrow = (e - 16 * HC - Sn * HC) / HC; rch = (e - 16 * HC - Sn * HC) % HC;
    }
    const T* src = nullptr;  // stays null for rows past Sn * R: they are zero
    int tab_row = 0;
    if (role == 0 && rrow < Sn * R) {
      const int i = rrow / R, h = rrow - i * R;
      src = reinterpret_cast<const T*>(p.q) + (size_t)b * p.q_sb + (size_t)i * p.q_ss + (size_t)(g * R + h) * p.q_sh;
      tab_row = i;
    } else if (role == 1) {
      src = reinterpret_cast<const T*>(p.k_new) + (size_t)b * p.kn_sb + (size_t)rrow * p.kn_ss + (size_t)g * p.kn_sh;
      tab_row = rrow;
    } else if (role == 2) {
      src = reinterpret_cast<const T*>(p.v_new) + (size_t)b * p.vn_sb + (size_t)rrow * p.vn_ss + (size_t)g * p.vn_sh;
    }
    if (src) {
      have = true;
      xa = __ldg(reinterpret_cast<const uint4*>(src + rch * 8));
      xb = __ldg(reinterpret_cast<const uint4*>(src + (rch + HC) * 8));
      if (p.rope && role != 2) {
        const float* cr = p.cos + (size_t)tab_row * p.cs_stride + rch * 8;
        const float* sr = p.sin + (size_t)tab_row * p.cs_stride + rch * 8;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          cra[u] = __ldg(reinterpret_cast<const float4*>(cr) + u);
          crb[u] = __ldg(reinterpret_cast<const float4*>(cr + D / 2) + u);
          sra[u] = __ldg(reinterpret_cast<const float4*>(sr) + u);
          srb[u] = __ldg(reinterpret_cast<const float4*>(sr + D / 2) + u);
        }
      }
    }
    if (tid < p.max_pages) btv = p.block_table[(size_t)b * p.max_pages + tid];
  }
  const int L = p.seq_lens[b];
  const int kv_len = L + Sn;
  int pad = p.pad_len ? p.pad_len[b] : 0;
  pad = max(0, min(pad, kv_len));
  if (vec && tid < p.max_pages) bt_s[tid] = btv;
  if (vec) __syncthreads();
  const int32_t* bt = vec ? bt_s : p.block_table + (size_t)b * p.max_pages;

  // Device-side bounds: capacity and page ids of every position touched.
  bool bad = L < 0 || kv_len > p.max_pages * p.page_size || (p.rope && p.rope_abs && kv_len > p.cos_rows);
  if (!bad) {
    for (int pg = tid; pg * p.page_size < kv_len; pg += kDecThreads) {
      const int id = bt[pg];
      if (id < 0 || id >= p.num_pages) bad = true;
    }
  }
  if (__syncthreads_or(bad)) {
    if (tid == 0 && p.status) atomicExch(p.status, (int)kDevBadShape);
    return;
  }

  const bool new_in_smem = Sn <= kSnSmem;
  const size_t page_stride = (size_t)p.Hkv * p.page_size * D;  // elements per page
  auto cache_off = [&](int pos) -> size_t {
    return (size_t)bt[pos / p.page_size] * page_stride + ((size_t)g * p.page_size + pos % p.page_size) * D;
  };
  auto cos_row = [&](int i) -> const float* {
    return p.cos + (size_t)(p.rope_abs ? L + i : i) * p.cs_stride;
  };
  auto sin_row = [&](int i) -> const float* {
    return p.sin + (size_t)(p.rope_abs ? L + i : i) * p.cs_stride;
  };

  // Cached positions [kb, min(kb + nk, L)) of a block: whole pages by TMA
  // (rows past L are rewritten or zero-filled once the copy has landed), or
  // 16-byte copies page by page (a page holds its positions of one KV head
  // contiguously).
  auto stage_prefix = [&](int kb, int nk) {
    const int pend = kb + max(0, min(nk, L - kb));  // one past the last cached position
    if (tma) {
      if (tid == 0) {
        const int pg0 = kb / p.page_size, pg1 = (pend + p.page_size - 1) / p.page_size;
        mbar_arrive_expect_tx(pbar, (uint32_t)(2 * max(0, pg1 - pg0) * p.page_size * SH::ROWB));
        for (int pg = pg0; pg < pg1; ++pg) {
          const int row = (bt[pg] * p.Hkv + g) * p.page_size;
          const int key = pg * p.page_size - kb;
          tma_load_2d(ks + key * SH::ROWB, &tmKp, pbar, 0, row);
          tma_load_2d(vs + key * SH::ROWB, &tmVp, pbar, 0, row);
        }
      }
      return;
    }
    for (int pos0 = kb; pos0 < pend;) {
      const int pg = pos0 / p.page_size;
      const int pos1 = min(pend, (pg + 1) * p.page_size);
      const size_t base = cache_off(pos0);
      const T* ksrc = reinterpret_cast<const T*>(p.k_pages) + base;
      const T* vsrc = reinterpret_cast<const T*>(p.v_pages) + base;
      const int key0 = pos0 - kb;
      for (int e = tid; e < (pos1 - pos0) * SH::CH; e += kDecThreads) {
        const int key = key0 + e / SH::CH, c = e % SH::CH;
        cp_async16(smem_u32(ks + dswz<D>(key, c)), ksrc + (size_t)e * 8);
        cp_async16(smem_u32(vs + dswz<D>(key, c)), vsrc + (size_t)e * 8);
      }
      pos0 = pos1;
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  // The first block's prefix is in flight while the new tokens are processed.
  stage_prefix(0, min(kKMax, kv_len));

  if (vec) {
    // Rotate (q, k) and place the rows: q into the query tile, new k / v into
    // the cache and into their staging rows.
    if (have && role <= 1 && p.rope) {
      const uint32_t wa[4] = {xa.x, xa.y, xa.z, xa.w}, wb[4] = {xb.x, xb.y, xb.z, xb.w};
      const float ca[8] = {cra[0].x, cra[0].y, cra[0].z, cra[0].w, cra[1].x, cra[1].y, cra[1].z, cra[1].w};
      const float cb[8] = {crb[0].x, crb[0].y, crb[0].z, crb[0].w, crb[1].x, crb[1].y, crb[1].z, crb[1].w};
      const float sa[8] = {sra[0].x, sra[0].y, sra[0].z, sra[0].w, sra[1].x, sra[1].y, sra[1].z, sra[1].w};
      const float sb[8] = {srb[0].x, srb[0].y, srb[0].z, srb[0].w, srb[1].x, srb[1].y, srb[1].z, srb[1].w};
      uint32_t ya[4], yb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 a2 = E::to_f2(wa[u]), b2 = E::to_f2(wb[u]);
        float y0, y1, z0, z1;
        if (p.rope == kRopeRefRound) {
          rope_pair_ref_round<BF16>(a2.x, b2.x, ca[2 * u], sa[2 * u], cb[2 * u], sb[2 * u], y0, z0);
          rope_pair_ref_round<BF16>(a2.y, b2.y, ca[2 * u + 1], sa[2 * u + 1], cb[2 * u + 1], sb[2 * u + 1], y1, z1);
        } else {
          rope_pair(a2.x, b2.x, ca[2 * u], sa[2 * u], cb[2 * u], sb[2 * u], y0, z0);
          rope_pair(a2.y, b2.y, ca[2 * u + 1], sa[2 * u + 1], cb[2 * u + 1], sb[2 * u + 1], y1, z1);
        }
        ya[u] = E::from_f2(y0, y1);
        yb[u] = E::from_f2(z0, z1);
      }
      xa = make_uint4(ya[0], ya[1], ya[2], ya[3]);
      xb = make_uint4(yb[0], yb[1], yb[2], yb[3]);
    }
    if (role == 0) {
      *reinterpret_cast<uint4*>(qs + dswz<D>(rrow, rch)) = xa;  // rows past Sn * R stay zero
      *reinterpret_cast<uint4*>(qs + dswz<D>(rrow, rch + HC)) = xb;
    } else if (role <= 2) {
      const size_t off = cache_off(L + rrow);
      T* dst = reinterpret_cast<T*>(role == 1 ? p.k_pages : p.v_pages) + off;
      *reinterpret_cast<uint4*>(dst + rch * 8) = xa;
      *reinterpret_cast<uint4*>(dst + (rch + HC) * 8) = xb;
      uint8_t* st = role == 1 ? kns : vns;
      *reinterpret_cast<uint4*>(st + dswz<D>(rrow, rch)) = xa;
      *reinterpret_cast<uint4*>(st + dswz<D>(rrow, rch + HC)) = xb;
    }
  }

  // ---- append: rotate the new keys, write new K/V into the paged cache.
  for (int e = tid; !vec && e < Sn * (D / 2); e += kDecThreads) {
    const int i = e / (D / 2), d = e - i * (D / 2);
    const T* kn = reinterpret_cast<const T*>(p.k_new) + (size_t)b * p.kn_sb + (size_t)i * p.kn_ss +
                  (size_t)g * p.kn_sh;
    const T* vn = reinterpret_cast<const T*>(p.v_new) + (size_t)b * p.vn_sb + (size_t)i * p.vn_ss +
                  (size_t)g * p.vn_sh;
    float k0 = (float)kn[d], k1 = (float)kn[d + D / 2];
    if (p.rope) {
      const float* cr = cos_row(i);
      const float* sr = sin_row(i);
      float y0, y1;
      if (p.rope == kRopeRefRound)
        rope_pair_ref_round<BF16>(k0, k1, cr[d], sr[d], cr[d + D / 2], sr[d + D / 2], y0, y1);
      else
        rope_pair(k0, k1, cr[d], sr[d], cr[d + D / 2], sr[d + D / 2], y0, y1);
      k0 = y0;
      k1 = y1;
    }
    const size_t off = cache_off(L + i);
    T* kc = reinterpret_cast<T*>(p.k_pages) + off;
    T* vc = reinterpret_cast<T*>(p.v_pages) + off;
    kc[d] = (T)k0;
    kc[d + D / 2] = (T)k1;
    vc[d] = vn[d];
    vc[d + D / 2] = vn[d + D / 2];
    if (new_in_smem) {
      reinterpret_cast<T*>(kns + dswz<D>(i, d / 8))[d % 8] = (T)k0;
      reinterpret_cast<T*>(kns + dswz<D>(i, (d + D / 2) / 8))[(d + D / 2) % 8] = (T)k1;
      reinterpret_cast<T*>(vns + dswz<D>(i, d / 8))[d % 8] = vn[d];
      reinterpret_cast<T*>(vns + dswz<D>(i, (d + D / 2) / 8))[(d + D / 2) % 8] = vn[d + D / 2];
    }
  }
  // ---- queries: rows r = i * R + h (i < Sn), rotated, into shared memory.
  const int nrows = Sn * R;
  const int ngroups = (nrows + 15) / 16;
  const float c2 = p.scale_log2;
  const float sd64 = p.scale_div64;
  // Make this CTA's cache writes visible to its own loads below (only the
  // path that re-reads new rows from the cache needs it).
  if (!new_in_smem) __threadfence_block();
  __syncthreads();
  uint32_t pphase = 0;  // page-copy barrier phase

  for (int rg = 0; rg < ngroups; ++rg) {
    for (int e = tid; !vec && e < 16 * (D / 2); e += kDecThreads) {
      const int rr = e / (D / 2), d = e - rr * (D / 2);
      const int row = rg * 16 + rr;
      float y0 = 0.f, y1 = 0.f;
      if (row < nrows) {
        const int i = row / R, h = row - (row / R) * R;
        const T* qr = reinterpret_cast<const T*>(p.q) + (size_t)b * p.q_sb + (size_t)i * p.q_ss +
                      (size_t)(g * R + h) * p.q_sh;
        float x0 = (float)qr[d], x1 = (float)qr[d + D / 2];
        if (p.rope) {
          const float* cr = cos_row(i);
          const float* sr = sin_row(i);
          if (p.rope == kRopeRefRound)
            rope_pair_ref_round<BF16>(x0, x1, cr[d], sr[d], cr[d + D / 2], sr[d + D / 2], y0, y1);
          else
            rope_pair(x0, x1, cr[d], sr[d], cr[d + D / 2], sr[d + D / 2], y0, y1);
        } else {
          y0 = x0;
          y1 = x1;
        }
      }
      // element d lives in chunk d / 8 (swizzled) at offset d % 8
      reinterpret_cast<T*>(qs + dswz<D>(rr, d / 8))[d % 8] = (T)y0;
      reinterpret_cast<T*>(qs + dswz<D>(rr, (d + D / 2) / 8))[(d + D / 2) % 8] = (T)y1;
    }
    __syncthreads();

    // A fragments of Q (16 rows x D) for every k16 step.
    uint32_t qa[D / 16][4];
    {
      const int r = lane & 15, cb = lane >> 4;  // row, 8-column block within the k16 step
#pragma unroll
      for (int s = 0; s < D / 16; ++s)
        ldsm_x4(smem_u32(qs + dswz<D>(r, 2 * s + cb)), qa[s][0], qa[s][1], qa[s][2], qa[s][3]);
    }
    // This thread's two rows: g8 and g8 + 8 (C-fragment layout).
    const int g8 = lane >> 2, t4 = lane & 3;
    int rpos[2], rlo[2], rhi[2];
    bool rpad[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int row = rg * 16 + g8 + 8 * k;
      const bool valid = row < nrows;
      const int i = valid ? row / R : 0;
      rpos[k] = L + i;  // absolute position of this query
      rpad[k] = valid && rpos[k] < pad;
      // Rows past the query rows are never stored: they take every key so
      // that they never force the masked path.
      rlo[k] = !valid ? -(1 << 30) : (rpad[k] ? 0 : pad);
      rhi[k] = valid ? rpos[k] : (1 << 30);
    }
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float oacc[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) oacc[j][0] = oacc[j][1] = oacc[j][2] = oacc[j][3] = 0.f;

    for (int kb = 0; kb < kv_len; kb += kKMax) {
      const int nk = min(kKMax, kv_len - kb);
      // ---- stage keys [kb, kb + nk) of K and V (swizzled rows): the cached
      // prefix by 16-byte cp.async (issued before the append for the first
      // block), the new tokens from shared memory or, past kSnSmem of them,
      // from the cache this CTA has just written.
      if (rg > 0 || kb > 0) {
        __syncthreads();  // previous block fully consumed
        stage_prefix(kb, nk);
      }
      if (tma) {
        // The pages of this block have landed before any row of it is rewritten.
        const bool ok = mbar_wait(pbar, pphase, nullptr, p.status);
        pphase ^= 1u;
        if (__syncthreads_or(!ok)) return;
      } else {
        cp_async_wait_all();
      }
      {
        const int n0 = max(kb, L), n1 = kb + nk;  // new positions in this block
        for (int e = tid; e < max(0, n1 - n0) * SH::CH; e += kDecThreads) {
          const int pos = n0 + e / SH::CH, c = e % SH::CH;
          const int key = pos - kb;
          if (new_in_smem) {
            *reinterpret_cast<uint4*>(ks + dswz<D>(key, c)) = *reinterpret_cast<const uint4*>(kns + dswz<D>(pos - L, c));
            *reinterpret_cast<uint4*>(vs + dswz<D>(key, c)) = *reinterpret_cast<const uint4*>(vns + dswz<D>(pos - L, c));
          } else {
            const size_t off = cache_off(pos) + (size_t)c * 8;
            cp_async16(smem_u32(ks + dswz<D>(key, c)), reinterpret_cast<const T*>(p.k_pages) + off);
            cp_async16(smem_u32(vs + dswz<D>(key, c)), reinterpret_cast<const T*>(p.v_pages) + off);
          }
        }
      }
      // zero-fill the tail of the last 16-key chunk so masked keys hold finite data
      const int nk16 = (nk + 15) & ~15;
      for (int e = tid; e < (nk16 - nk) * SH::CH; e += kDecThreads) {
        const int key = nk + e / SH::CH, c = e % SH::CH;
        *reinterpret_cast<uint4*>(ks + dswz<D>(key, c)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vs + dswz<D>(key, c)) = make_uint4(0, 0, 0, 0);
      }
      cp_async_wait_all();
      __syncthreads();

      // ---- this warp's 16-key chunks of the block (split-K across warps).
      const int nchunks = nk16 / 16;
      for (int ch = warp; ch < nchunks; ch += kDecWarps) {
        const int key0 = ch * 16;  // within block
        float sc[2][4];
#pragma unroll
        for (int j = 0; j < 2; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
        // S = Q K^T: key blocks j (8 keys), k16 steps s.
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int krow = key0 + 8 * j + (lane & 7);
#pragma unroll
          for (int s2 = 0; s2 < D / 32; ++s2) {
            // four 8x8 matrices: dims [32 s2 + 8 m, +8) for m = lane / 8
            uint32_t b0, b1, b2, b3;
            ldsm_x4(smem_u32(ks + dswz<D>(krow, 4 * s2 + (lane >> 3))), b0, b1, b2, b3);
            mma16816<BF16>(sc[j], qa[2 * s2], b0, b1);
            mma16816<BF16>(sc[j], qa[2 * s2 + 1], b2, b3);
          }
        }
        // Online softmax over these 16 keys (rows g8 / g8 + 8; cols 2 t4 + {0,1} per key block).
        float pv[2][4];
        const int kabs = kb + key0;
        const bool plain = __all_sync(0xffffffffu, !rpad[0] && !rpad[1] && kabs >= rlo[0] && kabs >= rlo[1] &&
                                                       kabs + 15 <= rhi[0] && kabs + 15 <= rhi[1]);
        if (plain) {
          // Every key of the chunk is allowed for every row of the warp.  The
          // row reference m only moves (a quad max and a rescale of O) when a
          // score exceeds it by more than 2^8; P <= 256 otherwise.
          float x[2];
#pragma unroll
          for (int k = 0; k < 2; ++k)
            x[k] = fmaxf(fmaxf(sc[0][2 * k], sc[0][2 * k + 1]), fmaxf(sc[1][2 * k], sc[1][2 * k + 1])) * c2;
          if (__any_sync(0xffffffffu, x[0] > m_run[0] + 8.f || x[1] > m_run[1] + 8.f)) {
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              float cmax = fmaxf(x[k], __shfl_xor_sync(0xffffffffu, x[k], 1));
              cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
              if (cmax > m_run[k] + 8.f) {  // quad-uniform
                const float alpha = ex2_approx(m_run[k] - cmax);  // m_run = -inf -> 0
                l_run[k] *= alpha;
#pragma unroll
                for (int jd = 0; jd < D / 8; ++jd) {
                  oacc[jd][2 * k] *= alpha;
                  oacc[jd][2 * k + 1] *= alpha;
                }
                m_run[k] = cmax;
              }
            }
          }
#pragma unroll
          for (int k = 0; k < 2; ++k)
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
              for (int e2 = 0; e2 < 2; ++e2) {
                const float pe = ex2_approx(fmaf(sc[j][2 * k + e2], c2, -m_run[k]));
                pv[j][2 * k + e2] = pe;
                l_run[k] += pe;  // this thread's keys; the quad sum is taken at the end
              }
        } else {
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          float cmax = -INFINITY;
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
              const int key = kb + key0 + 8 * j + 2 * t4 + e2;
              const bool ok = key >= rlo[k] && key <= rhi[k];
              const float v = sc[j][2 * k + e2];
              if (ok) cmax = fmaxf(cmax, v);
            }
          cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
          cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
          // Fully padded rows score their keys in the reference's 64-wide bands.
          const RowScore rs(rpad[k], c2, sd64);
          const float m_new = fmaxf(m_run[k], rs(cmax));
          const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
          const float alpha = ex2_approx(m_run[k] - m_use);  // m_run = -inf -> 0
          float lsum = 0.f;
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e2 = 0; e2 < 2; ++e2) {
              const int key = kb + key0 + 8 * j + 2 * t4 + e2;
              const bool ok = key >= rlo[k] && key <= rhi[k];
              const float sv = sc[j][2 * k + e2];
              const float pe = ok ? ex2_approx(rs(sv) - m_use) : 0.f;
              pv[j][2 * k + e2] = pe;
              lsum += pe;
            }
          l_run[k] = l_run[k] * alpha + lsum;  // this thread's keys
          m_run[k] = m_new;
#pragma unroll
          for (int jd = 0; jd < D / 8; ++jd) {
            oacc[jd][2 * k] *= alpha;
            oacc[jd][2 * k + 1] *= alpha;
          }
        }
        }
        // O += P V: P (16 rows x 16 keys) as the A fragment, V via ldmatrix.trans.
        uint32_t pa[4];
        pa[0] = E::from_f2(pv[0][0], pv[0][1]);
        pa[1] = E::from_f2(pv[0][2], pv[0][3]);
        pa[2] = E::from_f2(pv[1][0], pv[1][1]);
        pa[3] = E::from_f2(pv[1][2], pv[1][3]);
#pragma unroll
        for (int jd2 = 0; jd2 < D / 16; ++jd2) {
          // matrices: (keys 0-7 | 8-15) x (dims 16 jd2 + 0-7 | 8-15)
          const int vrow = key0 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int vch = 2 * jd2 + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(vs + dswz<D>(vrow, vch)), b0, b1, b2, b3);
          mma16816<BF16>(oacc[2 * jd2], pa, b0, b1);
          mma16816<BF16>(oacc[2 * jd2 + 1], pa, b2, b3);
        }
      }
    }
    // ---- merge the warps' partials (m, l, O) per row and store.
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      l_run[k] += __shfl_xor_sync(0xffffffffu, l_run[k], 1);
      l_run[k] += __shfl_xor_sync(0xffffffffu, l_run[k], 2);
    }
    __syncthreads();  // the partials go over the K / V rows
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int rr = g8 + 8 * k;
      float* rw = red + (warp * 16 + rr) * SH::RED_STRIDE;
      if (t4 == 0) {
        rw[D] = m_run[k];
        rw[D + 1] = l_run[k];
      }
#pragma unroll
      for (int jd = 0; jd < D / 8; ++jd) {
        rw[8 * jd + 2 * t4] = oacc[jd][2 * k];
        rw[8 * jd + 2 * t4 + 1] = oacc[jd][2 * k + 1];
      }
    }
    __syncthreads();
    // Per row: weights of the four partials, f_w / sum_w f_w l_w with
    // f_w = 2^(m_w - max m) (a warp that saw no allowed key contributes 0).
    float* wt = red + kDecWarps * 16 * SH::RED_STRIDE;  // [warps][16]
    if (tid < 16) {
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, red[(w * 16 + tid) * SH::RED_STRIDE + D]);
      const float Mu = (M == -INFINITY) ? 0.f : M;
      float f[kDecWarps], lt = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        const float mw = red[(w * 16 + tid) * SH::RED_STRIDE + D];
        f[w] = (mw == -INFINITY) ? (M == -INFINITY ? 1.f : 0.f) : ex2_approx(mw - Mu);
        lt += f[w] * red[(w * 16 + tid) * SH::RED_STRIDE + D + 1];
      }
      const float inv = 1.f / lt;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) wt[w * 16 + tid] = f[w] * inv;
    }
    __syncthreads();
    for (int e = tid; e < 16 * (D / 2); e += kDecThreads) {
      const int rr = e / (D / 2), d = 2 * (e - rr * (D / 2));
      const int row = rg * 16 + rr;
      if (row >= nrows) continue;
      float o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        const float* rw = red + (w * 16 + rr) * SH::RED_STRIDE;
        const float ww = wt[w * 16 + rr];
        o0 = fmaf(ww, rw[d], o0);
        o1 = fmaf(ww, rw[d + 1], o1);
      }
      const int i = row / R, h = row - (row / R) * R;
      T* orow = reinterpret_cast<T*>(p.o) + (size_t)b * p.o_sb + (size_t)i * p.o_ss + (size_t)(g * R + h) * p.o_sh;
      if (p.o_pairs) {
        *reinterpret_cast<uint32_t*>(orow + d) = E::from_f2(o0, o1);
      } else {
        orow[d] = (T)o0;
        orow[d + 1] = (T)o1;
      }
    }
    __syncthreads();
  }
}

cudaError_t launch_decode_sm100(const DecodeParams& prm, const CUtensorMap& kmap, const CUtensorMap& vmap, int D,
                                bool bf16, int grid, cudaStream_t stream) {
  auto go = [&](auto kfn, int smem) -> cudaError_t {
    cudaError_t e = smem_limit_once(reinterpret_cast<const void*>(kfn), smem);
    if (e != cudaSuccess) return e;
    kfn<<<grid, kDecThreads, smem, stream>>>(kmap, vmap, prm);
    return cudaGetLastError();
  };
  if (D == 32) return bf16 ? go(dt_decode_kernel<32, true>, DecShape<32>::SMEM)
                           : go(dt_decode_kernel<32, false>, DecShape<32>::SMEM);
  if (D == 64) return bf16 ? go(dt_decode_kernel<64, true>, DecShape<64>::SMEM)
                           : go(dt_decode_kernel<64, false>, DecShape<64>::SMEM);
  return cudaErrorInvalidValue;
}

}  // namespace dtk
