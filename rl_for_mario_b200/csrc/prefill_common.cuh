// Helpers shared by the prefill kernels: swizzled tile addressing and
// in-place rotate-half RoPE on a shared-memory tile.
#pragma once

#include "dt_common.cuh"

namespace dtk {

// Byte offset of 16-byte chunk c of row r inside a TMA/UMMA swizzled tile
// (64-byte rows use the 64B swizzle, 128-byte rows the 128B swizzle).
template <int ROWB>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  if constexpr (ROWB == 64) {
    return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
  } else {
    return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
  }
}

// Rotate one row of a swizzled tile in place:
//   y[d] = x[d] cos[d] - x[d+D/2] sin[d],  y[d+D/2] = x[d+D/2] cos[d+D/2] + x[d] sin[d+D/2]
// (rotate-half RoPE, reference :103-117).  Arithmetic in fp32, or with the
// reference's roundings in the activation dtype when ref_round
// (rope_pair_ref_round).
template <int D, bool BF16>
__device__ __forceinline__ void rope_row_inplace(uint8_t* tile, int r, const float* __restrict__ cr,
                                                 const float* __restrict__ sr, bool ref_round = false) {
  constexpr int NCH = D / 8;  // 16-byte chunks per row
  constexpr int HALF = NCH / 2;
#pragma unroll
  for (int c = 0; c < HALF; ++c) {
    uint4* pa = reinterpret_cast<uint4*>(tile + swz<D * 2>(r, c));
    uint4* pb = reinterpret_cast<uint4*>(tile + swz<D * 2>(r, c + HALF));
    uint4 a = *pa, b = *pb;
    const float4 ca0 = __ldg(reinterpret_cast<const float4*>(cr + c * 8));
    const float4 ca1 = __ldg(reinterpret_cast<const float4*>(cr + c * 8 + 4));
    const float4 sa0 = __ldg(reinterpret_cast<const float4*>(sr + c * 8));
    const float4 sa1 = __ldg(reinterpret_cast<const float4*>(sr + c * 8 + 4));
    const float4 cb0 = __ldg(reinterpret_cast<const float4*>(cr + (c + HALF) * 8));
    const float4 cb1 = __ldg(reinterpret_cast<const float4*>(cr + (c + HALF) * 8 + 4));
    const float4 sb0 = __ldg(reinterpret_cast<const float4*>(sr + (c + HALF) * 8));
    const float4 sb1 = __ldg(reinterpret_cast<const float4*>(sr + (c + HALF) * 8 + 4));
    const float ca[8] = {ca0.x, ca0.y, ca0.z, ca0.w, ca1.x, ca1.y, ca1.z, ca1.w};
    const float sa[8] = {sa0.x, sa0.y, sa0.z, sa0.w, sa1.x, sa1.y, sa1.z, sa1.w};
    const float cb[8] = {cb0.x, cb0.y, cb0.z, cb0.w, cb1.x, cb1.y, cb1.z, cb1.w};
    const float sb[8] = {sb0.x, sb0.y, sb0.z, sb0.w, sb1.x, sb1.y, sb1.z, sb1.w};
    uint32_t au[4] = {a.x, a.y, a.z, a.w}, bu[4] = {b.x, b.y, b.z, b.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xa = Elem<BF16>::to_f2(au[i]);
      const float2 xb = Elem<BF16>::to_f2(bu[i]);
      float y0, y1, z0, z1;
      if (ref_round) {
        rope_pair_ref_round<BF16>(xa.x, xb.x, ca[2 * i], sa[2 * i], cb[2 * i], sb[2 * i], y0, z0);
        rope_pair_ref_round<BF16>(xa.y, xb.y, ca[2 * i + 1], sa[2 * i + 1], cb[2 * i + 1], sb[2 * i + 1], y1, z1);
      } else {
        y0 = xa.x * ca[2 * i] - xb.x * sa[2 * i];
        y1 = xa.y * ca[2 * i + 1] - xb.y * sa[2 * i + 1];
        z0 = xb.x * cb[2 * i] + xa.x * sb[2 * i];
        z1 = xb.y * cb[2 * i + 1] + xa.y * sb[2 * i + 1];
      }
      ya[i] = Elem<BF16>::from_f2(y0, y1);
      yb[i] = Elem<BF16>::from_f2(z0, z1);
    }
    *pa = make_uint4(ya[0], ya[1], ya[2], ya[3]);
    *pb = make_uint4(yb[0], yb[1], yb[2], yb[3]);
  }
}

// Same rotation with the cos/sin row in shared memory (generic loads).
template <int D, bool BF16>
__device__ __forceinline__ void rope_row_inplace_smem(uint8_t* tile, int r, const float* cr, const float* sr) {
  constexpr int NCH = D / 8;
  constexpr int HALF = NCH / 2;
#pragma unroll
  for (int c = 0; c < HALF; ++c) {
    uint4* pa = reinterpret_cast<uint4*>(tile + swz<D * 2>(r, c));
    uint4* pb = reinterpret_cast<uint4*>(tile + swz<D * 2>(r, c + HALF));
    const uint4 a = *pa, b = *pb;
    const float4 ca0 = *reinterpret_cast<const float4*>(cr + c * 8);
    const float4 ca1 = *reinterpret_cast<const float4*>(cr + c * 8 + 4);
    const float4 sa0 = *reinterpret_cast<const float4*>(sr + c * 8);
    const float4 sa1 = *reinterpret_cast<const float4*>(sr + c * 8 + 4);
    const float4 cb0 = *reinterpret_cast<const float4*>(cr + (c + HALF) * 8);
    const float4 cb1 = *reinterpret_cast<const float4*>(cr + (c + HALF) * 8 + 4);
    const float4 sb0 = *reinterpret_cast<const float4*>(sr + (c + HALF) * 8);
    const float4 sb1 = *reinterpret_cast<const float4*>(sr + (c + HALF) * 8 + 4);
    const float ca[8] = {ca0.x, ca0.y, ca0.z, ca0.w, ca1.x, ca1.y, ca1.z, ca1.w};
    const float sa[8] = {sa0.x, sa0.y, sa0.z, sa0.w, sa1.x, sa1.y, sa1.z, sa1.w};
    const float cb[8] = {cb0.x, cb0.y, cb0.z, cb0.w, cb1.x, cb1.y, cb1.z, cb1.w};
    const float sb[8] = {sb0.x, sb0.y, sb0.z, sb0.w, sb1.x, sb1.y, sb1.z, sb1.w};
    const uint32_t au[4] = {a.x, a.y, a.z, a.w}, bu[4] = {b.x, b.y, b.z, b.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xa = Elem<BF16>::to_f2(au[i]);
      const float2 xb = Elem<BF16>::to_f2(bu[i]);
      ya[i] = Elem<BF16>::from_f2(xa.x * ca[2 * i] - xb.x * sa[2 * i], xa.y * ca[2 * i + 1] - xb.y * sa[2 * i + 1]);
      yb[i] = Elem<BF16>::from_f2(xb.x * cb[2 * i] + xa.x * sb[2 * i], xb.y * cb[2 * i + 1] + xa.y * sb[2 * i + 1]);
    }
    *pa = make_uint4(ya[0], ya[1], ya[2], ya[3]);
    *pb = make_uint4(yb[0], yb[1], yb[2], yb[3]);
  }
}

// Same rotation from a shared-memory cos / sin row whose sin entries of the
// first half are stored negated, in packed fp32 pairs (one multiply and one
// fused multiply-add instruction per two outputs).  ref_round: the
// reference's roundings instead (rope_pair_ref_round).
template <int D, bool BF16>
__device__ __forceinline__ void rope_row_inplace_f2(uint8_t* tile, int r, const float* cr, const float* sr,
                                                    bool ref_round = false) {
  constexpr int NCH = D / 8;
  constexpr int HALF = NCH / 2;
  using E = Elem<BF16>;
#pragma unroll
  for (int c = 0; c < HALF; ++c) {
    uint4* pa = reinterpret_cast<uint4*>(tile + swz<D * 2>(r, c));
    uint4* pb = reinterpret_cast<uint4*>(tile + swz<D * 2>(r, c + HALF));
    const uint4 a = *pa, b = *pb;
    const uint32_t au[4] = {a.x, a.y, a.z, a.w}, bu[4] = {b.x, b.y, b.z, b.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xa = E::to_f2(au[i]), xb = E::to_f2(bu[i]);
      const float2 ca = *reinterpret_cast<const float2*>(cr + c * 8 + 2 * i);
      const float2 cb = *reinterpret_cast<const float2*>(cr + (c + HALF) * 8 + 2 * i);
      const float2 sa = *reinterpret_cast<const float2*>(sr + c * 8 + 2 * i);  // negated
      const float2 sb = *reinterpret_cast<const float2*>(sr + (c + HALF) * 8 + 2 * i);
      if (ref_round) {
        // sa holds -sin: the products with it are rotate_half(x) * sin exactly.
        float y0, y1, z0, z1;
        rope_pair_ref_round<BF16>(xa.x, xb.x, ca.x, -sa.x, cb.x, sb.x, y0, z0);
        rope_pair_ref_round<BF16>(xa.y, xb.y, ca.y, -sa.y, cb.y, sb.y, y1, z1);
        ya[i] = E::from_f2(y0, y1);
        yb[i] = E::from_f2(z0, z1);
        continue;
      }
      const float2 y = ffma2(xa, ca, fmul2(xb, sa));
      const float2 z = ffma2(xb, cb, fmul2(xa, sb));
      ya[i] = E::from_f2(y.x, y.y);
      yb[i] = E::from_f2(z.x, z.y);
    }
    *pa = make_uint4(ya[0], ya[1], ya[2], ya[3]);
    *pb = make_uint4(yb[0], yb[1], yb[2], yb[3]);
  }
}

// Per-tile schedule, computed identically by every role.
struct TilePlan {
  int pos0, pos_end, kstart, kend, nblocks;
};

__device__ __forceinline__ TilePlan plan_tile(int t, int PT, int S, int pad) {
  TilePlan p;
  p.pos0 = t * PT;
  p.pos_end = min(S, p.pos0 + PT);
  p.kend = p.pos_end;
  // A tile without padded rows needs keys pad..q only; keys below pad carry
  // exactly zero weight.  Tiles that hold padded rows need keys from 0.
  p.kstart = (p.pos0 >= pad) ? (pad & ~15) : 0;
  p.nblocks = (p.kend - p.kstart + 127) / 128;
  return p;
}

__device__ __forceinline__ int block_cols(const TilePlan& p, int j) {
  const int kb0 = p.kstart + j * 128;
  const int rem = p.kend - kb0;
  return min(128, (rem + 15) & ~15);
}

}  // namespace dtk
