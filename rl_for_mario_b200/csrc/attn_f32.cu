// float32 attention kernels (CUDA cores) for float32 models.
//
// Same mathematics as the bf16 tensor-core kernels -- the prefill branch
// (model/model_decision_transformer.py:179-224) and the cached branch
// (:179-191, :225-245) of DecisionTransformerAttention.forward -- computed
// entirely in fp32 (exact dot products, exp2f, fp32 accumulation), so a float32
// model keeps the reference's float32 numerics.
//
// One CTA per (sample b, KV head g, group of 128 query rows); a thread owns
// one query row (position, head) and walks the keys it may attend to; K/V are
// staged (and K rotated) through shared memory in blocks of 64 keys.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kF32Threads = 128;
constexpr int kF32KB = 64;

// Online-softmax accumulation of one key for one row (log2 domain).
template <int D>
__device__ __forceinline__ void f32_accumulate(const float* __restrict__ kr, const float* __restrict__ vr,
                                               const float (&q)[D], float c2, float sd64, bool padded, float& m,
                                               float& l, float (&acc)[D]) {
  float s = 0.f;
#pragma unroll
  for (int d = 0; d < D; ++d) s = fmaf(q[d], kr[d], s);
  s = RowScore(padded, c2, sd64)(s);
  if (s > m) {
    const float sc = exp2f(m - s);  // m = -inf -> 0
    l *= sc;
#pragma unroll
    for (int d = 0; d < D; ++d) acc[d] *= sc;
    m = s;
  }
  const float p = exp2f(s - m);
  l += p;
#pragma unroll
  for (int d = 0; d < D; ++d) acc[d] = fmaf(p, vr[d], acc[d]);
}

__device__ __forceinline__ void rope_f32(float x0, float x1, const float* cr, const float* sr, int d, int half,
                                         float& y0, float& y1) {
  y0 = x0 * cr[d] - x1 * sr[d];
  y1 = x1 * cr[d + half] + x0 * sr[d + half];
}

// The reference's fp32 evaluation of q * cos + rotate_half(q) * sin: two
// rounded products and a rounded sum (no fused multiply-add).
__device__ __forceinline__ void rope_f32_ref(float x0, float x1, const float* cr, const float* sr, int d, int half,
                                             float& y0, float& y1) {
  y0 = __fadd_rn(__fmul_rn(x0, cr[d]), -__fmul_rn(x1, sr[d]));
  y1 = __fadd_rn(__fmul_rn(x1, cr[d + half]), __fmul_rn(x0, sr[d + half]));
}

__device__ __forceinline__ void rope_f32_mode(int mode, float x0, float x1, const float* cr, const float* sr, int d,
                                              int half, float& y0, float& y1) {
  if (mode == kRopeRefRound) rope_f32_ref(x0, x1, cr, sr, d, half, y0, y1);
  else rope_f32(x0, x1, cr, sr, d, half, y0, y1);
}

}  // namespace

// ---------------------------------------------------------------------------- prefill
template <int D>
__global__ void __launch_bounds__(kF32Threads) dt_prefill_f32_kernel(const PrefillF32Params p) {
  __shared__ float ks[kF32KB][D + 1];
  __shared__ float vs[kF32KB][D + 1];
  const int b = blockIdx.x / p.Hkv, g = blockIdx.x - (blockIdx.x / p.Hkv) * p.Hkv;
  const int R = p.R, S = p.S;
  int pad = p.pad_len ? p.pad_len[b] : 0;
  pad = max(0, min(pad, S));
  const int row = blockIdx.y * kF32Threads + threadIdx.x;  // (position, head) row of this unit
  const bool valid = row < S * R;
  const int pos = valid ? row / R : 0, h = valid ? row - (row / R) * R : 0;
  const bool padded = pos < pad;
  const int lo = padded ? 0 : pad, hi = valid ? pos : -1;
  const float c2 = p.scale_log2;

  float q[D];
  if (valid) {
    const float* qr = p.q + (size_t)b * p.q_sb + (size_t)pos * p.q_ss + (size_t)(g * R + h) * p.q_sh;
    if (p.rope) {
      const float* cr = p.cos + (size_t)pos * p.cs_stride;
      const float* sr = p.sin + (size_t)pos * p.cs_stride;
#pragma unroll
      for (int d = 0; d < D / 2; ++d) rope_f32_mode(p.rope, qr[d], qr[d + D / 2], cr, sr, d, D / 2, q[d], q[d + D / 2]);
    } else {
#pragma unroll
      for (int d = 0; d < D; ++d) q[d] = qr[d];
    }
  }
  float m = -INFINITY, l = 0.f, acc[D];
#pragma unroll
  for (int d = 0; d < D; ++d) acc[d] = 0.f;

  // Keys needed by this row group: [0, last position of the group].
  const int last_row = min(S * R, (int)(blockIdx.y + 1) * kF32Threads) - 1;
  const int kend = last_row / R + 1;
  for (int kb = 0; kb < kend; kb += kF32KB) {
    const int nk = min(kF32KB, kend - kb);
    __syncthreads();
    for (int e = threadIdx.x; e < nk * (D / 2); e += kF32Threads) {
      const int j = e / (D / 2), d = e - j * (D / 2);
      const int key = kb + j;
      const float* kr = p.k + (size_t)b * p.k_sb + (size_t)key * p.k_ss + (size_t)g * p.k_sh;
      const float* vr = p.v + (size_t)b * p.v_sb + (size_t)key * p.v_ss + (size_t)g * p.v_sh;
      float y0 = kr[d], y1 = kr[d + D / 2];
      if (p.rope) rope_f32_mode(p.rope, kr[d], kr[d + D / 2], p.cos + (size_t)key * p.cs_stride,
                           p.sin + (size_t)key * p.cs_stride, d, D / 2, y0, y1);
      ks[j][d] = y0;
      ks[j][d + D / 2] = y1;
      vs[j][d] = vr[d];
      vs[j][d + D / 2] = vr[d + D / 2];
    }
    __syncthreads();
    const int j0 = max(lo - kb, 0), j1 = min(hi - kb, nk - 1);
    for (int j = j0; j <= j1; ++j) f32_accumulate<D>(ks[j], vs[j], q, c2, p.scale_div64, padded, m, l, acc);
  }
  if (valid) {
    float* orow = p.o + (size_t)b * p.o_sb + (size_t)pos * p.o_ss + (size_t)(g * R + h) * p.o_sh;
    const float inv = 1.f / l;
#pragma unroll
    for (int d = 0; d < D; ++d) orow[d] = acc[d] * inv;
  }
}

// ---------------------------------------------------------------------------- decode
template <int D>
__global__ void __launch_bounds__(kF32Threads) dt_decode_f32_kernel(const DecodeParams p) {
  __shared__ float ks[kF32KB][D + 1];
  __shared__ float vs[kF32KB][D + 1];
  const int b = blockIdx.x / p.Hkv, g = blockIdx.x - (blockIdx.x / p.Hkv) * p.Hkv;
  const int R = p.R, Sn = p.Sn;
  const int L = p.seq_lens[b];
  const int kv_len = L + Sn;
  int pad = p.pad_len ? p.pad_len[b] : 0;
  pad = max(0, min(pad, kv_len));
  const int32_t* bt = p.block_table + (size_t)b * p.max_pages;
  bool bad = L < 0 || kv_len > p.max_pages * p.page_size || (p.rope && p.rope_abs && kv_len > p.cos_rows);
  if (!bad)
    for (int pg = threadIdx.x; pg * p.page_size < kv_len; pg += kF32Threads)
      if (bt[pg] < 0 || bt[pg] >= p.num_pages) bad = true;
  if (__syncthreads_or(bad)) {
    if (threadIdx.x == 0 && p.status) atomicExch(p.status, (int)kDevBadShape);
    return;
  }
  const size_t page_stride = (size_t)p.Hkv * p.page_size * D;
  auto cache_off = [&](int pos) -> size_t {
    return (size_t)bt[pos / p.page_size] * page_stride + ((size_t)g * p.page_size + pos % p.page_size) * D;
  };
  auto cs_row = [&](int i) -> size_t { return (size_t)(p.rope_abs ? L + i : i) * p.cs_stride; };
  const float* Kn = static_cast<const float*>(p.k_new);
  const float* Vn = static_cast<const float*>(p.v_new);
  // The first row group appends the new tokens to the cache (every group
  // stages them for itself from k_new / v_new below).
  if (blockIdx.y == 0) {
    for (int e = threadIdx.x; e < Sn * (D / 2); e += kF32Threads) {
      const int i = e / (D / 2), d = e - i * (D / 2);
      const float* kr = Kn + (size_t)b * p.kn_sb + (size_t)i * p.kn_ss + (size_t)g * p.kn_sh;
      const float* vr = Vn + (size_t)b * p.vn_sb + (size_t)i * p.vn_ss + (size_t)g * p.vn_sh;
      float y0 = kr[d], y1 = kr[d + D / 2];
      if (p.rope) rope_f32_mode(p.rope, kr[d], kr[d + D / 2], p.cos + cs_row(i), p.sin + cs_row(i), d, D / 2, y0, y1);
      float* kc = static_cast<float*>(p.k_pages) + cache_off(L + i);
      float* vc = static_cast<float*>(p.v_pages) + cache_off(L + i);
      kc[d] = y0;
      kc[d + D / 2] = y1;
      vc[d] = vr[d];
      vc[d + D / 2] = vr[d + D / 2];
    }
  }
  const int row = blockIdx.y * kF32Threads + threadIdx.x;
  const bool valid = row < Sn * R;
  const int i = valid ? row / R : 0, h = valid ? row - (row / R) * R : 0;
  const int qpos = L + i;
  const bool padded = qpos < pad;
  const int lo = padded ? 0 : pad, hi = valid ? qpos : -1;
  float q[D];
  if (valid) {
    const float* qr = static_cast<const float*>(p.q) + (size_t)b * p.q_sb + (size_t)i * p.q_ss +
                      (size_t)(g * R + h) * p.q_sh;
    if (p.rope) {
#pragma unroll
      for (int d = 0; d < D / 2; ++d)
        rope_f32_mode(p.rope, qr[d], qr[d + D / 2], p.cos + cs_row(i), p.sin + cs_row(i), d, D / 2, q[d], q[d + D / 2]);
    } else {
#pragma unroll
      for (int d = 0; d < D; ++d) q[d] = qr[d];
    }
  }
  float m = -INFINITY, l = 0.f, acc[D];
#pragma unroll
  for (int d = 0; d < D; ++d) acc[d] = 0.f;
  for (int kb = 0; kb < kv_len; kb += kF32KB) {
    const int nk = min(kF32KB, kv_len - kb);
    __syncthreads();
    for (int e = threadIdx.x; e < nk * (D / 2); e += kF32Threads) {
      const int j = e / (D / 2), d = e - j * (D / 2);
      const int key = kb + j;
      float k0, k1, v0, v1;
      if (key < L) {
        const float* kc = static_cast<const float*>(p.k_pages) + cache_off(key);
        const float* vc = static_cast<const float*>(p.v_pages) + cache_off(key);
        k0 = kc[d], k1 = kc[d + D / 2], v0 = vc[d], v1 = vc[d + D / 2];
      } else {
        const int ii = key - L;
        const float* kr = Kn + (size_t)b * p.kn_sb + (size_t)ii * p.kn_ss + (size_t)g * p.kn_sh;
        const float* vr = Vn + (size_t)b * p.vn_sb + (size_t)ii * p.vn_ss + (size_t)g * p.vn_sh;
        k0 = kr[d], k1 = kr[d + D / 2], v0 = vr[d], v1 = vr[d + D / 2];
        if (p.rope) rope_f32_mode(p.rope, kr[d], kr[d + D / 2], p.cos + cs_row(ii), p.sin + cs_row(ii), d, D / 2, k0, k1);
      }
      ks[j][d] = k0;
      ks[j][d + D / 2] = k1;
      vs[j][d] = v0;
      vs[j][d + D / 2] = v1;
    }
    __syncthreads();
    const int j0 = max(lo - kb, 0), j1 = min(hi - kb, nk - 1);
    for (int j = j0; j <= j1; ++j) f32_accumulate<D>(ks[j], vs[j], q, p.scale_log2, p.scale_div64, padded, m, l, acc);
  }
  if (valid) {
    float* orow = static_cast<float*>(p.o) + (size_t)b * p.o_sb + (size_t)i * p.o_ss + (size_t)(g * R + h) * p.o_sh;
    const float inv = 1.f / l;
#pragma unroll
    for (int d = 0; d < D; ++d) orow[d] = acc[d] * inv;
  }
}

cudaError_t launch_prefill_f32(const PrefillF32Params& prm, int D, int B, cudaStream_t stream) {
  dim3 grid(B * prm.Hkv, (prm.S * prm.R + kF32Threads - 1) / kF32Threads);
  if (D == 32) dt_prefill_f32_kernel<32><<<grid, kF32Threads, 0, stream>>>(prm);
  else if (D == 64) dt_prefill_f32_kernel<64><<<grid, kF32Threads, 0, stream>>>(prm);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_decode_f32(const DecodeParams& prm, int D, int B, cudaStream_t stream) {
  dim3 grid(B * prm.Hkv, (prm.Sn * prm.R + kF32Threads - 1) / kF32Threads);
  if (D == 32) dt_decode_f32_kernel<32><<<grid, kF32Threads, 0, stream>>>(prm);
  else if (D == 64) dt_decode_f32_kernel<64><<<grid, kF32Threads, 0, stream>>>(prm);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace dtk
