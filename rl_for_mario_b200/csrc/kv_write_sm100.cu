// Writes a run of tokens' K (rotated) and V into the paged cache.
//
// Restates the cache half of DecisionTransformerAttention.forward
// (model/model_decision_transformer.py:179-191): the cached K is post-RoPE,
// V is stored as projected.  Token s of sample b lands at position
// start_pos[b] + s.  A dense [B, Hkv, L, D] cache is the special case of one
// page per sample with page_size = L.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

template <int D, typename T>
__global__ void __launch_bounds__(256) dt_kv_write_kernel(const KvWriteParams p) {
  const int b = blockIdx.x / p.Hkv;
  const int g = blockIdx.x - b * p.Hkv;
  const int start = p.start_pos ? p.start_pos[b] : 0;
  const int32_t* bt = p.block_table + (size_t)b * p.max_pages;
  const size_t page_stride = (size_t)p.Hkv * p.page_size * D;
  for (int e = blockIdx.y * blockDim.x + threadIdx.x; e < p.S * (D / 2); e += gridDim.y * blockDim.x) {
    const int s = e / (D / 2), d = e - s * (D / 2);
    const int pos = start + s;
    if (pos < 0 || pos >= p.max_pages * p.page_size) {
      if (p.status) atomicExch(p.status, (int)kDevBadShape);
      continue;
    }
    const int page = bt[pos / p.page_size];
    if (page < 0 || page >= p.num_pages) {
      if (p.status) atomicExch(p.status, (int)kDevBadShape);
      continue;
    }
    const T* kr = reinterpret_cast<const T*>(p.k) + (size_t)b * p.k_sb + (size_t)s * p.k_ss + (size_t)g * p.k_sh;
    const T* vr = reinterpret_cast<const T*>(p.v) + (size_t)b * p.v_sb + (size_t)s * p.v_ss + (size_t)g * p.v_sh;
    float k0 = (float)kr[d], k1 = (float)kr[d + D / 2];
    if (p.rope) {
      const int row = p.rope_abs ? pos : s;
      if (row >= p.cos_rows) {
        if (p.status) atomicExch(p.status, (int)kDevBadShape);
        continue;
      }
      const float* cr = p.cos + (size_t)row * p.cs_stride;
      const float* sr = p.sin + (size_t)row * p.cs_stride;
      float y0, y1;
      if (p.rope == kRopeRefRound) {
        // The reference's roundings in T (rope_pair_ref_round; fp32: unfused products).
        auto rnd = [](float x) { return (float)(T)x; };
        y0 = rnd(__fadd_rn(rnd(__fmul_rn(k0, cr[d])), -rnd(__fmul_rn(k1, sr[d]))));
        y1 = rnd(__fadd_rn(rnd(__fmul_rn(k1, cr[d + D / 2])), rnd(__fmul_rn(k0, sr[d + D / 2]))));
      } else {
        y0 = k0 * cr[d] - k1 * sr[d];
        y1 = k1 * cr[d + D / 2] + k0 * sr[d + D / 2];
      }
      k0 = y0;
      k1 = y1;
    }
    const size_t off = (size_t)page * page_stride + ((size_t)g * p.page_size + pos % p.page_size) * D;
    T* kc = reinterpret_cast<T*>(p.k_pages) + off;
    T* vc = reinterpret_cast<T*>(p.v_pages) + off;
    kc[d] = (T)k0;
    kc[d + D / 2] = (T)k1;
    vc[d] = vr[d];
    vc[d + D / 2] = vr[d + D / 2];
  }
}

template <typename T>
static void kv_write_d(const KvWriteParams& prm, int D, dim3 grid, cudaStream_t stream) {
  if (D == 32) dt_kv_write_kernel<32, T><<<grid, 256, 0, stream>>>(prm);
  else dt_kv_write_kernel<64, T><<<grid, 256, 0, stream>>>(prm);
}

cudaError_t launch_kv_write_sm100(const KvWriteParams& prm, int D, int dtype, int B, cudaStream_t stream) {
  if (D != 32 && D != 64) return cudaErrorInvalidValue;
  const int per = prm.S * (D / 2);
  const int gy = (per + 255) / 256 < 64 ? (per + 255) / 256 : 64;
  dim3 grid(B * prm.Hkv, gy);
  if (dtype == 0) kv_write_d<__nv_bfloat16>(prm, D, grid, stream);
  else if (dtype == 1) kv_write_d<__half>(prm, D, grid, stream);
  else kv_write_d<float>(prm, D, grid, stream);
  return cudaGetLastError();
}

}  // namespace dtk
