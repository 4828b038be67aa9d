// Row RMSNorm, sm_100a: the reference's RMSNorm.forward
// (model/model_decision_transformer.py:76-86) for the norms that are not
// fused into a GEMM (embed_norm :420, the final norm :457).
//
//   r = rsqrt(mean(x^2) + eps)            fp32
//   y = w * cast(x * r)                   the normalised row is rounded to the
//                                         activation dtype before the weight
//                                         product, as `.type_as(x)` does
//
// One warp per row, 16-byte loads; the row's chunks stay in registers between
// the sum of squares and the scaling when K <= 32 * 8 * kHeld (768-wide rows:
// three chunks per lane), else the second pass re-reads them (L1 / L2).
// HBM-bound: 2 K bytes read and 2 K bytes written per row.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kHeld = 4;  // 16-byte chunks per lane kept in registers

template <bool BF16>
__device__ __forceinline__ uint32_t norm_pair(uint32_t xv, uint32_t wv, float r) {
  const float2 xf = Elem<BF16>::to_f2(xv);
  const float2 wf = Elem<BF16>::to_f2(wv);
  const float2 n = Elem<BF16>::to_f2(Elem<BF16>::from_f2(xf.x * r, xf.y * r));  // cast(x * r)
  return Elem<BF16>::from_f2(wf.x * n.x, wf.y * n.y);
}

template <bool BF16>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const uint16_t* __restrict__ x, long long x_stride,
                                                           const uint16_t* __restrict__ w, uint16_t* __restrict__ y,
                                                           long long y_stride, int M, int K, float eps) {
  const int lane = threadIdx.x & 31;
  const int nch = K >> 3;  // 16-byte chunks per row
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  for (long long row = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < M;
       row += ((long long)gridDim.x * blockDim.x) >> 5) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * x_stride);
    uint4* yr = reinterpret_cast<uint4*>(y + row * y_stride);
    uint4 held[kHeld];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
      const int c = lane + 32 * j;
      held[j] = c < nch ? __ldg(xr + c) : make_uint4(0u, 0u, 0u, 0u);
    }
    for (int c = lane + 32 * kHeld; c < nch; c += 32) {
      const uint4 u = __ldg(xr + c);
      const uint32_t q[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Elem<BF16>::to_f2(q[e]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
      const uint32_t q[4] = {held[j].x, held[j].y, held[j].z, held[j].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Elem<BF16>::to_f2(q[e]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / (float)K + eps);
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
      const int c = lane + 32 * j;
      if (c < nch) {
        const uint4 wu = __ldg(wv + c);
        yr[c] = make_uint4(norm_pair<BF16>(held[j].x, wu.x, r), norm_pair<BF16>(held[j].y, wu.y, r),
                           norm_pair<BF16>(held[j].z, wu.z, r), norm_pair<BF16>(held[j].w, wu.w, r));
      }
    }
    for (int c = lane + 32 * kHeld; c < nch; c += 32) {
      const uint4 u = __ldg(xr + c), wu = __ldg(wv + c);
      yr[c] = make_uint4(norm_pair<BF16>(u.x, wu.x, r), norm_pair<BF16>(u.y, wu.y, r),
                         norm_pair<BF16>(u.z, wu.z, r), norm_pair<BF16>(u.w, wu.w, r));
    }
  }
}

}  // namespace

cudaError_t launch_rmsnorm_sm100(const void* x, long long x_stride, const void* w, void* y, long long y_stride, int M,
                                 int K, float eps, bool bf16, int num_sms, cudaStream_t st) {
  // 8 rows per 256-thread block; enough blocks to fill every SM several times over.
  const long long want = ((long long)M + 7) / 8;
  const long long cap = (long long)num_sms * 16;
  const unsigned grid = (unsigned)(want < cap ? want : cap);
  auto xs = static_cast<const uint16_t*>(x);
  auto ws = static_cast<const uint16_t*>(w);
  auto ys = static_cast<uint16_t*>(y);
  if (bf16)
    rmsnorm_rows_kernel<true><<<grid, 256, 0, st>>>(xs, x_stride, ws, ys, y_stride, M, K, eps);
  else
    rmsnorm_rows_kernel<false><<<grid, 256, 0, st>>>(xs, x_stride, ws, ys, y_stride, M, K, eps);
  return cudaGetLastError();
}

}  // namespace dtk
