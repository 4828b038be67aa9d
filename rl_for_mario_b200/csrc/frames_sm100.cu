// Frame stacks -> space-to-depth blocks for the state encoder's first
// convolution, sm_100a.
//
// The reference encoder (model/model_decision_transformer.py:315-341) feeds
// uint8 frames [N, C, H, W] to an 8 x 8 stride-4 convolution after the
// division by 255 (:338).  That convolution equals a 2 x 2 stride-1
// convolution over the frames cut into 4 x 4 blocks, whose C * 16 channels
// are (c, dy, dx); this kernel writes those blocks, converted exactly to
// 16 bits (0..255 are exact in bf16 and fp16), channels-last:
//   out[n, Y, X, c * 16 + dy * 4 + dx] = frames[n, c, 4 Y + dy, 4 X + dx].
// The 1/255 goes into the convolution weight; the reference applies it only
// when the frames' maximum exceeds 1, so the kernel also folds the maximum
// byte into *frame_max (atomicMax, when non-null) instead of a separate
// reduction over the frames.  One thread per output block
// position: 4 rows x 4 bytes per channel as 32-bit loads (neighbouring
// threads read neighbouring words), 32 contiguous output bytes per channel
// as two 16-byte stores (neighbouring threads write neighbouring rows).
// HBM-bound: C*H*W bytes read and 2*C*H*W bytes written per frame.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

template <bool BF16>
__global__ void __launch_bounds__(256) frames_to_blocks_kernel(const uint8_t* __restrict__ frames,
                                                               uint16_t* __restrict__ out, long long n_pos, int C,
                                                               int H, int W, unsigned int* frame_max) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t bmax = 0;  // byte-wise maximum of every word this thread reads
  if (i < n_pos) {
    const int Wb = W >> 2, Hb = H >> 2;
    const long long per_frame = (long long)Hb * Wb;
    const long long n = i / per_frame;
    const int rem = (int)(i - n * per_frame);
    const int Y = rem / Wb, X = rem - (rem / Wb) * Wb;
    const uint8_t* src = frames + (size_t)n * C * H * W + (size_t)(4 * Y) * W + 4 * X;
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)i * C * 16);
    for (int c = 0; c < C; ++c) {
      uint32_t w[4];
#pragma unroll
      for (int dy = 0; dy < 4; ++dy) w[dy] = __ldg(reinterpret_cast<const uint32_t*>(src + (size_t)dy * W));
      uint32_t o[8];
#pragma unroll
      for (int dy = 0; dy < 4; ++dy) {
        const float b0 = (float)(w[dy] & 0xffu), b1 = (float)((w[dy] >> 8) & 0xffu);
        const float b2 = (float)((w[dy] >> 16) & 0xffu), b3 = (float)(w[dy] >> 24);
        o[2 * dy] = Elem<BF16>::from_f2(b0, b1);
        o[2 * dy + 1] = Elem<BF16>::from_f2(b2, b3);
        bmax = __vmaxu4(bmax, w[dy]);
      }
      dst[2 * c] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[2 * c + 1] = make_uint4(o[4], o[5], o[6], o[7]);
      src += (size_t)H * W;
    }
  }
  if (frame_max) {
    uint32_t m = max(max(bmax & 0xffu, (bmax >> 8) & 0xffu), max((bmax >> 16) & 0xffu, bmax >> 24));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m > 0) atomicMax(frame_max, m);
  }
}

}  // namespace

cudaError_t launch_frames_to_blocks_sm100(const void* frames, void* out, long long N, int C, int H, int W, bool bf16,
                                          unsigned int* frame_max, cudaStream_t st) {
  const long long n_pos = N * (long long)(H / 4) * (W / 4);
  const long long blocks = (n_pos + 255) / 256;
  if (bf16)
    frames_to_blocks_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const uint8_t*>(frames), static_cast<uint16_t*>(out), n_pos, C, H, W, frame_max);
  else
    frames_to_blocks_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(
        static_cast<const uint8_t*>(frames), static_cast<uint16_t*>(out), n_pos, C, H, W, frame_max);
  return cudaGetLastError();
}

}  // namespace dtk
