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
// threads read neighbouring words).  A CTA's outputs are one contiguous
// range (256 positions x C*32 bytes); with C = 4 (the Mario frame stacks) it
// is staged in shared memory, 16-byte pieces XOR-swizzled by position, and
// written back with every warp storing 512 contiguous bytes per instruction
// (direct per-thread stores touch 32 lines per warp instruction).
// HBM-bound: C*H*W bytes read and 2*C*H*W bytes written per frame.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

// STAGE: C == 4, outputs staged in shared memory (8 pieces of 16 bytes per position).
template <bool BF16, bool STAGE>
__global__ void __launch_bounds__(256) frames_to_blocks_kernel(const uint8_t* __restrict__ frames,
                                                               uint16_t* __restrict__ out, long long n_pos, int C,
                                                               int H, int W, unsigned int* frame_max) {
  __shared__ uint4 stage[STAGE ? 256 * 8 : 1];
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int t = threadIdx.x;
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
      if (STAGE) {
        stage[t * 8 + ((2 * c) ^ (t & 7))] = make_uint4(o[0], o[1], o[2], o[3]);
        stage[t * 8 + ((2 * c + 1) ^ (t & 7))] = make_uint4(o[4], o[5], o[6], o[7]);
      } else {
        dst[2 * c] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[2 * c + 1] = make_uint4(o[4], o[5], o[6], o[7]);
      }
      src += (size_t)H * W;
    }
  }
  if (STAGE) {
    __syncthreads();
    // Piece j of the CTA's range belongs to position j / 8, piece j % 8.
    const long long p0 = (long long)blockIdx.x * blockDim.x;
    const long long np = n_pos - p0 < 256 ? n_pos - p0 : 256;
    uint4* dst0 = reinterpret_cast<uint4*>(out + (size_t)p0 * 64);
    for (int j = t; j < np * 8; j += 256) {
      const int tp = j >> 3, k = j & 7;
      dst0[j] = stage[tp * 8 + (k ^ (tp & 7))];
    }
  }
  if (frame_max) {
    uint32_t m = max(max(bmax & 0xffu, (bmax >> 8) & 0xffu), max((bmax >> 16) & 0xffu, bmax >> 24));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m > 0) atomicMax(frame_max, m);
  }
}

// One CTA per frame: the frame (C*H*W bytes, a multiple of 16) is copied
// into shared memory with coalesced 16-byte loads, then output piece j
// (8 outputs: channel c = k / 2, rows 4 Y + 2 (k & 1) + {0, 1}, four columns,
// with position j / (2 C) and k = j % (2 C)) is built from two shared words
// and stored, consecutive threads writing consecutive pieces.
template <bool BF16>
__global__ void __launch_bounds__(256) frame_cta_to_blocks_kernel(const uint8_t* __restrict__ frames,
                                                                  uint16_t* __restrict__ out, int C, int H, int W,
                                                                  unsigned int* frame_max) {
  extern __shared__ uint4 fbuf[];
  const int fbytes = C * H * W;
  const uint4* src = reinterpret_cast<const uint4*>(frames + (size_t)blockIdx.x * fbytes);
  uint32_t bmax = 0;
  for (int i = threadIdx.x; i < fbytes / 16; i += blockDim.x) {
    const uint4 u = __ldg(src + i);
    fbuf[i] = u;
    bmax = __vmaxu4(__vmaxu4(bmax, u.x), __vmaxu4(__vmaxu4(u.y, u.z), u.w));
  }
  __syncthreads();
  const uint32_t* f32 = reinterpret_cast<const uint32_t*>(fbuf);
  const int Wb = W >> 2, per_frame = (H >> 2) * Wb, np = 2 * C;
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)blockIdx.x * per_frame * C * 16);
  for (int j = threadIdx.x; j < per_frame * np; j += blockDim.x) {
    const int pos = j / np, k = j - pos * np;
    const int Y = pos / Wb, X = pos - Y * Wb;
    const int row = (k >> 1) * H + 4 * Y + 2 * (k & 1);  // row of the channel plane
    const uint32_t w0 = f32[(row * W >> 2) + X], w1 = f32[((row + 1) * W >> 2) + X];
    dst[j] = make_uint4(
        Elem<BF16>::from_f2((float)(w0 & 0xffu), (float)((w0 >> 8) & 0xffu)),
        Elem<BF16>::from_f2((float)((w0 >> 16) & 0xffu), (float)(w0 >> 24)),
        Elem<BF16>::from_f2((float)(w1 & 0xffu), (float)((w1 >> 8) & 0xffu)),
        Elem<BF16>::from_f2((float)((w1 >> 16) & 0xffu), (float)(w1 >> 24)));
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
  auto fr = static_cast<const uint8_t*>(frames);
  auto o = static_cast<uint16_t*>(out);
  const long long fbytes = (long long)C * H * W;
  if (fbytes % 16 == 0 && fbytes <= 48 * 1024 && N < (1LL << 31) && (reinterpret_cast<uintptr_t>(frames) & 15) == 0) {
    const unsigned grid = (unsigned)N;
    if (bf16)
      frame_cta_to_blocks_kernel<true><<<grid, 256, (size_t)fbytes, st>>>(fr, o, C, H, W, frame_max);
    else
      frame_cta_to_blocks_kernel<false><<<grid, 256, (size_t)fbytes, st>>>(fr, o, C, H, W, frame_max);
  } else if (C == 4) {
    if (bf16)
      frames_to_blocks_kernel<true, true><<<(unsigned)blocks, 256, 0, st>>>(fr, o, n_pos, C, H, W, frame_max);
    else
      frames_to_blocks_kernel<false, true><<<(unsigned)blocks, 256, 0, st>>>(fr, o, n_pos, C, H, W, frame_max);
  } else {
    if (bf16)
      frames_to_blocks_kernel<true, false><<<(unsigned)blocks, 256, 0, st>>>(fr, o, n_pos, C, H, W, frame_max);
    else
      frames_to_blocks_kernel<false, false><<<(unsigned)blocks, 256, 0, st>>>(fr, o, n_pos, C, H, W, frame_max);
  }
  return cudaGetLastError();
}

}  // namespace dtk
