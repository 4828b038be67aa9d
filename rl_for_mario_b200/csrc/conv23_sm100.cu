// The state encoder's second and third convolutions with their ReLUs
// (model/model_decision_transformer.py:322-325: Conv2d(32, 64, 4, stride 2)
// on 20 x 20 and Conv2d(64, 64, 3, stride 1) on 9 x 9) fused in one
// persistent tcgen05 kernel, sm_100a: the second layer's output never leaves
// shared memory.
//
// Both convolutions are computed on padded output grids, so that for every
// kernel tap the rows of the A operand (one row per output position) are one
// contiguous window of the input positions, in the K-major, no-swizzle
// operand layout the MMA reads: no im2col copy and no per-tap gather.
//
//  * conv2: the 20 x 20 x 32 input as 10 x 10 blocks of 2 x 2 pixels (128
//    values per block); the 4 x 4 stride-2 kernel is a 2 x 2 stride-1 kernel
//    over blocks.  Output row m = 10 oy + ox on a 10-wide grid (ox = 9 and
//    m >= 90 are never stored) reads block m + 10 dy + dx for tap (dy, dx), so
//    a tap is the operand window starting at block 10 dy + dx.  The input lands
//    in that layout straight from HBM: cp.async copies each 16-byte piece
//    (8 channels of a pixel) to its place (block, 16-byte K group).
//  * conv3: conv2's 9 x 9 x 64 output, written by conv2's epilogue into
//    shared memory on a 9-wide grid; output row m = 9 oy + ox (ox >= 7,
//    m >= 63 never stored) reads position m + 9 ky + kx for tap (ky, kx).
//
// Operand buffers hold only real rows (100 blocks, 81 positions per K group);
// a 128-row window runs past them into the next K group or the next buffer,
// but only in rows that are never stored (a stored conv2 row reads blocks up
// to 88 + 11 = 99, a stored conv3 row positions up to 60 + 20 = 80).
//
// M = 128 rows, N = 64 output channels, K = 16 per MMA: conv2 is 4 taps x 8
// K steps, conv3 9 taps x 4; fp32 accumulators in TMEM, bias + ReLU in fp32,
// one rounding.  One CTA per SM, warp-specialised and pipelined over its
// frames: warp 0 issues the MMAs (conv2 of frame i, then conv3 of frame i - 1),
// warps 1-4 run the epilogues (thread = TMEM lane = output row: conv2's into
// shared memory as conv3's operand, conv3's to HBM), warp 5 loads frames two
// input buffers ahead.  Accumulators and conv3's operand are double-buffered,
// so the tensor core works on one frame while the epilogues finish the last.
// The weights of both layers stay in shared memory (staged once per CTA from
// the reference's [64, Cin, k, k] layout).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kC23Threads = 192;  // warp 0 MMA issuer, 1-4 epilogue, 5 loader
// K-major no-swizzle operands: a 16-byte piece holds 8 consecutive K values
// of one row; piece (K group j, row r) sits at (j * ROWS + r) * 16, so 8
// consecutive rows form a core matrix (SBO = 128 B) and the next K group is
// ROWS * 16 bytes on (LBO).
constexpr int kA2Rows = 100;  // conv2 input blocks
constexpr int kA2Bytes = 16 * kA2Rows * 16;
constexpr int kA3Rows = 81;   // conv3 input positions
constexpr int kA3Bytes = 8 * kA3Rows * 16;
constexpr int kW2Bytes = 4 * 16 * 64 * 16;  // [tap][K group][out channel][8 values]
constexpr int kW3Bytes = 9 * 8 * 64 * 16;
constexpr int kOffW2 = 0;
constexpr int kOffW3 = kOffW2 + kW2Bytes;
constexpr int kOffA2 = kOffW3 + kW3Bytes;    // two buffers
constexpr int kOffA3 = kOffA2 + 2 * kA2Bytes;  // two buffers; the A2 overhang (39 rows) lands here
constexpr int kOffGuard = kOffA3 + 2 * kA3Bytes;  // the last A3 window's overhang (66 rows)
constexpr int kOffBias = kOffGuard + 1280;   // 128 floats: conv2 then conv3
constexpr int kOffBar = kOffBias + 128 * 4;
// a2_full[2], a2_empty[2], c2_full[2], c2_empty[2], a3_full[2], a3_empty[2], c3_full[2], c3_empty[2]
constexpr int kC23Bars = 16;
constexpr int kC23Smem = kOffBar + kC23Bars * 8 + 16;
static_assert(kC23Smem <= 232448, "shared memory budget");
static_assert(16 * 39 <= 2 * kA3Bytes && 16 * 66 <= 1280, "window overhang stays inside the allocation");
constexpr int kFrameBytes = 20 * 20 * 32 * 2;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// 32 accumulator columns of this thread's row + bias, ReLU, 16-bit: four 16-byte pieces.
template <bool BF16>
__device__ __forceinline__ void relu_pieces(const float (&v)[32], const float* bias, uint4 (&out)[4]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = 8 * g + 2 * e;
      w[e] = pack2<BF16>(fmaxf(v[c] + bias[c], 0.0f), fmaxf(v[c + 1] + bias[c + 1], 0.0f));
    }
    out[g] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kC23Threads, 1)
    encoder_conv23_kernel(const uint8_t* __restrict__ x1, const uint16_t* __restrict__ w2,
                          const float* __restrict__ b2, uint8_t* __restrict__ y2, const uint16_t* __restrict__ w3,
                          const float* __restrict__ b3, uint8_t* __restrict__ y3, long long n_frames,
                          int* status) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint16_t* w2s = reinterpret_cast<uint16_t*>(smem + kOffW2);
  uint16_t* w3s = reinterpret_cast<uint16_t*>(smem + kOffW3);
  float* bias = reinterpret_cast<float*>(smem + kOffBias);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t *a2_full = bars, *a2_empty = bars + 2, *c2_full = bars + 4, *c2_empty = bars + 6;
  uint64_t *a3_full = bars + 8, *a3_empty = bars + 10, *c3_full = bars + 12, *c3_empty = bars + 14;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kC23Bars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  // Weights into [tap][K group][out channel][8 values]; conv2's K order within a
  // tap is (sub-pixel sy, sx; channel), the block layout of its input.
  for (int i = tid; i < 4 * 128 * 64; i += kC23Threads) {
    const int e = i & 7, n = (i >> 3) & 63, j = (i >> 9) & 15, t = i >> 13;
    const int k = j * 8 + e, sub = k >> 5, c = k & 31;
    const int ky = 2 * (t >> 1) + (sub >> 1), kx = 2 * (t & 1) + (sub & 1);
    w2s[((t * 16 + j) * 64 + n) * 8 + e] = w2[((n * 32 + c) * 4 + ky) * 4 + kx];
  }
  for (int i = tid; i < 9 * 64 * 64; i += kC23Threads) {
    const int e = i & 7, n = (i >> 3) & 63, j = (i >> 9) & 7, t = i >> 12;
    const int c = j * 8 + e, ky = t / 3, kx = t - 3 * (t / 3);
    w3s[((t * 8 + j) * 64 + n) * 8 + e] = w3[((n * 64 + c) * 3 + ky) * 3 + kx];
  }
  if (tid < 64) {
    bias[tid] = b2[tid];
    bias[64 + tid] = b3[tid];
  }
  // The overhang regions hold whatever the window reads past real rows: zero
  // them once so that even never-stored accumulator rows stay finite.
  for (int i = tid; i < (2 * kA2Bytes + 2 * kA3Bytes + 1280) / 16; i += kC23Threads)
    reinterpret_cast<uint4*>(smem + kOffA2)[i] = make_uint4(0, 0, 0, 0);
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a2_full[b], 32);  // every loader lane, once its copies have landed
      mbar_init(&a2_empty[b], 1);  // MMA commit
      mbar_init(&c2_full[b], 1);
      mbar_init(&c2_empty[b], 4);  // one arrival per epilogue warp
      mbar_init(&a3_full[b], 4);
      mbar_init(&a3_empty[b], 1);
      mbar_init(&c3_full[b], 1);
      mbar_init(&c3_empty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, 256);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the generic writes above, before the tensor core reads them
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // this CTA's frames: f = blockIdx.x + i * gridDim.x, i < nloc
  const long long nloc = n_frames > blockIdx.x ? (n_frames - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  auto frame = [&](long long i) { return blockIdx.x + i * (long long)gridDim.x; };

  if (warp == 0) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BF16, 128, 64, 0, 0);
      const uint32_t a2_base = smem_u32(smem + kOffA2), a3_base = smem_u32(smem + kOffA3);
      const uint32_t w2_base = smem_u32(smem + kOffW2), w3_base = smem_u32(smem + kOffW3);
      bool ok = true;
      auto conv3 = [&](long long i) -> bool {
        const int b = (int)(i & 1);
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(&a3_full[b], ph, abort_flag, status)) return false;
        if (!mbar_wait(&c3_empty[b], ph ^ 1u, abort_flag, status)) return false;
        tc_fence_after();
        const uint32_t a = a3_base + (uint32_t)(b * kA3Bytes), d = tmem + 128u + 64u * b;
#pragma unroll 1
        for (int t = 0; t < 9; ++t) {
          const uint32_t p0 = (uint32_t)((t / 3) * 9 + t % 3);
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint64_t ad = umma_smem_desc(a + ((2 * s) * kA3Rows + p0) * 16, kA3Rows * 16, 128, kSwNone);
            const uint64_t bd =
                umma_smem_desc(w3_base + (uint32_t)(((t * 8 + 2 * s) * 64) * 16), 64 * 16, 128, kSwNone);
            umma_f16_ss(d, ad, bd, idesc, (t | s) ? 1u : 0u);
          }
        }
        umma_commit(&a3_empty[b]);
        umma_commit(&c3_full[b]);
        return true;
      };
      for (long long i = 0; i < nloc && ok; ++i) {
        const int b = (int)(i & 1);
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!(ok = mbar_wait(&a2_full[b], ph, abort_flag, status))) break;
        if (!(ok = mbar_wait(&c2_empty[b], ph ^ 1u, abort_flag, status))) break;
        tc_fence_after();
        const uint32_t a = a2_base + (uint32_t)(b * kA2Bytes), d = tmem + 64u * b;
#pragma unroll 1
        for (int t = 0; t < 4; ++t) {
          const uint32_t p0 = (uint32_t)((t >> 1) * 10 + (t & 1));
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            const uint64_t ad = umma_smem_desc(a + ((2 * s) * kA2Rows + p0) * 16, kA2Rows * 16, 128, kSwNone);
            const uint64_t bd =
                umma_smem_desc(w2_base + (uint32_t)(((t * 16 + 2 * s) * 64) * 16), 64 * 16, 128, kSwNone);
            umma_f16_ss(d, ad, bd, idesc, (t | s) ? 1u : 0u);
          }
        }
        umma_commit(&a2_empty[b]);
        umma_commit(&c2_full[b]);
        if (i >= 1) ok = conv3(i - 1);
      }
      if (ok && nloc >= 1) conv3(nloc - 1);
    }
  } else if (warp <= 4) {
    // ------------------------------------------------------------ epilogues
    const int wq = warp & 3;                    // TMEM lane quarter of this warp
    const int m = wq * 32 + lane;               // accumulator row
    const uint32_t t_row = tmem + ((uint32_t)(wq * 32) << 16);
    bool ok = true;
    auto epi3 = [&](long long i) -> bool {
      const int b = (int)(i & 1);
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(&c3_full[b], ph, abort_flag, status))) return false;
      tc_fence_after();
      const long long f = frame(i);
      const int oy = m / 9, ox = m - 9 * (m / 9);
      const bool valid = m < 63 && ox < 7;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
        tmem_ld32(t_row + 128u + 64u * b + 32u * h, v);
        uint4 p[4];
        relu_pieces<BF16>(v, bias + 64 + 32 * h, p);
        if (valid) {
          uint8_t* dst = y3 + ((f * 49 + oy * 7 + ox) * 64 + 32 * h) * 2;
#pragma unroll
          for (int g = 0; g < 4; ++g) *reinterpret_cast<uint4*>(dst + g * 16) = p[g];
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c3_empty[b]);
      return true;
    };
    for (long long i = 0; i < nloc && ok; ++i) {
      const int b = (int)(i & 1);
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&c2_full[b], ph, abort_flag, status)))) break;
      // conv3's operand buffer b is free once frame i - 2's conv3 MMAs are done
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&a3_empty[b], ph ^ 1u, abort_flag, status)))) break;
      tc_fence_after();
      const long long f = frame(i);
      const int oy = m / 10, ox = m - 10 * (m / 10);
      const bool valid = m < 90 && ox < 9;
      const int q = oy * 9 + ox;
      uint8_t* a3 = smem + kOffA3 + b * kA3Bytes;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
        tmem_ld32(t_row + 64u * b + 32u * h, v);
        uint4 p[4];
        relu_pieces<BF16>(v, bias + 32 * h, p);
        if (valid) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            *reinterpret_cast<uint4*>(a3 + ((4 * h + g) * kA3Rows + q) * 16) = p[g];
            if (y2) *reinterpret_cast<uint4*>(y2 + ((f * 81 + q) * 64 + 32 * h + 8 * g) * 2) = p[g];
          }
        }
      }
      fence_proxy_async_smem();  // conv3's operand, before the tensor core reads it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&c2_empty[b]);
        mbar_arrive(&a3_full[b]);
      }
      if (i >= 1) ok = epi3(i - 1);
    }
    if (ok && nloc >= 1) epi3(nloc - 1);
  } else {
    // ------------------------------------------------------------ loader
    bool ok = true;
    for (long long i = 0; i < nloc && ok; ++i) {
      const int b = (int)(i & 1);
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&a2_empty[b], ph ^ 1u, abort_flag, status)))) break;
      const uint8_t* src = x1 + frame(i) * kFrameBytes;
      const uint32_t a2 = smem_u32(smem + kOffA2 + b * kA2Bytes);
      for (int k = lane; k < 1600; k += 32) {
        const int pix = k >> 2, cg = k & 3, y = pix / 20, x = pix - 20 * (pix / 20);
        const int blk = (y >> 1) * 10 + (x >> 1), j = (((y & 1) << 1) | (x & 1)) * 4 + cg;
        cp_async16(a2 + (uint32_t)((j * kA2Rows + blk) * 16), src + k * 16);
      }
      cp_async_commit();
      cp_async_wait<0>();
      fence_proxy_async_smem();  // these pieces, before the tensor core reads them
      mbar_arrive(&a2_full[b]);
    }
    cp_async_wait<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

cudaError_t launch_encoder_conv23_sm100(const void* x1, const void* w2, const float* b2, void* y2, const void* w3,
                                        const float* b3, void* y3, long long n_frames, bool bf16, int num_sms,
                                        int* status, cudaStream_t st) {
  const void* fn = bf16 ? reinterpret_cast<const void*>(encoder_conv23_kernel<true>)
                        : reinterpret_cast<const void*>(encoder_conv23_kernel<false>);
  cudaError_t e = smem_limit_once(fn, kC23Smem);
  if (e != cudaSuccess) return e;
  const long long grid = n_frames < num_sms ? n_frames : num_sms;
  auto args = [&](auto k) {
    k<<<(unsigned)grid, kC23Threads, kC23Smem, st>>>(
        static_cast<const uint8_t*>(x1), static_cast<const uint16_t*>(w2), b2, static_cast<uint8_t*>(y2),
        static_cast<const uint16_t*>(w3), b3, static_cast<uint8_t*>(y3), n_frames, status);
  };
  if (bf16) args(encoder_conv23_kernel<true>);
  else args(encoder_conv23_kernel<false>);
  return cudaGetLastError();
}

}  // namespace dtk
