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
//    in that layout straight from HBM: one TMA box per (sub-pixel, 8-channel
//    group) walks the frame's pixels with a traversal stride of 2 in x and y
//    and writes the 100 blocks' 16-byte pieces of that K group contiguously,
//    16 boxes per frame.
//  * conv3: conv2's 9 x 9 x 64 output, written by conv2's epilogue into
//    shared memory on a 9-wide grid; output row m = 9 oy + ox (ox >= 7,
//    m >= 63 never stored) reads position m + 9 ky + kx for tap (ky, kx).
//
// Operand buffers hold the real rows of a K group (100 blocks, padded to 104
// so that every TMA box starts on a 128-byte boundary; 81 positions for
// conv3); a 128-row window runs past them into the next K group or the next
// buffer, but only in rows that are never stored (a stored conv2 row reads
// blocks up to 88 + 11 = 99, a stored conv3 row positions up to 60 + 20 = 80).
//
// The A operand of a tap is shared by the taps that differ only in x: their
// weights are stacked along N, so one MMA computes every x tap of a row of
// taps, and the x shift is applied to the accumulator instead of the operand.
// conv2: N = 128 (dx = 0, 1 stacked), E_dx[m] = sum over dy, K of
// A[m + 10 dy] W[dy, dx], output row m = E_0[m] + E_1[m + 1];
// conv3: N = 192 (kx = 0, 1, 2), output row m = E_0[m] + E_1[m + 1] + E_2[m + 2].
// That is 2 x 8 MMAs for conv2 and 3 x 4 for conv3 (28 per frame instead of
// 68 with one tap per MMA): each MMA reads its 4 KB A window once for 2 or 3
// taps, and the shared-memory operand traffic per frame drops from 408 KB to
// 248 KB.  The epilogue thread of row m takes row m + 1 / m + 2 from its
// neighbour lanes (warp shuffles); the rows right after a warp's 32 lanes
// (32 and 64 for conv2, 32 and 33 for conv3) are published through shared
// memory by the warp that owns them.  fp32 accumulators in TMEM, bias + ReLU
// in fp32, one rounding.
//
// One CTA per SM, warp-specialised and pipelined over its frames: warp 0
// issues the MMAs (conv2 of frame i, then conv3 of frame i - 1), warps 1-8 run
// the epilogues (thread = TMEM lane = output row, warps 1-4 output channels
// 0-31, warps 5-8 channels 32-63: conv2's into shared memory as conv3's
// operand, conv3's to HBM), one thread of warp 9 issues the TMA loads of the
// frames into two input buffers.  conv2's accumulator (2 x 128
// columns) and conv3's operand are double-buffered, conv3's accumulator (192
// columns) single, so the tensor core works on one frame while the epilogues
// finish the last.  The weights of both layers stay in shared memory (staged
// once per CTA from the reference's [64, Cin, k, k] layout).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kC23Threads = 320;  // warp 0 MMA issuer, 1-8 epilogue, 9 loader
constexpr int kEpiWarps = 8;
// K-major no-swizzle operands: a 16-byte piece holds 8 consecutive K values
// of one row; piece (K group j, row r) sits at (j * ROWS + r) * 16, so 8
// consecutive rows form a core matrix (SBO = 128 B) and the next K group is
// ROWS * 16 bytes on (LBO).
constexpr int kA2Rows = 104;  // conv2 input blocks (100) padded to a 128-byte K-group pitch
constexpr int kA2Bytes = 16 * kA2Rows * 16;
constexpr int kA3Rows = 81;   // conv3 input positions
constexpr int kA3Bytes = 8 * kA3Rows * 16;
constexpr int kN2 = 128;      // conv2 MMA N: (dx, out channel)
constexpr int kN3 = 192;      // conv3 MMA N: (kx, out channel)
constexpr int kW2Bytes = 2 * 16 * kN2 * 16;  // [dy][K group][dx, out channel][8 values]
constexpr int kW3Bytes = 3 * 8 * kN3 * 16;   // [ky][K group][kx, out channel][8 values]
constexpr int kOffW2 = 0;
constexpr int kOffW3 = kOffW2 + kW2Bytes;
constexpr int kOffA2 = kOffW3 + kW3Bytes;    // two buffers
constexpr int kOffA3 = kOffA2 + 2 * kA2Bytes;  // two buffers; the A2 overhang lands here
constexpr int kOffGuard = kOffA3 + 2 * kA3Bytes;  // the last A3 window's overhang (66 rows)
constexpr int kOffX2 = kOffGuard + 1280;     // [2 buffers][rows 32, 64][64] floats: E_1 of those rows
constexpr int kOffX3 = kOffX2 + 2 * 2 * 64 * 4;  // [E_1 row 32, E_2 row 32, E_2 row 33][64] floats
constexpr int kOffBias = kOffX3 + 3 * 64 * 4;  // 128 floats: conv2 then conv3
constexpr int kOffBar = kOffBias + 128 * 4;
// a2_full[2], a2_empty[2], c2_full[2], c2_empty[2], a3_full[2], a3_empty[2], x2_full[2], c3_full, c3_empty,
// x3_full, drain
constexpr int kC23Bars = 18;
constexpr int kC23Smem = kOffBar + kC23Bars * 8 + 16;
static_assert(kC23Smem <= 232448, "shared memory budget");
static_assert(16 * (20 + 128 - kA2Rows) <= 2 * kA3Bytes && 16 * (18 + 128 - kA3Rows) <= 1280,
              "window overhang stays inside the allocation");
static_assert((kA2Rows * 16) % 128 == 0 && kOffA2 % 128 == 0 && kA2Bytes % 128 == 0,
              "TMA boxes start on 128-byte boundaries");
constexpr uint32_t kFrameBytes = 20 * 20 * 32 * 2;  // the 16 boxes of one frame
// TMEM columns: conv2 accumulators at 0 and 128, conv3's at 256.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemC3 = 256;

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

// v += the values of lane + d (d = 1, 2); the last d lanes take row 32 (w + 1) + ...
// from `next` (the published rows after this warp's 32), when given.
template <int D>
__device__ __forceinline__ void add_shifted(float (&v)[32], const float (&e)[32], int lane, const float* next) {
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    float x = __shfl_down_sync(0xffffffffu, e[c], D);
    if (lane >= 32 - D) x = next ? next[(lane - (32 - D)) * 64 + c] : 0.0f;
    v[c] += x;
  }
}

__device__ __forceinline__ void store_row(float* dst, const float (&e)[32]) {
#pragma unroll
  for (int c = 0; c < 32; c += 4) *reinterpret_cast<float4*>(dst + c) = make_float4(e[c], e[c + 1], e[c + 2], e[c + 3]);
}

template <bool BF16>
__global__ void __launch_bounds__(kC23Threads, 1)
    encoder_conv23_kernel(const __grid_constant__ CUtensorMap tmX, const uint16_t* __restrict__ w2,
                          const float* __restrict__ b2, uint8_t* __restrict__ y2, const uint16_t* __restrict__ w3,
                          const float* __restrict__ b3, uint8_t* __restrict__ y3, long long n_frames,
                          int* status) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint16_t* w2s = reinterpret_cast<uint16_t*>(smem + kOffW2);
  uint16_t* w3s = reinterpret_cast<uint16_t*>(smem + kOffW3);
  float* bias = reinterpret_cast<float*>(smem + kOffBias);
  float* x2s = reinterpret_cast<float*>(smem + kOffX2);
  float* x3s = reinterpret_cast<float*>(smem + kOffX3);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t *a2_full = bars, *a2_empty = bars + 2, *c2_full = bars + 4, *c2_empty = bars + 6;
  uint64_t *a3_full = bars + 8, *a3_empty = bars + 10, *x2_full = bars + 12;
  uint64_t *c3_full = bars + 14, *c3_empty = bars + 15, *x3_full = bars + 16, *drain = bars + 17;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kC23Bars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  // conv2 weights into [dy][K group][dx, out channel][8 values]; the K order
  // within a row of taps is (sub-pixel sy, sx; channel), the block layout of
  // its input.
#pragma unroll 8
  for (int i = tid; i < 2 * 16 * kN2 * 8; i += kC23Threads) {
    const int e = i & 7, nn = (i >> 3) & 127, j = (i >> 10) & 15, dy = i >> 14;
    const int dx = nn >> 6, n = nn & 63;
    const int k = j * 8 + e, sub = k >> 5, c = k & 31;
    const int ky = 2 * dy + (sub >> 1), kx = 2 * dx + (sub & 1);
    w2s[i] = w2[((n * 32 + c) * 4 + ky) * 4 + kx];
  }
  // conv3 weights into [ky][K group][kx, out channel][8 values].
#pragma unroll 8
  for (int i = tid; i < 3 * 8 * kN3 * 8; i += kC23Threads) {
    const int e = i & 7, r = i >> 3, nn = r % kN3, j = (r / kN3) & 7, ky = r / (kN3 * 8);
    const int kx = nn >> 6, n = nn & 63, c = j * 8 + e;
    w3s[i] = w3[((n * 64 + c) * 3 + ky) * 3 + kx];
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
      mbar_init(&a2_full[b], 1);   // the loader's expect_tx; the 16 boxes complete the bytes
      mbar_init(&a2_empty[b], 1);  // MMA commit
      mbar_init(&c2_full[b], 1);
      mbar_init(&c2_empty[b], kEpiWarps);  // one arrival per epilogue warp
      mbar_init(&a3_full[b], kEpiWarps);
      mbar_init(&a3_empty[b], 1);
      mbar_init(&x2_full[b], 4);   // the warps owning rows 32 and 64 (both channel halves)
    }
    mbar_init(c3_full, 1);
    mbar_init(c3_empty, kEpiWarps);
    mbar_init(x3_full, 2);         // the warps owning rows 32 and 33 (both channel halves)
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_holder, kTmemCols);
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
      const uint32_t idesc2 = umma_idesc_f16(BF16, 128, kN2, 0, 0);
      const uint32_t idesc3 = umma_idesc_f16(BF16, 128, kN3, 0, 0);
      const uint32_t a2_base = smem_u32(smem + kOffA2), a3_base = smem_u32(smem + kOffA3);
      // The descriptors' 14-bit start-address field (address / 16) has room for
      // every offset added below: the whole allocation is under 256 KB.
      const uint64_t w2_desc = umma_smem_desc(smem_u32(smem + kOffW2), kN2 * 16, 128, kSwNone);
      const uint64_t w3_desc = umma_smem_desc(smem_u32(smem + kOffW3), kN3 * 16, 128, kSwNone);
      bool ok = true;
      auto conv3 = [&](long long i) -> bool {
        const int b = (int)(i & 1);
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(&a3_full[b], ph, abort_flag, status)) return false;
        if (!mbar_wait(c3_empty, ((uint32_t)i & 1u) ^ 1u, abort_flag, status)) return false;
        tc_fence_after();
        const uint64_t a0 = umma_smem_desc(a3_base + (uint32_t)(b * kA3Bytes), kA3Rows * 16, 128, kSwNone);
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
          for (int s = 0; s < 4; ++s)
            umma_f16_ss(tmem + kTmemC3, a0 + (uint64_t)((2 * s) * kA3Rows + 9 * ky),
                        w3_desc + (uint64_t)((ky * 8 + 2 * s) * kN3), idesc3, (ky | s) ? 1u : 0u);
        }
        umma_commit(&a3_empty[b]);
        umma_commit(c3_full);
        return true;
      };
      for (long long i = 0; i < nloc && ok; ++i) {
        const int b = (int)(i & 1);
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!(ok = mbar_wait(&a2_full[b], ph, abort_flag, status))) break;
        if (!(ok = mbar_wait(&c2_empty[b], ph ^ 1u, abort_flag, status))) break;
        tc_fence_after();
        const uint64_t a0 = umma_smem_desc(a2_base + (uint32_t)(b * kA2Bytes), kA2Rows * 16, 128, kSwNone);
#pragma unroll
        for (int dy = 0; dy < 2; ++dy) {
#pragma unroll
          for (int s = 0; s < 8; ++s)
            umma_f16_ss(tmem + (uint32_t)(kN2 * b), a0 + (uint64_t)((2 * s) * kA2Rows + 10 * dy),
                        w2_desc + (uint64_t)((dy * 16 + 2 * s) * kN2), idesc2, (dy | s) ? 1u : 0u);
        }
        umma_commit(&a2_empty[b]);
        umma_commit(&c2_full[b]);
        if (i >= 1) ok = conv3(i - 1);
      }
      if (ok && nloc >= 1) conv3(nloc - 1);
      // every MMA issued has finished before TMEM is released
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else if (warp <= kEpiWarps) {
    // ------------------------------------------------------------ epilogues
    const int wq = warp & 3;                    // TMEM lane quarter of this warp
    const int h = (warp - 1) >> 2;              // output channels 32 h .. 32 h + 31
    const int m = wq * 32 + lane;               // accumulator row
    const uint32_t t_row = tmem + ((uint32_t)(wq * 32) << 16);
    bool ok = true;
    auto epi3 = [&](long long i) -> bool {
      const uint32_t ph = (uint32_t)i & 1u;
      if (!__all_sync(0xffffffffu, mbar_wait(c3_full, ph, abort_flag, status))) return false;
      tc_fence_after();
      // E_0, E_1, E_2 of this row and channel half: three loads in flight, one wait
      uint32_t r0[32], r1[32], r2[32];
      tmem_ld32_async(t_row + kTmemC3 + 32u * h, r0);
      tmem_ld32_async(t_row + kTmemC3 + 64u + 32u * h, r1);
      tmem_ld32_async(t_row + kTmemC3 + 128u + 32u * h, r2);
      tmem_wait_ld3(r0, r1, r2);
      float v[32], e1[32], e2[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        v[c] = __uint_as_float(r0[c]);
        e1[c] = __uint_as_float(r1[c]);
        e2[c] = __uint_as_float(r2[c]);
      }
      if (wq == 1) {
        // publish E_1 of row 32 and E_2 of rows 32, 33 for the rows 30, 31 above
        if (lane == 0) store_row(x3s + 32 * h, e1);
        if (lane < 2) store_row(x3s + (1 + lane) * 64 + 32 * h, e2);
        __syncwarp();
        if (lane == 0) mbar_arrive(x3_full);
      }
      if (wq == 0 && !__all_sync(0xffffffffu, mbar_wait(x3_full, ph, abort_flag, status))) return false;
      const long long f = frame(i);
      const int oy = m / 9, ox = m - 9 * (m / 9);
      const bool valid = m < 63 && ox < 7;
      {
        add_shifted<1>(v, e1, lane, wq == 0 ? x3s + 32 * h : nullptr);
        add_shifted<2>(v, e2, lane, wq == 0 ? x3s + 64 + 32 * h : nullptr);
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
      if (lane == 0) mbar_arrive(c3_empty);  // after this warp's reads of TMEM and of the published rows
      return true;
    };
    for (long long i = 0; i < nloc && ok; ++i) {
      const int b = (int)(i & 1);
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&c2_full[b], ph, abort_flag, status)))) break;
      // conv3's operand buffer b is free once frame i - 2's conv3 MMAs are done
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&a3_empty[b], ph ^ 1u, abort_flag, status)))) break;
      tc_fence_after();
      // E_0, E_1 of this row and channel half: both loads in flight, one wait
      uint32_t r0[32], r1[32];
      tmem_ld32_async(t_row + (uint32_t)(kN2 * b) + 32u * h, r0);
      tmem_ld32_async(t_row + (uint32_t)(kN2 * b) + 64u + 32u * h, r1);
      tmem_wait_ld(r0);
      tmem_wait_ld(r1);
      float v[32], e[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        v[c] = __uint_as_float(r0[c]);
        e[c] = __uint_as_float(r1[c]);
      }
      float* xb = x2s + b * 128;
      if (wq == 1 || wq == 2) {
        // publish E_1 of row 32 (warp quarter 1) / row 64 (quarter 2)
        if (lane == 0) store_row(xb + (wq - 1) * 64 + 32 * h, e);
        __syncwarp();
        if (lane == 0) mbar_arrive(&x2_full[b]);
      }
      if (wq <= 1 && !(ok = __all_sync(0xffffffffu, mbar_wait(&x2_full[b], ph, abort_flag, status)))) break;
      const long long f = frame(i);
      const int oy = m / 10, ox = m - 10 * (m / 10);
      const bool valid = m < 90 && ox < 9;
      const int q = oy * 9 + ox;
      uint8_t* a3 = smem + kOffA3 + b * kA3Bytes;
      {
        add_shifted<1>(v, e, lane, wq <= 1 ? xb + wq * 64 + 32 * h : nullptr);
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
        mbar_arrive(&c2_empty[b]);  // after this warp's reads of TMEM and of the published rows
        mbar_arrive(&a3_full[b]);
      }
      if (i >= 1) ok = epi3(i - 1);
    }
    if (ok && nloc >= 1) epi3(nloc - 1);
  } else if (lane == 0) {
    // ------------------------------------------------------------ loader
    // K group j = 4 (2 sy + sx) + cg of a frame: the box of channels 8 cg ..
    // 8 cg + 7 at pixels (2 by + sy, 2 bx + sx), block-major (by, bx).
    prefetch_tmap(&tmX);
    long long i = 0;
    bool ok = true;
    for (; i < nloc; ++i) {
      const int b = (int)(i & 1);
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!(ok = mbar_wait(&a2_empty[b], ph ^ 1u, abort_flag, status))) break;
      mbar_arrive_expect_tx(&a2_full[b], kFrameBytes);
      uint8_t* a2 = smem + kOffA2 + b * kA2Bytes;
      const int f = (int)frame(i);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        tma_load_4d(a2 + j * kA2Rows * 16, &tmX, &a2_full[b], 8 * (j & 3), (j >> 2) & 1, j >> 3, f);
    }
    if (!ok)  // copies already issued land before the CTA exits
      for (int b = 0; b < 2; ++b) {
        const long long uses = i / 2 + (b < (int)(i & 1) ? 1 : 0);
        if (uses > 0) mbar_wait(&a2_full[b], (uint32_t)((uses - 1) & 1), nullptr, nullptr);
      }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_encoder_conv23_sm100(const CUtensorMap& x1, const void* w2, const float* b2, void* y2, const void* w3,
                                        const float* b3, void* y3, long long n_frames, bool bf16, int num_sms,
                                        int* status, cudaStream_t st) {
  const void* fn = bf16 ? reinterpret_cast<const void*>(encoder_conv23_kernel<true>)
                        : reinterpret_cast<const void*>(encoder_conv23_kernel<false>);
  cudaError_t e = smem_limit_once(fn, kC23Smem);
  if (e != cudaSuccess) return e;
  const long long grid = n_frames < num_sms ? n_frames : num_sms;
  auto args = [&](auto k) {
    k<<<(unsigned)grid, kC23Threads, kC23Smem, st>>>(
        x1, static_cast<const uint16_t*>(w2), b2, static_cast<uint8_t*>(y2),
        static_cast<const uint16_t*>(w3), b3, static_cast<uint8_t*>(y3), n_frames, status);
  };
  if (bf16) args(encoder_conv23_kernel<true>);
  else args(encoder_conv23_kernel<false>);
  return cudaGetLastError();
}

}  // namespace dtk
