// The state encoder's first convolution straight from the uint8 frames,
// sm_100a (tcgen05 implicit GEMM).
//
// Reference: model/model_decision_transformer.py:315-341 — frames / 255 when
// the frames' maximum exceeds 1 (:338), then Conv2d(4, 32, 8, stride 4) and
// ReLU.  As a GEMM: one row per output position (n, oy, ox), K = 4 x 8 x 8
// pixels of its receptive field (order c, ky, kx: the weight's own layout),
// N = 32 output channels; y = relu(s (A W^T) + bias) with s = 1/255 or 1.
//
// Persistent CTAs over 128-row tiles of the flattened positions:
//   warps 8-23  build the A tile of the next position block in shared memory
//               (double-buffered), one (row, input channel) per thread, all its
//               loads in flight at once: per kernel row the 8 pixels
//               are two 32-bit loads, turned into exact 16-bit values (the
//               byte is placed in the mantissa of 2^23 with a byte permute,
//               2^23 subtracted) and stored as one 16-byte piece of the
//               128-byte-swizzled K-major layout the MMA reads;
//   warp 4      owns TMEM (two 32-column fp32 accumulators) and issues the 16
//               128 x 32 x 16 MMAs of a tile;
//   warps 0-3   read an accumulator (one TMEM lane quarter each), apply
//               scale, bias and ReLU and write the 32 channels of a position
//               (64 contiguous bytes, channels-last).
// The pixel values 0..255 are exact in bf16 / fp16; the 1/255 is applied to
// the fp32 accumulator.  Whether it applies (some byte > 1) is decided by a
// first kernel that stops reading as soon as any thread has seen such a byte.
#include <mutex>

#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kC1Threads = 768;
constexpr int kC1Builders = 16;  // warps 8..23
constexpr int kC1N = 32;        // output channels

struct C1Shape {
  static constexpr int A_ATOM = 128 * 128;   // 128 rows x 64 K-values of 16 bits (one input channel)
  static constexpr int A_BYTES = 4 * A_ATOM;  // K = 256
  static constexpr int B_ATOM = kC1N * 128;   // 32 rows x 64 K-values
  static constexpr int B_BYTES = 4 * B_ATOM;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = 2 * A_BYTES;
  static constexpr int OFF_BIAS = OFF_B + B_BYTES;  // 32 floats
  static constexpr int OFF_BAR = OFF_BIAS + kC1N * 4;
  // a_full[2], a_empty[2], acc_full[2], acc_empty[2], drain
  static constexpr int NBAR = 9;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Byte offset of 16-byte piece j of row r inside a 128-byte-swizzled K-major atom.
__device__ __forceinline__ uint32_t sw128_off(int r, int j) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

// Exact float of byte k of w: 0x4B0000bb is 2^23 + b.
__device__ __forceinline__ float byte_f(uint32_t w, int k) {
  return __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)k)) - 8388608.f;
}

// *frame_max ends > 1 exactly when some byte exceeds 1 (then it is such a
// byte; else it is the largest byte, 0 or 1).  A warp stops once the flag
// says > 1, so real frames cost a few reads instead of a pass; one atomic per
// warp and step.
__global__ void __launch_bounds__(256) frames_max_kernel(const uint4* __restrict__ f, long long n16,
                                                         unsigned int* frame_max) {
  const volatile unsigned int* vf = frame_max;
  const long long stride = (long long)gridDim.x * blockDim.x;
  // whole warps iterate together (the bound is warp-uniform)
  const long long start = (long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31);
  for (long long i0 = start; i0 < n16; i0 += stride) {
    unsigned int seen = 0;
    if ((threadIdx.x & 31) == 0) seen = *vf;
    if (__shfl_sync(0xffffffffu, seen, 0) > 1u) return;
    const long long i = i0 + (threadIdx.x & 31);
    uint32_t b = 0;
    if (i < n16) {
      const uint4 u = __ldg(f + i);
      const uint32_t m = __vmaxu4(__vmaxu4(u.x, u.y), __vmaxu4(u.z, u.w));
      b = max(max(m & 0xffu, (m >> 8) & 0xffu), max((m >> 16) & 0xffu, m >> 24));
    }
    b = __reduce_max_sync(0xffffffffu, b);
    if ((threadIdx.x & 31) == 0 && b > 0) atomicMax(frame_max, b);
    if (b > 1) return;
  }
}

// ROUND: the pixels enter the MMA as frames / 255 rounded to the 16-bit type
// (the reference's 16-bit evaluation of x / 255 before its convolution, :338)
// instead of exact integers with the 1/255 applied to the accumulator.
template <bool BF16, bool ROUND>
__global__ void __launch_bounds__(kC1Threads, 1)
    frames_conv1_kernel(const uint8_t* __restrict__ frames, const uint16_t* __restrict__ w,
                        const float* __restrict__ bias, const unsigned int* __restrict__ frame_max,
                        uint16_t* __restrict__ y, long long total, int H, int W, int OH, int OW, int* status) {
  using SH = C1Shape;
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = smem + SH::OFF_A;
  uint8_t* b_s = smem + SH::OFF_B;
  float* bias_s = reinterpret_cast<float*>(smem + SH::OFF_BIAS);
  uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* a_empty = a_full + 2;
  uint64_t* acc_full = a_empty + 2;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  __shared__ uint32_t tmem_holder;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long ntiles = (total + 127) / 128;

  if (tid == 0) {
    for (int j = 0; j < 2; ++j) {
      mbar_init(&a_full[j], kC1Builders);
      mbar_init(&a_empty[j], 1);
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], 4);
    }
    mbar_init(drain, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  // W [32][256] into the swizzled K-major B layout (atom = input channel), bias into shared memory.
  for (int e = tid; e < kC1N * 32; e += kC1Threads) {  // 32 rows x 32 pieces of 16 bytes
    const int r = e >> 5, piece = e & 31, atom = piece >> 3, j = piece & 7;
    const uint4 v = *reinterpret_cast<const uint4*>(w + (size_t)r * 256 + piece * 8);
    *reinterpret_cast<uint4*>(b_s + atom * SH::B_ATOM + sw128_off(r, j)) = v;
  }
  if (tid < kC1N) bias_s[tid] = bias[tid];
  if (warp == 4) {
    tmem_alloc(&tmem_holder, 64);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_holder;
  const int P = OH * OW;
  const long long fbytes = 4LL * H * W;

  if (warp >= 8) {
    // ---------------------------------------------------------------- A builders
    const int tb = tid - 256;  // 0..511
    // x / 255 in fp32, then rounded with the 16-bit conversion below: the same
    // value as the reference's 16-bit division for every byte.
    const float in_scale = (ROUND && *frame_max > 1u) ? (1.f / 255.f) : 1.f;
    int i = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!(ok = mbar_wait(&a_empty[buf], ((i >> 1) & 1) ^ 1, &abort_flag, status))) break;
      uint8_t* ab = a_s + buf * SH::A_BYTES;
      // This thread's row (position) of the tile and one of its four channels.
      const int r = tb & 127, c = tb >> 7;
      const long long p = t * 128 + r;
      const bool valid = p < total;
      const uint8_t* base = frames;
      if (valid) {
        const long long n = p / P;
        const int rem = (int)(p - n * P);
        const int oy = rem / OW, ox = rem - oy * OW;
        base = frames + n * fbytes + (size_t)(4 * oy) * W + 4 * ox;
      }
      // All 16 loads first (one round trip), then the conversions and stores.
      uint32_t px[8][2];
      const uint8_t* cbase = base + (size_t)c * H * W;
#pragma unroll
      for (int ky = 0; ky < 8; ++ky) {
        const uint8_t* src = cbase + (size_t)ky * W;
        px[ky][0] = valid ? __ldg(reinterpret_cast<const uint32_t*>(src)) : 0u;
        px[ky][1] = valid ? __ldg(reinterpret_cast<const uint32_t*>(src + 4)) : 0u;
      }
#pragma unroll
      for (int ky = 0; ky < 8; ++ky) {
        const uint32_t w0 = px[ky][0], w1 = px[ky][1];
        uint4 o;
        if (ROUND) {
          o.x = E::from_f2(byte_f(w0, 0) * in_scale, byte_f(w0, 1) * in_scale);
          o.y = E::from_f2(byte_f(w0, 2) * in_scale, byte_f(w0, 3) * in_scale);
          o.z = E::from_f2(byte_f(w1, 0) * in_scale, byte_f(w1, 1) * in_scale);
          o.w = E::from_f2(byte_f(w1, 2) * in_scale, byte_f(w1, 3) * in_scale);
        } else {
          o.x = E::from_f2(byte_f(w0, 0), byte_f(w0, 1));
          o.y = E::from_f2(byte_f(w0, 2), byte_f(w0, 3));
          o.z = E::from_f2(byte_f(w1, 0), byte_f(w1, 1));
          o.w = E::from_f2(byte_f(w1, 2), byte_f(w1, 3));
        }
        *reinterpret_cast<uint4*>(ab + c * SH::A_ATOM + sw128_off(r, ky)) = o;
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[buf]);
    }
  } else if (warp == 4) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BF16, 128, kC1N, 0, 0);
      int i = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!(ok = mbar_wait(&a_full[buf], (i >> 1) & 1, &abort_flag, status))) break;
        if (!(ok = mbar_wait(&acc_empty[buf], ((i >> 1) & 1) ^ 1, &abort_flag, status))) break;
        tc_fence_after();
#pragma unroll
        for (int atom = 0; atom < 4; ++atom) {
          const uint64_t ad = umma_smem_desc(smem_u32(a_s + buf * SH::A_BYTES + atom * SH::A_ATOM), 16, 1024, kSw128);
          const uint64_t bd = umma_smem_desc(smem_u32(b_s + atom * SH::B_ATOM), 16, 1024, kSw128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 32 bytes per K step inside the 128-byte atom
            umma_f16_ss(tmem + (uint32_t)(buf * kC1N), ad + 2 * kk, bd + 2 * kk, idesc,
                        (atom > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&a_empty[buf]);
        umma_commit(&acc_full[buf]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else if (warp < 4) {
    // ---------------------------------------------------------------- epilogue
    const int wq = warp;
    const int r = wq * 32 + lane;
    const float s = (!ROUND && *frame_max > 1u) ? (1.f / 255.f) : 1.f;
    const float* b = bias_s;
    int i = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (i >> 1) & 1, &abort_flag, status)))) break;
      tc_fence_after();
      float v[kC1N];
      tmem_ld32(tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(buf * kC1N), v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const long long p = t * 128 + r;
      if (p < total) {
        uint4* dst = reinterpret_cast<uint4*>(y + (size_t)p * kC1N);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = q * 8 + 2 * e;
            o[e] = E::from_f2(fmaxf(fmaf(v[j], s, b[j]), 0.f), fmaxf(fmaf(v[j + 1], s, b[j + 1]), 0.f));
          }
          dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// ---------------------------------------------------------------------------
// 84 x 84 frames (the Mario observation): the 8 x 8 stride-4 convolution over 4
// channels is a 2 x 2 stride-1 convolution over the frame cut into 21 x 21
// blocks of 4 x 4 pixels (64 channels: c * 16 + ry * 4 + rx).  Each frame's
// bytes are copied into shared memory once (one bulk copy, up to three frames
// in flight) and converted once into 16-bit blocks, stored as 128-byte rows
// (row = block row * 24 + block column, 128-byte swizzle).  A tile covers five
// output rows: tile row i = (oy, ox) = divmod(i, 24) of the tile's first output
// row, and the MMA reads atom (dy, dx = 0) of all 128 tile rows straight from
// the block rows starting at row (oy0 + dy) * 24 (rows 128 bytes apart, 8-row
// groups 1 KB apart, 1 KB aligned: 24 and 120 are multiples of 8).  The dx = 1
// atoms read the same rows into a second accumulator, and the epilogue adds
// row i + 1 of it to row i (a lane shuffle; a lane quarter's last row takes the
// next quarter's first from shared memory), which is the block one column to
// the right.  No position is ever gathered; tile rows 120-127 and columns
// ox >= 20 are padding (never stored).  A frame runs as two halves (output rows
// 0-9 and 10-19, block rows 0-10 and 10-20), double-buffered, so the
// conversion of one half overlaps the MMAs of the other.
//   warp 0      bulk copies of the frames' bytes (four frame buffers; frames
//               four ahead are pulled into L2 first);
//   warps 1, 6  TMEM owner (warp 1) and MMA issuers, one per tile of a half: 2
//               atoms dy x 4 K steps of 128 x 64 x 16, whose B stacks the dx = 0
//               and dx = 1 weights (64 rows), so one MMA fills both 32-column
//               accumulators of the pair from one read of the A rows; two pairs
//               per issuer (one per half parity);
//   warps 2-5,  epilogue of the first / second tile of every half: the dx = 1
//   11-14       shift, scale, bias, ReLU, 64 bytes of channels-last output per
//               position;
//   warps 7-10  convert a half's blocks (one (block, channel) per item: four
//               32-bit shared loads, 16 exact 16-bit values, two 16-byte stores).
// Without round_input the pixels enter the MMA as exact fp16 integers (a byte
// permute makes 1024 + b in fp16, one packed subtract of 1024 leaves b: one
// instruction per byte), and so do the weights: bf16 weights are converted to
// fp16 once per CTA, exactly for every |w| >= 2^-14 (smaller ones to the nearest
// fp16 subnormal, within 2^-25).  With round_input the pixels are frames / 255
// rounded to the model's dtype and both operands stay in that dtype.
constexpr int kB1Threads = 480;
constexpr int kB1Conv = 4;          // converter warps
constexpr int kB1Raw = 4;           // frame buffers
constexpr int kB1Batch = 4;         // converter items per thread with loads in flight together
constexpr int kB1FrameBytes = 4 * 84 * 84;
constexpr int kB1ArrRows = 272;     // 11 block rows x 24 and the rows the second tile's dy = 1 atoms read past them

struct B1Shape {
  static constexpr int RAW = (kB1FrameBytes + 1023) & ~1023;
  static constexpr int ARR = kB1ArrRows * 128;        // block rows of a half
  static constexpr int OFF_RAW = 0;                   // [kB1Raw frames]
  static constexpr int OFF_ARR = kB1Raw * RAW;        // [2 halves]
  static constexpr int OFF_B = OFF_ARR + 2 * ARR;     // 2 atoms dy x 64 rows (dx, o) x 128 B
  static constexpr int OFF_BIAS = OFF_B + 4 * 4096;
  static constexpr int OFF_XCH = OFF_BIAS + kC1N * 4;  // [group][tile parity][lane quarter][32] dx = 1 rows
  static constexpr int OFF_BAR = OFF_XCH + 2 * 2 * 4 * kC1N * 4;
  // raw_full[R], raw_empty[R], arr_full[2], arr_empty[2], acc_full[4], acc_empty[4], drain[2]
  static constexpr int NBAR = 2 * kB1Raw + 18;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
};

// One bulk copy (no tensor map) global -> this CTA's shared memory, completing on bar.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <bool BF16, bool ROUND>
__global__ void __launch_bounds__(kB1Threads, 1)
    frames_conv1_blocked_kernel(const uint8_t* __restrict__ frames, const uint16_t* __restrict__ w,
                                const float* __restrict__ bias, const unsigned int* __restrict__ frame_max,
                                uint16_t* __restrict__ y, long long n_frames, int* status) {
  using SH = B1Shape;
  using E = Elem<BF16>;
  constexpr bool AF16 = !ROUND || !BF16;  // MMA operands in fp16
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* raw_s = smem + SH::OFF_RAW;
  uint8_t* arr_s = smem + SH::OFF_ARR;
  uint8_t* b_s = smem + SH::OFF_B;
  float* bias_s = reinterpret_cast<float*>(smem + SH::OFF_BIAS);
  float* xch_s = reinterpret_cast<float*>(smem + SH::OFF_XCH);
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* raw_empty = raw_full + kB1Raw;
  uint64_t* arr_full = raw_empty + kB1Raw;
  uint64_t* arr_empty = arr_full + 2;
  uint64_t* acc_full = arr_empty + 2;  // [tile * 2 + half parity] (an accumulator pair)
  uint64_t* acc_empty = acc_full + 4;
  uint64_t* drain = acc_empty + 4;     // [issuer]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
    for (int j = 0; j < kB1Raw; ++j) {
      mbar_init(&raw_full[j], 1);
      mbar_init(&raw_empty[j], kB1Conv);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&arr_full[j], kB1Conv);
      mbar_init(&arr_empty[j], 2);  // both issuers' MMAs done with the half
      mbar_init(&drain[j], 1);
    }
    for (int j = 0; j < 4; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  // W [32][4 x 8 x 8] -> atom dy, B row dx * 32 + o, K-value q = c * 16 + ry * 4 + rx
  // holds W[o][c][4 dy + ry][4 dx + rx]; swizzled K-major rows of 128 bytes.
  for (int idx = tid; idx < 4 * kC1N * 8; idx += kB1Threads) {  // 16-byte pieces
    const int dy = idx >> 9, orow = (idx >> 3) & 63, j = idx & 7;
    const int dx = orow >> 5, o = orow & 31;
    uint32_t v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint32_t h[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int q = j * 8 + 2 * e + k, c = q >> 4, ry = (q >> 2) & 3, rx = q & 3;
        h[k] = w[o * 256 + c * 64 + (4 * dy + ry) * 8 + (4 * dx + rx)];
        if (AF16 && BF16) {  // bf16 bits -> fp16 bits
          const __half hv = __float2half_rn(__uint_as_float(h[k] << 16));
          h[k] = *reinterpret_cast<const uint16_t*>(&hv);
        }
      }
      v[e] = h[0] | (h[1] << 16);
    }
    *reinterpret_cast<uint4*>(b_s + dy * 8192 + sw128_off(orow, j)) = make_uint4(v[0], v[1], v[2], v[3]);
  }
  if (tid < kC1N) bias_s[tid] = bias[tid];
  if (warp == 1) {
    tmem_alloc(tmem_holder, 256);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- frame copies
    if (lane == 0) {
      int i = 0;
      bool ok = true;
      for (long long n = blockIdx.x; n < n_frames && ok; n += gridDim.x, ++i) {
        const int rb = i % kB1Raw;
        const long long nf = n + (long long)kB1Raw * gridDim.x;
        if (nf < n_frames) bulk_prefetch_l2(frames + nf * kB1FrameBytes, (uint32_t)kB1FrameBytes);
        if (!(ok = mbar_wait(&raw_empty[rb], ((i / kB1Raw) & 1) ^ 1, abort_flag, status))) break;
        mbar_arrive_expect_tx(&raw_full[rb], (uint32_t)kB1FrameBytes);
        bulk_load(raw_s + rb * SH::RAW, frames + n * kB1FrameBytes, (uint32_t)kB1FrameBytes, &raw_full[rb]);
      }
      if (!ok)  // copies already issued land before the CTA exits
        for (int j = 0; j < kB1Raw; ++j) {
          const int uses = i / kB1Raw + (j < i % kB1Raw ? 1 : 0);
          if (uses > 0) mbar_wait(&raw_full[j], (uses - 1) & 1, nullptr, nullptr);
        }
    }
  } else if (warp == 1 || warp == 6) {
    // ---------------------------------------------------------------- MMA issuers (tile t of every half)
    if (lane == 0) {
      const int t = warp == 1 ? 0 : 1;
      const uint32_t idesc = umma_idesc_f16(!AF16, 128, 2 * kC1N, 0, 0);
      int k = 0;  // halves
      bool ok = true;
      for (long long n = blockIdx.x; n < n_frames && ok; n += gridDim.x)
        for (int h = 0; h < 2 && ok; ++h, ++k) {
          const int hb = k & 1;
          const int ab = t * 2 + hb;  // accumulator pair: tile t, half parity
          if (!(ok = mbar_wait(&arr_full[hb], (k >> 1) & 1, abort_flag, status))) break;
          if (!(ok = mbar_wait(&acc_empty[ab], ((k >> 1) & 1) ^ 1, abort_flag, status))) break;
          tc_fence_after();
          const uint32_t arr = smem_u32(arr_s + hb * SH::ARR);
#pragma unroll
          for (int dy = 0; dy < 2; ++dy) {
            const uint64_t ad = umma_smem_desc(arr + (uint32_t)(120 * t + 24 * dy) * 128u, 16, 1024, kSw128);
            const uint64_t bd = umma_smem_desc(smem_u32(b_s + dy * 8192), 16, 1024, kSw128);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16_ss(tmem + (uint32_t)(ab * 64), ad + 2 * kk, bd + 2 * kk, idesc, (dy > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&acc_full[ab]);
          umma_commit(&arr_empty[hb]);
        }
      umma_commit(&drain[t]);
      mbar_wait(&drain[t], 0, nullptr, nullptr);
    }
  } else if (warp < 6 || warp >= 11) {
    // ---------------------------------------------------------------- epilogue (group g: tile g of every half)
    const int g = warp < 6 ? 0 : 1;
    const int wq = warp & 3;
    const int r = wq * 32 + lane;
    const float s = (!ROUND && *frame_max > 1u) ? (1.f / 255.f) : 1.f;
    int k = 0;  // halves (= this group's tiles)
    bool ok = true;
    for (long long n = blockIdx.x; n < n_frames && ok; n += gridDim.x)
      for (int h = 0; h < 2 && ok; ++h, ++k) {
          const int t = g, j = k;
          const int ab = t * 2 + (k & 1);
          const bool okw = __all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (k >> 1) & 1, abort_flag, status));
          float v0[kC1N], v1[kC1N];
          if (okw) {
            tc_fence_after();
            const uint32_t ta = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(ab * 64);
            tmem_ld32(ta, v0);
            tmem_ld32(ta + kC1N, v1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[ab]);
          }
          // Row r + 1 of the dx = 1 accumulator: the next lane, or for lane 31 the next
          // quarter's lane 0 through shared memory (16-byte accesses).
          float* xw = xch_s + ((g * 2 + (j & 1)) * 4 + wq) * kC1N;
          if (lane == 0 && okw) {
#pragma unroll
            for (int c = 0; c < kC1N; c += 4)
              *reinterpret_cast<float4*>(xw + c) = make_float4(v1[c], v1[c + 1], v1[c + 2], v1[c + 3]);
          }
          // All four epilogue warps pass here every tile; the barrier also agrees on
          // their waits' outcomes, so they leave together.
          ok = named_bar_and(1 + g, 128, okw);
          if (!ok) break;
          const float* xn = xch_s + ((g * 2 + (j & 1)) * 4 + ((wq + 1) & 3)) * kC1N;
          const int oyl = r / 24, ox = r - oyl * 24;
          const bool valid = r < 120 && ox < 20;
#pragma unroll
          for (int c = 0; c < kC1N; ++c) v1[c] = __shfl_down_sync(0xffffffffu, v1[c], 1);
          if (lane == 31) {
#pragma unroll
            for (int c = 0; c < kC1N; c += 4) {
              const float4 x4 = *reinterpret_cast<const float4*>(xn + c);
              v1[c] = x4.x, v1[c + 1] = x4.y, v1[c + 2] = x4.z, v1[c + 3] = x4.w;
            }
          }
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(y + ((size_t)(n * 20 + 10 * h + 5 * t + oyl) * 20 + ox) * kC1N);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 b0 = *reinterpret_cast<const float4*>(bias_s + q * 8);
              const float4 b1 = *reinterpret_cast<const float4*>(bias_s + q * 8 + 4);
              const float bq[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
              uint32_t o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int jj = q * 8 + 2 * e;
                o[e] = E::from_f2(fmaxf(fmaf(v0[jj] + v1[jj], s, bq[2 * e]), 0.f),
                                  fmaxf(fmaf(v0[jj + 1] + v1[jj + 1], s, bq[2 * e + 1]), 0.f));
              }
              dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
            }
          }
        }
  } else {
    // ---------------------------------------------------------------- block converters (warps 7-10)
    const int ct = tid - 224;  // 0..127
    const float in_scale = (ROUND && *frame_max > 1u) ? (1.f / 255.f) : 1.f;
    int i = 0, k = 0;
    bool ok = true;
    for (long long n = blockIdx.x; n < n_frames && ok; n += gridDim.x, ++i) {
      const int rb = i % kB1Raw;
      if (!(ok = mbar_wait(&raw_full[rb], (i / kB1Raw) & 1, abort_flag, status))) break;
      const uint8_t* raw = raw_s + rb * SH::RAW;
      for (int h = 0; h < 2 && ok; ++h, ++k) {
        const int hb = k & 1;
        if (!(ok = mbar_wait(&arr_empty[hb], ((k >> 1) & 1) ^ 1, abort_flag, status))) break;
        uint8_t* arr = arr_s + hb * SH::ARR;
        // items: (channel 0..3, local block row 0..10, block column 0..20), the column
        // fastest: a warp's 32-bit loads then cover consecutive words of a frame row
        // (and the next block row's, 20 banks further), nearly free of bank conflicts.
        // A thread takes kB1Batch items at a time with all their loads issued before
        // any conversion, so that one warp per scheduler keeps several shared-memory
        // loads in flight.
        constexpr int kItems = 11 * 21 * 4, kStride = kB1Conv * 32;
        for (int it0 = ct; it0 < kItems; it0 += kB1Batch * kStride) {
          uint32_t px[kB1Batch][4];
          int rows[kB1Batch], chans[kB1Batch];
#pragma unroll
          for (int u = 0; u < kB1Batch; ++u) {
            const int it = it0 + u * kStride;
            const int bx = it % 21, rest = it / 21, byl = rest % 11, c = rest / 11;
            rows[u] = byl * 24 + bx;
            chans[u] = c;
            if (it < kItems) {
              const uint8_t* src = raw + c * 7056 + (4 * (10 * h + byl)) * 84 + 4 * bx;
#pragma unroll
              for (int ry = 0; ry < 4; ++ry) px[u][ry] = *reinterpret_cast<const uint32_t*>(src + ry * 84);
            }
          }
#pragma unroll
          for (int u = 0; u < kB1Batch; ++u) {
            if (it0 + u * kStride >= kItems) break;
            uint32_t o[8];
#pragma unroll
            for (int ry = 0; ry < 4; ++ry) {
              if (ROUND) {
                o[2 * ry] = E::from_f2(byte_f(px[u][ry], 0) * in_scale, byte_f(px[u][ry], 1) * in_scale);
                o[2 * ry + 1] = E::from_f2(byte_f(px[u][ry], 2) * in_scale, byte_f(px[u][ry], 3) * in_scale);
              } else {
                // fp16 pairs (1024 + b0, 1024 + b1) and (1024 + b2, 1024 + b3), minus 1024: exact
                const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
                uint32_t lo = __byte_perm(px[u][ry], 0x64646464u, 0x5140);
                uint32_t hi = __byte_perm(px[u][ry], 0x64646464u, 0x7362);
                const __half2 l2 = __hsub2(*reinterpret_cast<const __half2*>(&lo), k1024);
                const __half2 h2 = __hsub2(*reinterpret_cast<const __half2*>(&hi), k1024);
                o[2 * ry] = *reinterpret_cast<const uint32_t*>(&l2);
                o[2 * ry + 1] = *reinterpret_cast<const uint32_t*>(&h2);
              }
            }
            *reinterpret_cast<uint4*>(arr + sw128_off(rows[u], 2 * chans[u])) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(arr + sw128_off(rows[u], 2 * chans[u] + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&arr_full[hb]);
      }
      __syncwarp();
      if (ok && lane == 0) mbar_arrive(&raw_empty[rb]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

cudaError_t launch_frames_conv1_sm100(const void* frames, long long N, int H, int W, const void* w,
                                      const float* bias, unsigned int* frame_max, void* y, bool bf16,
                                      bool round_input, int num_sms, int* status, cudaStream_t st) {
  const long long bytes = N * 4LL * H * W;
  cudaError_t e = cudaMemsetAsync(frame_max, 0, sizeof(unsigned int), st);
  if (e != cudaSuccess) return e;
  const long long n16 = bytes / 16;
  const long long want = (n16 + 255) / 256;
  const unsigned mgrid = (unsigned)(want < (long long)num_sms * 2 ? want : (long long)num_sms * 2);
  frames_max_kernel<<<mgrid, 256, 0, st>>>(static_cast<const uint4*>(frames), n16, frame_max);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (H == 84 && W == 84) {
    const unsigned grid = (unsigned)(N < num_sms ? N : num_sms);
    auto kb = bf16 ? (round_input ? frames_conv1_blocked_kernel<true, true> : frames_conv1_blocked_kernel<true, false>)
                   : (round_input ? frames_conv1_blocked_kernel<false, true> : frames_conv1_blocked_kernel<false, false>);
    e = smem_limit_once(reinterpret_cast<const void*>(kb), B1Shape::SMEM);
    if (e != cudaSuccess) return e;
    kb<<<grid, kB1Threads, B1Shape::SMEM, st>>>(static_cast<const uint8_t*>(frames), static_cast<const uint16_t*>(w),
                                                bias, frame_max, static_cast<uint16_t*>(y), N, status);
    return cudaGetLastError();
  }
  const int OH = (H - 8) / 4 + 1, OW = (W - 8) / 4 + 1;
  const long long total = N * OH * OW;
  const long long ntiles = (total + 127) / 128;
  const unsigned grid = (unsigned)(ntiles < num_sms ? ntiles : num_sms);
  auto kfn = bf16 ? (round_input ? frames_conv1_kernel<true, true> : frames_conv1_kernel<true, false>)
                  : (round_input ? frames_conv1_kernel<false, true> : frames_conv1_kernel<false, false>);
  e = smem_limit_once(reinterpret_cast<const void*>(kfn), C1Shape::SMEM);
  if (e != cudaSuccess) return e;
  kfn<<<grid, kC1Threads, C1Shape::SMEM, st>>>(static_cast<const uint8_t*>(frames), static_cast<const uint16_t*>(w),
                                                bias, frame_max, static_cast<uint16_t*>(y), total, H, W, OH, OW,
                                                status);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Scratch of the allocation-free entry point (dt_frames_conv1_noalloc): the
// frame-maximum word lives in this file-scope array instead of a buffer the
// caller allocates.  Host code must not pass the array's name to a kernel (on
// the host it names a shadow, not device memory); it passes the device address
// that conv1_noalloc_scratch() looked up for the current device.  Every call
// shares the array and the launch clears the word first; calls whose work
// overlaps on the GPU race on it.
static __device__ __align__(256) unsigned int g_conv1_noalloc_scratch[kConv1NoallocScratchWords];

cudaError_t conv1_noalloc_scratch(unsigned int** out) {
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static unsigned int* ptr[kMaxDev] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (!ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_conv1_noalloc_scratch);
    if (e != cudaSuccess) return e;
    ptr[dev] = static_cast<unsigned int*>(p);
  }
  *out = ptr[dev];
  return cudaSuccess;
}

}  // namespace dtk
