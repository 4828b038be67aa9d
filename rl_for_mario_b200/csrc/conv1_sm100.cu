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
