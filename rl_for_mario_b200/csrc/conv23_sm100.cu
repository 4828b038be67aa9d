// The state encoder's second and third convolutions with their ReLUs
// (model/model_decision_transformer.py:322-325: Conv2d(32, 64, 4, stride 2)
// on 20 x 20 and Conv2d(64, 64, 3, stride 1) on 9 x 9) as tcgen05 implicit
// GEMMs whose A tiles are single TMA copies, sm_100a.
//
// Rows of the GEMM are output positions, N = 64 output channels, K = the
// receptive field.  The K dimension is cut into atoms of 64 16-bit values (one
// 128-byte swizzled row each) chosen so that, for one atom, the input bytes of
// consecutive output positions sit at a regular stride in the channels-last
// input; one tensor-map copy then lands the atom's rows for a whole frame in
// the K-major 128-byte-swizzled layout the MMA reads, with no im2col pass:
//
//  * conv2 (input [N, 20, 20, 32]): view the input as 2 x 2 pixel blocks; the
//    4 x 4 stride-2 kernel is a 2 x 2 stride-1 kernel over blocks.  Atom
//    (dy, dx, sy) holds the two pixels (sx = 0, 1) of block row sy of block
//    (oy + dy, ox + dx): 64 values = 128 contiguous bytes.  A 5-D box
//    [64 values, 9 block columns (128 B apart), 1 block row parity, 9 block rows
//    (2 input rows apart), 1 frame] gives the 81 positions of a frame in (oy,
//    ox) order.  8 atoms, K = 512; one frame per 128-row tile (81 rows valid);
//  * conv3 (input [N, 9, 9, 64], conv2's output): atom (ky, kx) is the 64
//    channels of input pixel (oy + ky, ox + kx); a 4-D box [64 channels, 7
//    columns, 7 rows, 2 frames] gives 98 rows (two frames' 49 positions).  9
//    atoms, K = 576.
//
// Warps: 0 TMA producer (ring of stages; each unit's input bytes are also
// pulled into L2 two units ahead with one bulk prefetch), 1 TMEM owner + MMA issuer
// (M = 128, N = 64, K = 16 steps; two 64-column accumulators in TMEM), 2-5
// epilogue (bias + ReLU in fp32, one rounding, 128 bytes of channels-last
// output per position).  The weights of all atoms stay in shared memory,
// staged once per CTA from the reference's [64, Cin, k, k] layout.  Stages are
// packed at the box size (81 or 98 rows, rounded up to 1 KB) so that more copies
// are in flight; the MMA still reads 128 rows from a stage, so its rows past the
// box read the next stage (or the weights behind the ring): those accumulator
// rows belong to no position and are never stored.
#include "dt_common.cuh"
#include "dt_internal.h"

namespace dtk {

namespace {

constexpr int kCvThreads = 192;
constexpr int kCvBAtom = 64 * 128;   // one atom of the 64-row weight tile

template <int LAYER>
struct Cv;
template <>
struct Cv<2> {
  static constexpr int NATOM = 8, FRAMES = 1, P = 81, CIN = 32, KS = 4;
  static constexpr int ROWS = FRAMES * P;
  static constexpr int IN_BYTES = 20 * 20 * 32 * 2;  // one frame of input
  static constexpr int STAGES = 14;
  // Weight value of atom a, output channel o, K-value e (o, c, ky, kx of the reference layout).
  __device__ static int w_index(int a, int o, int e) {
    const int dy = a >> 2, dx = (a >> 1) & 1, sy = a & 1, sx = e >> 5, c = e & 31;
    return ((o * CIN + c) * KS + (2 * dy + sy)) * KS + (2 * dx + sx);
  }
};
template <>
struct Cv<3> {
  static constexpr int NATOM = 9, FRAMES = 2, P = 49, CIN = 64, KS = 3;
  static constexpr int ROWS = FRAMES * P;
  static constexpr int IN_BYTES = 9 * 9 * 64 * 2;
  static constexpr int STAGES = 11;
  __device__ static int w_index(int a, int o, int e) {
    const int ky = a / 3, kx = a % 3;
    return ((o * CIN + e) * KS + ky) * KS + kx;
  }
};

template <int LAYER>
struct CvShape {
  static constexpr int STAGES = Cv<LAYER>::STAGES;
  static constexpr int STAGE = (Cv<LAYER>::ROWS * 128 + 1023) & ~1023;  // box bytes, 1 KB aligned
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = STAGES * STAGE;  // the last stage's 128-row read ends inside B
  static_assert(OFF_B + kCvBAtom * Cv<LAYER>::NATOM >= (STAGES - 1) * STAGE + 128 * 128, "MMA overhang");
  static constexpr int OFF_BIAS = OFF_B + Cv<LAYER>::NATOM * kCvBAtom;
  static constexpr int OFF_BAR = OFF_BIAS + 64 * 4;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr int NBAR = 2 * STAGES + 5;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
};

// Byte offset of 16-byte piece j of row r inside a 128-byte-swizzled K-major atom.
__device__ __forceinline__ uint32_t cv_sw128(int r, int j) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

// Atom a of unit u as box coordinates of the layer's tensor map.
template <int LAYER>
__device__ __forceinline__ void cv_load(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int a, int u) {
  if constexpr (LAYER == 2) {
    // dims (innermost first): 64 values, block column, block-row parity, block row, frame
    const int dy = a >> 2, dx = (a >> 1) & 1, sy = a & 1;
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cta.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(0), "r"(dx), "r"(sy), "r"(dy), "r"(u)
        : "memory");
  } else {
    // dims: 64 channels, column, row, frame; a unit is two frames
    tma_load_4d(dst, map, bar, 0, a % 3, a / 3, 2 * u);
  }
}

template <int LAYER, bool BF16>
__global__ void __launch_bounds__(kCvThreads, 1)
    encoder_conv_kernel(const __grid_constant__ CUtensorMap tmX, const uint8_t* __restrict__ x,
                        const uint16_t* __restrict__ w, const float* __restrict__ bias, uint16_t* __restrict__ y,
                        long long n_frames, int* status) {
  using L = Cv<LAYER>;
  using SH = CvShape<LAYER>;
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = smem + SH::OFF_A;
  uint8_t* b_s = smem + SH::OFF_B;
  float* bias_s = reinterpret_cast<float*>(smem + SH::OFF_BIAS);
  constexpr int NST = SH::STAGES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SH::OFF_BAR);
  uint64_t* empty = full + NST;
  uint64_t* acc_full = empty + NST;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long units = (n_frames + L::FRAMES - 1) / L::FRAMES;

  if (tid == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Weights into the swizzled K-major B layout, one atom per 8 KB; bias into shared memory.
  for (int idx = tid; idx < L::NATOM * 64 * 8; idx += kCvThreads) {  // 16-byte pieces
    const int a = idx >> 9, o = (idx >> 3) & 63, j = idx & 7;
    uint32_t v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = w[L::w_index(a, o, j * 8 + 2 * q)];
      const uint32_t hi = w[L::w_index(a, o, j * 8 + 2 * q + 1)];
      v[q] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(b_s + a * kCvBAtom + cv_sw128(o, j)) = make_uint4(v[0], v[1], v[2], v[3]);
  }
  if (tid < 64) bias_s[tid] = bias[tid];
  if (warp == 1) {
    tmem_alloc(tmem_holder, 128);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tmX);
      int cnt = 0;
      bool ok = true;
      // The input bytes of unit v (FRAMES whole frames, contiguous) into L2.
      auto prefetch_unit = [&](long long v) {
        if (v >= units) return;
        const long long f0 = v * L::FRAMES;
        const long long nf = n_frames - f0 < L::FRAMES ? n_frames - f0 : L::FRAMES;
        bulk_prefetch_l2(x + f0 * L::IN_BYTES, (uint32_t)(nf * L::IN_BYTES));
      };
      prefetch_unit(blockIdx.x);
      prefetch_unit(blockIdx.x + (long long)gridDim.x);
      for (long long u = blockIdx.x; u < units && ok; u += gridDim.x) {
        prefetch_unit(u + 2LL * gridDim.x);
        for (int a = 0; a < L::NATOM; ++a, ++cnt) {
          const int s = cnt % NST;
          if (!(ok = mbar_wait(&empty[s], ((cnt / NST) & 1) ^ 1, abort_flag, status))) break;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(L::ROWS * 128));
          cv_load<LAYER>(a_s + s * SH::STAGE, &tmX, &full[s], a, (int)u);
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA can exit.
        for (int s = 0; s < NST; ++s) {
          const int uses = cnt / NST + (s < cnt % NST ? 1 : 0);
          if (uses > 0) mbar_wait(&full[s], (uses - 1) & 1, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(BF16, 128, 64, 0, 0);
      int cnt = 0, i = 0;
      bool ok = true;
      for (long long u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!(ok = mbar_wait(&acc_empty[buf], ((i >> 1) & 1) ^ 1, abort_flag, status))) break;
        for (int a = 0; a < L::NATOM; ++a, ++cnt) {
          const int s = cnt % NST;
          if (!(ok = mbar_wait(&full[s], (cnt / NST) & 1, abort_flag, status))) break;
          tc_fence_after();
          const uint64_t ad = umma_smem_desc(smem_u32(a_s + s * SH::STAGE), 16, 1024, kSw128);
          const uint64_t bd = umma_smem_desc(smem_u32(b_s + a * kCvBAtom), 16, 1024, kSw128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 32 bytes per K step inside the 128-byte atom
            umma_f16_ss(tmem + (uint32_t)(buf * 64), ad + 2 * kk, bd + 2 * kk, idesc,
                        (a > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int wq = warp & 3;
    const int r = wq * 32 + lane;  // tile row = TMEM lane
    const uint32_t t_row = tmem + ((uint32_t)(wq * 32) << 16);
    const int f_in = r / L::P, pos = r - f_in * L::P;
    int i = 0;
    bool ok = true;
    for (long long u = blockIdx.x; u < units && ok; u += gridDim.x, ++i) {
      const int buf = i & 1;
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (i >> 1) & 1, abort_flag, status)))) break;
      tc_fence_after();
      float v[64];
      tmem_ld32(t_row + (uint32_t)(buf * 64), *reinterpret_cast<float(*)[32]>(v));
      tmem_ld32(t_row + (uint32_t)(buf * 64 + 32), *reinterpret_cast<float(*)[32]>(v + 32));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      const long long n = u * L::FRAMES + f_in;
      if (r < L::ROWS && n < n_frames) {
        uint4* dst = reinterpret_cast<uint4*>(y + (size_t)(n * L::P + pos) * 64);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = q * 8 + 2 * e;
            o[e] = E::from_f2(fmaxf(v[j] + bias_s[j], 0.f), fmaxf(v[j + 1] + bias_s[j + 1], 0.f));
          }
          dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace

cudaError_t launch_encoder_conv_sm100(int layer, const CUtensorMap& x, const void* xp, const void* w,
                                      const float* bias, void* y, long long n_frames, bool bf16, int num_sms,
                                      int* status, cudaStream_t st) {
  const long long units = layer == 2 ? n_frames : (n_frames + 1) / 2;
  const unsigned grid = (unsigned)(units < num_sms ? units : num_sms);
  const void* fn;
  int smem;
  if (layer == 2) {
    fn = bf16 ? reinterpret_cast<const void*>(encoder_conv_kernel<2, true>)
              : reinterpret_cast<const void*>(encoder_conv_kernel<2, false>);
    smem = CvShape<2>::SMEM;
  } else {
    fn = bf16 ? reinterpret_cast<const void*>(encoder_conv_kernel<3, true>)
              : reinterpret_cast<const void*>(encoder_conv_kernel<3, false>);
    smem = CvShape<3>::SMEM;
  }
  cudaError_t e = smem_limit_once(fn, smem);
  if (e != cudaSuccess) return e;
  const uint8_t* xb = static_cast<const uint8_t*>(xp);
  const uint16_t* wp = static_cast<const uint16_t*>(w);
  uint16_t* yp = static_cast<uint16_t*>(y);
  if (layer == 2) {
    if (bf16)
      encoder_conv_kernel<2, true><<<grid, kCvThreads, smem, st>>>(x, xb, wp, bias, yp, n_frames, status);
    else
      encoder_conv_kernel<2, false><<<grid, kCvThreads, smem, st>>>(x, xb, wp, bias, yp, n_frames, status);
  } else {
    if (bf16)
      encoder_conv_kernel<3, true><<<grid, kCvThreads, smem, st>>>(x, xb, wp, bias, yp, n_frames, status);
    else
      encoder_conv_kernel<3, false><<<grid, kCvThreads, smem, st>>>(x, xb, wp, bias, yp, n_frames, status);
  }
  return cudaGetLastError();
}

}  // namespace dtk
