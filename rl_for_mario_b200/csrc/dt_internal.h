// Internal launch interfaces between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace dtk {

// Raises a kernel's dynamic shared-memory limit on the current device once:
// the attribute stays set in the device's context, and the launch paths are
// host-bound (the rollout enqueues dozens of launches per step), so later
// launches skip the driver call.  Thread-safe; one record per (kernel, device).
inline cudaError_t smem_limit_once(const void* func, int bytes) {
  struct Done {
    const void* f;
    int dev, bytes;
  };
  static std::mutex mu;
  static Done done[256];
  static int n = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (done[i].f == func && done[i].dev == dev && done[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && n < 256) done[n++] = Done{func, dev, bytes};
  return e;
}

// Kernel parameters of the fused prefill (everything except the TMA maps).
struct PrefillParams {
  void* o;                  // [B, S, Hq, D] output, element strides below
  const float* cos;         // [>= S, D] fp32, row stride cs_stride (positions 0..S-1)
  const float* sin;
  const int32_t* pad_len;   // [B] left-padding length in tokens, or null (no padding)
  int* status;              // device status word
  long long o_sb, o_ss, o_sh;
  int cs_stride;
  int S, Hkv, R, PT;        // R = Hq / Hkv query heads per KV head, PT = positions per 128-row tile
  float scale_log2;         // softmax scale * log2(e)
  float scale_div64;        // softmax scale / 64 (fully padded rows)
  int rope;                 // 1: rotate Q and K in the kernel
};

cudaError_t launch_prefill_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                 const PrefillParams& prm, int D, bool bf16, int grid, cudaStream_t stream);

// Persistent variant for head_dim 32 and S <= 192 (K/V resident per unit).
// A CTA stages the padding of at most kShortMaxUnitsPerCta units; the grid
// grows past the SM count when there are more.
constexpr int kShortMaxUnitsPerCta = 2048;
cudaError_t launch_prefill_short_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                       const PrefillParams& prm, bool bf16, int n_units, int grid,
                                       cudaStream_t stream);

// Persistent two-tile kernel for head_dim 64 with Q/K already rotated (any S).
cudaError_t launch_prefill_long_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                      const PrefillParams& prm, bool bf16, int n_units, int grid,
                                      cudaStream_t stream);

// Decode CTA shape: threads (warps split the keys) and keys staged per block.
constexpr int kDecodeThreads = 64;
constexpr int kDecodeKeyBlock = 128;

// Kernel parameters of the paged-cache decode (dt_attn_decode).
struct DecodeParams {
  const void* q;             // [B, Sn, Hq, D] new queries (pre-RoPE)
  const void* k_new;         // [B, Sn, Hkv, D] new keys (pre-RoPE)
  const void* v_new;         // [B, Sn, Hkv, D] new values
  void* o;                   // [B, Sn, Hq, D]
  void* k_pages;             // [num_pages, Hkv, page_size, D]
  void* v_pages;
  const int32_t* block_table;  // [B, max_pages]
  const int32_t* seq_lens;     // [B] cached positions before this call
  const int32_t* pad_len;      // [B] or null
  const float* cos;
  const float* sin;
  int* status;
  long long q_sb, q_ss, q_sh, kn_sb, kn_ss, kn_sh, vn_sb, vn_ss, vn_sh, o_sb, o_ss, o_sh;
  int cs_stride, rope, rope_abs;
  int cos_rows;
  int Sn, Hkv, R, page_size, max_pages, num_pages;
  int o_pairs;               // 1: o and its strides allow 4-byte stores of element pairs
  int vec_front;             // 1: 16-byte loads of the new rows in one round trip (see the kernel)
  int tma_pages;             // 1: cache pages copied by TMA (page_size a power of two in 16..256)
  float scale_log2;
  float scale_div64;
};

// Kernel parameters of dt_kv_write.
struct KvWriteParams {
  const void* k;               // [B, S, Hkv, D] keys (pre-RoPE)
  const void* v;               // [B, S, Hkv, D]
  void* k_pages;
  void* v_pages;
  const int32_t* block_table;  // [B, max_pages]
  const int32_t* start_pos;    // [B] or null (0)
  const float* cos;
  const float* sin;
  int* status;
  long long k_sb, k_ss, k_sh, v_sb, v_ss, v_sh;
  int cs_stride, cos_rows, rope, rope_abs;
  int S, Hkv, page_size, max_pages, num_pages;
};

// float32 prefill (CUDA cores).
struct PrefillF32Params {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  const float* cos;
  const float* sin;
  const int32_t* pad_len;
  long long q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh, o_sb, o_ss, o_sh;
  int cs_stride, rope;
  int S, Hkv, R;
  float scale_log2;
  float scale_div64;
};

cudaError_t launch_prefill_f32(const PrefillF32Params& prm, int D, int B, cudaStream_t stream);
cudaError_t launch_decode_f32(const DecodeParams& prm, int D, int B, cudaStream_t stream);

// Fused RMSNorm + QKV projection.
struct RmsQkvParams {
  void* y;            // [M, N] output rows, row stride y_stride elements
  int* status;
  const float* cos;   // RoPE tables (rope_cols > 0): row (m mod seq_len), stride cs_stride
  const float* sin;
  long long y_stride;
  int M, K, N, bf16;
  int rope_cols, head_dim, seq_len, cs_stride;  // rope_cols = 0: no rotation
  int swiglu;  // 1: W rows are 64-row gate / up blocks, y[:, j] = silu(gate_j) * up_j (N / 2 columns)
  int resid;   // 1: y += x @ W^T in place (no RMSNorm scale; y is read as the residual)
  int nonorm;  // 1: no RMSNorm scale (y = x @ W^T, with the RoPE epilogue when rope_cols > 0)
  float eps;
};

int rmsnorm_qkv_ncta(int N);
constexpr int kPersistKChunk = 64;  // K elements per stage of the persistent RMSNorm GEMM (x / W box width)

// Static scratch of dt_frames_conv1_noalloc: 64 32-bit words (256 bytes) of
// device memory that every GPU loading the library holds until exit.  A call
// uses kConv1NoallocWordsPerCall of them (the frame-maximum word), whatever
// its frame count.
constexpr int kConv1NoallocScratchWords = 64;
constexpr int kConv1NoallocWordsPerCall = 1;

// Device address of that array on the current device, looked up once per
// device (cudaGetSymbolAddress with the device current) and cached.
cudaError_t conv1_noalloc_scratch(unsigned int** out);


cudaError_t launch_frames_to_blocks_sm100(const void* frames, void* out, long long N, int C, int H, int W, bool bf16,
                                          unsigned int* frame_max, cudaStream_t st);
// round_input: frames / 255 rounded to the output dtype before the
// convolution (the reference's 16-bit rounding) instead of exact pixels.
// Residual GEMM y += x W^T on CTA pairs (N a multiple of 256; x, w maps with
// 64 x 128 boxes, y map with 64 x 32 boxes, all 128-byte swizzle).
cudaError_t launch_gemm_residual_pair_sm100(const CUtensorMap& x, const CUtensorMap& w, const CUtensorMap& y, int M,
                                            int N, int K, bool bf16, int num_sms, int* status, cudaStream_t st);

// The state encoder's second and third convolutions + ReLU, fused; x1 is the
// map of the [N, 20, 20, 32] input as (channel, x, y, frame) with traversal
// strides (1, 2, 2, 1) and 8 x 20 x 20 x 1 boxes (one K group of the
// space-to-depth operand per box; encoded in capi.cu).
cudaError_t launch_encoder_conv23_sm100(const CUtensorMap& x1, const void* w2, const float* b2, void* y2, const void* w3,
                                        const float* b3, void* y3, long long n_frames, bool bf16, int num_sms,
                                        int* status, cudaStream_t st);

cudaError_t launch_frames_conv1_sm100(const void* frames, long long N, int H, int W, const void* w,
                                      const float* bias, unsigned int* frame_max, void* y, bool bf16,
                                      bool round_input, int num_sms, int* status, cudaStream_t st);
cudaError_t launch_rmsnorm_sm100(const void* x, long long x_stride, const void* w, void* y, long long y_stride, int M,
                                 int K, float eps, bool bf16, int num_sms, cudaStream_t st);
cudaError_t launch_rmsnorm_qkv_sm100(const CUtensorMap& x, const CUtensorMap& w, const CUtensorMap& y,
                                     const RmsQkvParams& p, int ncta, int num_sms, cudaStream_t st);

// dtype: 0 bf16, 1 fp16, 2 fp32
cudaError_t launch_kv_write_sm100(const KvWriteParams& prm, int D, int dtype, int B, cudaStream_t stream);

cudaError_t launch_decode_sm100(const DecodeParams& prm, const CUtensorMap& kmap, const CUtensorMap& vmap, int D,
                                bool bf16, int grid, cudaStream_t stream);


// Batched NES emulation (nes_sm100.cu).  op: 0 run frames, 1 reset, 2 buttons,
// 3 observation, 4 environment bookkeeping.  Unused fields may be left zero.
struct NesLaunch {
  uint8_t* regs;
  uint8_t* ram;
  uint8_t* vram;
  uint8_t* oam;
  uint8_t* pal;
  uint8_t* fb;
  const uint8_t* prg;
  uint32_t prg_size;
  const uint8_t* chr;
  int n;
  int num_frames;
  const uint8_t* mask;
  int mirroring;
  const uint8_t* buttons;
  const int64_t* actions;
  int32_t* boot;
  int boot_settle, boot_total, frame_skip;
  int* status;
  uint8_t* obs;
  uint8_t* stacked;
  int stack;
  int32_t* prev_x;
  int32_t* init_lives;
  float* reward;
  uint8_t* done;
  int32_t* x_pos;
  int32_t* lives;
  uint8_t* flag;
};
cudaError_t launch_nes(int op, const NesLaunch& L, cudaStream_t st);

}  // namespace dtk
