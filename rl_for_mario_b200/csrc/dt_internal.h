// Internal launch interfaces between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace dtk {

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
  int rope;                 // 1: rotate Q and K in the kernel
};

cudaError_t launch_prefill_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                 const PrefillParams& prm, int D, bool bf16, int grid, cudaStream_t stream);

// Persistent variant for head_dim 32 and S <= 192 (K/V resident per unit).
cudaError_t launch_prefill_short_sm100(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                                       const PrefillParams& prm, bool bf16, int n_units, int grid,
                                       cudaStream_t stream);

}  // namespace dtk
