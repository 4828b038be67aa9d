// C-ABI entry points (include/dt_attn.h): argument validation, TMA tensor-map
// encoding and kernel dispatch.  No entry point allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/dt_attn.h"
#include "dt_internal.h"

namespace {

// NVTX range around an entry point (host-side validation, descriptor encoding
// and the launch), so a timeline profiler shows each attention call by name.
// NVTX v3 is header-only: without a profiler attached a range costs a few
// nanoseconds.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Device status word, one per device context (static device memory).
__device__ int g_dev_status;

constexpr int kMaxDevices = 64;
int* g_status_ptr[kMaxDevices] = {};
int g_cc_major[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};
std::mutex g_dev_mu;

// Resolves, once per device, the status word's device address and the
// compute capability.
int device_setup(int* dev_out, int** status_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(DT_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (!g_status_ptr[dev]) {
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dev_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    g_cc_major[dev] = major;
    g_num_sms[dev] = sms;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  *dev_out = dev;
  *status_out = g_status_ptr[dev];
  return DT_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 4-D map over a [B, S, H, D] tensor (dims innermost first: D, H, S, B).
int encode_bshd(CUtensorMap* map, const void* base, bool is16, int B, int S, int H, int D, int64_t sb,
                int64_t ss, int64_t sh, uint32_t box_h, uint32_t box_s, const char* name) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const int esz = 2;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(sh * esz), (cuuint64_t)(ss * esz), (cuuint64_t)(sb * esz)};
  cuuint32_t box[4] = {(cuuint32_t)D, box_h, box_s, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle swz = (D * esz == 64) ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = enc(map, is16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DT_ERR_INVALID, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name, (int)r);
  return DT_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D map over the rows of a paged cache ([num_pages * Hkv * page_size, D]),
// box = one page of one KV head, swizzled like the decode kernel's rows.
int encode_pages(CUtensorMap* map, const void* base, bool is16, int D, uint64_t rows, uint32_t page_size,
                 const char* name) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)D, rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {(cuuint32_t)D, page_size};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle swz = D == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = enc(map, is16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DT_ERR_INVALID, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name, (int)r);
  return DT_OK;
}

}  // namespace

extern "C" {

int dt_version(void) { return (0 << 16) | 1; }

const char* dt_last_error(void) { return g_err; }

int dt_device_status(void* stream) {
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return -rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return -cuda_fail(e, "cudaStreamSynchronize");
  int value = 0;
  e = cudaMemcpyFromSymbol(&value, g_dev_status, sizeof(int));
  if (e != cudaSuccess) return -cuda_fail(e, "cudaMemcpyFromSymbol");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_dev_status, &zero, sizeof(int));
  if (e != cudaSuccess) return -cuda_fail(e, "cudaMemcpyToSymbol");
  return value;
}

int dt_attn_prefill(const void* q, const void* k, const void* v, void* o, const float* cos_tab,
                    const float* sin_tab, int cos_rows, int64_t cos_stride, const int32_t* pad_len, int B,
                    int S, int Hq, int Hkv, int D, int64_t q_sb, int64_t q_ss, int64_t q_sh, int64_t k_sb,
                    int64_t k_ss, int64_t k_sh, int64_t v_sb, int64_t v_ss, int64_t v_sh, int64_t o_sb,
                    int64_t o_ss, int64_t o_sh, float scale, int apply_rope, int dtype, void* stream) {
  NvtxRange nvtx_range("dt_attn_prefill");
  if (!q || !k || !v || !o) return fail(DT_ERR_INVALID, "dt_attn_prefill: null q/k/v/o pointer");
  if (B < 1 || S < 1 || Hq < 1 || Hkv < 1)
    return fail(DT_ERR_INVALID, "dt_attn_prefill: sizes must be positive (B=%d S=%d Hq=%d Hkv=%d)", B, S, Hq, Hkv);
  if (Hq % Hkv != 0)
    return fail(DT_ERR_INVALID, "dt_attn_prefill: num_attention_heads (%d) must be divisible by "
                                "num_key_value_heads (%d)", Hq, Hkv);
  if (D != 32 && D != 64) return fail(DT_ERR_UNSUPPORTED, "dt_attn_prefill: head_dim %d not in {32, 64}", D);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16 && dtype != DT_DTYPE_FP32)
    return fail(DT_ERR_UNSUPPORTED, "dt_attn_prefill: dtype %d not supported", dtype);
  const int R = Hq / Hkv;
  if (R > 128) return fail(DT_ERR_UNSUPPORTED, "dt_attn_prefill: group size %d > 128", R);
  if ((long long)B * Hkv > 0x7fffffffLL) return fail(DT_ERR_UNSUPPORTED, "dt_attn_prefill: B*Hkv too large");
  const bool f32 = dtype == DT_DTYPE_FP32;
  if (!f32 && (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)))
    return fail(DT_ERR_INVALID, "dt_attn_prefill: q/k/v/o must be 16-byte aligned");
  const int64_t strides[12] = {q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh, o_sb, o_ss, o_sh};
  for (int i = 0; i < 12; ++i)
    if (strides[i] <= 0 || (!f32 && strides[i] % 8 != 0))
      return fail(DT_ERR_INVALID, "dt_attn_prefill: stride #%d (%lld) must be a positive multiple of 8", i,
                  (long long)strides[i]);
  if (apply_rope < 0 || apply_rope > 2)
    return fail(DT_ERR_INVALID, "dt_attn_prefill: apply_rope must be 0, 1 or 2 (got %d)", apply_rope);
  if (apply_rope) {
    if (!cos_tab || !sin_tab) return fail(DT_ERR_INVALID, "dt_attn_prefill: null cos/sin with apply_rope");
    if (cos_rows < S) return fail(DT_ERR_INVALID, "dt_attn_prefill: cos/sin have %d rows < S=%d", cos_rows, S);
    if (!f32 && (!aligned16(cos_tab) || !aligned16(sin_tab) || cos_stride % 4 != 0))
      return fail(DT_ERR_INVALID, "dt_attn_prefill: cos/sin must be 16-byte aligned with row stride %% 4 == 0");
    if (cos_stride < D)
      return fail(DT_ERR_INVALID, "dt_attn_prefill: cos/sin must be 16-byte aligned with row stride >= D, %% 4");
  }
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  if (g_cc_major[dev] != 10)
    return fail(DT_ERR_UNSUPPORTED, "dt_attn_prefill: needs an sm_100 GPU (device %d is cc %d.x)", dev,
                g_cc_major[dev]);

  const float sc0 = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  if (f32) {
    dtk::PrefillF32Params fp;
    fp.q = static_cast<const float*>(q); fp.k = static_cast<const float*>(k); fp.v = static_cast<const float*>(v);
    fp.o = static_cast<float*>(o); fp.cos = cos_tab; fp.sin = sin_tab; fp.pad_len = pad_len;
    fp.q_sb = q_sb; fp.q_ss = q_ss; fp.q_sh = q_sh; fp.k_sb = k_sb; fp.k_ss = k_ss; fp.k_sh = k_sh;
    fp.v_sb = v_sb; fp.v_ss = v_ss; fp.v_sh = v_sh; fp.o_sb = o_sb; fp.o_ss = o_ss; fp.o_sh = o_sh;
    fp.cs_stride = (int)cos_stride; fp.rope = apply_rope; fp.S = S; fp.Hkv = Hkv; fp.R = R;
    fp.scale_log2 = sc0 * 1.4426950408889634f;
    fp.scale_div64 = sc0 / 64.f;
    cudaError_t e = dtk::launch_prefill_f32(fp, D, B, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "dt_attn_prefill (fp32) launch");
    return DT_OK;
  }
  const bool bf16 = dtype == DT_DTYPE_BF16;
  const int PT = 128 / R;
  // Short sequences with head_dim 32 (the DT's 192-token context) use the
  // persistent kernel that keeps a unit's whole K/V in shared memory.
  const bool short_path = (D == 32 && S <= 192);
  // Longer sequences with head_dim 64: the persistent kernel over pairs of
  // query tiles with 64-key blocks.
  const bool long_path = !short_path && D == 64;
  const uint32_t kv_box = short_path ? (uint32_t)((S + 15) & ~15) : (long_path ? 64u : 128u);
  CUtensorMap mq, mk, mv;
  if ((rc = encode_bshd(&mq, q, bf16, B, S, Hq, D, q_sb, q_ss, q_sh, (uint32_t)R, (uint32_t)PT, "q"))) return rc;
  if ((rc = encode_bshd(&mk, k, bf16, B, S, Hkv, D, k_sb, k_ss, k_sh, 1, kv_box, "k"))) return rc;
  if ((rc = encode_bshd(&mv, v, bf16, B, S, Hkv, D, v_sb, v_ss, v_sh, 1, kv_box, "v"))) return rc;

  dtk::PrefillParams prm;
  prm.o = o;
  prm.cos = cos_tab;
  prm.sin = sin_tab;
  prm.pad_len = pad_len;
  prm.status = status;
  prm.o_sb = o_sb;
  prm.o_ss = o_ss;
  prm.o_sh = o_sh;
  prm.cs_stride = (int)cos_stride;
  prm.S = S;
  prm.Hkv = Hkv;
  prm.R = R;
  prm.PT = PT;
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  prm.scale_log2 = sc * 1.4426950408889634f;
  prm.scale_div64 = sc / 64.f;
  prm.rope = apply_rope;
  const int units = B * Hkv;
  cudaError_t e;
  if (short_path) {
    int grid = units < g_num_sms[dev] ? units : g_num_sms[dev];
    // The persistent kernel stages at most kShortMaxUnitsPerCta units' padding per CTA.
    const int cap = dtk::kShortMaxUnitsPerCta;
    if ((units + grid - 1) / grid > cap) grid = (units + cap - 1) / cap;
    e = dtk::launch_prefill_short_sm100(mq, mk, mv, prm, bf16, units, grid, static_cast<cudaStream_t>(stream));
  } else if (long_path) {
    const long long ntiles = (S + PT - 1) / PT;
    const long long items = (long long)units * ((ntiles + 1) / 2);
    if (items > 0x7fffffffLL) return fail(DT_ERR_UNSUPPORTED, "dt_attn_prefill: too many query tiles");
    const int grid = items < g_num_sms[dev] ? (int)items : g_num_sms[dev];
    e = dtk::launch_prefill_long_sm100(mq, mk, mv, prm, bf16, units, grid, static_cast<cudaStream_t>(stream));
  } else {
    e = dtk::launch_prefill_sm100(mq, mk, mv, prm, D, bf16, units, static_cast<cudaStream_t>(stream));
  }
  if (e != cudaSuccess) return cuda_fail(e, "dt_attn_prefill launch");
  return DT_OK;
}

}  // extern "C"

namespace {
// Shared checks of the paged-cache arguments.
int check_cache(const char* fn, const void* k_pages, const void* v_pages, int num_pages, int page_size,
                const int32_t* block_table, int max_pages, int D, int dtype) {
  if (!k_pages || !v_pages || !block_table) return fail(DT_ERR_INVALID, "%s: null cache pointer", fn);
  if (num_pages < 1 || page_size < 1 || max_pages < 1)
    return fail(DT_ERR_INVALID, "%s: num_pages, page_size, max_pages must be positive", fn);
  if (D != 32 && D != 64) return fail(DT_ERR_UNSUPPORTED, "%s: head_dim %d not in {32, 64}", fn, D);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16 && dtype != DT_DTYPE_FP32)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported", fn, dtype);
  if (!aligned16(k_pages) || !aligned16(v_pages)) return fail(DT_ERR_INVALID, "%s: cache pages must be 16-byte aligned", fn);
  return DT_OK;
}
}  // namespace

extern "C" {

int dt_attn_decode(const void* q, const void* k_new, const void* v_new, void* o, void* k_pages, void* v_pages,
                   int num_pages, int page_size, const int32_t* block_table, int max_pages,
                   const int32_t* seq_lens, const int32_t* pad_len, const float* cos_tab, const float* sin_tab,
                   int cos_rows, int64_t cos_stride, int rope_abs, int B, int Sn, int Hq, int Hkv, int D,
                   int64_t q_sb, int64_t q_ss, int64_t q_sh, int64_t kn_sb, int64_t kn_ss, int64_t kn_sh,
                   int64_t vn_sb, int64_t vn_ss, int64_t vn_sh, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                   float scale, int apply_rope, int dtype, void* stream) {
  const char* fn = "dt_attn_decode";
  NvtxRange nvtx_range("dt_attn_decode");
  if (!q || !k_new || !v_new || !o || !seq_lens) return fail(DT_ERR_INVALID, "%s: null q/k_new/v_new/o/seq_lens", fn);
  if (B < 1 || Sn < 1 || Hq < 1 || Hkv < 1) return fail(DT_ERR_INVALID, "%s: sizes must be positive", fn);
  if (Hq % Hkv != 0)
    return fail(DT_ERR_INVALID, "%s: num_attention_heads (%d) must be divisible by num_key_value_heads (%d)", fn,
                Hq, Hkv);
  int rc = check_cache(fn, k_pages, v_pages, num_pages, page_size, block_table, max_pages, D, dtype);
  if (rc) return rc;
  if ((long long)max_pages * page_size > 0x7fffffffLL) return fail(DT_ERR_INVALID, "%s: cache capacity too large", fn);
  if (apply_rope < 0 || apply_rope > 2) return fail(DT_ERR_INVALID, "%s: apply_rope must be 0, 1 or 2", fn);
  if (apply_rope) {
    if (!cos_tab || !sin_tab) return fail(DT_ERR_INVALID, "%s: null cos/sin with apply_rope", fn);
    if (!rope_abs && cos_rows < Sn) return fail(DT_ERR_INVALID, "%s: cos/sin have %d rows < Sn=%d", fn, cos_rows, Sn);
    if (cos_stride < D) return fail(DT_ERR_INVALID, "%s: cos/sin row stride < D", fn);
  }
  int dev = 0;
  int* status = nullptr;
  if ((rc = device_setup(&dev, &status))) return rc;
  if (g_cc_major[dev] != 10) return fail(DT_ERR_UNSUPPORTED, "%s: needs an sm_100 GPU", fn);
  dtk::DecodeParams p;
  p.q = q; p.k_new = k_new; p.v_new = v_new; p.o = o; p.k_pages = k_pages; p.v_pages = v_pages;
  p.block_table = block_table; p.seq_lens = seq_lens; p.pad_len = pad_len; p.cos = cos_tab; p.sin = sin_tab;
  p.status = status;
  p.q_sb = q_sb; p.q_ss = q_ss; p.q_sh = q_sh; p.kn_sb = kn_sb; p.kn_ss = kn_ss; p.kn_sh = kn_sh;
  p.vn_sb = vn_sb; p.vn_ss = vn_ss; p.vn_sh = vn_sh; p.o_sb = o_sb; p.o_ss = o_ss; p.o_sh = o_sh;
  p.cs_stride = (int)cos_stride; p.rope = apply_rope; p.rope_abs = rope_abs ? 1 : 0; p.cos_rows = cos_rows;
  p.Sn = Sn; p.Hkv = Hkv; p.R = Hq / Hkv; p.page_size = page_size; p.max_pages = max_pages; p.num_pages = num_pages;
  p.o_pairs = ((reinterpret_cast<uintptr_t>(o) & 3u) == 0 && o_sb % 2 == 0 && o_ss % 2 == 0 && o_sh % 2 == 0) ? 1 : 0;
  {
    const int hc = D / 16;
    const bool rows_ok = aligned16(q) && aligned16(k_new) && aligned16(v_new) && q_sb % 8 == 0 && q_ss % 8 == 0 &&
                         q_sh % 8 == 0 && kn_sb % 8 == 0 && kn_ss % 8 == 0 && kn_sh % 8 == 0 && vn_sb % 8 == 0 &&
                         vn_ss % 8 == 0 && vn_sh % 8 == 0;
    const bool tabs_ok = !apply_rope || (!rope_abs && aligned16(cos_tab) && aligned16(sin_tab) && cos_stride % 4 == 0);
    p.vec_front = (dtype != DT_DTYPE_FP32 && Sn * (Hq / Hkv) <= 16 && Sn <= 16 && 16 * hc + 2 * Sn * hc <= dtk::kDecodeThreads &&
                   max_pages <= dtk::kDecodeThreads && rows_ok && tabs_ok) ? 1 : 0;
  }
  const float sc = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = sc * 1.4426950408889634f;
  p.scale_div64 = sc / 64.f;
  if ((long long)B * Hkv > 0x7fffffffLL) return fail(DT_ERR_UNSUPPORTED, "%s: B*Hkv too large", fn);
  CUtensorMap kmap, vmap;
  memset(&kmap, 0, sizeof(kmap));
  memset(&vmap, 0, sizeof(vmap));
  const long long cache_rows = (long long)num_pages * Hkv * page_size;
  p.tma_pages = (dtype != DT_DTYPE_FP32 && page_size >= 16 && page_size <= dtk::kDecodeKeyBlock && (page_size & (page_size - 1)) == 0 &&
                 cache_rows <= 0x7fffffffLL) ? 1 : 0;
  if (p.tma_pages) {
    const bool is16 = dtype == DT_DTYPE_BF16;
    if ((rc = encode_pages(&kmap, k_pages, is16, D, (uint64_t)cache_rows, (uint32_t)page_size, "k_pages"))) return rc;
    if ((rc = encode_pages(&vmap, v_pages, is16, D, (uint64_t)cache_rows, (uint32_t)page_size, "v_pages"))) return rc;
  }
  cudaError_t e = dtype == DT_DTYPE_FP32
                      ? dtk::launch_decode_f32(p, D, B, static_cast<cudaStream_t>(stream))
                      : dtk::launch_decode_sm100(p, kmap, vmap, D, dtype == DT_DTYPE_BF16, B * Hkv,
                                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dt_attn_decode launch");
  return DT_OK;
}

int dt_kv_write(const void* k, const void* v, void* k_pages, void* v_pages, int num_pages, int page_size,
                const int32_t* block_table, int max_pages, const int32_t* start_pos, const float* cos_tab,
                const float* sin_tab, int cos_rows, int64_t cos_stride, int rope_abs, int B, int S, int Hkv, int D,
                int64_t k_sb, int64_t k_ss, int64_t k_sh, int64_t v_sb, int64_t v_ss, int64_t v_sh, int apply_rope,
                int dtype, void* stream) {
  const char* fn = "dt_kv_write";
  NvtxRange nvtx_range("dt_kv_write");
  if (!k || !v) return fail(DT_ERR_INVALID, "%s: null k/v", fn);
  if (B < 1 || S < 1 || Hkv < 1) return fail(DT_ERR_INVALID, "%s: sizes must be positive", fn);
  int rc = check_cache(fn, k_pages, v_pages, num_pages, page_size, block_table, max_pages, D, dtype);
  if (rc) return rc;
  if (apply_rope < 0 || apply_rope > 2) return fail(DT_ERR_INVALID, "%s: apply_rope must be 0, 1 or 2", fn);
  if (apply_rope) {
    if (!cos_tab || !sin_tab) return fail(DT_ERR_INVALID, "%s: null cos/sin with apply_rope", fn);
    if (!rope_abs && cos_rows < S) return fail(DT_ERR_INVALID, "%s: cos/sin have %d rows < S=%d", fn, cos_rows, S);
  }
  int dev = 0;
  int* status = nullptr;
  if ((rc = device_setup(&dev, &status))) return rc;
  dtk::KvWriteParams p;
  p.k = k; p.v = v; p.k_pages = k_pages; p.v_pages = v_pages; p.block_table = block_table; p.start_pos = start_pos;
  p.cos = cos_tab; p.sin = sin_tab; p.status = status;
  p.k_sb = k_sb; p.k_ss = k_ss; p.k_sh = k_sh; p.v_sb = v_sb; p.v_ss = v_ss; p.v_sh = v_sh;
  p.cs_stride = (int)cos_stride; p.cos_rows = cos_rows; p.rope = apply_rope; p.rope_abs = rope_abs ? 1 : 0;
  p.S = S; p.Hkv = Hkv; p.page_size = page_size; p.max_pages = max_pages; p.num_pages = num_pages;
  cudaError_t e = dtk::launch_kv_write_sm100(p, D, dtype, B, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dt_kv_write launch");
  return DT_OK;
}

}  // extern "C"

namespace {
int encode_2d(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t rows, uint64_t row_stride_el,
              uint32_t box_inner, uint32_t box_rows, const char* name, int swizzle_bytes = 128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {row_stride_el * 2};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DT_ERR_INVALID, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name, (int)r);
  return DT_OK;
}
}  // namespace

namespace {
int rmsnorm_qkv_impl(const char* fn, const void* x, int64_t x_row_stride, const void* w_fused, void* y,
                     int64_t y_row_stride, int M, int K, int N, float eps, const float* cos_tab, const float* sin_tab,
                     int64_t cos_stride, int cos_rows, int seq_len, int rope_cols, int head_dim, int dtype,
                     void* stream, int swiglu = 0, int resid = 0, int nonorm = 0) {
  // N counts rows of w_fused; with swiglu, y has N / 2 columns.
  if (!x || !w_fused || !y) return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (M < 1 || K < 1 || N < 1) return fail(DT_ERR_INVALID, "%s: sizes must be positive", fn);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16 / fp16)", fn, dtype);
  const int y_cols = swiglu ? N / 2 : N;
  if (K % 8 || N % 8 || x_row_stride % 8 || y_row_stride % 8 || x_row_stride < K || y_row_stride < y_cols)
    return fail(DT_ERR_INVALID, "%s: K, N and row strides must be multiples of 8 (strides >= K / N)", fn);
  if (!aligned16(x) || !aligned16(w_fused) || !aligned16(y)) return fail(DT_ERR_INVALID, "%s: 16-byte alignment", fn);
  if (!(eps > 0.f)) return fail(DT_ERR_INVALID, "%s: eps must be positive", fn);
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  if (g_cc_major[dev] != 10) return fail(DT_ERR_UNSUPPORTED, "%s: needs an sm_100 GPU", fn);
  const bool bf16 = dtype == DT_DTYPE_BF16;
  if (resid && N % 256 == 0 && g_num_sms[dev] >= 2 &&
      (long long)((M + 255) / 256) * (N / 256) >= 2LL * g_num_sms[dev]) {
    // Residual GEMM on CTA pairs (256 x 256 tiles, each CTA stages half of the
    // tile's x rows and half of its W rows per K chunk), for problems with at
    // least four tiles per pair; smaller ones (a rollout step's 24,576 rows) run
    // faster on the single-CTA kernel below, measured.
    CUtensorMap px, pw, py;
    if ((rc = encode_2d(&px, x, bf16, (uint64_t)K, (uint64_t)M, (uint64_t)x_row_stride, 64, 128, "x", 128))) return rc;
    if ((rc = encode_2d(&pw, w_fused, bf16, (uint64_t)K, (uint64_t)N, (uint64_t)K, 64, 128, "w", 128))) return rc;
    if ((rc = encode_2d(&py, y, bf16, (uint64_t)N, (uint64_t)M, (uint64_t)y_row_stride, 64, 32, "y", 128))) return rc;
    cudaError_t e = dtk::launch_gemm_residual_pair_sm100(px, pw, py, M, N, K, bf16, g_num_sms[dev], status,
                                                         static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
    return DT_OK;
  }
  // 0: persistent kernel, 256-column tiles (the only one with the SwiGLU epilogue)
  const int ncta = (swiglu || resid) ? 0 : dtk::rmsnorm_qkv_ncta(N);
  const int nsub = ncta == 0 ? 256 : (ncta <= 256 ? ncta : ncta / 2);
  CUtensorMap mx, mw, my;
  // The persistent kernel stages kPersistKChunk-wide K slices (32: 64-byte rows, 64-byte swizzle).
  const uint32_t kbox = ncta == 0 ? dtk::kPersistKChunk : 64;
  const int ksw = (int)kbox * 2;
  if ((rc = encode_2d(&mx, x, bf16, (uint64_t)K, (uint64_t)M, (uint64_t)x_row_stride, kbox, 128, "x", ksw))) return rc;
  if ((rc = encode_2d(&mw, w_fused, bf16, (uint64_t)K, (uint64_t)N, (uint64_t)K, kbox, (uint32_t)nsub, "w", ksw)))
    return rc;
  memset(&my, 0, sizeof(my));
  // The persistent kernel stores 32 x 64 output slices (one per epilogue warp) by TMA.
  if (ncta == 0 &&
      (rc = encode_2d(&my, y, bf16, (uint64_t)y_cols, (uint64_t)M, (uint64_t)y_row_stride, 64, 32, "y")))
    return rc;
  dtk::RmsQkvParams p;
  p.y = y; p.status = status; p.y_stride = y_row_stride; p.M = M; p.K = K; p.N = N; p.bf16 = bf16 ? 1 : 0; p.eps = eps;
  p.cos = cos_tab; p.sin = sin_tab; p.rope_cols = rope_cols; p.head_dim = head_dim; p.seq_len = seq_len;
  p.cs_stride = (int)cos_stride;
  p.swiglu = swiglu;
  p.resid = resid;
  p.nonorm = nonorm;
  cudaError_t e = dtk::launch_rmsnorm_qkv_sm100(mx, mw, my, p, ncta, g_num_sms[dev],
                                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}
}  // namespace

extern "C" int dt_rmsnorm_qkv(const void* x, int64_t x_row_stride, const void* w_fused, void* y,
                              int64_t y_row_stride, int M, int K, int N, float eps, int dtype, void* stream) {
  return rmsnorm_qkv_impl("dt_rmsnorm_qkv", x, x_row_stride, w_fused, y, y_row_stride, M, K, N, eps, nullptr,
                          nullptr, 0, 0, 1, 0, 0, dtype, stream);
}

extern "C" int dt_rmsnorm_qkv_rope(const void* x, int64_t x_row_stride, const void* w_fused, void* y,
                                   int64_t y_row_stride, int M, int K, int N, float eps, const float* cos_tab,
                                   const float* sin_tab, int64_t cos_stride, int cos_rows, int seq_len,
                                   int rope_cols, int head_dim, int dtype, void* stream) {
  const char* fn = "dt_rmsnorm_qkv_rope";
  if (!cos_tab || !sin_tab) return fail(DT_ERR_INVALID, "%s: null cos / sin", fn);
  if (head_dim != 32 && head_dim != 64) return fail(DT_ERR_UNSUPPORTED, "%s: head_dim %d not in {32, 64}", fn, head_dim);
  if (rope_cols < 0 || rope_cols > N || rope_cols % head_dim)
    return fail(DT_ERR_INVALID, "%s: rope_cols must be a multiple of head_dim within N", fn);
  if (seq_len < 1 || M % seq_len) return fail(DT_ERR_INVALID, "%s: M must be a multiple of seq_len", fn);
  if (cos_rows < seq_len) return fail(DT_ERR_INVALID, "%s: cos / sin have %d rows < seq_len %d", fn, cos_rows, seq_len);
  if (cos_stride < head_dim || cos_stride % 4 || cos_stride > 0x7fffffffLL || !aligned16(cos_tab) ||
      !aligned16(sin_tab))
    return fail(DT_ERR_INVALID, "%s: cos / sin must be 16-byte aligned with row stride >= head_dim, %% 4", fn);
  return rmsnorm_qkv_impl(fn, x, x_row_stride, w_fused, y, y_row_stride, M, K, N, eps, cos_tab, sin_tab, cos_stride,
                          cos_rows, seq_len, rope_cols, head_dim, dtype, stream);
}

extern "C" int dt_qkv_rope(const void* x, int64_t x_row_stride, const void* w, void* y, int64_t y_row_stride, int M,
                           int K, int N, const float* cos_tab, const float* sin_tab, int64_t cos_stride, int cos_rows,
                           int seq_len, int rope_cols, int head_dim, int dtype, void* stream) {
  const char* fn = "dt_qkv_rope";
  if (head_dim != 32 && head_dim != 64) return fail(DT_ERR_UNSUPPORTED, "%s: head_dim %d not in {32, 64}", fn, head_dim);
  if (rope_cols < 0 || rope_cols > N || rope_cols % head_dim)
    return fail(DT_ERR_INVALID, "%s: rope_cols must be a multiple of head_dim within [0, N]", fn);
  if (!cos_tab || !sin_tab) return fail(DT_ERR_INVALID, "%s: null cos / sin", fn);
  if (seq_len < 1 || M % seq_len) return fail(DT_ERR_INVALID, "%s: M must be a multiple of seq_len", fn);
  if (cos_rows < seq_len) return fail(DT_ERR_INVALID, "%s: cos / sin have %d rows < seq_len %d", fn, cos_rows, seq_len);
  if (cos_stride < head_dim || cos_stride % 4 || cos_stride > 0x7fffffffLL || !aligned16(cos_tab) ||
      !aligned16(sin_tab))
    return fail(DT_ERR_INVALID, "%s: cos / sin must be 16-byte aligned with row stride >= head_dim, %% 4", fn);
  return rmsnorm_qkv_impl(fn, x, x_row_stride, w, y, y_row_stride, M, K, N, 1.f, cos_tab, sin_tab, cos_stride,
                          cos_rows, seq_len, rope_cols, head_dim, dtype, stream, 0, 0, 1);
}

extern "C" int dt_gemm_residual(const void* x, int64_t x_row_stride, const void* w, void* y, int64_t y_row_stride,
                                int M, int K, int N, int dtype, void* stream) {
  const char* fn = "dt_gemm_residual";
  if (N % 64) return fail(DT_ERR_INVALID, "%s: N must be a multiple of 64 (got %d)", fn, N);
  return rmsnorm_qkv_impl(fn, x, x_row_stride, w, y, y_row_stride, M, K, N, 1.f, nullptr, nullptr, 0, 0, 1, 0, 0,
                          dtype, stream, 0, 1);
}

extern "C" int dt_frames_to_blocks(const void* frames, void* out, int64_t N, int C, int H, int W,
                                   unsigned int* frame_max, int dtype, void* stream) {
  const char* fn = "dt_frames_to_blocks";
  if (!frames || !out) return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (N < 1 || C < 1 || H < 4 || W < 4 || H % 4 || W % 4)
    return fail(DT_ERR_INVALID, "%s: N, C >= 1 and H, W positive multiples of 4 required", fn);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16 / fp16)", fn, dtype);
  if ((reinterpret_cast<uintptr_t>(frames) & 3) || !aligned16(out))
    return fail(DT_ERR_INVALID, "%s: frames must be 4-byte and out 16-byte aligned", fn);
  if (N * (int64_t)(H / 4) * (W / 4) > (int64_t)0x7fffffff * 255)
    return fail(DT_ERR_INVALID, "%s: too many frames for one launch", fn);
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  cudaError_t e = dtk::launch_frames_to_blocks_sm100(frames, out, N, C, H, W, dtype == DT_DTYPE_BF16, frame_max,
                                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}

extern "C" int dt_frames_conv1(const void* frames, int64_t N, int C, int H, int W, const void* w, const float* bias,
                               unsigned int* frame_max, void* y, int round_input, int dtype, void* stream) {
  const char* fn = "dt_frames_conv1";
  if (!frames || !w || !bias || !frame_max || !y) return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (C != 4) return fail(DT_ERR_UNSUPPORTED, "%s: %d input channels (the kernel takes 4)", fn, C);
  if (N < 1 || H < 8 || W < 8 || (H - 8) % 4 || (W - 8) % 4)
    return fail(DT_ERR_INVALID, "%s: N >= 1 and H, W = 8 + 4 k required", fn);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16 / fp16)", fn, dtype);
  if (!aligned16(frames) || (N * (int64_t)C * H * W) % 16 || !aligned16(w) || !aligned16(y) ||
      (reinterpret_cast<uintptr_t>(bias) & 3) || (reinterpret_cast<uintptr_t>(frame_max) & 3))
    return fail(DT_ERR_INVALID, "%s: frames, w and y 16-byte aligned, frame bytes a multiple of 16", fn);
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  if (g_cc_major[dev] != 10) return fail(DT_ERR_UNSUPPORTED, "%s: needs an sm_100 GPU", fn);
  cudaError_t e = dtk::launch_frames_conv1_sm100(frames, N, H, W, w, bias, frame_max, y, dtype == DT_DTYPE_BF16,
                                                 round_input != 0, g_num_sms[dev], status,
                                                 static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}

extern "C" int dt_encoder_conv23(const void* x1, int64_t N, const void* w2, const float* b2, void* y2, const void* w3,
                                 const float* b3, void* y3, int dtype, void* stream) {
  const char* fn = "dt_encoder_conv23";
  if (!x1 || !w2 || !b2 || !w3 || !b3 || !y3) return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (N < 1 || N > 0x3fffffffLL) return fail(DT_ERR_INVALID, "%s: N must be in [1, 2^30)", fn);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16 / fp16)", fn, dtype);
  if (!aligned16(x1) || (y2 && !aligned16(y2)) || !aligned16(y3) || (reinterpret_cast<uintptr_t>(w2) & 1) ||
      (reinterpret_cast<uintptr_t>(w3) & 1) || (reinterpret_cast<uintptr_t>(b2) & 3) ||
      (reinterpret_cast<uintptr_t>(b3) & 3))
    return fail(DT_ERR_INVALID, "%s: x1, y2 and y3 must be 16-byte aligned", fn);
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  if (g_cc_major[dev] != 10) return fail(DT_ERR_UNSUPPORTED, "%s: needs an sm_100 GPU", fn);
  // x1 [N, 20, 20, 32] as (channel, x, y, frame), walked with a stride of 2
  // pixels in x and y: a box of 8 channels x 20 x 20 pixels from (8 cg, sx,
  // sy, f) holds the 10 x 10 pixels (2 bx + sx, 2 by + sy), i.e. one K group
  // of the 2 x 2 space-to-depth blocks, 1,600 bytes in block order.
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(DT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  CUtensorMap mx;
  {
    const cuuint64_t dims[4] = {32, 20, 20, (cuuint64_t)N};
    const cuuint64_t strides[3] = {64, 1280, 25600};
    const cuuint32_t box[4] = {8, 20, 20, 1};
    const cuuint32_t estr[4] = {1, 2, 2, 1};
    CUresult r = enc(&mx, dtype == DT_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                     4, const_cast<void*>(x1), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DT_ERR_INVALID, "%s: cuTensorMapEncodeTiled(x1) failed with CUresult %d", fn, (int)r);
  }
  cudaError_t e = dtk::launch_encoder_conv23_sm100(mx, w2, b2, y2, w3, b3, y3, N, dtype == DT_DTYPE_BF16,
                                                   g_num_sms[dev], status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}

extern "C" int dt_frames_conv1_noalloc(const void* frames, int64_t N, int C, int H, int W, const void* w,
                                       const float* bias, void* y, int round_input, int dtype, void* stream) {
  const char* fn = "dt_frames_conv1_noalloc";
  if (!frames || !w || !bias || !y) return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (C != 4) return fail(DT_ERR_UNSUPPORTED, "%s: %d input channels (the kernel takes 4)", fn, C);
  if (N < 1 || H < 8 || W < 8 || (H - 8) % 4 || (W - 8) % 4)
    return fail(DT_ERR_INVALID, "%s: N >= 1 and H, W = 8 + 4 k required", fn);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16 / fp16)", fn, dtype);
  if (!aligned16(frames) || (N * (int64_t)C * H * W) % 16 || !aligned16(w) || !aligned16(y) ||
      (reinterpret_cast<uintptr_t>(bias) & 3))
    return fail(DT_ERR_INVALID, "%s: frames, w and y 16-byte aligned, frame bytes a multiple of 16", fn);
  // The static scratch must hold what this call needs (one word, whatever N).
  if (dtk::kConv1NoallocWordsPerCall > dtk::kConv1NoallocScratchWords)
    return fail(DT_ERR_INVALID, "%s: needs %d scratch words, the static array holds %d", fn,
                dtk::kConv1NoallocWordsPerCall, dtk::kConv1NoallocScratchWords);
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  if (g_cc_major[dev] != 10) return fail(DT_ERR_UNSUPPORTED, "%s: needs an sm_100 GPU", fn);
  unsigned int* scratch = nullptr;
  cudaError_t e = dtk::conv1_noalloc_scratch(&scratch);
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s: scratch address: %s", fn, cudaGetErrorString(e));
  e = dtk::launch_frames_conv1_sm100(frames, N, H, W, w, bias, scratch, y, dtype == DT_DTYPE_BF16, round_input != 0,
                                     g_num_sms[dev], status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}

extern "C" int dt_rmsnorm(const void* x, int64_t x_row_stride, const void* w, void* y, int64_t y_row_stride, int M,
                          int K, float eps, int dtype, void* stream) {
  const char* fn = "dt_rmsnorm";
  if (!x || !w || !y) return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (M < 1 || K < 8 || K % 8 || x_row_stride < K || y_row_stride < K || x_row_stride % 8 || y_row_stride % 8)
    return fail(DT_ERR_INVALID, "%s: K a positive multiple of 8, row strides >= K and multiples of 8", fn);
  if (dtype != DT_DTYPE_BF16 && dtype != DT_DTYPE_FP16)
    return fail(DT_ERR_UNSUPPORTED, "%s: dtype %d not supported (bf16 / fp16)", fn, dtype);
  if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return fail(DT_ERR_INVALID, "%s: 16-byte alignment", fn);
  if (!(eps > 0.f)) return fail(DT_ERR_INVALID, "%s: eps must be positive", fn);
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  cudaError_t e = dtk::launch_rmsnorm_sm100(x, x_row_stride, w, y, y_row_stride, M, K, eps, dtype == DT_DTYPE_BF16,
                                            g_num_sms[dev], static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}

extern "C" int dt_rmsnorm_swiglu(const void* x, int64_t x_row_stride, const void* w_fused, void* y,
                                 int64_t y_row_stride, int M, int K, int N, float eps, int dtype, void* stream) {
  const char* fn = "dt_rmsnorm_swiglu";
  if (N < 128 || N % 64) return fail(DT_ERR_INVALID, "%s: the output width must be a multiple of 64, >= 128", fn);
  if (N > (1 << 29)) return fail(DT_ERR_INVALID, "%s: output width too large", fn);
  return rmsnorm_qkv_impl(fn, x, x_row_stride, w_fused, y, y_row_stride, M, K, 2 * N, eps, nullptr, nullptr, 0, 0, 1,
                          0, 0, dtype, stream, 1);
}

// ------------------------------------------------------------------ NES emulation
namespace {
int nes_check(const char* fn, const DtNesState* s, int n, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr,
              uint32_t chr_size, bool need_rom) {
  if (!s || !s->regs || !s->ram || !s->vram || !s->oam || !s->palette)
    return fail(DT_ERR_INVALID, "%s: null state pointer", fn);
  if (reinterpret_cast<uintptr_t>(s->regs) & 15) return fail(DT_ERR_INVALID, "%s: regs must be 16-byte aligned", fn);
  if (s->framebuffer && (reinterpret_cast<uintptr_t>(s->framebuffer) & 7))
    return fail(DT_ERR_INVALID, "%s: framebuffer must be 8-byte aligned", fn);
  if (n < 1) return fail(DT_ERR_INVALID, "%s: n must be >= 1", fn);
  if (need_rom) {
    if (!prg || !chr) return fail(DT_ERR_INVALID, "%s: null ROM pointer", fn);
    if (prg_size != 0x4000u && prg_size != 0x8000u)
      return fail(DT_ERR_UNSUPPORTED, "%s: PRG ROM must be 16 or 32 KB (got %u bytes)", fn, prg_size);
    if (chr_size != 0x2000u) return fail(DT_ERR_UNSUPPORTED, "%s: CHR ROM must be 8 KB (got %u bytes)", fn, chr_size);
  }
  return DT_OK;
}
dtk::NesLaunch nes_launch(const DtNesState* s, int n, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr) {
  dtk::NesLaunch L;
  memset(&L, 0, sizeof(L));
  L.regs = s->regs; L.ram = s->ram; L.vram = s->vram; L.oam = s->oam; L.pal = s->palette; L.fb = s->framebuffer;
  L.prg = prg; L.prg_size = prg_size; L.chr = chr; L.n = n;
  return L;
}
int nes_run(const char* fn, int op, dtk::NesLaunch& L, void* stream) {
  int dev = 0;
  int* status = nullptr;
  int rc = device_setup(&dev, &status);
  if (rc) return rc;
  L.status = status;
  cudaError_t e = dtk::launch_nes(op, L, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(DT_ERR_CUDA, "%s launch: %s", fn, cudaGetErrorString(e));
  return DT_OK;
}
}  // namespace

extern "C" int dt_nes_reset(const DtNesState* s, int n, const uint8_t* mask, int mirroring, const uint8_t* prg,
                            uint32_t prg_size, const uint8_t* chr, uint32_t chr_size, void* stream) {
  const char* fn = "dt_nes_reset";
  if (int rc = nes_check(fn, s, n, prg, prg_size, chr, chr_size, true)) return rc;
  if (mirroring < -1 || mirroring > 4) return fail(DT_ERR_INVALID, "%s: mirroring must be -1..4", fn);
  dtk::NesLaunch L = nes_launch(s, n, prg, prg_size, chr);
  L.mask = mask;
  L.mirroring = mirroring;
  return nes_run(fn, 1, L, stream);
}

extern "C" int dt_nes_run_frames(const DtNesState* s, int n, int num_frames, const uint8_t* prg, uint32_t prg_size,
                                 const uint8_t* chr, uint32_t chr_size, void* stream) {
  const char* fn = "dt_nes_run_frames";
  if (int rc = nes_check(fn, s, n, prg, prg_size, chr, chr_size, true)) return rc;
  if (num_frames < 1) return fail(DT_ERR_INVALID, "%s: num_frames must be >= 1", fn);
  dtk::NesLaunch L = nes_launch(s, n, prg, prg_size, chr);
  L.num_frames = num_frames;
  return nes_run(fn, 0, L, stream);
}

extern "C" int dt_nes_set_buttons(const DtNesState* s, int n, const uint8_t* buttons, void* stream) {
  const char* fn = "dt_nes_set_buttons";
  if (int rc = nes_check(fn, s, n, nullptr, 0, nullptr, 0, false)) return rc;
  if (!buttons) return fail(DT_ERR_INVALID, "%s: null buttons", fn);
  dtk::NesLaunch L = nes_launch(s, n, nullptr, 0, nullptr);
  L.buttons = buttons;
  return nes_run(fn, 2, L, stream);
}

extern "C" int dt_nes_set_actions(const DtNesState* s, int n, const int64_t* actions, const int32_t* boot,
                                  int boot_settle, void* stream) {
  const char* fn = "dt_nes_set_actions";
  if (int rc = nes_check(fn, s, n, nullptr, 0, nullptr, 0, false)) return rc;
  if (!actions) return fail(DT_ERR_INVALID, "%s: null actions", fn);
  dtk::NesLaunch L = nes_launch(s, n, nullptr, 0, nullptr);
  L.actions = actions;
  L.boot = const_cast<int32_t*>(boot);
  L.boot_settle = boot_settle;
  return nes_run(fn, 2, L, stream);
}

extern "C" int dt_nes_observe(const DtNesState* s, int n, uint8_t* obs, uint8_t* stacked, int stack, void* stream) {
  const char* fn = "dt_nes_observe";
  if (int rc = nes_check(fn, s, n, nullptr, 0, nullptr, 0, false)) return rc;
  if (!s->framebuffer) return fail(DT_ERR_INVALID, "%s: rendering is off (no framebuffer)", fn);
  if (!obs && !stacked) return fail(DT_ERR_INVALID, "%s: no output", fn);
  if (stacked && (stack < 1 || stack > 64)) return fail(DT_ERR_INVALID, "%s: stack must be 1..64", fn);
  if ((obs && (reinterpret_cast<uintptr_t>(obs) & 3)) || (stacked && (reinterpret_cast<uintptr_t>(stacked) & 3)))
    return fail(DT_ERR_INVALID, "%s: outputs must be 4-byte aligned", fn);
  dtk::NesLaunch L = nes_launch(s, n, nullptr, 0, nullptr);
  L.obs = obs;
  L.stacked = stacked;
  L.stack = stack;
  return nes_run(fn, 3, L, stream);
}

extern "C" int dt_nes_env_update(const DtNesState* s, int n, int frame_skip, int boot_total, int32_t* boot,
                                 int32_t* prev_x, int32_t* init_lives, float* reward, uint8_t* done, int32_t* x_pos,
                                 int32_t* lives, uint8_t* flag_get, const uint8_t* prg, uint32_t prg_size,
                                 const uint8_t* chr, uint32_t chr_size, void* stream) {
  const char* fn = "dt_nes_env_update";
  if (int rc = nes_check(fn, s, n, prg, prg_size, chr, chr_size, true)) return rc;
  if (!boot || !prev_x || !init_lives || !reward || !done || !x_pos || !lives || !flag_get)
    return fail(DT_ERR_INVALID, "%s: null pointer", fn);
  if (frame_skip < 1 || boot_total < 0) return fail(DT_ERR_INVALID, "%s: frame_skip >= 1, boot_total >= 0", fn);
  dtk::NesLaunch L = nes_launch(s, n, prg, prg_size, chr);
  L.frame_skip = frame_skip;
  L.boot_total = boot_total;
  L.boot = boot;
  L.prev_x = prev_x;
  L.init_lives = init_lives;
  L.reward = reward;
  L.done = done;
  L.x_pos = x_pos;
  L.lives = lives;
  L.flag = flag_get;
  return nes_run(fn, 4, L, stream);
}
