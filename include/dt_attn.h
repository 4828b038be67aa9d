/*
 * dt_attn.h -- C ABI of the sm_100a Decision Transformer attention library
 * (libdt_attn_sm100.so).
 *
 * The library replaces the attention core of DecisionTransformerAttention in
 * FujiM3/RL_for_Mario (model/model_decision_transformer.py:137-249).  Every
 * entry point takes raw device pointers, sizes, element strides and a
 * cudaStream_t (passed as void*), allocates no device memory, launches
 * asynchronously on that stream and returns a status code.  On a nonzero
 * status, dt_last_error() returns a message for the calling thread.
 *
 * Layout conventions (element strides; the innermost dimension, D, is
 * contiguous):
 *   q, o       [B, S, Hq, D]   -- the reference's q_proj(x).view(B, S, Hq, D)
 *   k, v       [B, S, Hkv, D]  -- k_proj / v_proj views (:175-177)
 *   cos, sin   [rows, D] fp32  -- precompute_freqs_cis tables (:93-99), already
 *                                 sliced so that row i is the angle of token i
 *                                 of this call (:440-443)
 *   pad_len    [B] int32       -- number of leading padding tokens per sample
 *                                 (left padding, attention_mask == 0 prefix)
 */
#ifndef DT_ATTN_H_
#define DT_ATTN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define DT_OK 0
#define DT_ERR_INVALID 1     /* bad pointer, size, stride or alignment */
#define DT_ERR_UNSUPPORTED 2 /* shape / dtype / device not supported */
#define DT_ERR_CUDA 3        /* a CUDA runtime call failed */
#define DT_ERR_DEVICE 4      /* a kernel reported a device-side error */

/* Element types. */
#define DT_DTYPE_BF16 0
#define DT_DTYPE_FP16 1
#define DT_DTYPE_FP32 2

/* Library version, (major << 16) | minor. */
int dt_version(void);

/* Message describing the last nonzero status returned on this thread. */
const char* dt_last_error(void);

/*
 * Fused causal grouped-query prefill attention.
 *
 * Replaces, for one layer, the prefill branch of
 * DecisionTransformerAttention.forward (model_decision_transformer.py:179-224):
 * RoPE on q and k (apply_rotary_pos_emb, :108-117, when apply_rope != 0),
 * repeat_kv (:121-130, never materialised here), and
 * F.scaled_dot_product_attention with the causal mask and the additive
 * (1 - attention_mask) * -1e9 padding mask (:206-224), scale 1/sqrt(D) unless
 * `scale` > 0 is given.  Writes the attention output (before o_proj, :247) to o.
 *
 * Supported: dtype BF16 or FP16, D in {32, 64}, Hq % Hkv == 0,
 * Hq / Hkv <= 128.  Base pointers 16-byte aligned, strides multiples of 8
 * elements, cos/sin rows >= S.
 */
int dt_attn_prefill(const void* q, const void* k, const void* v, void* o, const float* cos_tab,
                    const float* sin_tab, int cos_rows, int64_t cos_stride, const int32_t* pad_len, int B,
                    int S, int Hq, int Hkv, int D, int64_t q_sb, int64_t q_ss, int64_t q_sh, int64_t k_sb,
                    int64_t k_ss, int64_t k_sh, int64_t v_sb, int64_t v_ss, int64_t v_sh, int64_t o_sb,
                    int64_t o_ss, int64_t o_sh, float scale, int apply_rope, int dtype, void* stream);

/*
 * KV-cached decode step with an in-place paged cache.
 *
 * Replaces the cached branch of DecisionTransformerAttention.forward
 * (model_decision_transformer.py:179-191 and :225-245): rotates q and k_new
 * (RoPE at the new tokens' positions), appends the rotated k_new and v_new to
 * the cache at positions seq_lens[b] .. seq_lens[b] + Sn - 1 (the reference
 * builds a new tensor with torch.cat, :188-190), then attends the Sn new
 * queries over all seq_lens[b] + Sn keys: causal on the new columns
 * (:230-237), optional left padding pad_len[b] of the [B, kv_len] mask
 * (:238-242), softmax in fp32 (:243).  seq_lens is read, not advanced.
 *
 * Cache: k_pages / v_pages [num_pages, Hkv, page_size, D]; block_table
 * [B, max_pages] int32 page ids.  cos/sin rows are indexed by absolute
 * position when rope_abs != 0, else by the new-token index 0..Sn-1 (the
 * reference passes tables already sliced at start_pos, :439-443).
 * Out-of-range positions or page ids are rejected on the device: the kernel
 * skips the sample and sets the status word (dt_device_status).
 */
int dt_attn_decode(const void* q, const void* k_new, const void* v_new, void* o, void* k_pages, void* v_pages,
                   int num_pages, int page_size, const int32_t* block_table, int max_pages,
                   const int32_t* seq_lens, const int32_t* pad_len, const float* cos_tab, const float* sin_tab,
                   int cos_rows, int64_t cos_stride, int rope_abs, int B, int Sn, int Hq, int Hkv, int D,
                   int64_t q_sb, int64_t q_ss, int64_t q_sh, int64_t kn_sb, int64_t kn_ss, int64_t kn_sh,
                   int64_t vn_sb, int64_t vn_ss, int64_t vn_sh, int64_t o_sb, int64_t o_ss, int64_t o_sh,
                   float scale, int apply_rope, int dtype, void* stream);

/*
 * Writes S tokens of K (rotated when apply_rope) and V into the paged cache at
 * positions start_pos[b] + s (start_pos may be null: 0).  This is the cache
 * produced by the prefill branch with use_cache=True
 * (model_decision_transformer.py:179-191: present = (RoPE(k), v)); a dense
 * [B, Hkv, L, D] cache is the case page_size = L, block_table[b] = {b}.
 */
int dt_kv_write(const void* k, const void* v, void* k_pages, void* v_pages, int num_pages, int page_size,
                const int32_t* block_table, int max_pages, const int32_t* start_pos, const float* cos_tab,
                const float* sin_tab, int cos_rows, int64_t cos_stride, int rope_abs, int B, int S, int Hkv, int D,
                int64_t k_sb, int64_t k_ss, int64_t k_sh, int64_t v_sb, int64_t v_ss, int64_t v_sh, int apply_rope,
                int dtype, void* stream);

/*
 * Fused RMSNorm + Q/K/V projection: y[m, :] = rsqrt(mean(x[m, :]^2) + eps) *
 * (x[m, :] @ w_fused^T), with w_fused = [Wq; Wk; Wv] * diag(w_norm) ([N, K],
 * K contiguous).  Replaces the block's input_layernorm (RMSNorm,
 * model_decision_transformer.py:76-86, called at :296) followed by the
 * attention's q_proj / k_proj / v_proj (:175-177); a row of y is the fused
 * [q | k | v] the prefill / decode entry points take as strided views.
 * x [M, K] (row stride x_row_stride), y [M, N] (row stride y_row_stride);
 * bf16 or fp16; K, N and strides multiples of 8, 16-byte aligned pointers.
 */
int dt_rmsnorm_qkv(const void* x, int64_t x_row_stride, const void* w_fused, void* y, int64_t y_row_stride, int M,
                   int K, int N, float eps, int dtype, void* stream);

/*
 * dt_rmsnorm_qkv followed, in the same epilogue, by the rotate-half RoPE of
 * the q and k heads (apply_rotary_pos_emb, model_decision_transformer.py:103-117,
 * applied at :179-183): columns [0, rope_cols) of y are groups of head_dim
 * (32 or 64) and row m is rotated with table row (m mod seq_len) of cos / sin
 * ([>= seq_len, head_dim] fp32, row stride cos_stride, 16-byte aligned).  The
 * v columns (>= rope_cols) are left as projected.  The result feeds the
 * attention entry points with apply_rope = 0.
 */
int dt_rmsnorm_qkv_rope(const void* x, int64_t x_row_stride, const void* w_fused, void* y, int64_t y_row_stride,
                        int M, int K, int N, float eps, const float* cos_tab, const float* sin_tab,
                        int64_t cos_stride, int cos_rows, int seq_len, int rope_cols, int head_dim, int dtype,
                        void* stream);

/*
 * Fused post-attention RMSNorm + SwiGLU up-projection:
 *   y[m, j] = silu(g[m, j]) * u[m, j],  [g | u] = rsqrt(mean(x[m, :]^2) + eps) * (x[m, :] @ W^T)
 * Replaces post_attention_layernorm (RMSNorm, model_decision_transformer.py:76-86,
 * called at :302-303) and FeedForward's gate_proj / up_proj / silu / product
 * (:256-271, before down_proj).  w_fused ([2 N, K], K contiguous) holds the
 * gate and up rows, each scaled by the norm weight, interleaved in blocks of
 * 64 rows: rows [128 b, 128 b + 64) are gate rows [64 b, 64 b + 64) and rows
 * [128 b + 64, 128 b + 128) the matching up rows.  x [M, K], y [M, N]; N (the
 * FFN width) a multiple of 64 and >= 128; bf16 or fp16; K and row strides
 * multiples of 8, 16-byte aligned pointers.
 */
int dt_rmsnorm_swiglu(const void* x, int64_t x_row_stride, const void* w_fused, void* y, int64_t y_row_stride,
                      int M, int K, int N, float eps, int dtype, void* stream);

/*
 * Q/K/V projection + RoPE without a norm: y = x @ w^T with the rotate-half RoPE
 * of the q and k heads (columns [0, rope_cols)) applied in the epilogue, as
 * dt_rmsnorm_qkv_rope does after its norm.  Replaces q_proj / k_proj / v_proj
 * (model_decision_transformer.py:175-177) and apply_rotary_pos_emb (:103-117,
 * applied at :179-183) when the caller has already normalised x (the drop-in
 * module inside the reference's block, whose input_layernorm runs first,
 * :296); the attention entry points then take q / k with apply_rope = 0.
 * w = [Wq; Wk; Wv] ([N, K]); other arguments as dt_rmsnorm_qkv_rope.
 */
int dt_qkv_rope(const void* x, int64_t x_row_stride, const void* w, void* y, int64_t y_row_stride, int M, int K,
                int N, const float* cos_tab, const float* sin_tab, int64_t cos_stride, int cos_rows, int seq_len,
                int rope_cols, int head_dim, int dtype, void* stream);

/*
 * Residual GEMM of the DT block: y[m, :] += x[m, :] @ w^T in place, in fp32
 * with one rounding of the sum (the residual is the GEMM's accumulator input).
 * Replaces o_proj and its residual add (model_decision_transformer.py:247-248,
 * :300) and down_proj and its residual add (:271, :303).  x [M, K], w [N, K]
 * (K contiguous), y [M, N], row strides in elements; bf16 or fp16; K, N and
 * the strides multiples of 8, N a multiple of 64, 16-byte aligned pointers.
 * Runs on the persistent tcgen05 GEMM of dt_rmsnorm_qkv (256-column tiles).
 */
int dt_gemm_residual(const void* x, int64_t x_row_stride, const void* w, void* y, int64_t y_row_stride, int M, int K,
                     int N, int dtype, void* stream);

/*
 * The state encoder's first layer from the uint8 frames: frames / 255 (when
 * their maximum exceeds 1, model_decision_transformer.py:338), Conv2d(4, 32,
 * 8, stride 4) and ReLU (:315-341), as one implicit GEMM on the tensor cores.
 * frames [N, 4, H, W] uint8 (H, W = 8 + 4k; 16-byte aligned, N*4*H*W a
 * multiple of 16); w [32, 256] 16-bit, the conv weight [32, 4, 8, 8] as is
 * (unscaled); bias [32] fp32; y [N, OH, OW, 32] 16-bit (channels-last, OH =
 * (H - 8) / 4 + 1); frame_max (device) ends > 1 exactly when some byte of the
 * frames exceeds 1 (the reference's test; the scan stops at the first such byte).
 * Rounding (round_input = 0): the pixels enter the MMA as exact 16-bit
 * integers, the 1/255 is applied to the fp32 accumulator and the output is
 * rounded once: the fp32 convolution of frames / 255 to within one output
 * rounding.  round_input = 1: frames / 255 is rounded to the output dtype
 * first, as the reference's 16-bit model evaluates x / 255 before its
 * convolution; the products then accumulate in fp32 and the output is
 * rounded once.
 */
int dt_frames_conv1(const void* frames, int64_t N, int C, int H, int W, const void* w, const float* bias,
                    unsigned int* frame_max, void* y, int round_input, int dtype, void* stream);

/*
 * The state encoder's second and third layers: Conv2d(32, 64, 4, stride 2) +
 * ReLU on the first layer's 20 x 20 output, then Conv2d(64, 64, 3, stride 1) +
 * ReLU (model_decision_transformer.py:322-325), fused in one tensor-core
 * kernel that keeps the second layer's output in shared memory.  x1
 * [N, 20, 20, 32] and y3 [N, 7, 7, 64] channels-last 16-bit tensors (16-byte
 * aligned); y2 [N, 9, 9, 64] (nullable) also receives the second layer's
 * output (conv2 + ReLU) when given.  w2 [64, 32, 4, 4],
 * w3 [64, 64, 3, 3] 16-bit in the reference's own layout; b2, b3 [64] fp32.
 * Products accumulate in fp32, the bias is added in fp32 and each output is
 * rounded once.  bf16 or fp16; N in [1, 2^30).
 */
int dt_encoder_conv23(const void* x1, int64_t N, const void* w2, const float* b2, void* y2, const void* w3,
                      const float* b3, void* y3, int dtype, void* stream);

/*
 * dt_frames_conv1 for callers that cannot allocate device memory.  No
 * counterpart in the reference: it exists for callers such as an environment
 * host written in C or C++ that hands the library frames it already holds on
 * the GPU and owns no allocator, or a process whose memory pool has reserved
 * the device's memory, where a cudaMalloc would fail or stall the step loop.
 * Same arguments and result as dt_frames_conv1 without frame_max: the
 * frame-maximum word lives in a 256-byte static device array of the library
 * (held on every GPU that loads it, until exit).  A call needs one word of it
 * whatever the frame count, and is rejected with DT_ERR_INVALID if the array
 * cannot hold that.  The call allocates nothing (no cudaMalloc, cudaFree or
 * allocating library routine).  Its first call on a device looks up the
 * array's device address there; make that first call before any stream
 * capture.  Every call shares the array (each clears its word first), so
 * calls whose work overlaps on the GPU, on different streams, race.
 */
int dt_frames_conv1_noalloc(const void* frames, int64_t N, int C, int H, int W, const void* w, const float* bias,
                            void* y, int round_input, int dtype, void* stream);

/*
 * RMSNorm with the reference's rounding: y = w * cast(x * rsqrt(mean(x^2) +
 * eps)) with the mean and rsqrt in fp32, the normalised row cast to the
 * activation dtype before the weight product (model_decision_transformer.py:
 * 76-86; used for embed_norm and the final norm, :420 and :457).  x, y
 * [M, K] with row strides; w [K]; bf16 or fp16; K and strides multiples of
 * 8, 16-byte aligned pointers.
 */
int dt_rmsnorm(const void* x, int64_t x_row_stride, const void* w, void* y, int64_t y_row_stride, int M, int K,
               float eps, int dtype, void* stream);

/*
 * State-encoder input: uint8 frame stacks [N, C, H, W] -> 16-bit 4 x 4
 * space-to-depth blocks, channels-last [N, H/4, W/4, C*16] with channel
 * c*16 + dy*4 + dx = frames[n, c, 4Y + dy, 4X + dx] (values 0..255, exact).
 * With the first convolution's weight regrouped the same way (and scaled by
 * 1/255), the reference's frames / 255 -> Conv2d(C, 32, 8, stride 4)
 * (model_decision_transformer.py:315-341, division at :338) becomes a 2 x 2
 * stride-1 convolution over C*16 channels.  frame_max (nullable, device):
 * raised by atomicMax to the largest byte read (the reference's x.max() > 1
 * test, :338, without a separate pass).  H, W multiples of 4; frames 4-byte
 * aligned, out 16-byte aligned; bf16 or fp16 output.
 */
int dt_frames_to_blocks(const void* frames, void* out, int64_t N, int C, int H, int W, unsigned int* frame_max,
                        int dtype, void* stream);

/*
 * ---- Batched NES emulation: the Mario environment step (scope row f4) ----
 *
 * Replaces the reference's GPU emulator class NESBatchGpu and its kernels
 * (nes_emulator_gpu/src/cuda/host/nes_batch_gpu.{h,cu}, src/cuda/kernels/
 * nes_batch_kernel.cu) and the bookkeeping of GpuMarioVecEnv.step
 * (scripts/mario/gpu_vec_env.py:271-404), with the same results (the same
 * instructions, cycle counts, PPU model, frame loop and observation).  The
 * caller owns every buffer; nothing here allocates.  Instances are grouped 32
 * to a group; buffers hold n_pad = n rounded up to 32 instances:
 *   regs        [n_pad][48]  packed registers, little-endian: A X Y SP, PC(16)
 *               P nmi_pending, irq_pending joypad1 joypad_shift joypad_strobe,
 *               PPUCTRL PPUMASK PPUSTATUS OAMADDR, v(16) t(16), fine_x w
 *               read_buffer mirroring, scanline(16) cycle(16), frame_ready 0
 *               active_sprite_count far_dma_count, total_cycles(64),
 *               sprite-0-in-list flag, 0 (16-byte aligned)
 *   ram, vram   [n_pad/32][2048][32]   byte a of instance i at
 *                                       ((i/32)*2048 + a)*32 + i%32
 *   oam         [n_pad/32][256][32],  palette [n_pad/32][32][32]
 *   framebuffer [n_pad/32][240][32][32][8] palette values; pixel (y, x) of
 *               instance i at (((i/32)*240 + y)*32 + x/8)*256 + (i%32)*8 + x%8;
 *               NULL renders nothing (and, as in the reference, then never
 *               sets the sprite 0 hit flag)
 * PRG ROM 16 or 32 KB, CHR ROM 8 KB (NROM), device memory.
 * Defined where the reference is not: an OAM DMA from page >= 8 copies from
 * the RAM mirror (pages < 0x20), PRG ROM (pages >= 0x80) or zeros (the
 * reference reads past the instance's RAM); reset clears the controller latch.
 */
typedef struct DtNesState {
  uint8_t* regs;
  uint8_t* ram;
  uint8_t* vram;
  uint8_t* oam;
  uint8_t* palette;
  uint8_t* framebuffer;
} DtNesState;

/* Power-on reset (NESBatchGpu::reset_all / reset_selected,
 * nes_batch_kernel.cu:86-110, :231-254) of every instance, or of those with
 * mask[i] != 0 (device, nullable).  mirroring 0..4 sets it (MIRROR_*); -1 keeps
 * each instance's. */
int dt_nes_reset(const DtNesState* s, int n, const uint8_t* mask, int mirroring, const uint8_t* prg,
                 uint32_t prg_size, const uint8_t* chr, uint32_t chr_size, void* stream);

/* num_frames frames of every instance, all but the last without background
 * rendering (NESBatchGpu::run_frames_all, nes_batch_kernel.cu:116-160;
 * num_frames = 1 is run_frame_all, :46-80). */
int dt_nes_run_frames(const DtNesState* s, int n, int num_frames, const uint8_t* prg, uint32_t prg_size,
                      const uint8_t* chr, uint32_t chr_size, void* stream);

/* Controller bytes (device [n]) and a fresh serial latch
 * (NESBatchGpu::set_buttons_batch, nes_batch_gpu.cu:424-430). */
int dt_nes_set_buttons(const DtNesState* s, int n, const uint8_t* buttons, void* stream);

/* Controller bytes from SIMPLE_MOVEMENT action indices (device int64 [n],
 * 0..6), overridden during the boot sequence (boot[i] > boot_settle: START;
 * 0 < boot[i] <= boot_settle: none) as GpuMarioVecEnv.step does
 * (gpu_vec_env.py:327-342).  An index out of 0..6 sets the device status. */
int dt_nes_set_actions(const DtNesState* s, int n, const int64_t* actions, const int32_t* boot,
                       int boot_settle, void* stream);

/* 84 x 84 grayscale observation of every framebuffer (palette -> luma,
 * bilinear; nes_batch_kernel.cu:180-216) into obs [n][84][84] (nullable) and,
 * when stacked [n][stack][84][84] is given, shifts each instance's stack by one
 * frame (oldest first) and appends it (the frame ring of gpu_vec_env.py:
 * 250-267). */
int dt_nes_observe(const DtNesState* s, int n, uint8_t* obs, uint8_t* stacked, int stack, void* stream);

/* The rest of GpuMarioVecEnv.step (gpu_vec_env.py:344-404) after the frames and
 * the observation: x position ($006D * 256 + $0086), lives ($075A) and the
 * stage-clear flag ($07D7 == 0x80) from RAM; boot counters (boot[i] -= frame_skip
 * while > 0); reward = clip(dx / 40, -1, 1), -1 on a lost life, +1 on the
 * flag; done; and, for done instances, a reset and boot[i] = boot_total.  All
 * arrays are device [n] and updated in place. */
int dt_nes_env_update(const DtNesState* s, int n, int frame_skip, int boot_total, int32_t* boot, int32_t* prev_x,
                      int32_t* init_lives, float* reward, uint8_t* done, int32_t* x_pos, int32_t* lives,
                      uint8_t* flag_get, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr,
                      uint32_t chr_size, void* stream);

/*
 * Synchronises `stream`, then returns and clears the device status word that
 * the kernels of this library write when a bounded wait runs out or a
 * device-side check fails (0 = no error).  Used by tests and debugging.
 */
int dt_device_status(void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DT_ATTN_H_ */
