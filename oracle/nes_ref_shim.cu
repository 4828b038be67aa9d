// ORACLE (test infrastructure only): extern "C" wrappers around the reference's
// own batched NES emulator (class NESBatchGpu, nes_emulator_gpu/src/cuda/host/
// nes_batch_gpu.{h,cu}, and its kernels in src/cuda/kernels/nes_batch_kernel.cu),
// compiled from the reference's sources by oracle/build_ref.py into
// oracle/_ref/libnes_ref.so.  Tests use it to pin the CPU oracle
// (oracle/nes_oracle.c) to the reference's GPU code on synthetic cartridges.
// Errors (the class throws) come back as -1.
#include <cstdint>
#include <cstring>
#include <exception>

#include "nes_batch_gpu.h"

extern "C" {
void* ref_nes_create(int n) {
  try {
    return new NESBatchGpu(n);
  } catch (const std::exception&) {
    return nullptr;
  }
}
void ref_nes_destroy(void* h) { delete static_cast<NESBatchGpu*>(h); }

#define REF_TRY(stmt)                 \
  try {                               \
    stmt;                             \
    return 0;                         \
  } catch (const std::exception&) {   \
    return -1;                        \
  }

int ref_nes_load_rom(void* h, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr, uint32_t chr_size) {
  REF_TRY(static_cast<NESBatchGpu*>(h)->load_rom(prg, prg_size, chr, chr_size))
}
int ref_nes_reset_all(void* h, int mirroring) {
  REF_TRY(static_cast<NESBatchGpu*>(h)->reset_all((uint8_t)mirroring))
}
int ref_nes_run_frame_all(void* h) { REF_TRY(static_cast<NESBatchGpu*>(h)->run_frame_all()) }
int ref_nes_run_frames_all(void* h, int k) { REF_TRY(static_cast<NESBatchGpu*>(h)->run_frames_all(k)) }
int ref_nes_set_buttons(void* h, const uint8_t* b, int n) {
  REF_TRY(static_cast<NESBatchGpu*>(h)->set_buttons_batch(b, n))
}
int ref_nes_get_ram(void* h, uint8_t* out) { REF_TRY(static_cast<NESBatchGpu*>(h)->get_ram_batch(out)) }
int ref_nes_get_obs(void* h, uint8_t* out) { REF_TRY(static_cast<NESBatchGpu*>(h)->get_obs_batch(out)) }
int ref_nes_get_framebuffers(void* h, uint32_t* out) {
  REF_TRY(static_cast<NESBatchGpu*>(h)->get_framebuffers(out))
}
int ref_nes_reset_selected(void* h, const uint8_t* mask, int n) {
  REF_TRY(static_cast<NESBatchGpu*>(h)->reset_selected(mask, n))
}
// Scalars of instance i, in the oracle's order (oracle/nes.py SCALARS, without dma_far).
int ref_nes_get_scalars(void* h, int i, int64_t* out) {
  try {
    NESState s;
    std::memset(&s, 0, sizeof(s));
    static_cast<NESBatchGpu*>(h)->get_state(i, s);
    const int64_t v[27] = {s.cpu.A, s.cpu.X, s.cpu.Y, s.cpu.SP, s.cpu.PC, s.cpu.P, (int64_t)s.cpu.total_cycles,
                           s.cpu.nmi_pending, s.cpu.irq_pending, 0, 0, 0, s.ppu.ctrl, s.ppu.mask, s.ppu.status,
                           s.ppu.oam_addr, s.ppu.v, s.ppu.t, s.ppu.fine_x, s.ppu.w, s.ppu.read_buffer,
                           s.ppu.mirroring, s.ppu.scanline, s.ppu.cycle, s.ppu.frame_ready, s.ppu.nmi_flag,
                           s.ppu.active_sprite_count};
    std::memcpy(out, v, sizeof(v));
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}
}
