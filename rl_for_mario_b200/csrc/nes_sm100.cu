// Batched NES emulation for the Mario environment step (rows f4 of the hot-path
// scope), sm_100a: one thread per emulator instance, the instance's CPU and PPU
// registers in registers, and its memories interleaved 32 instances to a group
// in HBM so that a warp's accesses to one address of its 32 instances are one
// 32-byte sector.
//
// Behaviour is the reference's batched CUDA emulator, exactly
// (nes_emulator_gpu/src/cuda/kernels/nes_batch_kernel.cu, device/cpu_device.cuh,
// device/ppu_device.cuh): the same instruction set, cycle counts and bus, the same
// simplified PPU (tile background from the PPUCTRL nametable, per-pixel sprites,
// sprite 0 hit, vblank NMI), the same frame loop (an instruction, then 3 PPU dots
// per CPU cycle, until the dot that enters scanline 261; at most 65,000 CPU cycles)
// and the same headless intermediate frames of a multi-frame step.  Two places
// where the reference's behaviour is undefined are defined here: an OAM DMA from
// page >= 8 reads the RAM mirror (pages < 0x20), PRG ROM (pages >= 0x80) or 0 --
// the reference copies from memory past the instance's RAM -- and reset leaves the
// controller latch at 0.
//
// What differs is how the work is laid out:
//   - the PPU advances by ranges of dots between CPU instructions, visiting only
//     the dots where something happens (sprite evaluation at the start of a
//     visible line, rendered pixels, vblank, pre-render); the reference calls its
//     dot function 3 times per CPU cycle.  CPU accesses happen only between
//     instructions, so the result is the same;
//   - a background tile is kept in a 64-bit register while its 8 pixels are
//     rendered and the sprites drawn over it, then stored with one 8-byte store;
//   - OAM, palette RAM, the line's sprite list and the decode table sit in shared
//     memory; PRG / CHR ROM are read through the read-only cache;
//   - instructions are decoded through a 256-entry table (addressing mode, operation,
//     base cycles, page-cross cycle) instead of a 256-way switch, so instances on
//     different opcodes of the same mode share the address code.
#include <cuda_runtime.h>
#include <stdint.h>

#include "dt_internal.h"

namespace dtk {
namespace {

// mode (bits 0-3) | kind << 4 | base cycles << 10 | page-cross cycle << 14
__constant__ uint32_t kNesDecode[256] = {
    0x1DA0u, 0x1868u, 0x0710u, 0x0710u, 0x0F0Cu, 0x0C62u, 0x14F2u, 0x0710u,
    0x0DC0u, 0x0861u, 0x08FEu, 0x0710u, 0x130Du, 0x1065u, 0x18F5u, 0x0710u,
    0x095Au, 0x5469u, 0x0710u, 0x0710u, 0x130Cu, 0x1063u, 0x18F3u, 0x0710u,
    0x0A90u, 0x5067u, 0x0B00u, 0x0710u, 0x5306u, 0x5066u, 0x1CF6u, 0x0710u,
    0x1975u, 0x1878u, 0x0710u, 0x0710u, 0x0CE2u, 0x0C72u, 0x1512u, 0x0710u,
    0x11E0u, 0x0871u, 0x091Eu, 0x0710u, 0x10E5u, 0x1075u, 0x1915u, 0x0710u,
    0x095Au, 0x5479u, 0x0710u, 0x0710u, 0x130Cu, 0x1073u, 0x1913u, 0x0710u,
    0x0AA0u, 0x5077u, 0x0B00u, 0x0710u, 0x5306u, 0x5076u, 0x1D16u, 0x0710u,
    0x1990u, 0x1888u, 0x0710u, 0x0710u, 0x0F0Cu, 0x0C82u, 0x1502u, 0x0710u,
    0x0DB0u, 0x0881u, 0x090Eu, 0x0710u, 0x0D65u, 0x1085u, 0x1905u, 0x0710u,
    0x095Au, 0x5489u, 0x0710u, 0x0710u, 0x130Cu, 0x1083u, 0x1903u, 0x0710u,
    0x0AB0u, 0x5087u, 0x0B00u, 0x0710u, 0x5306u, 0x5086u, 0x1D06u, 0x0710u,
    0x1980u, 0x1898u, 0x0710u, 0x0710u, 0x0F0Cu, 0x0C92u, 0x1522u, 0x0710u,
    0x11D0u, 0x0891u, 0x092Eu, 0x0710u, 0x156Bu, 0x1095u, 0x1925u, 0x0710u,
    0x095Au, 0x5499u, 0x0710u, 0x0710u, 0x130Cu, 0x1093u, 0x1923u, 0x0710u,
    0x0AC0u, 0x5097u, 0x0B00u, 0x0710u, 0x5306u, 0x5096u, 0x1D26u, 0x0710u,
    0x0B0Cu, 0x1838u, 0x0B0Cu, 0x0710u, 0x0C52u, 0x0C32u, 0x0C42u, 0x0710u,
    0x0A80u, 0x0B0Cu, 0x0A10u, 0x0710u, 0x1055u, 0x1035u, 0x1045u, 0x0710u,
    0x095Au, 0x1839u, 0x0710u, 0x0710u, 0x1053u, 0x1033u, 0x1044u, 0x0710u,
    0x0A20u, 0x1437u, 0x0A40u, 0x0710u, 0x0710u, 0x1436u, 0x0710u, 0x0710u,
    0x0821u, 0x1808u, 0x0811u, 0x0710u, 0x0C22u, 0x0C02u, 0x0C12u, 0x0710u,
    0x0A00u, 0x0801u, 0x09F0u, 0x0710u, 0x1025u, 0x1005u, 0x1015u, 0x0710u,
    0x095Au, 0x5409u, 0x0710u, 0x0710u, 0x1023u, 0x1003u, 0x1014u, 0x0710u,
    0x0AD0u, 0x5007u, 0x0A30u, 0x0710u, 0x5026u, 0x5006u, 0x5017u, 0x0710u,
    0x08D1u, 0x18B8u, 0x0B0Cu, 0x0710u, 0x0CD2u, 0x0CB2u, 0x1542u, 0x0710u,
    0x0A60u, 0x08B1u, 0x0A70u, 0x0710u, 0x10D5u, 0x10B5u, 0x1945u, 0x0710u,
    0x095Au, 0x54B9u, 0x0710u, 0x0710u, 0x130Cu, 0x10B3u, 0x1943u, 0x0710u,
    0x0AE0u, 0x50B7u, 0x0B00u, 0x0710u, 0x5306u, 0x50B6u, 0x1D46u, 0x0710u,
    0x08C1u, 0x18A8u, 0x0B0Cu, 0x0710u, 0x0CC2u, 0x0CA2u, 0x1532u, 0x0710u,
    0x0A50u, 0x08A1u, 0x0B00u, 0x0710u, 0x10C5u, 0x10A5u, 0x1935u, 0x0710u,
    0x095Au, 0x54A9u, 0x0710u, 0x0710u, 0x130Cu, 0x10A3u, 0x1933u, 0x0710u,
    0x0AF0u, 0x50A7u, 0x0B00u, 0x0710u, 0x5306u, 0x50A6u, 0x1D36u, 0x0710u,
};
enum NesMode {NM_IMP, NM_IMM, NM_ZP, NM_ZPX, NM_ZPY, NM_ABS, NM_ABX, NM_ABY, NM_IZX, NM_IZY, NM_REL, NM_IND, NM_SK1, NM_SK2, NM_ACC};
enum NesKind {NK_LDA, NK_LDX, NK_LDY, NK_STA, NK_STX, NK_STY, NK_ORA, NK_AND, NK_EOR, NK_ADC, NK_SBC, NK_CMP, NK_CPX, NK_CPY, NK_BIT, NK_ASL, NK_LSR, NK_ROL, NK_ROR, NK_INC, NK_DEC, NK_BR, NK_JMP, NK_JSR, NK_RTS, NK_RTI, NK_BRK, NK_PHA, NK_PHP, NK_PLA, NK_PLP, NK_TAX, NK_TAY, NK_TXA, NK_TYA, NK_TSX, NK_TXS, NK_INX, NK_INY, NK_DEX, NK_DEY, NK_CLC, NK_SEC, NK_CLI, NK_SEI, NK_CLV, NK_CLD, NK_SED, NK_NOP, NK_UNK};


constexpr int kNesThreads = 128;  // instances per CTA (4 groups of 32)
constexpr int kG = 32;            // instances per interleave group

struct NesMem {
  uint8_t* ram;   // this instance's byte 0 of [group][2048][32]
  uint8_t* vram;  // [group][2048][32]
  uint8_t* oam;   // shared: [256][kNesThreads] (column tid)
  uint8_t* pal;   // shared: [32][kNesThreads]
  uint32_t* spr;  // shared: [8][kNesThreads]: x | attr << 8 | pattern << 16
  uint8_t* ntc;   // shared: [40][kNesThreads]: the current tile row's 32 tile indices and 8 attribute bytes
  uint8_t* fbrow; // this instance's tile words of row 0: [group][240][32 tiles][32][8 B] or null
  const uint8_t* prg;
  uint32_t prg_mask;
  const uint8_t* chr;
  const uint32_t* dec;  // shared decode table
};

struct NesCpu {
  uint32_t A, X, Y, SP, P, PC, nmi, irq, pad, pad_shift, pad_strobe;
  uint32_t ctrl, mask, status, oam_addr, v, t, fine_x, w, rbuf, mir;
  int scanline, cycle;
  uint32_t frame_ready, count, s0, dma_far, headless;
  uint32_t spr_tiles;  // tiles of this line that some listed sprite covers (bit per 8-pixel tile)
  uint32_t tile_done;  // the current tile was finished at its first pixel (no sprite over it)
  uint32_t nt_key;     // (nametable select, tile row) held in ntc; ~0 after any VRAM write
  unsigned long long total;
  unsigned long long tbuf;  // background tile being rendered (8 palette values)
};

__device__ __forceinline__ uint32_t nt_index(uint32_t mir, uint32_t addr) {
  addr = (addr - 0x2000u) & 0x0FFFu;
  switch (mir) {
    case 0: return ((addr >> 10) & 2u) ? 0x400u + (addr & 0x3FFu) : (addr & 0x3FFu);
    case 1: return addr & 0x7FFu;
    case 2: return addr & 0x3FFu;
    case 3: return 0x400u | (addr & 0x3FFu);
    default: return addr & 0x7FFu;
  }
}
__device__ __forceinline__ uint32_t pal_index(uint32_t a) {
  a &= 0x1Fu;
  return ((a & 0x13u) == 0x10u) ? (a & 0x0Fu) : a;
}

// ---------------------------------------------------------------- PPU rendering
__device__ __forceinline__ uint32_t chr_byte(const NesMem& m, uint32_t a) { return __ldg(m.chr + a); }

__device__ __forceinline__ void bg_tile(NesCpu& s, const NesMem& m, int tx) {
  const uint32_t p0 = m.pal[0];
  if (!(s.mask & 0x08u)) {
    s.tbuf = 0x0101010101010101ull * p0;
    return;
  }
  const int y = s.scanline, ty = y >> 3, fy = y & 7;
  const uint32_t base = 0x2000u | ((s.ctrl & 3u) << 10);
  // The 8 lines of a tile row read the same 32 tile indices and 8 attribute
  // bytes: read them once, all at once, into shared memory (VRAM only changes
  // through PPUDATA writes, which drop this copy).
  const uint32_t key = ((s.ctrl & 3u) << 8) | (uint32_t)ty;
  if (key != s.nt_key) {
    // a row's tiles (and its attribute bytes) are consecutive bytes of one nametable
    const uint8_t* row = m.vram + nt_index(s.mir, base + ty * 32) * kG;
    const uint8_t* att = m.vram + nt_index(s.mir, base + 0x3C0u + (ty >> 2) * 8) * kG;
#pragma unroll 1
    for (int b = 0; b < 5; ++b) {
      const uint8_t* src = b < 4 ? row + b * 8 * kG : att;
      uint32_t v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = src[i * kG];
#pragma unroll
      for (int i = 0; i < 8; ++i) m.ntc[(b * 8 + i) * kNesThreads] = (uint8_t)v[i];
    }
    s.nt_key = key;
  }
  const uint32_t tile = m.ntc[tx * kNesThreads];
  const uint32_t attr = m.ntc[(32 + (tx >> 2)) * kNesThreads];
  const uint32_t pal = (attr >> ((((ty & 3) >> 1) * 2 + ((tx & 3) >> 1)) * 2)) & 3u;
  const uint32_t pa = ((s.ctrl & 0x10u) ? 0x1000u : 0u) + tile * 16u + fy;
  const uint32_t lo = chr_byte(m, pa), hi = chr_byte(m, pa + 8);
  unsigned long long t = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t px = (((hi >> (7 - i)) & 1u) << 1) | ((lo >> (7 - i)) & 1u);
    const uint32_t col = px ? m.pal[(pal * 4 + px) * kNesThreads] : p0;
    t |= (unsigned long long)col << (8 * i);
  }
  s.tbuf = t;
}
__device__ __forceinline__ void flush_tile(const NesCpu& s, const NesMem& m, int tx) {
  *reinterpret_cast<unsigned long long*>(m.fbrow + ((size_t)s.scanline * 32 + tx) * (kG * 8)) = s.tbuf;
}
__device__ __forceinline__ void sprite_pixel(NesCpu& s, const NesMem& m, int x) {
  for (uint32_t i = 0; i < s.count; ++i) {
    const uint32_t e = m.spr[i * kNesThreads];
    int dx = x - (int)(e & 0xFFu);
    if ((unsigned)dx >= 8u) continue;
    const uint32_t attr = (e >> 8) & 0xFFu, pat = e >> 16;
    if (attr & 0x40u) dx = 7 - dx;
    const uint32_t px = (((pat >> (7 - dx)) & 1u) << 1) | ((pat >> (15 - dx)) & 1u);
    if (!px) continue;
    const uint32_t bgp = (uint32_t)(s.tbuf >> (8 * (x & 7))) & 0xFFu;
    if (i == 0 && s.s0 && x != 255 && (s.mask & 0x08u)) {
      if (s.headless || bgp != m.pal[0]) s.status |= 0x40u;
    }
    if (s.headless) return;
    const uint32_t col = m.pal[pal_index(0x10u + (attr & 3u) * 4 + px) * kNesThreads];
    if ((attr & 0x20u) && bgp != m.pal[0]) continue;
    const int sh = 8 * (x & 7);
    s.tbuf = (s.tbuf & ~(0xFFull << sh)) | ((unsigned long long)col << sh);
    return;
  }
}
// Pixels [xa, xb) of the current visible line.  A tile that no listed sprite
// covers is final once its background is drawn at its first pixel (nothing
// else can change it), so it is stored then and its other pixels are skipped;
// covered tiles take every pixel.  Headless frames only look for sprite 0 hits,
// so they visit only sprite 0's 8 pixels.
__device__ __forceinline__ void render_range(NesCpu& s, const NesMem& m, int xa, int xb) {
  if (s.headless) {
    if (!s.count || !(s.mask & 0x10u)) return;  // (headless lists hold sprite 0 only)
    const int sx = (int)(m.spr[0] & 0xFFu);
    const int lo = max(xa, sx), hi = min(xb, sx + 8);
    for (int x = lo; x < hi; ++x) sprite_pixel(s, m, x);
    return;
  }
  int x = xa;
  while (x < xb) {
    const int tx = x >> 3;
    if ((x & 7) == 0) {
      bg_tile(s, m, tx);
      s.tile_done = !((s.spr_tiles >> tx) & 1u);
      if (s.tile_done) flush_tile(s, m, tx);
    }
    if (s.tile_done) {
      x = (x | 7) + 1;  // next tile
      continue;
    }
    if (s.mask & 0x10u) sprite_pixel(s, m, x);
    if ((x & 7) == 7) flush_tile(s, m, tx);
    ++x;
  }
}
__device__ __forceinline__ void eval_sprites(NesCpu& s, const NesMem& m) {
  s.count = 0;
  s.s0 = 0;
  s.spr_tiles = 0;
  const int n = s.headless ? 1 : 64;
  for (int i = 0; i < n; ++i) {
    const int row = s.scanline - ((int)m.oam[(4 * i) * kNesThreads] + 1);
    if ((unsigned)row >= 8u) continue;
    if (s.count >= 8) {
      s.status |= 0x20u;
      break;
    }
    const uint32_t tile = m.oam[(4 * i + 1) * kNesThreads], attr = m.oam[(4 * i + 2) * kNesThreads];
    const uint32_t x = m.oam[(4 * i + 3) * kNesThreads];
    const uint32_t fy = (attr & 0x80u) ? 7 - row : row;
    const uint32_t a = ((s.ctrl & 0x08u) ? 0x1000u : 0u) + tile * 16u + fy;
    const uint32_t pat = (chr_byte(m, a) << 8) | chr_byte(m, a + 8);
    m.spr[s.count * kNesThreads] = x | (attr << 8) | (pat << 16);
    s.spr_tiles |= (1u << (x >> 3)) | ((x + 7) < 256 ? (1u << ((x + 7) >> 3)) : 0u);
    if (i == 0) s.s0 = 1;
    s.count++;
  }
}
// n PPU dots, as n calls of the reference's dot function with its NMI hand-off.
__device__ __forceinline__ void ppu_advance(NesCpu& s, const NesMem& m, int n) {
  while (n > 0) {
    if (s.scanline < 240) {
      const int span = min(n, 340 - s.cycle);  // dots that stay on this line
      if (span > 0) {
        if (m.fbrow && s.cycle < 256) render_range(s, m, s.cycle, min(s.cycle + span, 256));
        s.cycle += span;
        n -= span;
        if (!n) break;
      }
    } else {
      const int c0 = s.cycle, span = min(n, 340 - c0), c1 = c0 + span;  // dots c0+1 .. c1
      if (s.scanline == 241 && c0 < 1 && c1 >= 1) {
        s.status |= 0x80u;
        if (s.ctrl & 0x80u) s.nmi = 1;
      } else if (s.scanline == 261) {
        if (c0 < 1 && c1 >= 1) s.status &= ~0xE0u;
        if (c0 < 304 && c1 >= 280 && (s.mask & 0x18u)) s.v = (s.v & 0x841Fu) | (s.t & 0x7BE0u);
      }
      s.cycle = c1;
      n -= span;
      if (!n) break;
    }
    // the dot that ends the line
    s.cycle = 0;
    if (++s.scanline > 261) s.scanline = 0;
    if (s.scanline == 261) s.frame_ready = 1;
    if (s.scanline < 240) eval_sprites(s, m);
    --n;
  }
}

// ---------------------------------------------------------------- PPU registers
__device__ __forceinline__ uint32_t ppu_mem_read(const NesCpu& s, const NesMem& m, uint32_t a) {
  a &= 0x3FFFu;
  if (a < 0x2000u) return chr_byte(m, a);
  if (a < 0x3F00u) return m.vram[nt_index(s.mir, a) * kG];
  return m.pal[pal_index(a - 0x3F00u) * kNesThreads];
}
__device__ __forceinline__ void inc_v(NesCpu& s) { s.v = (s.v + ((s.ctrl & 4u) ? 32u : 1u)) & 0x7FFFu; }
__device__ __forceinline__ uint32_t ppu_reg_read(NesCpu& s, const NesMem& m, uint32_t addr) {
  switch (addr & 7u) {
    case 2: {
      const uint32_t r = (s.status & 0xE0u) | (s.rbuf & 0x1Fu);
      s.status &= ~0x80u;
      s.w = 0;
      return r;
    }
    case 4: return m.oam[s.oam_addr * kNesThreads];
    case 7: {
      uint32_t r = ppu_mem_read(s, m, s.v);
      if ((s.v & 0x3F00u) == 0x3F00u) {
        s.rbuf = ppu_mem_read(s, m, s.v & 0x2FFFu);
      } else {
        const uint32_t old = s.rbuf;
        s.rbuf = r;
        r = old;
      }
      inc_v(s);
      return r;
    }
    default: return 0;
  }
}
__device__ __forceinline__ void ppu_reg_write(NesCpu& s, const NesMem& m, uint32_t addr, uint32_t val) {
  switch (addr & 7u) {
    case 0: s.ctrl = val; s.t = (s.t & 0xF3FFu) | ((val & 3u) << 10); break;
    case 1: s.mask = val; break;
    case 3: s.oam_addr = val; break;
    case 4: m.oam[s.oam_addr * kNesThreads] = (uint8_t)val; s.oam_addr = (s.oam_addr + 1) & 0xFFu; break;
    case 5:
      if (!s.w) {
        s.t = (s.t & 0xFFE0u) | (val >> 3);
        s.fine_x = val & 7u;
        s.w = 1;
      } else {
        s.t = (s.t & 0x8FFFu) | ((val & 7u) << 12);
        s.t = (s.t & 0xFC1Fu) | ((val & 0xF8u) << 2);
        s.w = 0;
      }
      break;
    case 6:
      if (!s.w) {
        s.t = (s.t & 0x80FFu) | ((val & 0x3Fu) << 8);
        s.w = 1;
      } else {
        s.t = (s.t & 0xFF00u) | val;
        s.v = s.t;
        s.w = 0;
      }
      break;
    case 7: {
      const uint32_t a = s.v & 0x3FFFu;
      if (a >= 0x2000u) {
        if (a < 0x3F00u) {
          m.vram[nt_index(s.mir, a) * kG] = (uint8_t)val;
          s.nt_key = ~0u;
        }
        else {
          m.pal[pal_index(a - 0x3F00u) * kNesThreads] = (uint8_t)val;
        }
      }
      inc_v(s);
      break;
    }
    default: break;
  }
}

// ---------------------------------------------------------------- CPU bus
__device__ __forceinline__ uint32_t prg_byte(const NesMem& m, uint32_t a) { return __ldg(m.prg + (a & m.prg_mask)); }
__device__ __forceinline__ uint32_t rd(NesCpu& s, const NesMem& m, uint32_t a) {
  if (a < 0x2000u) return m.ram[(a & 0x7FFu) * kG];
  if (a >= 0x8000u) return prg_byte(m, a);
  if (a < 0x4000u) return ppu_reg_read(s, m, a);
  if (a == 0x4016u) {
    if (s.pad_strobe) return s.pad & 1u;
    if (s.pad_shift < 8u) return (s.pad >> s.pad_shift++) & 1u;
    return 1u;
  }
  return 0u;
}
__device__ __forceinline__ void oam_dma(NesCpu& s, const NesMem& m, uint32_t page) {
  if (page >= 8u && s.dma_far < 255u) s.dma_far++;
  for (uint32_t i = 0; i < 256u; ++i) {
    uint32_t b;
    if (page < 0x20u) b = m.ram[(((page & 7u) << 8) | i) * kG];
    else if (page >= 0x80u) b = prg_byte(m, (page << 8) | i);
    else b = 0;
    m.oam[((s.oam_addr + i) & 0xFFu) * kNesThreads] = (uint8_t)b;
  }
  s.total += 513;
}
__device__ __forceinline__ void wr(NesCpu& s, const NesMem& m, uint32_t a, uint32_t v) {
  if (a < 0x2000u) {
    m.ram[(a & 0x7FFu) * kG] = (uint8_t)v;
  } else if (a < 0x4000u) {
    ppu_reg_write(s, m, a, v);
  } else if (a == 0x4014u) {
    oam_dma(s, m, v);
  } else if (a == 0x4016u) {
    if (v & 1u) {
      s.pad_strobe = 1;
    } else if (s.pad_strobe) {
      s.pad_strobe = 0;
      s.pad_shift = 0;
    }
  }
}
__device__ __forceinline__ uint32_t rd16(NesCpu& s, const NesMem& m, uint32_t a) {
  const uint32_t lo = rd(s, m, a);
  return lo | (rd(s, m, (a + 1) & 0xFFFFu) << 8);
}
__device__ __forceinline__ void push(NesCpu& s, const NesMem& m, uint32_t v) {
  m.ram[(0x100u + s.SP) * kG] = (uint8_t)v;  // 0x100 + SP < 0x2000: RAM
  s.SP = (s.SP - 1) & 0xFFu;
}
__device__ __forceinline__ uint32_t pop(NesCpu& s, const NesMem& m) {
  s.SP = (s.SP + 1) & 0xFFu;
  return m.ram[(0x100u + s.SP) * kG];
}

// ---------------------------------------------------------------- CPU
enum : uint32_t { FC = 1, FZ = 2, FI = 4, FD = 8, FB = 16, FU = 32, FV = 64, FN = 128 };
__device__ __forceinline__ void zn(NesCpu& s, uint32_t v) {
  s.P = (s.P & ~(FZ | FN)) | (v ? 0u : FZ) | (v & FN);
}
__device__ __forceinline__ void setc(NesCpu& s, bool c) { s.P = c ? (s.P | FC) : (s.P & ~FC); }
__device__ __forceinline__ void interrupt(NesCpu& s, const NesMem& m, uint32_t vec, uint32_t pushed_p) {
  push(s, m, s.PC >> 8);
  push(s, m, s.PC & 0xFFu);
  push(s, m, pushed_p);
  s.P |= FI;
  s.PC = rd16(s, m, vec);
}

__device__ __forceinline__ int cpu_step(NesCpu& s, const NesMem& m) {
  if (s.nmi) {
    s.nmi = 0;
    interrupt(s, m, 0xFFFAu, (s.P & ~FB) | FU);
    s.total += 7;
    return 7;
  }
  if (s.irq && !(s.P & FI)) {
    s.irq = 0;
    interrupt(s, m, 0xFFFEu, (s.P & ~FB) | FU);
    s.total += 7;
    return 7;
  }
  // In PRG ROM (no read side effects) the two bytes after the opcode are read
  // with it, so the operand fetch does not wait for the decode; the values are
  // the bus reads the instruction makes at PC + 1 and PC + 2.
  const uint32_t pc0 = s.PC;
  const bool fast = pc0 >= 0x8000u && pc0 <= 0xFFFDu;
  uint32_t op, p1 = 0, p2 = 0;
  if (fast) {
    op = prg_byte(m, pc0);
    p1 = prg_byte(m, pc0 + 1);
    p2 = prg_byte(m, pc0 + 2);
  } else {
    op = rd(s, m, pc0);
  }
  s.PC = (pc0 + 1) & 0xFFFFu;
  auto opb = [&]() -> uint32_t { return fast ? p1 : rd(s, m, s.PC); };
  auto opw = [&]() -> uint32_t { return fast ? (p1 | (p2 << 8)) : rd16(s, m, s.PC); };
  const uint32_t d = m.dec[op];
  const uint32_t mode = d & 15u, kind = (d >> 4) & 63u;
  int cyc = (int)((d >> 10) & 15u);
  uint32_t a = 0;
  bool crossed = false;
  switch (mode) {
    case NM_IMM: a = s.PC; s.PC = (s.PC + 1) & 0xFFFFu; break;
    case NM_ZP: a = opb(); s.PC = (s.PC + 1) & 0xFFFFu; break;
    case NM_ZPX: a = (opb() + s.X) & 0xFFu; s.PC = (s.PC + 1) & 0xFFFFu; break;
    case NM_ZPY: a = (opb() + s.Y) & 0xFFu; s.PC = (s.PC + 1) & 0xFFFFu; break;
    case NM_ABS: a = opw(); s.PC = (s.PC + 2) & 0xFFFFu; break;
    case NM_ABX:
    case NM_ABY: {
      const uint32_t b = opw();
      s.PC = (s.PC + 2) & 0xFFFFu;
      a = (b + (mode == NM_ABX ? s.X : s.Y)) & 0xFFFFu;
      crossed = (a ^ b) & 0xFF00u;
      break;
    }
    case NM_IZX: {
      const uint32_t zp = (opb() + s.X) & 0xFFu;
      s.PC = (s.PC + 1) & 0xFFFFu;
      a = rd16(s, m, zp);
      break;
    }
    case NM_IZY: {
      const uint32_t zp = opb();
      s.PC = (s.PC + 1) & 0xFFFFu;
      const uint32_t b = rd16(s, m, zp);
      a = (b + s.Y) & 0xFFFFu;
      crossed = (a ^ b) & 0xFF00u;
      break;
    }
    case NM_REL: a = opb(); s.PC = (s.PC + 1) & 0xFFFFu; break;
    case NM_IND: {
      const uint32_t p = opw();
      s.PC = (s.PC + 2) & 0xFFFFu;
      const uint32_t lo = rd(s, m, p);
      a = lo | (rd(s, m, (p & 0xFF00u) | ((p + 1) & 0xFFu)) << 8);
      break;
    }
    case NM_SK1: s.PC = (s.PC + 1) & 0xFFFFu; break;
    case NM_SK2: s.PC = (s.PC + 2) & 0xFFFFu; break;
    default: break;
  }
  if (crossed && (d & 0x4000u)) ++cyc;
  // data operand of the read kinds: the immediate byte comes from the prefetch
  const bool imm_fast = fast && mode == NM_IMM;
  auto rdv = [&]() -> uint32_t { return imm_fast ? p1 : rd(s, m, a); };
  switch (kind) {
    case NK_LDA: s.A = rdv(); zn(s, s.A); break;
    case NK_LDX: s.X = rdv(); zn(s, s.X); break;
    case NK_LDY: s.Y = rdv(); zn(s, s.Y); break;
    case NK_STA: wr(s, m, a, s.A); break;
    case NK_STX: wr(s, m, a, s.X); break;
    case NK_STY: wr(s, m, a, s.Y); break;
    case NK_ORA: s.A |= rdv(); zn(s, s.A); break;
    case NK_AND: s.A &= rdv(); zn(s, s.A); break;
    case NK_EOR: s.A ^= rdv(); zn(s, s.A); break;
    case NK_ADC:
    case NK_SBC: {
      uint32_t v = rdv();
      // A - v - !C == A + ~v + C (8 bits): one adder for both
      if (kind == NK_SBC) v ^= 0xFFu;
      const uint32_t sum = s.A + v + (s.P & FC);
      const uint32_t r = sum & 0xFFu;
      s.P = (s.P & ~(FC | FV)) | (sum > 0xFFu ? FC : 0u) | ((~(s.A ^ v) & (s.A ^ r) & 0x80u) ? FV : 0u);
      s.A = r;
      zn(s, r);
      break;
    }
    case NK_CMP:
    case NK_CPX:
    case NK_CPY: {
      const uint32_t reg = kind == NK_CMP ? s.A : kind == NK_CPX ? s.X : s.Y;
      const uint32_t v = rdv();
      setc(s, reg >= v);
      zn(s, (reg - v) & 0xFFu);
      break;
    }
    case NK_BIT: {
      const uint32_t v = rd(s, m, a);
      s.P = (s.P & ~(FZ | FV | FN)) | ((s.A & v) ? 0u : FZ) | (v & (FV | FN));
      break;
    }
    case NK_ASL:
    case NK_LSR:
    case NK_ROL:
    case NK_ROR:
    case NK_INC:
    case NK_DEC: {
      const uint32_t v = mode == NM_ACC ? s.A : rd(s, m, a);
      uint32_t r;
      const uint32_t c = s.P & FC;
      switch (kind) {
        case NK_ASL: setc(s, v & 0x80u); r = (v << 1) & 0xFFu; break;
        case NK_ROL: setc(s, v & 0x80u); r = ((v << 1) | c) & 0xFFu; break;
        case NK_LSR: setc(s, v & 1u); r = v >> 1; break;
        case NK_ROR: setc(s, v & 1u); r = (v >> 1) | (c << 7); break;
        case NK_INC: r = (v + 1) & 0xFFu; break;
        default: r = (v - 1) & 0xFFu; break;
      }
      if (mode == NM_ACC) s.A = r;
      else wr(s, m, a, r);
      zn(s, r);
      break;
    }
    case NK_BR: {
      // flag: 0 N, 1 V, 2 C, 3 Z (op bits 7-6); taken when it equals op bit 5
      const uint32_t sel = op >> 6;
      const uint32_t f = sel == 0 ? (s.P >> 7) : sel == 1 ? (s.P >> 6) : sel == 2 ? s.P : (s.P >> 1);
      if ((f & 1u) == ((op >> 5) & 1u)) {
        const uint32_t np = (s.PC + (uint32_t)(int32_t)(int8_t)a) & 0xFFFFu;
        cyc = 3 + (((np ^ s.PC) & 0xFF00u) ? 1 : 0);
        s.PC = np;
      }
      break;
    }
    case NK_JMP: s.PC = a; break;
    case NK_JSR: {
      const uint32_t ret = (s.PC - 1) & 0xFFFFu;
      push(s, m, ret >> 8);
      push(s, m, ret & 0xFFu);
      s.PC = a;
      break;
    }
    case NK_RTS: {
      const uint32_t lo = pop(s, m);
      s.PC = ((lo | (pop(s, m) << 8)) + 1) & 0xFFFFu;
      break;
    }
    case NK_RTI: {
      s.P = (pop(s, m) & ~FB) | FU;
      const uint32_t lo = pop(s, m);
      s.PC = lo | (pop(s, m) << 8);
      break;
    }
    case NK_BRK:
      s.PC = (s.PC + 1) & 0xFFFFu;
      interrupt(s, m, 0xFFFEu, s.P | FB | FU);
      break;
    case NK_PHA: push(s, m, s.A); break;
    case NK_PHP: push(s, m, s.P | FB | FU); break;
    case NK_PLA: s.A = pop(s, m); zn(s, s.A); break;
    case NK_PLP: s.P = (pop(s, m) & ~FB) | FU; break;
    case NK_TAX: s.X = s.A; zn(s, s.X); break;
    case NK_TAY: s.Y = s.A; zn(s, s.Y); break;
    case NK_TXA: s.A = s.X; zn(s, s.A); break;
    case NK_TYA: s.A = s.Y; zn(s, s.A); break;
    case NK_TSX: s.X = s.SP; zn(s, s.X); break;
    case NK_TXS: s.SP = s.X; break;
    case NK_INX: s.X = (s.X + 1) & 0xFFu; zn(s, s.X); break;
    case NK_INY: s.Y = (s.Y + 1) & 0xFFu; zn(s, s.Y); break;
    case NK_DEX: s.X = (s.X - 1) & 0xFFu; zn(s, s.X); break;
    case NK_DEY: s.Y = (s.Y - 1) & 0xFFu; zn(s, s.Y); break;
    case NK_CLC: s.P &= ~FC; break;
    case NK_SEC: s.P |= FC; break;
    case NK_CLI: s.P &= ~FI; break;
    case NK_SEI: s.P |= FI; break;
    case NK_CLV: s.P &= ~FV; break;
    case NK_CLD: s.P &= ~FD; break;
    case NK_SED: s.P |= FD; break;
    default: break;  // NOPs and unknown opcodes (1 cycle, 1 byte)
  }
  s.total += (unsigned long long)cyc;
  return cyc;
}

// ---------------------------------------------------------------- state I/O
// Packed registers, 48 bytes per instance (see include/dt_attn.h).
__device__ __forceinline__ void load_regs(NesCpu& s, const uint8_t* regs) {
  const uint4 a = reinterpret_cast<const uint4*>(regs)[0];
  const uint4 b = reinterpret_cast<const uint4*>(regs)[1];
  const uint4 c = reinterpret_cast<const uint4*>(regs)[2];
  s.A = a.x & 0xFFu; s.X = (a.x >> 8) & 0xFFu; s.Y = (a.x >> 16) & 0xFFu; s.SP = a.x >> 24;
  s.PC = a.y & 0xFFFFu; s.P = (a.y >> 16) & 0xFFu; s.nmi = a.y >> 24;
  s.irq = a.z & 0xFFu; s.pad = (a.z >> 8) & 0xFFu; s.pad_shift = (a.z >> 16) & 0xFFu; s.pad_strobe = a.z >> 24;
  s.ctrl = a.w & 0xFFu; s.mask = (a.w >> 8) & 0xFFu; s.status = (a.w >> 16) & 0xFFu; s.oam_addr = a.w >> 24;
  s.v = b.x & 0xFFFFu; s.t = b.x >> 16;
  s.fine_x = b.y & 0xFFu; s.w = (b.y >> 8) & 0xFFu; s.rbuf = (b.y >> 16) & 0xFFu; s.mir = b.y >> 24;
  s.scanline = (int)(b.z & 0xFFFFu); s.cycle = (int)(b.z >> 16);
  s.frame_ready = b.w & 0xFFu; s.count = (b.w >> 16) & 0xFFu; s.dma_far = b.w >> 24;
  s.total = (unsigned long long)c.x | ((unsigned long long)c.y << 32);
  s.s0 = c.z & 1u;
  s.headless = 0;
  s.tbuf = 0;
  s.spr_tiles = 0;
  s.tile_done = 0;
  s.nt_key = ~0u;
}
__device__ __forceinline__ void store_regs(const NesCpu& s, uint8_t* regs) {
  uint4 a, b, c;
  a.x = s.A | (s.X << 8) | (s.Y << 16) | (s.SP << 24);
  a.y = s.PC | (s.P << 16) | (s.nmi << 24);
  a.z = s.irq | (s.pad << 8) | (s.pad_shift << 16) | (s.pad_strobe << 24);
  a.w = s.ctrl | (s.mask << 8) | (s.status << 16) | (s.oam_addr << 24);
  b.x = s.v | (s.t << 16);
  b.y = s.fine_x | (s.w << 8) | (s.rbuf << 16) | (s.mir << 24);
  b.z = (uint32_t)s.scanline | ((uint32_t)s.cycle << 16);
  b.w = s.frame_ready | (s.count << 16) | (s.dma_far << 24);  // byte 1: nmi_flag, always 0 between dots
  c.x = (uint32_t)s.total;
  c.y = (uint32_t)(s.total >> 32);
  c.z = s.s0;
  c.w = 0;
  reinterpret_cast<uint4*>(regs)[0] = a;
  reinterpret_cast<uint4*>(regs)[1] = b;
  reinterpret_cast<uint4*>(regs)[2] = c;
}

struct NesArgs {
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
};

__device__ __forceinline__ size_t grp_off(int i, int bytes) {
  return (size_t)(i >> 5) * (size_t)bytes * kG + (size_t)(i & 31);
}

__global__ void __launch_bounds__(kNesThreads) nes_frames_kernel(NesArgs g, int num_frames) {
  __shared__ uint32_t dec_s[256];
  __shared__ uint8_t oam_s[256 * kNesThreads];
  __shared__ uint8_t pal_s[32 * kNesThreads];
  __shared__ uint32_t spr_s[8 * kNesThreads];
  __shared__ uint8_t ntc_s[40 * kNesThreads];
  const int tid = threadIdx.x;
  for (int i = tid; i < 256; i += kNesThreads) dec_s[i] = kNesDecode[i];
  const int inst = blockIdx.x * kNesThreads + tid;
  const bool live = inst < g.n;
  NesMem m;
  m.oam = oam_s + tid;
  m.pal = pal_s + tid;
  m.spr = spr_s + tid;
  m.ntc = ntc_s + tid;
  m.dec = dec_s;
  m.prg = g.prg;
  m.prg_mask = g.prg_size - 1;
  m.chr = g.chr;
  NesCpu s;
  if (live) {
    m.ram = g.ram + grp_off(inst, 2048);
    m.vram = g.vram + grp_off(inst, 2048);
    m.fbrow = g.fb ? g.fb + (size_t)(inst >> 5) * (240 * 32 * kG * 8) + (size_t)(inst & 31) * 8 : nullptr;
    const uint8_t* go = g.oam + grp_off(inst, 256);
    for (int i = 0; i < 256; ++i) m.oam[i * kNesThreads] = go[i * kG];
    const uint8_t* gp = g.pal + grp_off(inst, 32);
    for (int i = 0; i < 32; ++i) m.pal[i * kNesThreads] = gp[i * kG];
    load_regs(s, g.regs + (size_t)inst * 48);
  }
  __syncthreads();
  if (!live) return;
  for (int f = 0; f < num_frames; ++f) {
    s.headless = f < num_frames - 1;
    s.frame_ready = 0;
    int total = 0;
    while (!s.frame_ready && total < 65000) {
      const int c = cpu_step(s, m);
      total += c;
      ppu_advance(s, m, 3 * c);
    }
  }
  s.headless = 0;
  store_regs(s, g.regs + (size_t)inst * 48);
  uint8_t* go = g.oam + grp_off(inst, 256);
  for (int i = 0; i < 256; ++i) go[i * kG] = m.oam[i * kNesThreads];
  uint8_t* gp = g.pal + grp_off(inst, 32);
  for (int i = 0; i < 32; ++i) gp[i * kG] = m.pal[i * kNesThreads];
}

// Power-on reset of the selected instances (all when mask is null).
__device__ void reset_instance(const NesArgs& g, int inst, int mirroring) {
  uint8_t* ram = g.ram + grp_off(inst, 2048);
  uint8_t* vram = g.vram + grp_off(inst, 2048);
  for (int i = 0; i < 2048; ++i) ram[i * kG] = 0, vram[i * kG] = 0;
  uint8_t* oam = g.oam + grp_off(inst, 256);
  for (int i = 0; i < 256; ++i) oam[i * kG] = 0;
  uint8_t* pal = g.pal + grp_off(inst, 32);
  for (int i = 0; i < 32; ++i) pal[i * kG] = 0;
  uint8_t* regs = g.regs + (size_t)inst * 48;
  const uint32_t mir = mirroring >= 0 ? (uint32_t)mirroring : regs[23];
  NesCpu s = {};
  s.SP = 0xFD;
  s.P = FU | FI;
  s.mir = mir;
  const uint32_t mask = g.prg_size - 1;
  s.PC = __ldg(g.prg + (0xFFFCu & mask)) | (__ldg(g.prg + (0xFFFDu & mask)) << 8);
  store_regs(s, regs);
}
__global__ void nes_reset_kernel(NesArgs g, const uint8_t* mask, int mirroring) {
  const int inst = blockIdx.x * blockDim.x + threadIdx.x;
  if (inst >= g.n || (mask && !mask[inst])) return;
  reset_instance(g, inst, mirroring);
}

// Controller bytes of every instance (and a fresh serial latch), as the
// reference's set_buttons_batch.  actions != null: SIMPLE_MOVEMENT indices with
// the boot sequence's override (START, then no button) where boot > 0.
__constant__ uint8_t kSimpleMovement[7] = {0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40};
__global__ void nes_buttons_kernel(uint8_t* regs, int n, const uint8_t* buttons, const int64_t* actions,
                                   const int32_t* boot, int boot_settle, int* status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t b;
  if (actions) {
    const int64_t act = actions[i];
    if (act < 0 || act > 6) {
      atomicExch(status, 3);  // invalid action index
      b = 0;
    } else {
      b = kSimpleMovement[act];
    }
    const int bt = boot ? boot[i] : 0;
    if (bt > boot_settle) b = 0x08;
    else if (bt > 0) b = 0;
  } else {
    b = buttons[i];
  }
  uint8_t* r = regs + (size_t)i * 48;
  r[9] = (uint8_t)b;
  r[10] = 0;
  r[11] = 0;
}

// Framebuffer -> 84 x 84 observation (palette -> luma, bilinear), the
// reference's arithmetic in its order with one rounding per operation; the new
// frame also goes into the stack buffer [n][stack][84][84] (oldest first,
// shifted by one).
__constant__ uint32_t kNesRgb[64] = {
    0x666666u, 0x002A88u, 0x1412A7u, 0x3B00A4u, 0x5C007Eu, 0x6E0040u, 0x6C0600u, 0x561D00u,
    0x333500u, 0x0B4800u, 0x005200u, 0x004F08u, 0x00404Du, 0x000000u, 0x000000u, 0x000000u,
    0xADADADu, 0x155FD9u, 0x4240FFu, 0x7527FEu, 0xA01ACCu, 0xB71E7Bu, 0xB53120u, 0x994E00u,
    0x6B6D00u, 0x388700u, 0x0C9300u, 0x008F32u, 0x007C8Du, 0x000000u, 0x000000u, 0x000000u,
    0xFFFEFFu, 0x64B0FFu, 0x9290FFu, 0xC676FFu, 0xF36AFFu, 0xFE6ECCu, 0xFE8170u, 0xEA9E22u,
    0xBCBE00u, 0x88D800u, 0x5CE430u, 0x45E082u, 0x48CDDEu, 0x4F4F4Fu, 0x000000u, 0x000000u,
    0xFFFEFFu, 0xC0DFFFu, 0xD3D2FFu, 0xE8C8FFu, 0xFBC2FFu, 0xFEC4EAu, 0xFECCC5u, 0xF7D8A5u,
    0xE4E594u, 0xCFEF96u, 0xBDF4ABu, 0xB3F3CCu, 0xB5EBF2u, 0xB8B8B8u, 0x000000u, 0x000000u,
};
__global__ void __launch_bounds__(128) nes_observe_kernel(const uint8_t* fb, int n, uint8_t* obs,
                                                          uint8_t* stacked, int stack) {
  __shared__ float gray_s[256];
  __shared__ int x0_s[84], x1_s[84];
  __shared__ float wx_s[84];
  const int tid = threadIdx.x;
  for (int i = tid; i < 256; i += blockDim.x) {
    const uint32_t c = kNesRgb[i & 63];
    const float r = (float)((c >> 16) & 0xFFu), gg = (float)((c >> 8) & 0xFFu), b = (float)(c & 0xFFu);
    gray_s[i] = __fadd_rn(__fadd_rn(__fmul_rn(0.299f, r), __fmul_rn(0.587f, gg)), __fmul_rn(0.114f, b));
  }
  for (int ox = tid; ox < 84; ox += blockDim.x) {
    const float fx = __fsub_rn(__fmul_rn(__fadd_rn((float)ox, 0.5f), 256.0f / 84.0f), 0.5f);
    const int x0 = fx < 0.0f ? 0 : (int)fx;
    x0_s[ox] = x0;
    x1_s[ox] = x0 + 1 < 256 ? x0 + 1 : 255;
    const float wx = __fsub_rn(fx, (float)x0);
    wx_s[ox] = wx < 0.0f ? 0.0f : wx;
  }
  __syncthreads();
  // thread = (instance, output row): a warp covers 32 instances of one group
  const long long item = (long long)blockIdx.x * blockDim.x + tid;
  const int inst = (int)(((item / (32 * 84)) * 32) + (item % 32));
  const int oy = (int)((item / 32) % 84);
  if (inst >= n) return;
  const float fy = __fsub_rn(__fmul_rn(__fadd_rn((float)oy, 0.5f), 240.0f / 84.0f), 0.5f);
  const int y0 = fy < 0.0f ? 0 : (int)fy, y1 = y0 + 1 < 240 ? y0 + 1 : 239;
  float wy = __fsub_rn(fy, (float)y0);
  if (wy < 0.0f) wy = 0.0f;
  const uint8_t* base = fb + (size_t)(inst >> 5) * (240 * 32 * kG * 8) + (size_t)(inst & 31) * 8;
  auto px = [&](int y, int x) -> float {
    return gray_s[base[((size_t)y * 32 + (x >> 3)) * (kG * 8) + (x & 7)]];
  };
  uint8_t* o = obs ? obs + (size_t)inst * 7056 + oy * 84 : nullptr;
  uint8_t* st = stacked ? stacked + ((size_t)inst * stack + (stack - 1)) * 7056 + oy * 84 : nullptr;
  if (st) {
    // shift this row of the older frames down by one
    for (int j = 0; j + 1 < stack; ++j) {
      const uint8_t* src = stacked + ((size_t)inst * stack + j + 1) * 7056 + oy * 84;
      uint8_t* dst = stacked + ((size_t)inst * stack + j) * 7056 + oy * 84;
      for (int q = 0; q < 21; ++q) reinterpret_cast<uint32_t*>(dst)[q] = reinterpret_cast<const uint32_t*>(src)[q];
    }
  }
  const float a0 = __fsub_rn(1.0f, wy);
  for (int q = 0; q < 21; ++q) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int ox = q * 4 + e;
      const int x0 = x0_s[ox], x1 = x1_s[ox];
      const float wx = wx_s[ox], b0 = __fsub_rn(1.0f, wx);
      float g = __fmul_rn(__fmul_rn(a0, b0), px(y0, x0));
      g = __fadd_rn(g, __fmul_rn(__fmul_rn(a0, wx), px(y0, x1)));
      g = __fadd_rn(g, __fmul_rn(__fmul_rn(wy, b0), px(y1, x0)));
      g = __fadd_rn(g, __fmul_rn(__fmul_rn(wy, wx), px(y1, x1)));
      word |= (uint32_t)(uint8_t)(int)__fadd_rn(g, 0.5f) << (8 * e);
    }
    if (o) reinterpret_cast<uint32_t*>(o)[q] = word;
    if (st) reinterpret_cast<uint32_t*>(st)[q] = word;
  }
}

// The environment's bookkeeping after a step (the reference's GpuMarioVecEnv.step
// after run_frames_all and the observation): x position, lives and the
// stage-clear flag from RAM, boot counters, rewards, done flags, and the reset of
// the instances that are done (they re-enter the boot sequence).
__global__ void nes_env_post_kernel(NesArgs g, int frame_skip, int boot_total, int32_t* boot, int32_t* prev_x,
                                    int32_t* init_lives, float* reward, uint8_t* done, int32_t* x_pos,
                                    int32_t* lives_out, uint8_t* flag) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= g.n) return;
  const uint8_t* ram = g.ram + grp_off(i, 2048);
  const int x = (int)ram[0x006D * kG] * 256 + (int)ram[0x0086 * kG];
  const int lives = ram[0x075A * kG];
  bool clear = ram[0x07D7 * kG] == 0x80;
  const int pb = boot[i];
  int b = pb > 0 ? max(0, pb - frame_skip) : pb;
  int il = init_lives[i], px = prev_x[i];
  if (pb > 0 && b <= 0) {
    il = lives;
    px = x;
  }
  const bool booting = b > 0;
  const bool died = lives < il && !booting;
  clear = clear && !booting;
  const bool d = died || clear;
  float r = booting ? 0.0f : __fdiv_rn((float)(x - px), 40.0f);
  r = fminf(fmaxf(r, -1.0f), 1.0f);
  if (died) r = -1.0f;
  if (clear) r = 1.0f;
  reward[i] = r;
  done[i] = d;
  x_pos[i] = x;
  lives_out[i] = lives;
  flag[i] = clear;
  if (d) {
    reset_instance(g, i, -1);
    b = boot_total;
    px = 0;
  } else if (!booting) {
    px = x;
  }
  boot[i] = b;
  prev_x[i] = px;
  init_lives[i] = il;
}

}  // namespace

cudaError_t launch_nes(int op, const NesLaunch& L, cudaStream_t st) {
  NesArgs g;
  g.regs = L.regs; g.ram = L.ram; g.vram = L.vram; g.oam = L.oam; g.pal = L.pal; g.fb = L.fb;
  g.prg = L.prg; g.prg_size = L.prg_size; g.chr = L.chr; g.n = L.n;
  const int blocks = (L.n + kNesThreads - 1) / kNesThreads;
  switch (op) {
    case 0: nes_frames_kernel<<<blocks, kNesThreads, 0, st>>>(g, L.num_frames); break;
    case 1: nes_reset_kernel<<<blocks, kNesThreads, 0, st>>>(g, L.mask, L.mirroring); break;
    case 2:
      nes_buttons_kernel<<<blocks, kNesThreads, 0, st>>>(L.regs, L.n, L.buttons, L.actions, L.boot,
                                                          L.boot_settle, L.status);
      break;
    case 3: {
      const long long items = (long long)((L.n + 31) / 32) * 32 * 84;
      nes_observe_kernel<<<(unsigned)((items + 127) / 128), 128, 0, st>>>(L.fb, L.n, L.obs, L.stacked, L.stack);
      break;
    }
    case 4:
      nes_env_post_kernel<<<blocks, kNesThreads, 0, st>>>(g, L.frame_skip, L.boot_total, L.boot, L.prev_x,
                                                           L.init_lives, L.reward, L.done, L.x_pos, L.lives,
                                                           L.flag);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace dtk
