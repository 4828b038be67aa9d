/*
 * ORACLE (test infrastructure only): a plain-C CPU restatement of the
 * reference's batched NES emulator, used as the checker for the CUDA
 * environment-step kernels (rl_for_mario_b200/csrc/nes_sm100.cu).  Nothing in
 * the product path loads this file.
 *
 * It follows the reference's CUDA emulator function by function, one PPU dot
 * at a time, exactly as the reference ticks it:
 *   - frame loop:       nes_emulator_gpu/src/cuda/kernels/nes_batch_kernel.cu:46-80 (one frame),
 *                       :116-160 (k frames, all but the last "headless")
 *   - reset:            nes_batch_kernel.cu:86-110, cpu_device.cuh (cpu_reset), ppu_device.cuh (ppu_reset)
 *   - CPU bus:          nes_emulator_gpu/src/cuda/device/cpu_device.cuh (cpu_read / cpu_write)
 *   - CPU instructions: cpu_device.cuh (cpu_step): the official opcodes with the
 *                       reference's cycle counts, its unofficial NOPs, and 1 cycle
 *                       for every other opcode; indirect pointers are fetched as
 *                       two bus reads at zp and zp + 1 (no zero-page wrap)
 *   - PPU:              nes_emulator_gpu/src/cuda/device/ppu_device.cuh (registers,
 *                       ppu_tick, tile background, per-pixel sprites, sprite 0 hit)
 *   - observation:      nes_batch_kernel.cu:180-216 (palette -> luma, bilinear 256x240 -> 84x84)
 *
 * Two behaviours are defined here where the reference's are not:
 *   - OAM DMA from a page >= 8: the reference copies from raw memory past the
 *     instance's 2 KB RAM (other instances' RAM or past the allocation).  Here
 *     pages 0x00-0x1F read the RAM mirror, pages 0x80-0xFF read PRG ROM and the
 *     rest read 0; dma_far counts such copies so tests can leave them out of
 *     comparisons with the reference.
 *   - reset leaves the controller latch at 0 (the reference stores
 *     uninitialised values there until the next set_buttons_batch).
 * Floating point: built with -ffp-contract=off; the observation uses the
 * reference's operation order, one rounding per operation.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  uint8_t x, y, tile, attr, oam_index;
  uint16_t pattern; /* lo plane in the high byte, hi plane in the low byte */
} OSprite;

typedef struct {
  /* CPU */
  uint8_t A, X, Y, SP, P, nmi_pending, irq_pending, joypad1, joypad_shift, joypad_strobe;
  uint16_t PC;
  uint64_t total_cycles;
  /* PPU */
  uint8_t ctrl, mask, status, oam_addr, fine_x, w, read_buffer, mirroring, frame_ready, nmi_flag, headless;
  uint16_t v, t;
  int scanline, cycle, active_count;
  OSprite spr[8];
  uint8_t ram[2048], vram[2048], oam[256], palette[32];
  uint32_t dma_far;
} NesO;

typedef struct {
  const uint8_t* prg;
  uint32_t prg_size;
  const uint8_t* chr;
  int render; /* framebuffer present */
} Cart;

static const uint32_t kPal[64] = {
    0xFF666666u, 0xFF002A88u, 0xFF1412A7u, 0xFF3B00A4u, 0xFF5C007Eu, 0xFF6E0040u, 0xFF6C0600u, 0xFF561D00u,
    0xFF333500u, 0xFF0B4800u, 0xFF005200u, 0xFF004F08u, 0xFF00404Du, 0xFF000000u, 0xFF000000u, 0xFF000000u,
    0xFFADADADu, 0xFF155FD9u, 0xFF4240FFu, 0xFF7527FEu, 0xFFA01ACCu, 0xFFB71E7Bu, 0xFFB53120u, 0xFF994E00u,
    0xFF6B6D00u, 0xFF388700u, 0xFF0C9300u, 0xFF008F32u, 0xFF007C8Du, 0xFF000000u, 0xFF000000u, 0xFF000000u,
    0xFFFFFEFFu, 0xFF64B0FFu, 0xFF9290FFu, 0xFFC676FFu, 0xFFF36AFFu, 0xFFFE6ECCu, 0xFFFE8170u, 0xFFEA9E22u,
    0xFFBCBE00u, 0xFF88D800u, 0xFF5CE430u, 0xFF45E082u, 0xFF48CDDEu, 0xFF4F4F4Fu, 0xFF000000u, 0xFF000000u,
    0xFFFFFEFFu, 0xFFC0DFFFu, 0xFFD3D2FFu, 0xFFE8C8FFu, 0xFFFBC2FFu, 0xFFFEC4EAu, 0xFFFECCC5u, 0xFFF7D8A5u,
    0xFFE4E594u, 0xFFCFEF96u, 0xFFBDF4ABu, 0xFFB3F3CCu, 0xFFB5EBF2u, 0xFFB8B8B8u, 0xFF000000u, 0xFF000000u,
};

/* The reference's 256-entry palette table repeats these 64 colours four times. */
uint32_t nes_o_palette_rgba(int idx) { return kPal[idx & 63]; }

/* ------------------------------------------------------------------ PPU memory */
static uint16_t nt_index(const NesO* s, uint16_t addr) {
  addr = (uint16_t)((addr - 0x2000u) & 0x0FFFu);
  switch (s->mirroring) {
    case 0: return (uint16_t)(((addr / 0x400u) & 2u) ? 0x400u + (addr & 0x3FFu) : (addr & 0x3FFu));
    case 1: return (uint16_t)(addr & 0x7FFu);
    case 2: return (uint16_t)(addr & 0x3FFu);
    case 3: return (uint16_t)(0x400u | (addr & 0x3FFu));
    default: return (uint16_t)(addr & 0x7FFu);
  }
}
static uint8_t pal_index(uint16_t a) {
  uint8_t p = (uint8_t)(a & 0x1Fu);
  if ((p & 0x13u) == 0x10u) p &= 0x0Fu;
  return p;
}
static uint8_t ppu_read(NesO* s, const Cart* c, uint16_t addr) {
  addr &= 0x3FFFu;
  if (addr < 0x2000u) return c->chr[addr];
  if (addr < 0x3F00u) return s->vram[nt_index(s, addr)];
  return s->palette[pal_index((uint16_t)(addr - 0x3F00u))];
}
static void ppu_write(NesO* s, uint16_t addr, uint8_t v) {
  addr &= 0x3FFFu;
  if (addr < 0x2000u) return;
  if (addr < 0x3F00u) s->vram[nt_index(s, addr)] = v;
  else s->palette[pal_index((uint16_t)(addr - 0x3F00u))] = v;
}
static void inc_v(NesO* s) { s->v = (uint16_t)((s->v + ((s->ctrl & 4u) ? 32u : 1u)) & 0x7FFFu); }

static uint8_t ppu_reg_read(NesO* s, const Cart* c, uint16_t addr) {
  switch (addr & 7u) {
    case 2: {
      uint8_t r = (uint8_t)((s->status & 0xE0u) | (s->read_buffer & 0x1Fu));
      s->status &= (uint8_t)~0x80u;
      s->w = 0;
      return r;
    }
    case 4: return s->oam[s->oam_addr];
    case 7: {
      uint8_t r = ppu_read(s, c, s->v);
      if ((s->v & 0x3F00u) == 0x3F00u) {
        s->read_buffer = ppu_read(s, c, (uint16_t)(s->v & 0x2FFFu));
      } else {
        uint8_t old = s->read_buffer;
        s->read_buffer = r;
        r = old;
      }
      inc_v(s);
      return r;
    }
    default: return 0;
  }
}
static void ppu_reg_write(NesO* s, uint16_t addr, uint8_t val) {
  switch (addr & 7u) {
    case 0:
      s->ctrl = val;
      s->t = (uint16_t)((s->t & 0xF3FFu) | ((val & 3u) << 10));
      break;
    case 1: s->mask = val; break;
    case 3: s->oam_addr = val; break;
    case 4: s->oam[s->oam_addr++] = val; break;
    case 5:
      if (!s->w) {
        s->t = (uint16_t)((s->t & 0xFFE0u) | (val >> 3));
        s->fine_x = val & 7u;
        s->w = 1;
      } else {
        s->t = (uint16_t)((s->t & 0x8FFFu) | ((val & 7u) << 12));
        s->t = (uint16_t)((s->t & 0xFC1Fu) | ((val & 0xF8u) << 2));
        s->w = 0;
      }
      break;
    case 6:
      if (!s->w) {
        s->t = (uint16_t)((s->t & 0x80FFu) | ((val & 0x3Fu) << 8));
        s->w = 1;
      } else {
        s->t = (uint16_t)((s->t & 0xFF00u) | val);
        s->v = s->t;
        s->w = 0;
      }
      break;
    case 7:
      ppu_write(s, s->v, val);
      inc_v(s);
      break;
    default: break;
  }
}

/* ------------------------------------------------------------------ rendering */
static void bg_tile(NesO* s, const Cart* c, uint8_t* fb, int tx, int y) {
  uint8_t* row = fb + y * 256 + tx * 8;
  if (!(s->mask & 0x08u)) {
    for (int i = 0; i < 8; ++i) row[i] = s->palette[0];
    return;
  }
  const uint16_t base = (uint16_t)(0x2000u | ((s->ctrl & 3u) << 10));
  const int ty = y / 8, fy = y % 8;
  const uint8_t tile = s->vram[nt_index(s, (uint16_t)(base + ty * 32 + tx))];
  const uint8_t attr = s->vram[nt_index(s, (uint16_t)(base + 0x3C0u + (ty / 4) * 8 + tx / 4))];
  const int shift = (((ty % 4) / 2) * 2 + ((tx % 4) / 2)) * 2;
  const uint8_t pal = (uint8_t)((attr >> shift) & 3u);
  const uint16_t pa = (uint16_t)(((s->ctrl & 0x10u) ? 0x1000u : 0u) + tile * 16);
  const uint8_t lo = c->chr[pa + fy], hi = c->chr[pa + fy + 8];
  for (int i = 0; i < 8; ++i) {
    const int b = 7 - i;
    const uint8_t px = (uint8_t)((((hi >> b) & 1u) << 1) | ((lo >> b) & 1u));
    row[i] = px == 0 ? s->palette[0] : s->palette[pal * 4 + px];
  }
}
static uint16_t spr_pattern(const NesO* s, const Cart* c, uint8_t tile, int fy, int vflip) {
  if (vflip) fy = 7 - fy;
  const uint16_t a = (uint16_t)(((s->ctrl & 0x08u) ? 0x1000u : 0u) + tile * 16 + fy);
  return (uint16_t)((c->chr[a] << 8) | c->chr[a + 8]);
}
static void take_sprite(NesO* s, const Cart* c, int i, int row) {
  OSprite* p = &s->spr[s->active_count++];
  p->x = s->oam[i * 4 + 3];
  p->y = s->oam[i * 4];
  p->tile = s->oam[i * 4 + 1];
  p->attr = s->oam[i * 4 + 2];
  p->oam_index = (uint8_t)i;
  p->pattern = spr_pattern(s, c, p->tile, row, (p->attr & 0x80u) != 0);
}
static void eval_sprites(NesO* s, const Cart* c) {
  s->active_count = 0;
  if (s->headless) {
    const int row = s->scanline - ((int)s->oam[0] + 1);
    if (row >= 0 && row < 8) take_sprite(s, c, 0, row);
    return;
  }
  for (int i = 0; i < 64; ++i) {
    const int row = s->scanline - ((int)s->oam[i * 4] + 1);
    if (row >= 0 && row < 8) {
      if (s->active_count < 8) {
        take_sprite(s, c, i, row);
      } else {
        s->status |= 0x20u;
        break;
      }
    }
  }
}
static void sprite_pixel(NesO* s, uint8_t* fb, int x, int y) {
  if (!(s->mask & 0x10u)) return;
  for (int i = 0; i < s->active_count; ++i) {
    const OSprite* p = &s->spr[i];
    int dx = x - (int)p->x;
    if (dx < 0 || dx >= 8) continue;
    if (p->attr & 0x40u) dx = 7 - dx;
    const uint8_t px = (uint8_t)((((p->pattern >> (7 - dx)) & 1u) << 1) | ((p->pattern >> (15 - dx)) & 1u));
    if (px == 0) continue;
    if (p->oam_index == 0 && x != 255 && (s->mask & 0x08u)) {
      if (s->headless || fb[y * 256 + x] != s->palette[0]) s->status |= 0x40u;
    }
    if (s->headless) return;
    const uint8_t col = s->palette[pal_index((uint16_t)(0x10u + (p->attr & 3u) * 4 + px))];
    if ((p->attr & 0x20u) && fb[y * 256 + x] != s->palette[0]) continue;
    fb[y * 256 + x] = col;
    return;
  }
}
static void ppu_tick(NesO* s, const Cart* c, uint8_t* fb) {
  if (++s->cycle > 340) {
    s->cycle = 0;
    if (++s->scanline > 261) s->scanline = 0;
    if (s->scanline == 261) s->frame_ready = 1;
  }
  if (s->scanline < 240) {
    if (s->cycle == 0) {
      eval_sprites(s, c);
      return;
    }
    if (s->cycle <= 256 && fb) {
      const int x = s->cycle - 1;
      if (!s->headless && (x & 7) == 0) bg_tile(s, c, fb, x >> 3, s->scanline);
      sprite_pixel(s, fb, x, s->scanline);
    }
    return;
  }
  if (s->scanline == 241 && s->cycle == 1) {
    s->status |= 0x80u;
    if (s->ctrl & 0x80u) s->nmi_flag = 1;
    return;
  }
  if (s->scanline == 261) {
    if (s->cycle == 1) {
      s->status &= (uint8_t)~0xE0u;
      s->nmi_flag = 0;
    } else if (s->cycle >= 280 && s->cycle <= 304 && (s->mask & 0x18u)) {
      s->v = (uint16_t)((s->v & 0x841Fu) | (s->t & 0x7BE0u));
    }
  }
}

/* ------------------------------------------------------------------ CPU bus */
static uint8_t prg_byte(const Cart* c, uint16_t addr) {
  return c->prg_size == 0x4000u ? c->prg[(addr - 0x8000u) & 0x3FFFu] : c->prg[addr - 0x8000u];
}
static uint8_t rd(NesO* s, const Cart* c, uint16_t addr) {
  if (addr < 0x2000u) return s->ram[addr & 0x7FFu];
  if (addr < 0x4000u) return ppu_reg_read(s, c, addr);
  if (addr == 0x4016u) {
    if (s->joypad_strobe) return s->joypad1 & 1u;
    if (s->joypad_shift < 8u) return (uint8_t)((s->joypad1 >> s->joypad_shift++) & 1u);
    return 1;
  }
  if (addr >= 0x8000u) return prg_byte(c, addr);
  return 0;
}
static void wr(NesO* s, const Cart* c, uint16_t addr, uint8_t v) {
  if (addr < 0x2000u) {
    s->ram[addr & 0x7FFu] = v;
  } else if (addr < 0x4000u) {
    ppu_reg_write(s, addr, v);
  } else if (addr == 0x4014u) {
    if (v >= 8u) s->dma_far++;
    for (int i = 0; i < 256; ++i) {
      uint8_t b;
      if (v < 0x20u) b = s->ram[((v & 7u) << 8) | (unsigned)i];
      else if (v >= 0x80u) b = prg_byte(c, (uint16_t)((v << 8) | i));
      else b = 0;
      s->oam[(s->oam_addr + i) & 0xFF] = b;
    }
    s->total_cycles += 513;
  } else if (addr == 0x4016u) {
    if (v & 1u) {
      s->joypad_strobe = 1;
    } else if (s->joypad_strobe) {
      s->joypad_strobe = 0;
      s->joypad_shift = 0;
    }
  }
}
static uint16_t rd16(NesO* s, const Cart* c, uint16_t a) {
  const uint8_t lo = rd(s, c, a);
  const uint8_t hi = rd(s, c, (uint16_t)(a + 1));
  return (uint16_t)((hi << 8) | lo);
}
static void push(NesO* s, const Cart* c, uint8_t v) { wr(s, c, (uint16_t)(0x100u + s->SP--), v); }
static uint8_t pop(NesO* s, const Cart* c) { return rd(s, c, (uint16_t)(0x100u + ++s->SP)); }

/* ------------------------------------------------------------------ CPU */
enum { FC = 1, FZ = 2, FI = 4, FD = 8, FB = 16, FU = 32, FV = 64, FN = 128 };
static void setf(NesO* s, uint8_t f, int on) { s->P = on ? (uint8_t)(s->P | f) : (uint8_t)(s->P & ~f); }
static void zn(NesO* s, uint8_t v) {
  setf(s, FZ, v == 0);
  setf(s, FN, (v & 0x80u) != 0);
}
static int cross(uint16_t a, uint16_t b) { return (a & 0xFF00u) != (b & 0xFF00u); }

/* Operand address of the read-type addressing modes; *extra gets the page-cross cycle. */
typedef enum { M_IMM, M_ZP, M_ZPX, M_ZPY, M_ABS, M_ABX, M_ABY, M_INX, M_INY } Mode;
static uint16_t ea(NesO* s, const Cart* c, Mode m, int* extra) {
  uint16_t base, a;
  switch (m) {
    case M_IMM: return s->PC++;
    case M_ZP: return rd(s, c, s->PC++);
    case M_ZPX: return (uint16_t)((rd(s, c, s->PC++) + s->X) & 0xFFu);
    case M_ZPY: return (uint16_t)((rd(s, c, s->PC++) + s->Y) & 0xFFu);
    case M_ABS: a = rd16(s, c, s->PC); s->PC += 2; return a;
    case M_ABX: base = rd16(s, c, s->PC); s->PC += 2; a = (uint16_t)(base + s->X); *extra = cross(base, a); return a;
    case M_ABY: base = rd16(s, c, s->PC); s->PC += 2; a = (uint16_t)(base + s->Y); *extra = cross(base, a); return a;
    case M_INX: return rd16(s, c, (uint16_t)(uint8_t)(rd(s, c, s->PC++) + s->X));
    case M_INY:
      base = rd16(s, c, (uint16_t)rd(s, c, s->PC++));
      a = (uint16_t)(base + s->Y);
      *extra = cross(base, a);
      return a;
  }
  return 0;
}
/* Base cycles of the read-type modes (LDA / AND / ORA / EOR / ADC / SBC / CMP). */
static const int kReadCycles[9] = {2, 3, 4, 4, 4, 4, 4, 6, 5};

static void adc(NesO* s, uint8_t v) {
  const uint16_t sum = (uint16_t)(s->A + v + ((s->P & FC) ? 1 : 0));
  const uint8_t r = (uint8_t)sum;
  setf(s, FC, sum > 0xFFu);
  setf(s, FV, ((s->A ^ v) & 0x80u) == 0 && ((s->A ^ r) & 0x80u) != 0);
  s->A = r;
  zn(s, r);
}
static void sbc(NesO* s, uint8_t v) {
  const uint16_t d = (uint16_t)(s->A - v - ((s->P & FC) ? 0 : 1));
  const uint8_t r = (uint8_t)d;
  setf(s, FC, d < 0x100u);
  setf(s, FV, ((s->A ^ v) & 0x80u) != 0 && ((s->A ^ r) & 0x80u) != 0);
  s->A = r;
  zn(s, r);
}
static void cmpv(NesO* s, uint8_t reg, uint8_t v) {
  setf(s, FC, reg >= v);
  setf(s, FZ, reg == v);
  setf(s, FN, ((uint8_t)(reg - v) & 0x80u) != 0);
}
static int branch(NesO* s, const Cart* c, int take) {
  const int8_t off = (int8_t)rd(s, c, s->PC++);
  if (!take) return 2;
  const uint16_t np = (uint16_t)(s->PC + off);
  const int cyc = 3 + cross(s->PC, np);
  s->PC = np;
  return cyc;
}

/* Read-modify-write ops: 0 ASL, 1 ROL, 2 LSR, 3 ROR, 4 INC, 5 DEC. */
static uint8_t rmw(NesO* s, int op, uint8_t v) {
  uint8_t r;
  const int oc = (s->P & FC) != 0;
  switch (op) {
    case 0: setf(s, FC, v & 0x80u); r = (uint8_t)(v << 1); break;
    case 1: setf(s, FC, v & 0x80u); r = (uint8_t)((v << 1) | oc); break;
    case 2: setf(s, FC, v & 1u); r = (uint8_t)(v >> 1); break;
    case 3: setf(s, FC, v & 1u); r = (uint8_t)((v >> 1) | (oc ? 0x80u : 0u)); break;
    case 4: r = (uint8_t)(v + 1); break;
    default: r = (uint8_t)(v - 1); break;
  }
  zn(s, r);
  return r;
}

static int cpu_step(NesO* s, const Cart* c) {
  if (s->nmi_pending) {
    s->nmi_pending = 0;
    push(s, c, (uint8_t)(s->PC >> 8));
    push(s, c, (uint8_t)s->PC);
    push(s, c, (uint8_t)((s->P & ~FB) | FU));
    setf(s, FI, 1);
    s->PC = rd16(s, c, 0xFFFAu);
    s->total_cycles += 7;
    return 7;
  }
  if (s->irq_pending && !(s->P & FI)) {
    s->irq_pending = 0;
    push(s, c, (uint8_t)(s->PC >> 8));
    push(s, c, (uint8_t)s->PC);
    push(s, c, (uint8_t)((s->P & ~FB) | FU));
    setf(s, FI, 1);
    s->PC = rd16(s, c, 0xFFFEu);
    s->total_cycles += 7;
    return 7;
  }
  const uint8_t op = rd(s, c, s->PC++);
  int cyc = 2, x = 0;
  /* read-type groups: the low bits select the mode (standard 6502 encoding) */
  static const Mode g1[8] = {M_INX, M_ZP, M_IMM, M_ABS, M_INY, M_ZPX, M_ABY, M_ABX};
  const int aaa = op >> 5, bbb = (op >> 2) & 7;
  if ((op & 3u) == 1u && op != 0x89) { /* ORA AND EOR ADC STA LDA CMP SBC (0x89: a NOP below) */
    const Mode m = g1[bbb];
    if (aaa == 4) { /* STA */
      const uint16_t a = ea(s, c, m, &x);
      wr(s, c, a, s->A);
      cyc = (m == M_ZP) ? 3 : (m == M_ZPX || m == M_ABS) ? 4 : (m == M_ABX || m == M_ABY) ? 5 : 6;
    } else {
      const uint16_t a = ea(s, c, m, &x);
      const uint8_t v = rd(s, c, a);
      switch (aaa) {
        case 0: s->A |= v; zn(s, s->A); break;
        case 1: s->A &= v; zn(s, s->A); break;
        case 2: s->A ^= v; zn(s, s->A); break;
        case 3: adc(s, v); break;
        case 5: s->A = v; zn(s, v); break;
        case 6: cmpv(s, s->A, v); break;
        default: sbc(s, v); break;
      }
      cyc = kReadCycles[m] + x;
    }
    s->total_cycles += (uint64_t)cyc;
    return cyc;
  }
  switch (op) {
    /* LDX / LDY */
    case 0xA2: s->X = rd(s, c, ea(s, c, M_IMM, &x)); zn(s, s->X); cyc = 2; break;
    case 0xA6: s->X = rd(s, c, ea(s, c, M_ZP, &x)); zn(s, s->X); cyc = 3; break;
    case 0xB6: s->X = rd(s, c, ea(s, c, M_ZPY, &x)); zn(s, s->X); cyc = 4; break;
    case 0xAE: s->X = rd(s, c, ea(s, c, M_ABS, &x)); zn(s, s->X); cyc = 4; break;
    case 0xBE: s->X = rd(s, c, ea(s, c, M_ABY, &x)); zn(s, s->X); cyc = 4 + x; break;
    case 0xA0: s->Y = rd(s, c, ea(s, c, M_IMM, &x)); zn(s, s->Y); cyc = 2; break;
    case 0xA4: s->Y = rd(s, c, ea(s, c, M_ZP, &x)); zn(s, s->Y); cyc = 3; break;
    case 0xB4: s->Y = rd(s, c, ea(s, c, M_ZPX, &x)); zn(s, s->Y); cyc = 4; break;
    case 0xAC: s->Y = rd(s, c, ea(s, c, M_ABS, &x)); zn(s, s->Y); cyc = 4; break;
    case 0xBC: s->Y = rd(s, c, ea(s, c, M_ABX, &x)); zn(s, s->Y); cyc = 4 + x; break;
    /* STX / STY */
    case 0x86: wr(s, c, ea(s, c, M_ZP, &x), s->X); cyc = 3; break;
    case 0x96: wr(s, c, ea(s, c, M_ZPY, &x), s->X); cyc = 4; break;
    case 0x8E: wr(s, c, ea(s, c, M_ABS, &x), s->X); cyc = 4; break;
    case 0x84: wr(s, c, ea(s, c, M_ZP, &x), s->Y); cyc = 3; break;
    case 0x94: wr(s, c, ea(s, c, M_ZPX, &x), s->Y); cyc = 4; break;
    case 0x8C: wr(s, c, ea(s, c, M_ABS, &x), s->Y); cyc = 4; break;
    /* transfers, increments */
    case 0xAA: s->X = s->A; zn(s, s->X); break;
    case 0xA8: s->Y = s->A; zn(s, s->Y); break;
    case 0x8A: s->A = s->X; zn(s, s->A); break;
    case 0x98: s->A = s->Y; zn(s, s->A); break;
    case 0xBA: s->X = s->SP; zn(s, s->X); break;
    case 0x9A: s->SP = s->X; break;
    case 0xE8: s->X++; zn(s, s->X); break;
    case 0xC8: s->Y++; zn(s, s->Y); break;
    case 0xCA: s->X--; zn(s, s->X); break;
    case 0x88: s->Y--; zn(s, s->Y); break;
    /* stack */
    case 0x48: push(s, c, s->A); cyc = 3; break;
    case 0x08: push(s, c, (uint8_t)(s->P | FB | FU)); cyc = 3; break;
    case 0x68: s->A = pop(s, c); zn(s, s->A); cyc = 4; break;
    case 0x28: s->P = (uint8_t)((pop(s, c) & ~FB) | FU); cyc = 4; break;
    /* BIT */
    case 0x24: case 0x2C: {
      const uint8_t v = rd(s, c, ea(s, c, op == 0x24 ? M_ZP : M_ABS, &x));
      setf(s, FZ, (s->A & v) == 0);
      setf(s, FN, v & 0x80u);
      setf(s, FV, v & 0x40u);
      cyc = op == 0x24 ? 3 : 4;
      break;
    }
    /* CPX / CPY */
    case 0xE0: cmpv(s, s->X, rd(s, c, ea(s, c, M_IMM, &x))); cyc = 2; break;
    case 0xE4: cmpv(s, s->X, rd(s, c, ea(s, c, M_ZP, &x))); cyc = 3; break;
    case 0xEC: cmpv(s, s->X, rd(s, c, ea(s, c, M_ABS, &x))); cyc = 4; break;
    case 0xC0: cmpv(s, s->Y, rd(s, c, ea(s, c, M_IMM, &x))); cyc = 2; break;
    case 0xC4: cmpv(s, s->Y, rd(s, c, ea(s, c, M_ZP, &x))); cyc = 3; break;
    case 0xCC: cmpv(s, s->Y, rd(s, c, ea(s, c, M_ABS, &x))); cyc = 4; break;
    /* shifts on A */
    case 0x0A: s->A = rmw(s, 0, s->A); break;
    case 0x2A: s->A = rmw(s, 1, s->A); break;
    case 0x4A: s->A = rmw(s, 2, s->A); break;
    case 0x6A: s->A = rmw(s, 3, s->A); break;
    /* read-modify-write on memory: ASL ROL LSR ROR (0x06..0x7E) and DEC INC (0xC6..0xFE) */
    case 0x06: case 0x16: case 0x0E: case 0x1E: case 0x26: case 0x36: case 0x2E: case 0x3E:
    case 0x46: case 0x56: case 0x4E: case 0x5E: case 0x66: case 0x76: case 0x6E: case 0x7E:
    case 0xC6: case 0xD6: case 0xCE: case 0xDE: case 0xE6: case 0xF6: case 0xEE: case 0xFE: {
      static const int kOp[8] = {0, 1, 2, 3, -1, -1, 5, 4};
      const Mode m = bbb == 1 ? M_ZP : bbb == 5 ? M_ZPX : bbb == 3 ? M_ABS : M_ABS;
      uint16_t a;
      if (bbb == 7) { /* abs,X without the page-cross cycle */
        a = (uint16_t)(rd16(s, c, s->PC) + s->X);
        s->PC += 2;
      } else {
        a = ea(s, c, m, &x);
      }
      const uint8_t r = rmw(s, kOp[aaa], rd(s, c, a));
      wr(s, c, a, r);
      cyc = bbb == 1 ? 5 : bbb == 7 ? 7 : 6;
      break;
    }
    /* branches */
    case 0x10: cyc = branch(s, c, !(s->P & FN)); break;
    case 0x30: cyc = branch(s, c, (s->P & FN) != 0); break;
    case 0x50: cyc = branch(s, c, !(s->P & FV)); break;
    case 0x70: cyc = branch(s, c, (s->P & FV) != 0); break;
    case 0x90: cyc = branch(s, c, !(s->P & FC)); break;
    case 0xB0: cyc = branch(s, c, (s->P & FC) != 0); break;
    case 0xD0: cyc = branch(s, c, !(s->P & FZ)); break;
    case 0xF0: cyc = branch(s, c, (s->P & FZ) != 0); break;
    /* jumps */
    case 0x4C: s->PC = rd16(s, c, s->PC); cyc = 3; break;
    case 0x6C: {
      const uint16_t p = rd16(s, c, s->PC);
      s->PC += 2;
      const uint8_t lo = rd(s, c, p);
      const uint8_t hi = rd(s, c, (uint16_t)((p & 0xFF00u) | ((p + 1) & 0xFFu)));
      s->PC = (uint16_t)((hi << 8) | lo);
      cyc = 5;
      break;
    }
    case 0x20: {
      const uint16_t a = rd16(s, c, s->PC);
      s->PC += 2;
      const uint16_t ret = (uint16_t)(s->PC - 1);
      push(s, c, (uint8_t)(ret >> 8));
      push(s, c, (uint8_t)ret);
      s->PC = a;
      cyc = 6;
      break;
    }
    case 0x60: {
      const uint8_t lo = pop(s, c), hi = pop(s, c);
      s->PC = (uint16_t)(((hi << 8) | lo) + 1);
      cyc = 6;
      break;
    }
    case 0x40: {
      s->P = (uint8_t)((pop(s, c) & ~FB) | FU);
      const uint8_t lo = pop(s, c), hi = pop(s, c);
      s->PC = (uint16_t)((hi << 8) | lo);
      cyc = 6;
      break;
    }
    case 0x00:
      s->PC++;
      push(s, c, (uint8_t)(s->PC >> 8));
      push(s, c, (uint8_t)s->PC);
      push(s, c, (uint8_t)(s->P | FB | FU));
      setf(s, FI, 1);
      s->PC = rd16(s, c, 0xFFFEu);
      cyc = 7;
      break;
    /* flags */
    case 0x18: setf(s, FC, 0); break;
    case 0x38: setf(s, FC, 1); break;
    case 0x58: setf(s, FI, 0); break;
    case 0x78: setf(s, FI, 1); break;
    case 0xB8: setf(s, FV, 0); break;
    case 0xD8: setf(s, FD, 0); break;
    case 0xF8: setf(s, FD, 1); break;
    /* NOPs */
    case 0xEA: case 0x1A: case 0x3A: case 0x5A: case 0x7A: case 0xDA: case 0xFA: break;
    case 0x80: case 0x82: case 0x89: case 0xC2: case 0xE2: s->PC++; break;
    case 0x04: case 0x44: case 0x64: s->PC++; cyc = 3; break;
    case 0x14: case 0x34: case 0x54: case 0x74: case 0xD4: case 0xF4: s->PC++; cyc = 4; break;
    case 0x0C: s->PC += 2; cyc = 4; break;
    case 0x1C: case 0x3C: case 0x5C: case 0x7C: case 0xDC: case 0xFC: {
      const uint16_t b = rd16(s, c, s->PC);
      s->PC += 2;
      cyc = 4 + cross(b, (uint16_t)(b + s->X));
      break;
    }
    default: cyc = 1; break;
  }
  s->total_cycles += (uint64_t)cyc;
  return cyc;
}

/* ------------------------------------------------------------------ frames */
static void run_one_frame(NesO* s, const Cart* c, uint8_t* fb) {
  s->frame_ready = 0;
  int total = 0;
  while (!s->frame_ready && total < 65000) {
    const int cy = cpu_step(s, c);
    total += cy;
    for (int i = 0; i < cy * 3; ++i) {
      ppu_tick(s, c, fb);
      if (s->nmi_flag) {
        s->nmi_flag = 0;
        s->nmi_pending = 1;
      }
    }
  }
}

static void reset_one(NesO* s, const Cart* c) {
  const uint8_t mir = s->mirroring;
  memset(s, 0, sizeof(*s));
  s->mirroring = mir;
  s->SP = 0xFD;
  s->P = FU | FI;
  s->PC = rd16(s, c, 0xFFFCu);
}

/* ------------------------------------------------------------------ batch API */
typedef struct {
  int n;
  NesO* st;
  uint8_t* fb; /* [n][240][256] or NULL */
} NesOBatch;

void* nes_o_create(int n, int render) {
  NesOBatch* b = (NesOBatch*)calloc(1, sizeof(NesOBatch));
  b->n = n;
  b->st = (NesO*)calloc((size_t)n, sizeof(NesO));
  b->fb = render ? (uint8_t*)calloc((size_t)n * 61440u, 1) : NULL;
  return b;
}
void nes_o_free(void* h) {
  NesOBatch* b = (NesOBatch*)h;
  free(b->st);
  free(b->fb);
  free(b);
}
static Cart cart(const NesOBatch* b, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr) {
  Cart c = {prg, prg_size, chr, b->fb != NULL};
  return c;
}
void nes_o_set_mirroring(void* h, int m) {
  NesOBatch* b = (NesOBatch*)h;
  for (int i = 0; i < b->n; ++i) b->st[i].mirroring = (uint8_t)m;
}
/* mask == NULL resets every instance */
void nes_o_reset(void* h, const uint8_t* mask, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr) {
  NesOBatch* b = (NesOBatch*)h;
  const Cart c = cart(b, prg, prg_size, chr);
  for (int i = 0; i < b->n; ++i)
    if (!mask || mask[i]) reset_one(&b->st[i], &c);
}
void nes_o_set_buttons(void* h, const uint8_t* buttons) {
  NesOBatch* b = (NesOBatch*)h;
  for (int i = 0; i < b->n; ++i) {
    b->st[i].joypad1 = buttons[i];
    b->st[i].joypad_shift = 0;
    b->st[i].joypad_strobe = 0;
  }
}
/* k frames, all but the last headless (k == 1: one fully rendered frame) */
void nes_o_step_frames(void* h, int k, const uint8_t* prg, uint32_t prg_size, const uint8_t* chr) {
  NesOBatch* b = (NesOBatch*)h;
  const Cart c = cart(b, prg, prg_size, chr);
  for (int i = 0; i < b->n; ++i) {
    for (int f = 0; f < k; ++f) {
      b->st[i].headless = (uint8_t)(f < k - 1);
      run_one_frame(&b->st[i], &c, b->fb ? b->fb + (size_t)i * 61440u : NULL);
    }
    b->st[i].headless = 0;
  }
}
void nes_o_get_ram(void* h, uint8_t* out) {
  NesOBatch* b = (NesOBatch*)h;
  for (int i = 0; i < b->n; ++i) memcpy(out + (size_t)i * 2048u, b->st[i].ram, 2048);
}
void nes_o_get_mem(void* h, uint8_t* vram, uint8_t* oam, uint8_t* pal) {
  NesOBatch* b = (NesOBatch*)h;
  for (int i = 0; i < b->n; ++i) {
    memcpy(vram + (size_t)i * 2048u, b->st[i].vram, 2048);
    memcpy(oam + (size_t)i * 256u, b->st[i].oam, 256);
    memcpy(pal + (size_t)i * 32u, b->st[i].palette, 32);
  }
}
void nes_o_get_fb(void* h, uint8_t* out) {
  NesOBatch* b = (NesOBatch*)h;
  if (b->fb) memcpy(out, b->fb, (size_t)b->n * 61440u);
}
/* Scalars per instance, in this order (int64 each):
 * A X Y SP PC P total_cycles nmi_pending irq_pending joypad1 joypad_shift joypad_strobe
 * ctrl mask status oam_addr v t fine_x w read_buffer mirroring scanline cycle
 * frame_ready nmi_flag active_sprite_count dma_far */
#define NES_O_NSCALAR 28
int nes_o_nscalar(void) { return NES_O_NSCALAR; }
void nes_o_get_scalars(void* h, int64_t* out) {
  NesOBatch* b = (NesOBatch*)h;
  for (int i = 0; i < b->n; ++i) {
    const NesO* s = &b->st[i];
    int64_t* o = out + (size_t)i * NES_O_NSCALAR;
    const int64_t v[NES_O_NSCALAR] = {s->A, s->X, s->Y, s->SP, s->PC, s->P, (int64_t)s->total_cycles,
                                      s->nmi_pending, s->irq_pending, s->joypad1, s->joypad_shift,
                                      s->joypad_strobe, s->ctrl, s->mask, s->status, s->oam_addr, s->v, s->t,
                                      s->fine_x, s->w, s->read_buffer, s->mirroring, s->scanline, s->cycle,
                                      s->frame_ready, s->nmi_flag, s->active_count, s->dma_far};
    memcpy(o, v, sizeof(v));
  }
}

/* Observation: palette index -> luma, bilinear 256 x 240 -> 84 x 84, rounded half up. */
static float gray_of(uint8_t idx) {
  const uint32_t rgba = kPal[idx & 63];
  const float r = (float)((rgba >> 16) & 0xFFu), g = (float)((rgba >> 8) & 0xFFu), b = (float)(rgba & 0xFFu);
  return 0.299f * r + 0.587f * g + 0.114f * b;
}
void nes_o_obs_from_fb(const uint8_t* fb, int n, uint8_t* out) {
  for (int i = 0; i < n; ++i) {
    const uint8_t* f = fb + (size_t)i * 61440u;
    for (int oy = 0; oy < 84; ++oy)
      for (int ox = 0; ox < 84; ++ox) {
        const float fy = ((float)oy + 0.5f) * (240.0f / 84.0f) - 0.5f;
        const float fx = ((float)ox + 0.5f) * (256.0f / 84.0f) - 0.5f;
        const int y0 = fy < 0.0f ? 0 : (int)fy, x0 = fx < 0.0f ? 0 : (int)fx;
        const int y1 = y0 + 1 < 240 ? y0 + 1 : 239, x1 = x0 + 1 < 256 ? x0 + 1 : 255;
        float wy = fy - (float)y0, wx = fx - (float)x0;
        if (wy < 0.0f) wy = 0.0f;
        if (wx < 0.0f) wx = 0.0f;
        const float g = (1.0f - wy) * (1.0f - wx) * gray_of(f[y0 * 256 + x0]) +
                        (1.0f - wy) * wx * gray_of(f[y0 * 256 + x1]) +
                        wy * (1.0f - wx) * gray_of(f[y1 * 256 + x0]) + wy * wx * gray_of(f[y1 * 256 + x1]);
        out[(size_t)i * 7056u + oy * 84 + ox] = (uint8_t)(g + 0.5f);
      }
  }
}
