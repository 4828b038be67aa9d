"""Synthetic NES cartridges for the batched emulator (the Super Mario Bros. ROM
that the reference's environment loads is not distributed with this library).

- ``Asm``: a small two-pass 6502 assembler (official opcodes, labels).
- ``demo_rom()``: an NROM program that exercises what the reference emulator
  models: palette, nametable and attribute writes through $2006/$2007, OAM DMA
  from $0200 in the NMI handler, controller reads through $4016, sprite 0 hit
  polling, scroll and control writes, and the RAM cells the reference's
  environment reads (x position at $006D/$0086, lives at $075A, the stage-clear
  flag at $07D7; ``scripts/mario/gpu_vec_env.py:200-215``): Right moves the
  player 3 pixels a frame, Left 1 back, holding B for 12 frames in a row costs a
  life, and reaching x = 0x240 sets the stage-clear flag.
- ``random_rom(seed)``: random PRG / CHR bytes with vectors into PRG; with
  ``prologue=True`` a fixed prologue first fills the palette, the nametables
  and OAM with random bytes and turns rendering and NMI on, then jumps into
  the random code.

Cartridges are returned as ``(prg, chr, mirroring)``: PRG of 16 or 32 KB, CHR of
8 KB, mirroring 0 (horizontal) or 1 (vertical), as the reference's iNES loader
returns them (``gpu_vec_env.py:_load_nes_rom``).
"""
from __future__ import annotations

import random
from typing import Dict, List, Tuple

# -------------------------------------------------------------------- assembler
_ALU = {"ORA": 0, "AND": 1, "EOR": 2, "ADC": 3, "STA": 4, "LDA": 5, "CMP": 6, "SBC": 7}
_ALU_MODE = {"izx": 0, "zp": 1, "imm": 2, "abs": 3, "izy": 4, "zpx": 5, "aby": 6, "abx": 7}
_OPS: Dict[Tuple[str, str], int] = {}
for _m, _a in _ALU.items():
    for _mode, _b in _ALU_MODE.items():
        if not (_m == "STA" and _mode == "imm"):
            _OPS[(_m, _mode)] = (_a << 5) | (_b << 2) | 1
_RMW = {"ASL": 0x00, "ROL": 0x20, "LSR": 0x40, "ROR": 0x60, "DEC": 0xC0, "INC": 0xE0}
for _m, _base in _RMW.items():
    for _mode, _off in (("zp", 0x06), ("zpx", 0x16), ("abs", 0x0E), ("abx", 0x1E)):
        _OPS[(_m, _mode)] = _base + _off
    if _m in ("ASL", "ROL", "LSR", "ROR"):
        _OPS[(_m, "acc")] = _base + 0x0A
_OPS.update({
    ("LDX", "imm"): 0xA2, ("LDX", "zp"): 0xA6, ("LDX", "zpy"): 0xB6, ("LDX", "abs"): 0xAE, ("LDX", "aby"): 0xBE,
    ("LDY", "imm"): 0xA0, ("LDY", "zp"): 0xA4, ("LDY", "zpx"): 0xB4, ("LDY", "abs"): 0xAC, ("LDY", "abx"): 0xBC,
    ("STX", "zp"): 0x86, ("STX", "zpy"): 0x96, ("STX", "abs"): 0x8E,
    ("STY", "zp"): 0x84, ("STY", "zpx"): 0x94, ("STY", "abs"): 0x8C,
    ("CPX", "imm"): 0xE0, ("CPX", "zp"): 0xE4, ("CPX", "abs"): 0xEC,
    ("CPY", "imm"): 0xC0, ("CPY", "zp"): 0xC4, ("CPY", "abs"): 0xCC,
    ("BIT", "zp"): 0x24, ("BIT", "abs"): 0x2C,
    ("JMP", "abs"): 0x4C, ("JMP", "ind"): 0x6C, ("JSR", "abs"): 0x20,
})
_IMPLIED = {"BRK": 0x00, "PHP": 0x08, "CLC": 0x18, "PLP": 0x28, "SEC": 0x38, "RTI": 0x40, "PHA": 0x48,
            "CLI": 0x58, "RTS": 0x60, "PLA": 0x68, "SEI": 0x78, "DEY": 0x88, "TXA": 0x8A, "TYA": 0x98,
            "TXS": 0x9A, "TAY": 0xA8, "TAX": 0xAA, "CLV": 0xB8, "TSX": 0xBA, "INY": 0xC8, "DEX": 0xCA,
            "CLD": 0xD8, "INX": 0xE8, "NOP": 0xEA, "SED": 0xF8}
_BRANCH = {"BPL": 0x10, "BMI": 0x30, "BVC": 0x50, "BVS": 0x70, "BCC": 0x90, "BCS": 0xB0, "BNE": 0xD0, "BEQ": 0xF0}
_SIZE = {"imm": 2, "zp": 2, "zpx": 2, "zpy": 2, "izx": 2, "izy": 2, "abs": 3, "abx": 3, "aby": 3, "ind": 3, "acc": 1}


class Asm:
    """Two-pass assembler: ``op(mnemonic, mode, arg)`` where arg is an int or a
    label name (absolute modes and branches)."""

    def __init__(self, org: int = 0x8000):
        self.org = org
        self.items: List[tuple] = []
        self.labels: Dict[str, int] = {}
        self.pc = org

    def label(self, name: str) -> "Asm":
        self.labels[name] = self.pc
        return self

    def op(self, mn: str, mode: str = "", arg=None) -> "Asm":
        if mn in _IMPLIED and not mode:
            self.items.append(("b", bytes([_IMPLIED[mn]])))
            self.pc += 1
        elif mn in _BRANCH:
            self.items.append(("br", _BRANCH[mn], arg, self.pc))
            self.pc += 2
        else:
            code = _OPS[(mn, mode)]
            self.items.append(("op", code, mode, arg))
            self.pc += _SIZE[mode]
        return self

    def data(self, bs) -> "Asm":
        bs = bytes(bs)
        self.items.append(("b", bs))
        self.pc += len(bs)
        return self

    def assemble(self) -> bytes:
        out = bytearray()
        for it in self.items:
            if it[0] == "b":
                out += it[1]
            elif it[0] == "br":
                _, code, target, at = it
                dest = self.labels[target] if isinstance(target, str) else target
                off = dest - (at + 2)
                if not -128 <= off <= 127:
                    raise ValueError(f"branch to {target} out of range ({off})")
                out += bytes([code, off & 0xFF])
            else:
                _, code, mode, arg = it
                val = self.labels[arg] if isinstance(arg, str) else (arg or 0)
                if _SIZE[mode] == 1:
                    out += bytes([code])
                elif _SIZE[mode] == 2:
                    out += bytes([code, val & 0xFF])
                else:
                    out += bytes([code, val & 0xFF, (val >> 8) & 0xFF])
        return bytes(out)


def _cart(code: bytes, vectors: Tuple[int, int, int], prg_size: int = 0x8000, fill: int = 0xEA) -> bytes:
    prg = bytearray([fill]) * prg_size
    prg[: len(code)] = code
    nmi, reset, irq = vectors
    prg[prg_size - 6: prg_size] = bytes([nmi & 0xFF, nmi >> 8, reset & 0xFF, reset >> 8, irq & 0xFF, irq >> 8])
    return bytes(prg)


def _chr(seed: int) -> bytes:
    """8 KB of tiles: structured patterns (stripes, checkers, diagonals) with
    some transparent rows, so backgrounds and sprites overlap in every way."""
    rng = random.Random(seed)
    out = bytearray()
    for t in range(512):
        kind = t % 4
        for plane in range(2):
            for r in range(8):
                if kind == 0:
                    b = 0xFF if (r + plane + t) % 3 else 0x00
                elif kind == 1:
                    b = 0xAA if (r + plane) % 2 else 0x55
                elif kind == 2:
                    b = (0x80 >> ((r + t) % 8)) * (1 + plane) & 0xFF
                else:
                    b = rng.randrange(256)
                out.append(b)
    return bytes(out)


# -------------------------------------------------------------------- demo
RAM_PAGE, RAM_X, RAM_LIVES, RAM_CLEAR = 0x006D, 0x0086, 0x075A, 0x07D7


def demo_rom(prg_size: int = 0x8000, mirroring: int = 0) -> Tuple[bytes, bytes, int]:
    a = Asm(0x8000 if prg_size == 0x8000 else 0xC000)
    # ---- reset
    a.label("reset")
    a.op("SEI").op("CLD").op("LDX", "imm", 0xFF).op("TXS")
    a.op("LDA", "imm", 0).op("STA", "abs", 0x2000).op("STA", "abs", 0x2001)
    for w in ("vb1", "vb2"):
        a.label(w).op("BIT", "abs", 0x2002).op("BPL", "", w)
    # palette: 32 entries
    a.op("LDA", "imm", 0x3F).op("STA", "abs", 0x2006).op("LDA", "imm", 0x00).op("STA", "abs", 0x2006)
    a.op("LDX", "imm", 0).label("pal").op("LDA", "abx", "paldata").op("STA", "abs", 0x2007)
    a.op("INX").op("CPX", "imm", 32).op("BNE", "", "pal")
    # nametables 0 and 1 (2 KB incl. attributes): byte = (i * 7 + (i >> 5)) & 0xFF
    a.op("LDA", "imm", 0x20).op("STA", "abs", 0x2006).op("LDA", "imm", 0).op("STA", "abs", 0x2006)
    a.op("LDY", "imm", 0).op("LDX", "imm", 8)  # 8 pages of 256
    a.op("LDA", "imm", 0).op("STA", "zp", 0x00)
    a.label("nt").op("LDA", "zp", 0x00).op("CLC").op("ADC", "imm", 7).op("STA", "zp", 0x00)
    a.op("TYA").op("LSR", "acc").op("LSR", "acc").op("LSR", "acc").op("LSR", "acc").op("LSR", "acc")
    a.op("ADC", "zp", 0x00).op("STA", "abs", 0x2007)
    a.op("INY").op("BNE", "", "nt").op("DEX").op("BNE", "", "nt")
    # OAM buffer at $0200: sprite i: y = 3 i + 20, tile = i, attr = i & 0xE3, x = 4 i
    a.op("LDX", "imm", 0).op("LDY", "imm", 0)
    a.label("oam").op("TYA").op("STA", "zp", 0x01).op("ASL", "acc").op("CLC").op("ADC", "zp", 0x01)
    a.op("ADC", "imm", 20).op("STA", "abx", 0x0200)
    a.op("TYA").op("STA", "abx", 0x0201).op("AND", "imm", 0xE3).op("STA", "abx", 0x0202)
    a.op("TYA").op("ASL", "acc").op("ASL", "acc").op("STA", "abx", 0x0203)
    a.op("INX").op("INX").op("INX").op("INX").op("INY").op("CPY", "imm", 64).op("BNE", "", "oam")
    # sprite 0 over the background at (40, 60), tile 1, front
    a.op("LDA", "imm", 60).op("STA", "abs", 0x0200).op("LDA", "imm", 1).op("STA", "abs", 0x0201)
    a.op("LDA", "imm", 0).op("STA", "abs", 0x0202).op("LDA", "imm", 40).op("STA", "abs", 0x0203)
    # game state
    a.op("LDA", "imm", 2).op("STA", "abs", RAM_LIVES)
    a.op("LDA", "imm", 0).op("STA", "zp", RAM_PAGE).op("STA", "zp", RAM_X).op("STA", "abs", RAM_CLEAR)
    a.op("STA", "zp", 0x14).op("STA", "zp", 0x10).op("STA", "zp", 0x11)
    # NMI on, sprites from $0000, background from $1000; show both
    a.op("LDA", "imm", 0x90).op("STA", "abs", 0x2000).op("LDA", "imm", 0x1E).op("STA", "abs", 0x2001)
    # ---- main loop: count iterations and sprite 0 hits
    a.label("main").op("INC", "zp", 0x10).op("BIT", "abs", 0x2002).op("BVC", "", "main")
    a.op("INC", "zp", 0x11).op("JMP", "abs", "main")
    # ---- NMI
    a.label("nmi").op("PHA").op("TXA").op("PHA").op("TYA").op("PHA")
    a.op("LDA", "imm", 0).op("STA", "abs", 0x2003).op("LDA", "imm", 0x02).op("STA", "abs", 0x4014)
    # controller: 8 reads, A first, into $12 (A in bit 7 ... Right in bit 0)
    a.op("LDA", "imm", 1).op("STA", "abs", 0x4016).op("LDA", "imm", 0).op("STA", "abs", 0x4016)
    a.op("LDX", "imm", 8).label("pad").op("LDA", "abs", 0x4016).op("LSR", "acc").op("ROL", "zp", 0x12)
    a.op("DEX").op("BNE", "", "pad")
    # Right: x += 3 (carry into the page byte)
    a.op("LDA", "zp", 0x12).op("AND", "imm", 0x01).op("BEQ", "", "noright")
    a.op("LDA", "zp", RAM_X).op("CLC").op("ADC", "imm", 3).op("STA", "zp", RAM_X)
    a.op("LDA", "zp", RAM_PAGE).op("ADC", "imm", 0).op("STA", "zp", RAM_PAGE)
    a.label("noright").op("LDA", "zp", 0x12).op("AND", "imm", 0x02).op("BEQ", "", "noleft")
    a.op("LDA", "zp", RAM_X).op("SEC").op("SBC", "imm", 1).op("STA", "zp", RAM_X)
    a.op("LDA", "zp", RAM_PAGE).op("SBC", "imm", 0).op("STA", "zp", RAM_PAGE)
    # B held 12 frames in a row: lose a life
    a.label("noleft").op("LDA", "zp", 0x12).op("AND", "imm", 0x40).op("BEQ", "", "nob")
    a.op("INC", "zp", 0x14).op("LDA", "zp", 0x14).op("CMP", "imm", 12).op("BNE", "", "bdone")
    a.op("DEC", "abs", RAM_LIVES)
    a.label("nob").op("LDA", "imm", 0).op("STA", "zp", 0x14)
    # x >= 0x240: stage clear
    a.label("bdone").op("LDA", "zp", RAM_PAGE).op("CMP", "imm", 2).op("BCC", "", "noclear")
    a.op("LDA", "zp", RAM_X).op("CMP", "imm", 0x40).op("BCC", "", "noclear")
    a.op("LDA", "imm", 0x80).op("STA", "abs", RAM_CLEAR)
    a.label("noclear")
    # sprites drift: x of sprite i += (i & 3); sprite 0 follows the player's x
    a.op("LDX", "imm", 4).op("LDY", "imm", 1)
    a.label("drift").op("TYA").op("AND", "imm", 3).op("CLC").op("ADC", "abx", 0x0203).op("STA", "abx", 0x0203)
    a.op("INX").op("INX").op("INX").op("INX").op("INY").op("CPY", "imm", 64).op("BNE", "", "drift")
    a.op("LDA", "zp", RAM_X).op("STA", "abs", 0x0203)
    # animate palette entry 1 with the frame counter, then scroll / control
    a.op("INC", "zp", 0x13).op("LDA", "imm", 0x3F).op("STA", "abs", 0x2006).op("LDA", "imm", 0x01)
    a.op("STA", "abs", 0x2006).op("LDA", "zp", 0x13).op("LSR", "acc").op("LSR", "acc").op("AND", "imm", 0x3F)
    a.op("STA", "abs", 0x2007)
    a.op("LDA", "zp", RAM_X).op("STA", "abs", 0x2005).op("LDA", "imm", 0).op("STA", "abs", 0x2005)
    a.op("LDA", "zp", RAM_PAGE).op("AND", "imm", 1).op("ORA", "imm", 0x90).op("STA", "abs", 0x2000)
    a.op("PLA").op("TAY").op("PLA").op("TAX").op("PLA").op("RTI")
    a.label("irq").op("RTI")
    a.label("paldata").data([0x0F, 0x30, 0x16, 0x27, 0x0F, 0x1A, 0x2A, 0x3A, 0x0F, 0x12, 0x22, 0x32,
                             0x0F, 0x05, 0x15, 0x25, 0x0F, 0x37, 0x17, 0x07, 0x0F, 0x21, 0x11, 0x01,
                             0x0F, 0x28, 0x18, 0x08, 0x0F, 0x3C, 0x2C, 0x1C])
    code = a.assemble()
    prg = _cart(code, (a.labels["nmi"], a.labels["reset"], a.labels["irq"]), prg_size)
    return prg, _chr(1), mirroring


# -------------------------------------------------------------------- random
def random_rom(seed: int, prologue: bool = True, prg_size: int = 0x8000) -> Tuple[bytes, bytes, int]:
    rng = random.Random(seed)
    org = 0x10000 - prg_size
    body = bytearray(rng.randrange(256) for _ in range(prg_size))
    entry = org + rng.randrange(0x100, prg_size - 0x100)
    if prologue:
        a = Asm(org)
        a.op("SEI").op("LDX", "imm", 0xFF).op("TXS")
        # palette, both nametables and OAM from PRG bytes (random), via $2007 / $2004
        a.op("LDA", "imm", 0x3F).op("STA", "abs", 0x2006).op("LDA", "imm", 0).op("STA", "abs", 0x2006)
        a.op("LDX", "imm", 0).label("p").op("LDA", "abx", org + 0x400).op("STA", "abs", 0x2007)
        a.op("INX").op("CPX", "imm", 32).op("BNE", "", "p")
        a.op("LDA", "imm", 0x20).op("STA", "abs", 0x2006).op("LDA", "imm", 0).op("STA", "abs", 0x2006)
        a.op("LDY", "imm", 0).op("LDX", "imm", 8)
        a.label("n").op("LDA", "aby", org + 0x500).op("EOR", "zp", 0x00).op("STA", "abs", 0x2007)
        a.op("INY").op("BNE", "", "n").op("INC", "zp", 0x00).op("DEX").op("BNE", "", "n")
        a.op("LDA", "imm", 0).op("STA", "abs", 0x2003)
        a.label("o").op("LDA", "aby", org + 0x600).op("STA", "abs", 0x2004).op("INY").op("BNE", "", "o")
        a.op("LDA", "imm", rng.choice([0x80, 0x88, 0x90, 0x98])).op("STA", "abs", 0x2000)
        a.op("LDA", "imm", rng.choice([0x1E, 0x18, 0x16, 0x1E])).op("STA", "abs", 0x2001)
        a.op("JMP", "abs", entry)
        code = a.assemble()
        body[: len(code)] = code
        reset = org
    else:
        reset = entry
    nmi = org + rng.randrange(0x100, prg_size - 0x100)
    irq = org + rng.randrange(0x100, prg_size - 0x100)
    body[prg_size - 6:] = bytes([nmi & 0xFF, nmi >> 8, reset & 0xFF, reset >> 8, irq & 0xFF, irq >> 8])
    chr_rom = bytes(rng.randrange(256) for _ in range(8192))
    return bytes(body), chr_rom, rng.randrange(2)
