"""The CPU oracle of the NES environment step (oracle/nes_oracle.c) against
golden vectors of the reference's own GPU emulator (tests/golden/nes_ref.npz,
made by tests/golden/make_nes_golden.py from the reference's NESBatchGpu on
the same synthetic cartridges and schedules), and the assembler / cartridge
builders."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).parent / "golden" / "nes_ref.npz"


def _replay(name, make, ci):
    import sys
    sys.path.insert(0, str(Path(__file__).parent / "golden"))
    from make_nes_golden import N, schedule
    from oracle.nes import OracleNES

    prg, chr_rom, mir = make()
    ora = OracleNES(N, prg, chr_rom, mir)
    ora.reset()
    for op, arg in schedule(ci):
        if op == "b":
            ora.set_buttons(arg)
        elif op == "f":
            ora.run_frames(1)
        elif op == "k":
            ora.run_frames(arg)
        else:
            ora.reset(arg)
    return ora


def _carts():
    import sys
    sys.path.insert(0, str(Path(__file__).parent / "golden"))
    from make_nes_golden import CARTS
    return list(CARTS.items())


@pytest.mark.parametrize("ci", range(12))
def test_oracle_matches_reference_goldens(ci):
    from oracle.nes import SCALARS, palette_rgba

    g = np.load(GOLDEN)
    name, make = _carts()[ci]
    ora = _replay(name, make, ci)
    keep = g[f"{name}/keep"]
    assert keep.sum() >= 4
    sc = ora.scalars()
    cols = [i for i, k in enumerate(SCALARS[:27]) if not k.startswith("joypad")]
    o_sc = np.stack([sc[k] for k in SCALARS[:27]], 1)
    assert np.array_equal(g[f"{name}/scalars"][keep][:, cols], o_sc[keep][:, cols])
    assert np.array_equal(g[f"{name}/ram"][keep], ora.ram()[keep])
    assert np.array_equal(g[f"{name}/obs"][keep], ora.obs()[keep])
    rgba = palette_rgba()[ora.framebuffer()]
    sha = np.array([int.from_bytes(hashlib.sha256(f.tobytes()).digest()[:8], "little") for f in rgba], np.uint64)
    assert np.array_equal(g[f"{name}/fb_sha"][keep], sha[keep])


def test_assembler_encodings():
    from rl_for_mario_b200.nes_roms import Asm

    a = Asm(0x8000)
    a.label("top").op("LDA", "imm", 0x42).op("STA", "abs", 0x2006).op("LDA", "izy", 0x10).op("ASL", "acc")
    a.op("INC", "abx", 0x0300).op("JMP", "ind", 0x02FF).op("BNE", "", "top").op("RTI")
    assert a.assemble() == bytes([0xA9, 0x42, 0x8D, 0x06, 0x20, 0xB1, 0x10, 0x0A, 0xFE, 0x00, 0x03,
                                  0x6C, 0xFF, 0x02, 0xD0, 0xF0, 0x40])


def test_known_answers():
    """Instruction semantics the reference's unit tests check (flags of ADC / SBC
    / CMP, the JMP-indirect page wrap, the stack), run as a cartridge."""
    from oracle.nes import OracleNES
    from rl_for_mario_b200.nes_roms import Asm, _cart

    a = Asm(0x8000)
    a.label("reset").op("LDA", "imm", 0x50).op("CLC").op("ADC", "imm", 0x50).op("PHP").op("STA", "zp", 0x00)
    a.op("PLA").op("STA", "zp", 0x01)                          # 0x50 + 0x50 = 0xA0, V and N set
    a.op("LDA", "imm", 0x50).op("SEC").op("SBC", "imm", 0xB0).op("PHP").op("STA", "zp", 0x02)
    a.op("PLA").op("STA", "zp", 0x03)                          # 0x50 - 0xB0 = 0xA0, V N set, C clear
    a.op("LDA", "imm", 0x34).op("STA", "abs", 0x02FF).op("LDA", "imm", 0x92).op("STA", "abs", 0x0200)
    a.op("LDA", "imm", 0x99).op("STA", "abs", 0x0300)
    a.op("JMP", "ind", 0x02FF)                                 # page wrap: high byte from $0200 -> $9234
    code = a.assemble()
    prg = bytearray(_cart(code, (0x8000, 0x8000, 0x8000)))
    tail = Asm(0x9234).op("STX", "zp", 0x04).op("TSX").op("STX", "zp", 0x05).label("h").op("JMP", "abs", "h").assemble()
    prg[0x1234: 0x1234 + len(tail)] = tail
    ora = OracleNES(1, bytes(prg), bytes(8192), 0)
    ora.reset()
    ora.set_buttons(np.zeros(1, np.uint8))
    ora.run_frames(1)
    ram = ora.ram()[0]
    assert ram[0] == 0xA0 and ram[1] & 0xC1 == 0xC0
    assert ram[2] == 0xA0 and ram[3] & 0xC1 == 0xC0
    assert ram[5] == 0xFD  # stack back where reset put it
    assert ora.scalars()["PC"][0] in range(0x9236, 0x923C)
