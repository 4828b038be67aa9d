"""ORACLE (test infrastructure only): ctypes binding of ``oracle/nes_oracle.c``
(the CPU restatement of the reference's batched NES emulator) and a numpy
restatement of the reference's environment step
(``scripts/mario/gpu_vec_env.py:271-404``: boot override, rewards from RAM,
done detection, auto-reset, frame ring).  Only tests/ and bench.py's CPU
baseline use it.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

_DIR = Path(__file__).resolve().parent
_SRC = _DIR / "nes_oracle.c"
_LIB = _DIR / "_native" / "libnes_oracle.so"
_lib = None

SCALARS = ("A X Y SP PC P total_cycles nmi_pending irq_pending joypad1 joypad_shift joypad_strobe ctrl mask "
           "status oam_addr v t fine_x w read_buffer mirroring scanline cycle frame_ready nmi_flag "
           "active_sprite_count dma_far").split()


def build(force: bool = False) -> Path:
    """Compiles the oracle with gcc (no FP contraction) into oracle/_native/."""
    if force or not _LIB.exists() or _LIB.stat().st_mtime < _SRC.stat().st_mtime:
        _LIB.parent.mkdir(exist_ok=True)
        subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(_LIB),
                        str(_SRC)], check=True)
    return _LIB


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(str(build()))
        P, I, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32
        for name, res, args in (
            ("nes_o_create", P, [I, I]), ("nes_o_free", None, [P]), ("nes_o_set_mirroring", None, [P, I]),
            ("nes_o_reset", None, [P, P, P, U, P]), ("nes_o_set_buttons", None, [P, P]),
            ("nes_o_step_frames", None, [P, I, P, U, P]), ("nes_o_get_ram", None, [P, P]),
            ("nes_o_get_mem", None, [P, P, P, P]), ("nes_o_get_fb", None, [P, P]),
            ("nes_o_get_scalars", None, [P, P]), ("nes_o_nscalar", I, []),
            ("nes_o_obs_from_fb", None, [P, I, P]), ("nes_o_palette_rgba", U, [I]),
        ):
            f = getattr(_lib, name)
            f.restype, f.argtypes = res, args
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class OracleNES:
    """N emulator instances on the CPU with the reference's NESBatchGpu calls."""

    def __init__(self, n: int, prg: bytes, chr_rom: bytes, mirroring: int = 0, render: bool = True):
        if len(prg) not in (0x4000, 0x8000) or len(chr_rom) != 0x2000:
            raise ValueError("PRG must be 16 or 32 KB and CHR 8 KB")
        self.n, self.render = n, render
        self._prg = np.frombuffer(prg, np.uint8).copy()
        self._chr = np.frombuffer(chr_rom, np.uint8).copy()
        self._h = lib().nes_o_create(n, 1 if render else 0)
        lib().nes_o_set_mirroring(self._h, mirroring)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().nes_o_free(self._h)
            self._h = None

    def _rom(self):
        return _ptr(self._prg), len(self._prg), _ptr(self._chr)

    def reset(self, mask=None):
        m = None if mask is None else _ptr(np.ascontiguousarray(mask, np.uint8))
        lib().nes_o_reset(self._h, m, *self._rom())

    def set_buttons(self, buttons):
        b = np.ascontiguousarray(buttons, np.uint8)
        lib().nes_o_set_buttons(self._h, _ptr(b))

    def run_frames(self, k: int):
        lib().nes_o_step_frames(self._h, k, *self._rom())

    def ram(self) -> np.ndarray:
        out = np.empty((self.n, 2048), np.uint8)
        lib().nes_o_get_ram(self._h, _ptr(out))
        return out

    def mem(self):
        vram, oam, pal = (np.empty((self.n, s), np.uint8) for s in (2048, 256, 32))
        lib().nes_o_get_mem(self._h, _ptr(vram), _ptr(oam), _ptr(pal))
        return vram, oam, pal

    def framebuffer(self) -> np.ndarray:
        out = np.zeros((self.n, 240, 256), np.uint8)
        lib().nes_o_get_fb(self._h, _ptr(out))
        return out

    def scalars(self) -> dict:
        k = lib().nes_o_nscalar()
        out = np.empty((self.n, k), np.int64)
        lib().nes_o_get_scalars(self._h, _ptr(out))
        return {name: out[:, i] for i, name in enumerate(SCALARS)}

    def obs(self) -> np.ndarray:
        return obs_from_framebuffer(self.framebuffer())


def obs_from_framebuffer(fb: np.ndarray) -> np.ndarray:
    fb = np.ascontiguousarray(fb, np.uint8)
    out = np.empty((fb.shape[0], 84, 84), np.uint8)
    lib().nes_o_obs_from_fb(_ptr(fb), fb.shape[0], _ptr(out))
    return out


def palette_rgba() -> np.ndarray:
    return np.array([lib().nes_o_palette_rgba(i) for i in range(256)], np.uint32)


# ---------------------------------------------------------------- environment
SIMPLE_MOVEMENT = np.array([0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40], np.uint8)
BOOT_TOTAL, BOOT_SETTLE, START = 286, 250, 0x08


class OracleEnv:
    """numpy restatement of the reference's GpuMarioVecEnv over OracleNES."""

    def __init__(self, n, prg, chr_rom, mirroring=0, frame_skip=4, frame_stack=4):
        self.nes = OracleNES(n, prg, chr_rom, mirroring, True)
        self.n, self.frame_skip, self.frame_stack = n, frame_skip, frame_stack
        self.ring = np.zeros((frame_stack, n, 84, 84), np.uint8)
        self.idx = 0
        self.prev_x = np.zeros(n, np.int32)
        self.init_lives = np.zeros(n, np.int32)
        self.boot = np.zeros(n, np.int32)

    @staticmethod
    def _x(ram):
        return ram[:, 0x6D].astype(np.int32) * 256 + ram[:, 0x86].astype(np.int32)

    def stacked(self):
        return np.stack([self.ring[(self.idx + i) % self.frame_stack] for i in range(self.frame_stack)], axis=1)

    def reset(self):
        self.nes.reset()
        self.boot[:] = 0
        self.idx = 0
        start, none = np.full(self.n, START, np.uint8), np.zeros(self.n, np.uint8)
        for f in range(BOOT_TOTAL - BOOT_SETTLE):
            self.nes.set_buttons(start if f % 4 < 2 else none)
            self.nes.run_frames(1)
        self.nes.set_buttons(none)
        self.nes.run_frames(BOOT_SETTLE)
        obs, ram = self.nes.obs(), self.nes.ram()
        self.ring[:] = obs[None]
        self.prev_x = self._x(ram)
        self.init_lives = ram[:, 0x75A].astype(np.int32)
        return self.stacked()

    def step(self, actions):
        actions = np.asarray(actions, np.int64)
        prev_boot = self.boot.copy()
        eff = SIMPLE_MOVEMENT[actions].copy()
        booting = self.boot > 0
        phase1 = booting & (self.boot > BOOT_SETTLE)
        eff[phase1] = START
        eff[booting & ~phase1] = 0
        self.nes.set_buttons(eff)
        self.nes.run_frames(self.frame_skip)
        self.boot[booting] = np.maximum(0, self.boot[booting] - self.frame_skip)
        obs, ram = self.nes.obs(), self.nes.ram()
        self.ring[self.idx] = obs
        self.idx = (self.idx + 1) % self.frame_stack
        cur_x = self._x(ram)
        lives = ram[:, 0x75A].astype(np.int32)
        clear = ram[:, 0x7D7] == 0x80
        just = (prev_boot > 0) & (self.boot <= 0)
        self.init_lives[just] = lives[just]
        self.prev_x[just] = cur_x[just]
        booting = self.boot > 0
        died = (lives < self.init_lives) & ~booting
        clear = clear & ~booting
        dones = died | clear
        dx = (cur_x - self.prev_x).astype(np.float32)
        dx[booting] = 0.0
        rew = np.clip(dx / 40.0, -1.0, 1.0).astype(np.float32)
        rew[died] = -1.0
        rew[clear] = 1.0
        info = {"x_pos": cur_x.copy(), "lives": lives.copy(), "flag_get": clear.copy()}
        if dones.any():
            self.nes.reset(dones.astype(np.uint8))
            self.boot[dones] = BOOT_TOTAL
            self.prev_x[dones] = 0
        active = ~booting & ~dones
        self.prev_x[active] = cur_x[active]
        return self.stacked(), rew, dones, info


# ---------------------------------------------------------------- the reference
_REF = _DIR / "_ref" / "libnes_ref.so"


class RefNESBatch:
    """The reference's own NESBatchGpu (built from its sources into
    oracle/_ref/libnes_ref.so by oracle/build_ref.py), through the extern "C"
    shim oracle/nes_ref_shim.cu.  Host numpy arrays in and out, as its pybind
    module takes them."""

    def __init__(self, n: int):
        if not _REF.exists():
            raise FileNotFoundError(f"{_REF} is not built (python oracle/build_ref.py)")
        self.lib = ctypes.CDLL(str(_REF))
        P, I, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32
        sig = {"ref_nes_create": (P, [I]), "ref_nes_destroy": (None, [P]),
               "ref_nes_load_rom": (I, [P, P, U, P, U]), "ref_nes_reset_all": (I, [P, I]),
               "ref_nes_run_frame_all": (I, [P]), "ref_nes_run_frames_all": (I, [P, I]),
               "ref_nes_set_buttons": (I, [P, P, I]), "ref_nes_get_ram": (I, [P, P]),
               "ref_nes_get_obs": (I, [P, P]), "ref_nes_get_framebuffers": (I, [P, P]),
               "ref_nes_reset_selected": (I, [P, P, I]), "ref_nes_get_scalars": (I, [P, I, P])}
        for k, (r, a) in sig.items():
            getattr(self.lib, k).restype, getattr(self.lib, k).argtypes = r, a
        self.n = n
        self.h = self.lib.ref_nes_create(n)
        if not self.h:
            raise RuntimeError("NESBatchGpu construction failed")

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.ref_nes_destroy(self.h)
            self.h = None

    def _ok(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"reference {what} failed")

    def load_rom(self, prg: bytes, chr_rom: bytes):
        self._prg = np.frombuffer(prg, np.uint8).copy()
        self._chr = np.frombuffer(chr_rom, np.uint8).copy()
        self._ok(self.lib.ref_nes_load_rom(self.h, _ptr(self._prg), len(prg), _ptr(self._chr), len(chr_rom)),
                 "load_rom")

    def reset_all(self, mirroring: int = 0):
        self._ok(self.lib.ref_nes_reset_all(self.h, mirroring), "reset_all")

    def run_frame_all(self):
        self._ok(self.lib.ref_nes_run_frame_all(self.h), "run_frame_all")

    def run_frames_all(self, k: int):
        self._ok(self.lib.ref_nes_run_frames_all(self.h, k), "run_frames_all")

    def set_buttons_batch(self, buttons):
        b = np.ascontiguousarray(buttons, np.uint8)
        self._ok(self.lib.ref_nes_set_buttons(self.h, _ptr(b), len(b)), "set_buttons_batch")

    def get_ram_batch(self) -> np.ndarray:
        out = np.empty((self.n, 2048), np.uint8)
        self._ok(self.lib.ref_nes_get_ram(self.h, _ptr(out)), "get_ram_batch")
        return out

    def get_obs_batch(self) -> np.ndarray:
        out = np.empty((self.n, 84, 84), np.uint8)
        self._ok(self.lib.ref_nes_get_obs(self.h, _ptr(out)), "get_obs_batch")
        return out

    def get_framebuffers(self) -> np.ndarray:
        out = np.empty((self.n, 240, 256), np.uint32)
        self._ok(self.lib.ref_nes_get_framebuffers(self.h, _ptr(out)), "get_framebuffers")
        return out

    def reset_selected(self, mask):
        m = np.ascontiguousarray(mask, np.uint8)
        self._ok(self.lib.ref_nes_reset_selected(self.h, _ptr(m), len(m)), "reset_selected")

    def scalars(self) -> np.ndarray:
        """[n, 27] in the order of SCALARS[:27] (the controller fields read 0)."""
        out = np.empty((self.n, 27), np.int64)
        for i in range(self.n):
            self._ok(self.lib.ref_nes_get_scalars(self.h, i, _ptr(out[i])), "get_state")
        return out
