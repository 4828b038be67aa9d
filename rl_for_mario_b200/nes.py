"""Batched NES emulation on this library's sm_100a kernels: drop-in for the
reference's ``nes_gpu`` extension (``NESBatchGpu``,
``nes_emulator_gpu/src/python/nes_gpu_py.cu:28-145``) and its vectorised Mario
environment (``GpuMarioVecEnv``, ``scripts/mario/gpu_vec_env.py:165-404``).

``NESBatchGpu`` keeps the reference's method names, argument meanings and
numpy return values (host copies, as the reference returns).  ``GpuMarioVecEnv``
keeps ``reset()`` / ``step(actions)``; ``step_device(actions)`` does the same
step with device tensors in and out and no host synchronisation, so the frames
it returns can feed the Decision Transformer's state encoder directly.

The emulator state lives in device memory owned by this object (torch
allocations); every kernel call goes through the C ABI (``include/dt_attn.h``,
``dt_nes_*``).  There is no CPU path: without the CUDA library these classes
raise.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple, Union

import numpy as np
import torch

from . import _lib

MIRROR_HORIZONTAL, MIRROR_VERTICAL, MIRROR_SINGLE_A, MIRROR_SINGLE_B, MIRROR_FOUR_SCREEN = range(5)
SIMPLE_MOVEMENT_BITMASK = np.array([0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40], np.uint8)
NUM_ACTIONS = 7
BOOT_FRAMES_TOTAL, BOOT_FRAMES_SETTLE, START_BTN = 286, 250, 0x08

# NES palette (RGBA32 as the reference's NES_PALETTE_CONST, ppu_device.cuh), 64 colours x 4
_PALETTE = np.array([
    0xFF666666, 0xFF002A88, 0xFF1412A7, 0xFF3B00A4, 0xFF5C007E, 0xFF6E0040, 0xFF6C0600, 0xFF561D00,
    0xFF333500, 0xFF0B4800, 0xFF005200, 0xFF004F08, 0xFF00404D, 0xFF000000, 0xFF000000, 0xFF000000,
    0xFFADADAD, 0xFF155FD9, 0xFF4240FF, 0xFF7527FE, 0xFFA01ACC, 0xFFB71E7B, 0xFFB53120, 0xFF994E00,
    0xFF6B6D00, 0xFF388700, 0xFF0C9300, 0xFF008F32, 0xFF007C8D, 0xFF000000, 0xFF000000, 0xFF000000,
    0xFFFFFEFF, 0xFF64B0FF, 0xFF9290FF, 0xFFC676FF, 0xFFF36AFF, 0xFFFE6ECC, 0xFFFE8170, 0xFFEA9E22,
    0xFFBCBE00, 0xFF88D800, 0xFF5CE430, 0xFF45E082, 0xFF48CDDE, 0xFF4F4F4F, 0xFF000000, 0xFF000000,
    0xFFFFFEFF, 0xFFC0DFFF, 0xFFD3D2FF, 0xFFE8C8FF, 0xFFFBC2FF, 0xFFFEC4EA, 0xFFFECCC5, 0xFFF7D8A5,
    0xFFE4E594, 0xFFCFEF96, 0xFFBDF4AB, 0xFFB3F3CC, 0xFFB5EBF2, 0xFFB8B8B8, 0xFF000000, 0xFF000000,
] * 4, np.uint32)

STATE_FIELDS = ("A", "X", "Y", "SP", "PC", "P", "total_cycles", "nmi_pending", "irq_pending", "joypad1",
                "joypad_shift", "joypad_strobe", "ctrl", "mask", "status", "oam_addr", "v", "t", "fine_x", "w",
                "read_buffer", "mirroring", "scanline", "cycle", "frame_ready", "nmi_flag",
                "active_sprite_count", "far_dma_count")


class _State(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in ("regs", "ram", "vram", "oam", "palette", "framebuffer")]


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(dev: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def load_nes_rom(path: Union[str, Path]) -> Tuple[bytes, bytes, int]:
    """iNES file -> (PRG, CHR, mirroring), as gpu_vec_env.py:_load_nes_rom."""
    data = Path(path).read_bytes()
    if data[:4] != b"NES\x1a":
        raise ValueError(f"{path} is not a valid iNES ROM (missing header magic)")
    prg_banks, chr_banks, flags6 = data[4], data[5], data[6]
    off = 16 + (512 if flags6 & 0x04 else 0)
    prg = data[off: off + prg_banks * 16384]
    chr_rom = data[off + prg_banks * 16384: off + prg_banks * 16384 + chr_banks * 8192]
    return bytes(prg), bytes(chr_rom), int(flags6 & 1)


class NESBatchGpu:
    """N NES instances in device memory; the reference's NESBatchGpu calls."""

    def __init__(self, num_instances: int, device: Optional[Union[int, str, torch.device]] = None):
        if num_instances < 1:
            raise ValueError("num_instances must be >= 1")
        if not torch.cuda.is_available():
            raise RuntimeError("NESBatchGpu needs a CUDA device (there is no CPU path)")
        self._lib = _lib.load()
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.n = num_instances
        g = (num_instances + 31) // 32
        z = lambda *shape: torch.zeros(*shape, dtype=torch.uint8, device=self.device)  # noqa: E731
        self.regs = z(g * 32, 48)
        self.ram = z(g, 2048, 32)
        self.vram = z(g, 2048, 32)
        self.oam = z(g, 256, 32)
        self.palette = z(g, 32, 32)
        self.framebuffer: Optional[torch.Tensor] = z(g, 240, 32, 32, 8)
        self.prg: Optional[torch.Tensor] = None
        self.chr: Optional[torch.Tensor] = None
        self._state = _State()
        self._sync_state()

    # ------------------------------------------------------------------ plumbing
    def _sync_state(self):
        s = self._state
        s.regs, s.ram, s.vram = self.regs.data_ptr(), self.ram.data_ptr(), self.vram.data_ptr()
        s.oam, s.palette = self.oam.data_ptr(), self.palette.data_ptr()
        s.framebuffer = self.framebuffer.data_ptr() if self.framebuffer is not None else None

    def _call(self, name: str, *args):
        rc = getattr(self._lib, name)(ctypes.byref(self._state), self.n, *args)
        _lib.check(name, rc)

    def _rom(self):
        if self.prg is None:
            raise RuntimeError("Call load_rom() first")
        return (_ptr(self.prg), self.prg.numel(), _ptr(self.chr), self.chr.numel())

    def _u8(self, a) -> torch.Tensor:
        if isinstance(a, torch.Tensor):
            t = a.to(device=self.device, dtype=torch.uint8)
        else:
            t = torch.from_numpy(np.ascontiguousarray(a, np.uint8)).to(self.device)
        if t.numel() < self.n:
            t = torch.cat([t.reshape(-1), torch.zeros(self.n - t.numel(), dtype=torch.uint8, device=self.device)])
        return t.reshape(-1)[: self.n].contiguous()

    # ------------------------------------------------------------------ reference API
    def load_rom(self, prg_data: bytes, chr_data: bytes) -> None:
        if len(prg_data) not in (0x4000, 0x8000) or len(chr_data) != 0x2000:
            raise ValueError("NROM cartridges only: PRG 16 or 32 KB, CHR 8 KB")
        self.prg = torch.frombuffer(bytearray(prg_data), dtype=torch.uint8).to(self.device)
        self.chr = torch.frombuffer(bytearray(chr_data), dtype=torch.uint8).to(self.device)

    def reset_all(self, mirroring: int = MIRROR_HORIZONTAL) -> None:
        self._call("dt_nes_reset", None, int(mirroring), *self._rom(), _stream(self.device))

    def run_frame_all(self) -> None:
        self.run_frames_all(1)

    def run_frames_all(self, num_frames: int) -> None:
        self._call("dt_nes_run_frames", int(num_frames), *self._rom(), _stream(self.device))

    def set_rendering_enabled(self, enabled: bool) -> None:
        if enabled and self.framebuffer is None:
            self.framebuffer = torch.zeros(self.ram.shape[0], 240, 32, 32, 8, dtype=torch.uint8, device=self.device)
        elif not enabled:
            self.framebuffer = None
        self._sync_state()

    def rendering_enabled(self) -> bool:
        return self.framebuffer is not None

    def set_buttons_batch(self, buttons) -> None:
        b = self._u8(buttons)
        self._call("dt_nes_set_buttons", _ptr(b), _stream(self.device))

    def get_obs_batch(self) -> np.ndarray:
        return self.obs_device().cpu().numpy()

    def get_ram_batch(self) -> np.ndarray:
        return self.ram_device().cpu().numpy()

    def reset_selected(self, done_mask) -> None:
        m = self._u8(done_mask)
        self._call("dt_nes_reset", _ptr(m), -1, *self._rom(), _stream(self.device))

    def get_framebuffers(self) -> np.ndarray:
        return _PALETTE[self.framebuffer_device().cpu().numpy()]

    def num_instances(self) -> int:
        return self.n

    # ------------------------------------------------------------------ device-side views
    def obs_device(self, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """[N, 84, 84] uint8 observation of the current framebuffers (device)."""
        if self.framebuffer is None:
            raise RuntimeError("Call set_rendering_enabled(True) before get_obs_batch()")
        if out is None:
            out = torch.empty(self.n, 84, 84, dtype=torch.uint8, device=self.device)
        self._call("dt_nes_observe", _ptr(out), None, 0, _stream(self.device))
        return out

    def ram_device(self) -> torch.Tensor:
        """[N, 2048] RAM in the reference's per-instance layout (a device copy)."""
        return self.ram.permute(0, 2, 1).reshape(-1, 2048)[: self.n]

    def framebuffer_device(self) -> torch.Tensor:
        """[N, 240, 256] palette values (a device copy)."""
        if self.framebuffer is None:
            raise RuntimeError("rendering is disabled")
        fb = self.framebuffer.permute(0, 3, 1, 2, 4).reshape(-1, 240, 256)
        return fb[: self.n]

    def memories_device(self):
        """(vram [N, 2048], oam [N, 256], palette [N, 32]) in per-instance layout."""
        f = lambda t, k: t.permute(0, 2, 1).reshape(-1, k)[: self.n]  # noqa: E731
        return f(self.vram, 2048), f(self.oam, 256), f(self.palette, 32)

    def get_state(self, instance_idx: int) -> Dict[str, int]:
        """Registers of one instance (NESBatchGpu::get_state)."""
        if not 0 <= instance_idx < self.n:
            raise IndexError("instance_idx out of range")
        return self.states()[instance_idx]

    def states(self) -> List[Dict[str, int]]:
        r = self.regs[: self.n].cpu().numpy().astype(np.int64)
        u16 = lambda i: r[:, i] | (r[:, i + 1] << 8)  # noqa: E731
        total = sum(r[:, 32 + k] << (8 * k) for k in range(8))
        cols = [r[:, 0], r[:, 1], r[:, 2], r[:, 3], u16(4), r[:, 6], total, r[:, 7], r[:, 8], r[:, 9], r[:, 10],
                r[:, 11], r[:, 12], r[:, 13], r[:, 14], r[:, 15], u16(16), u16(18), r[:, 20], r[:, 21], r[:, 22],
                r[:, 23], u16(24), u16(26), r[:, 28], r[:, 29], r[:, 30], r[:, 31]]
        return [dict(zip(STATE_FIELDS, (int(c[i]) for c in cols))) for i in range(self.n)]


class GpuMarioVecEnv:
    """The reference's GPU-vectorised Mario environment on NESBatchGpu above.

    ``rom``: an iNES path, or a ``(prg, chr, mirroring)`` tuple (the synthetic
    cartridges of ``nes_roms``); the reference's default is the SMB ROM from
    gym-super-mario-bros, which is not shipped here.
    """

    def __init__(self, num_envs: int = 1000, rom=None, frame_skip: int = 4, frame_stack: int = 4,
                 render: bool = True, device=None):
        if rom is None:
            raise FileNotFoundError("pass rom= (an iNES path or (prg, chr, mirroring))")
        prg, chr_rom, mirroring = load_nes_rom(rom) if isinstance(rom, (str, Path)) else rom
        self.num_envs, self.frame_skip, self.frame_stack = num_envs, frame_skip, frame_stack
        self._mirroring = mirroring
        self._batch = NESBatchGpu(num_envs, device)
        self._batch.load_rom(prg, chr_rom)
        self._batch.set_rendering_enabled(render)
        dev = self._batch.device
        self._device = dev
        i32 = lambda: torch.zeros(num_envs, dtype=torch.int32, device=dev)  # noqa: E731
        self._boot, self._prev_x, self._init_lives = i32(), i32(), i32()
        self._x_pos, self._lives = i32(), i32()
        self._reward = torch.zeros(num_envs, dtype=torch.float32, device=dev)
        self._done = torch.zeros(num_envs, dtype=torch.uint8, device=dev)
        self._flag = torch.zeros(num_envs, dtype=torch.uint8, device=dev)
        # [N, frame_stack, 84, 84], oldest first: the reference's frame ring, stacked
        self._stacked = torch.zeros(num_envs, frame_stack, 84, 84, dtype=torch.uint8, device=dev)
        self.observation_space_shape = (frame_stack, 84, 84)
        self.action_space_n = NUM_ACTIONS

    def _update(self):
        b = self._batch
        b._call("dt_nes_env_update", self.frame_skip, BOOT_FRAMES_TOTAL, _ptr(self._boot), _ptr(self._prev_x),
                _ptr(self._init_lives), _ptr(self._reward), _ptr(self._done), _ptr(self._x_pos),
                _ptr(self._lives), _ptr(self._flag), *b._rom(), _stream(b.device))

    def reset(self) -> torch.Tensor:
        b = self._batch
        b.reset_all(self._mirroring)
        self._boot.zero_()
        n = self.num_envs
        start = torch.full((n,), START_BTN, dtype=torch.uint8, device=self._device)
        none = torch.zeros(n, dtype=torch.uint8, device=self._device)
        for f in range(BOOT_FRAMES_TOTAL - BOOT_FRAMES_SETTLE):
            b.set_buttons_batch(start if f % 4 < 2 else none)
            b.run_frame_all()
        b.set_buttons_batch(none)
        b.run_frames_all(BOOT_FRAMES_SETTLE)
        obs = b.obs_device()
        self._stacked.copy_(obs[:, None].expand_as(self._stacked))
        ram = b.ram_device()
        self._prev_x.copy_(ram[:, 0x6D].int() * 256 + ram[:, 0x86].int())
        self._init_lives.copy_(ram[:, 0x75A].int())
        return self._stacked.clone()

    def step_device(self, actions: torch.Tensor):
        """One step on device: actions int64 [N] (device) -> (stacked obs
        [N, frame_stack, 84, 84] uint8 (this env's buffer: clone to keep), reward
        float32 [N], done uint8 [N], info dict of x_pos / lives / flag_get)."""
        b = self._batch
        a = actions.to(device=self._device, dtype=torch.int64).contiguous()
        b._call("dt_nes_set_actions", _ptr(a), _ptr(self._boot), BOOT_FRAMES_SETTLE, _stream(b.device))
        b.run_frames_all(self.frame_skip)
        b._call("dt_nes_observe", None, _ptr(self._stacked), self.frame_stack, _stream(b.device))
        self._update()
        info = {"x_pos": self._x_pos, "lives": self._lives, "flag_get": self._flag}
        return self._stacked, self._reward, self._done, info

    def step(self, actions) -> Tuple[torch.Tensor, np.ndarray, np.ndarray, List[Dict[str, Any]]]:
        """The reference's step: numpy actions -> (obs [N, stack, 84, 84] CUDA
        tensor, rewards float32 numpy, dones bool numpy, per-env info dicts)."""
        a = torch.as_tensor(np.asarray(actions, dtype=np.int64))
        obs, rew, done, info = self.step_device(a)
        x, lv, fl = (t.cpu().numpy() for t in (info["x_pos"], info["lives"], info["flag_get"]))
        infos = [{"x_pos": int(x[i]), "lives": int(lv[i]), "flag_get": bool(fl[i])} for i in range(self.num_envs)]
        return obs.clone(), rew.cpu().numpy(), done.cpu().numpy().astype(bool), infos

    def close(self) -> None:
        del self._batch


@torch.no_grad()
def run_policy(env: GpuMarioVecEnv, rollout, steps: int, target_return: float = 1.0,
               deterministic: bool = True, start_obs: Optional[torch.Tensor] = None):
    """Closed loop on the device, as the reference's batched rollout
    (trainer/train_ppo_finetune.py:397-437: policy -> actions for all
    environments -> environment step): the Decision Transformer's cached
    rollout (``rollout.DTRollout``) reads the environment's stacked frames,
    its actions step the emulators (``step_device``), and the new frames feed
    the next policy step -- no host round trip in between.  With the
    environments sharded over ranks (``env`` holds this rank's slice, the
    rollout gathers every rank's logits), each rank steps its emulators with
    its slice of the gathered actions.  Returns device tensors (actions,
    rewards, dones), each [steps, N] for this rank's N environments; the return-to-go
    falls by each step's reward, the timestep counts steps.  ``start_obs``:
    the frames of the first step (default: ``env.reset()``)."""
    n = env.num_envs
    dev = env._device
    obs = env.reset() if start_obs is None else start_obs
    rtg = torch.full((n,), float(target_return), dtype=torch.float32, device=dev)
    ts = torch.zeros(n, dtype=torch.long, device=dev)
    acts = torch.empty(steps, n, dtype=torch.long, device=dev)
    rews = torch.empty(steps, n, dtype=torch.float32, device=dev)
    dones = torch.empty(steps, n, dtype=torch.uint8, device=dev)
    rollout.reset()
    for t in range(steps):
        a, _ = rollout.step(obs, rtg, ts, deterministic=deterministic)
        a = a[rollout.lo:rollout.hi]
        obs, r, d, _ = env.step_device(a)
        acts[t], rews[t], dones[t] = a, r, d
        rtg -= r
        ts += 1
    return acts, rews, dones
