"""Golden vectors of the reference's own batched NES emulator on synthetic
cartridges, and the check that the CPU oracle reproduces them.

Runs on a machine with a GPU and oracle/_ref/libnes_ref.so (the reference's
NESBatchGpu and kernels, built by oracle/build_ref.py).  For every cartridge of
``CARTS`` it drives the reference and the oracle through the same schedule
(reset_all, buttons, single rendered frames, 4-frame steps, reset_selected),
compares RAM, CPU/PPU registers, RGBA framebuffers and 84 x 84 observations,
and stores the reference's results in tests/golden/nes_ref.npz:

    python tests/golden/make_nes_golden.py [OUT]

Instances whose program ran an OAM DMA from a page >= 8 (the reference then
copies from memory past the instance's RAM) are excluded; the oracle counts
those in dma_far.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.nes import OracleNES, RefNESBatch, SCALARS, palette_rgba  # noqa: E402
from rl_for_mario_b200.nes_roms import demo_rom, random_rom  # noqa: E402

N = 6
CARTS = {
    "demo32": lambda: demo_rom(0x8000, 0),
    "demo16v": lambda: demo_rom(0x4000, 1),
    **{f"rand{s}": (lambda s=s: random_rom(s, True)) for s in range(8)},
    **{f"raw{s}": (lambda s=s: random_rom(100 + s, False)) for s in range(2)},
}
# (op, arg): "b" buttons per instance, "f" one rendered frame, "k" k frames, "r" reset_selected mask
def schedule(seed: int):
    rng = np.random.default_rng(seed)
    ops = [("b", rng.integers(0, 256, N, dtype=np.uint8))]
    ops += [("f", 1)] * 3
    for _ in range(5):
        ops += [("b", rng.choice(np.array([0, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40, 0x08], np.uint8), N)),
                ("k", 4)]
    ops += [("r", (rng.random(N) < 0.5).astype(np.uint8)), ("b", rng.integers(0, 256, N, dtype=np.uint8)),
            ("k", 4), ("k", 2)]
    return ops


def fb_sha(rgba: np.ndarray) -> np.ndarray:
    return np.array([int.from_bytes(hashlib.sha256(f.tobytes()).digest()[:8], "little") for f in rgba], np.uint64)


def run(out_path: Path) -> int:
    pal = palette_rgba()
    golden, bad = {}, 0
    for ci, (name, make) in enumerate(CARTS.items()):
        prg, chr_rom, mir = make()
        ref = RefNESBatch(N)
        ref.load_rom(prg, chr_rom)
        ref.reset_all(mir)
        ora = OracleNES(N, prg, chr_rom, mir)
        ora.reset()
        for op, arg in schedule(ci):
            if op == "b":
                ref.set_buttons_batch(arg)
                ora.set_buttons(arg)
            elif op == "f":
                ref.run_frame_all()
                ora.run_frames(1)
            elif op == "k":
                ref.run_frames_all(arg)
                ora.run_frames(arg)
            else:
                ref.reset_selected(arg)
                ora.reset(arg)
        ram, obs, rgba, sc = ref.get_ram_batch(), ref.get_obs_batch(), ref.get_framebuffers(), ref.scalars()
        del ref
        os_ = ora.scalars()
        keep = os_["dma_far"] == 0
        o_sc = np.stack([os_[k] for k in SCALARS[:27]], 1)
        cols = [i for i, k in enumerate(SCALARS[:27]) if not k.startswith("joypad")]
        o_rgba = pal[ora.framebuffer()]
        o_obs = ora.obs()
        checks = {
            "ram": np.array_equal(ram[keep], ora.ram()[keep]),
            "scalars": np.array_equal(sc[keep][:, cols], o_sc[keep][:, cols]),
            "framebuffer": np.array_equal(rgba[keep], o_rgba[keep]),
            "obs_max_diff": int(np.abs(obs[keep].astype(int) - o_obs[keep].astype(int)).max(initial=0)),
            "obs_diff_frac": float((obs[keep] != o_obs[keep]).mean()) if keep.any() else 0.0,
        }
        ok = checks["ram"] and checks["scalars"] and checks["framebuffer"] and checks["obs_max_diff"] <= 1
        bad += 0 if ok else 1
        print(name, "kept", int(keep.sum()), "of", N, checks, "OK" if ok else "MISMATCH", flush=True)
        if not ok:
            for i in np.nonzero(keep)[0]:
                d = [SCALARS[c] for c in cols if sc[i, c] != o_sc[i, c]]
                if d or not np.array_equal(ram[i], ora.ram()[i]):
                    print("  instance", i, "scalars differ:", {k: (int(sc[i, SCALARS.index(k)]),
                                                                  int(o_sc[i, SCALARS.index(k)])) for k in d},
                          "ram diff bytes:", int((ram[i] != ora.ram()[i]).sum()))
        golden[f"{name}/keep"] = keep
        golden[f"{name}/ram"] = ram
        golden[f"{name}/scalars"] = sc
        golden[f"{name}/obs"] = obs
        golden[f"{name}/fb_sha"] = fb_sha(rgba)
    np.savez_compressed(out_path, **golden)
    return bad


if __name__ == "__main__":
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else ROOT / "tests" / "golden" / "nes_ref.npz"
    sys.exit(1 if run(out) else 0)
