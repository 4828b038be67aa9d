"""GPU parity of the batched NES emulation kernels (dt_nes_*): bit-exact
against the CPU oracle (oracle/nes_oracle.c) on every byte of state, against
the reference's own emulator through its golden vectors
(tests/golden/nes_ref.npz), and the environment step against the oracle's
restatement of GpuMarioVecEnv.step."""
import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).parent / "golden"))


def _run_schedule(nes, ora, ops):
    for op, arg in ops:
        if op == "b":
            nes.set_buttons_batch(arg)
            if ora is not None:
                ora.set_buttons(arg)
        elif op in ("f", "k"):
            nes.run_frames_all(arg)
            if ora is not None:
                ora.run_frames(arg)
        else:
            nes.reset_selected(arg)
            if ora is not None:
                ora.reset(arg)


def _compare_full(nes, ora):
    from oracle.nes import SCALARS

    assert np.array_equal(nes.get_ram_batch(), ora.ram())
    vram, oam, pal = (t.cpu().numpy() for t in nes.memories_device())
    o_vram, o_oam, o_pal = ora.mem()
    assert np.array_equal(vram, o_vram)
    assert np.array_equal(oam, o_oam)
    assert np.array_equal(pal, o_pal)
    assert np.array_equal(nes.framebuffer_device().cpu().numpy(), ora.framebuffer())
    assert np.array_equal(nes.get_obs_batch(), ora.obs())
    sc = ora.scalars()
    st = nes.states()
    for k in SCALARS:
        mine = np.array([s["far_dma_count" if k == "dma_far" else k] for s in st])
        ref = np.minimum(sc[k], 255) if k == "dma_far" else sc[k]
        assert np.array_equal(mine, ref), k


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(12))
def test_frames_match_oracle_every_byte(ci):
    """The 12 cartridges and schedules of the golden vectors, 6 instances each:
    registers, RAM, VRAM, OAM, palette RAM, framebuffers and observations."""
    from make_nes_golden import CARTS, N, schedule
    from oracle.nes import OracleNES
    from rl_for_mario_b200.nes import NESBatchGpu

    name, make = list(CARTS.items())[ci]
    prg, chr_rom, mir = make()
    nes = NESBatchGpu(N)
    nes.load_rom(prg, chr_rom)
    nes.reset_all(mir)
    ora = OracleNES(N, prg, chr_rom, mir)
    ora.reset()
    _run_schedule(nes, ora, schedule(ci))
    _compare_full(nes, ora)


@pytest.mark.gpu
@pytest.mark.parametrize("ci", range(12))
def test_frames_match_reference_goldens(ci):
    """Against the reference's own NESBatchGpu results (RAM, registers, RGBA
    framebuffer digests, observations) on the instances it defines."""
    from make_nes_golden import CARTS, N, schedule
    from oracle.nes import SCALARS
    from rl_for_mario_b200.nes import NESBatchGpu

    g = np.load(Path(__file__).parent / "golden" / "nes_ref.npz")
    name, make = list(CARTS.items())[ci]
    prg, chr_rom, mir = make()
    nes = NESBatchGpu(N)
    nes.load_rom(prg, chr_rom)
    nes.reset_all(mir)
    _run_schedule(nes, None, schedule(ci))
    keep = g[f"{name}/keep"]
    assert np.array_equal(nes.get_ram_batch()[keep], g[f"{name}/ram"][keep])
    assert np.array_equal(nes.get_obs_batch()[keep], g[f"{name}/obs"][keep])
    sha = np.array([int.from_bytes(hashlib.sha256(f.tobytes()).digest()[:8], "little")
                    for f in nes.get_framebuffers()], np.uint64)
    assert np.array_equal(sha[keep], g[f"{name}/fb_sha"][keep])
    st = nes.states()
    for c, k in enumerate(SCALARS[:27]):
        if k.startswith("joypad"):
            continue
        assert np.array_equal(np.array([s[k] for s in st])[keep], g[f"{name}/scalars"][keep][:, c]), k


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 33, 517])
def test_ragged_batches_and_random_buttons(n):
    """Instance counts that are not multiples of the 32-instance group, and of
    the 128-instance CTA; every instance with its own buttons each step."""
    from oracle.nes import OracleNES
    from rl_for_mario_b200.nes import NESBatchGpu
    from rl_for_mario_b200.nes_roms import demo_rom

    prg, chr_rom, mir = demo_rom()
    nes = NESBatchGpu(n)
    nes.load_rom(prg, chr_rom)
    nes.reset_all(mir)
    ora = OracleNES(n, prg, chr_rom, mir)
    ora.reset()
    rng = np.random.default_rng(n)
    for step in range(6):
        b = rng.integers(0, 256, n, dtype=np.uint8)
        _run_schedule(nes, ora, [("b", b), ("k", 1 + step % 4)])
    _compare_full(nes, ora)


@pytest.mark.gpu
def test_rendering_disabled_and_single_frames():
    """Without a framebuffer nothing is drawn and sprite 0 never hits (the
    reference skips per-pixel work when it has no framebuffer)."""
    from oracle.nes import OracleNES
    from rl_for_mario_b200.nes import NESBatchGpu
    from rl_for_mario_b200.nes_roms import demo_rom

    prg, chr_rom, mir = demo_rom()
    nes = NESBatchGpu(40)
    nes.set_rendering_enabled(False)
    nes.load_rom(prg, chr_rom)
    nes.reset_all(mir)
    ora = OracleNES(40, prg, chr_rom, mir, render=False)
    ora.reset()
    b = np.full(40, 0x81, np.uint8)
    _run_schedule(nes, ora, [("b", b), ("f", 1), ("f", 1), ("k", 5)])
    assert np.array_equal(nes.get_ram_batch(), ora.ram())
    assert int(nes.get_ram_batch()[:, 0x11].max()) == 0  # no sprite 0 hits counted
    with pytest.raises(RuntimeError):
        nes.get_obs_batch()


@pytest.mark.gpu
def test_vec_env_matches_oracle_env():
    """GpuMarioVecEnv.reset / step against the oracle's restatement of the
    reference's environment: stacked frames, rewards, dones, infos, through
    deaths (B held), stage clears, auto-resets and the boot sequence."""
    from oracle.nes import OracleEnv
    from rl_for_mario_b200.nes import GpuMarioVecEnv
    from rl_for_mario_b200.nes_roms import demo_rom

    n = 16
    rom = demo_rom()
    env = GpuMarioVecEnv(n, rom=rom)
    ora = OracleEnv(n, *rom)
    o0 = env.reset()
    r0 = ora.reset()
    assert np.array_equal(o0.cpu().numpy(), r0)
    rng = np.random.default_rng(0)
    seen_done = seen_reset_done = 0
    for t in range(90):
        acts = rng.choice([1, 1, 2, 3, 4, 0, 6, 5], n)
        obs, rew, done, info = env.step(acts)
        r_obs, r_rew, r_done, r_info = ora.step(acts)
        assert np.array_equal(obs.cpu().numpy(), r_obs), t
        assert np.array_equal(rew, r_rew), t
        assert np.array_equal(done, r_done), t
        assert [i["x_pos"] for i in info] == r_info["x_pos"].tolist()
        assert [i["lives"] for i in info] == r_info["lives"].tolist()
        assert [i["flag_get"] for i in info] == r_info["flag_get"].tolist()
        seen_done += int(done.sum())
        seen_reset_done += int((ora.boot[done] == 286).all()) if done.any() else 0
    assert seen_done > 0


@pytest.mark.gpu
def test_step_device_keeps_everything_on_device():
    """step_device: device tensors in and out; the same results as step()."""
    from rl_for_mario_b200.nes import GpuMarioVecEnv
    from rl_for_mario_b200.nes_roms import demo_rom

    rom = demo_rom()
    a, b = GpuMarioVecEnv(40, rom=rom), GpuMarioVecEnv(40, rom=rom)
    a.reset(), b.reset()
    acts = torch.randint(0, 7, (40,), generator=torch.Generator().manual_seed(1))
    for _ in range(5):
        o1, r1, d1, i1 = a.step_device(acts.cuda())
        o2, r2, d2, _ = b.step(acts.numpy())
        assert o1.is_cuda and r1.is_cuda and d1.is_cuda and i1["x_pos"].is_cuda
        assert torch.equal(o1.cpu(), o2.cpu())
        assert np.array_equal(r1.cpu().numpy(), r2) and np.array_equal(d1.cpu().numpy().astype(bool), d2)


@pytest.mark.gpu
def test_bad_arguments_are_rejected():
    from rl_for_mario_b200._lib import DTKernelError
    from rl_for_mario_b200.kernels import device_status
    from rl_for_mario_b200.nes import GpuMarioVecEnv, NESBatchGpu
    from rl_for_mario_b200.nes_roms import demo_rom

    nes = NESBatchGpu(4)
    with pytest.raises(RuntimeError):
        nes.run_frames_all(1)  # no ROM
    with pytest.raises(ValueError):
        nes.load_rom(bytes(0x2000), bytes(0x2000))
    prg, chr_rom, _ = demo_rom()
    nes.load_rom(prg, chr_rom)
    with pytest.raises(DTKernelError):
        nes.reset_all(7)
    with pytest.raises(DTKernelError):
        nes.run_frames_all(0)
    env = GpuMarioVecEnv(4, rom=demo_rom())
    env.reset()
    env.step_device(torch.tensor([0, 1, 9, 2], device="cuda"))
    assert device_status() != 0


@pytest.mark.gpu
@pytest.mark.parametrize("graphs", [False, True])
def test_policy_loop_on_device_matches_oracle_env(graphs):
    """run_policy: the Decision Transformer's cached rollout reads the
    environment's frames and its actions step the emulators, all on the
    device.  The same policy driven by the oracle's environment (frames copied
    from the host) sees bit-identical frames, so it chooses the same actions at
    every step, and rewards and dones agree."""
    from oracle.dt_ref import dt_param_shapes
    from oracle.nes import OracleEnv
    from oracle.seeded import seeded_state_dict
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT
    from rl_for_mario_b200.nes import GpuMarioVecEnv, run_policy
    from rl_for_mario_b200.nes_roms import demo_rom
    from rl_for_mario_b200.rollout import DTRollout

    cfg = DTConfig(hidden_size=256, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
                   context_len=32, dropout=0.0)
    cfgd = {k: getattr(cfg, k) for k in ("state_shape", "act_dim", "max_ep_len", "context_len", "hidden_size",
                                         "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                                         "intermediate_size")}
    model = MarioDT(cfg)
    model.load_state_dict(seeded_state_dict(dt_param_shapes(cfgd), 4), strict=True)
    model = model.cuda().to(torch.bfloat16).eval()
    n, T = 16, 24
    rom = demo_rom()
    env = GpuMarioVecEnv(n, rom=rom)
    policy = DTRollout(model, n, T, page_size=16, graphs=graphs)
    acts, rews, dones = run_policy(env, policy, T, target_return=2.0)
    assert acts.is_cuda and rews.is_cuda and dones.is_cuda
    if graphs:
        # episode 2 captures one graph per step, episode 3 replays them: same decisions
        for _ in range(2):
            a2, r2, d2 = run_policy(env, policy, T, target_return=2.0)
            assert torch.equal(a2, acts) and torch.equal(r2, rews) and torch.equal(d2, dones)

    ora = OracleEnv(n, *rom)
    ro = DTRollout(model, n, T, page_size=16, graphs=graphs)
    obs = torch.from_numpy(ora.reset()).cuda()
    rtg = torch.full((n,), 2.0, device="cuda")
    ts = torch.zeros(n, dtype=torch.long, device="cuda")
    with torch.no_grad():
        for t in range(T):
            a, _ = ro.step(obs, rtg, ts)
            assert torch.equal(a, acts[t]), t
            o, r, d, _ = ora.step(a.cpu().numpy())
            assert np.array_equal(r, rews[t].cpu().numpy()) and np.array_equal(d, dones[t].cpu().numpy().astype(bool))
            obs = torch.from_numpy(o).cuda()
            rtg -= torch.from_numpy(r).cuda()
            ts += 1
    assert len(set(acts.flatten().tolist())) > 1  # the policy does not collapse to one action
