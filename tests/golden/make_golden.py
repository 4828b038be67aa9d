"""Generates the golden vectors that pin the oracle to the reference.

Runs the UNMODIFIED reference modules from a checkout of FujiM3/RL_for_Mario
(default /root/reference, or $RL_FOR_MARIO_REF) in float32 on the CPU with
seeded weights (oracle/seeded.py) and writes tests/golden/*.npz.  The
fixtures store inputs and outputs; weights are regenerated from their seed by
the tests, with a checksum stored to detect drift.

    python tests/golden/make_golden.py

Only this script reads the reference tree; the tests read the .npz files.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("RL_FOR_MARIO_REF", "/root/reference"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

from oracle.dt_ref import dt_param_shapes  # noqa: E402
from oracle.seeded import checksum, seeded_normal, seeded_state_dict, seeded_uniform, seeded_uniform_int  # noqa: E402

from model.model_decision_transformer import (  # noqa: E402
    DecisionTransformerAttention,
    DecisionTransformerConfig,
    MarioDecisionTransformer,
    RMSNorm,
    precompute_freqs_cis,
)


def attn_case(name, hidden, nh, nkv, B, S, pads, seed, decode_new=0, decode_mask=False):
    """Reference DecisionTransformerAttention on seeded weights / inputs."""
    cfg = DecisionTransformerConfig(hidden_size=hidden, num_attention_heads=nh, num_key_value_heads=nkv,
                                    context_len=max(64, (S + decode_new + 2) // 3 + 1), dropout=0.0)
    mod = DecisionTransformerAttention(cfg).eval()
    shapes = [(n, tuple(p.shape)) for n, p in mod.named_parameters()]
    sd = seeded_state_dict(shapes, seed)
    mod.load_state_dict(sd)
    D = hidden // nh
    cos, sin = precompute_freqs_cis(D, S + decode_new + 8, 1e4)
    x = seeded_normal((B, S, hidden), seed, name + ":x")
    out = {"hidden": hidden, "nh": nh, "nkv": nkv, "B": B, "S": S, "seed": seed,
           "x_checksum": np.float64(checksum(x)),
           "w_checksum": np.float64(sum(checksum(sd[k]) for k in sorted(sd)))}
    mask = None
    if pads is not None:
        pads_t = torch.tensor(pads, dtype=torch.int64)
        mask = (torch.arange(S)[None] >= pads_t[:, None]).float()
        out["pad_len"] = pads_t.numpy().astype(np.int32)
    with torch.no_grad():
        y, past = mod(x, (cos[:S], sin[:S]), past_key_value=None, use_cache=True, attention_mask=mask)
    out["out"] = y.numpy()
    out["past_k"] = past[0].numpy()
    out["past_v"] = past[1].numpy()
    if decode_new:
        xn = seeded_normal((B, decode_new, hidden), seed, name + ":xn")
        out["x_new_checksum"] = np.float64(checksum(xn))
        dmask = None
        if decode_mask:
            L = S + decode_new
            dmask = (torch.arange(L)[None] >= torch.tensor(pads)[:, None]).float()
        with torch.no_grad():
            yd, pd = mod(xn, (cos[S:S + decode_new], sin[S:S + decode_new]), past_key_value=past,
                         use_cache=True, attention_mask=dmask)
        out["dec_out"] = yd.numpy()
        out["dec_k"] = pd[0].numpy()
        out["dec_v"] = pd[1].numpy()
        out["decode_mask"] = np.int32(1 if decode_mask else 0)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, {k: getattr(v, "shape", v) for k, v in out.items() if k not in ("w_checksum",)})


def dt_case(name, seed, cfgd, B, T, pad_steps, decode_steps=0):
    """Reference MarioDecisionTransformer forward (and an optional cached step)."""
    cfg = DecisionTransformerConfig(**cfgd, dropout=0.0)
    model = MarioDecisionTransformer(cfg).eval()
    names = dict(model.named_parameters())
    shapes = dt_param_shapes(cfgd)
    assert sorted(n for n, _ in shapes) == sorted(names), "param list drift"
    sd = seeded_state_dict(shapes, seed)
    model.load_state_dict(sd, strict=True)
    Ttot = T + decode_steps
    states = seeded_uniform_int((B, Ttot, *cfgd["state_shape"]), 0, 256, seed, name + ":states").to(torch.uint8)
    actions = seeded_uniform_int((B, Ttot), 0, cfgd["act_dim"], seed, name + ":actions")
    rtg = seeded_uniform((B, Ttot), 0.0, 3000.0, seed, name + ":rtg")
    start = seeded_uniform_int((B, 1), 0, 4000, seed, name + ":start")
    timesteps = start + torch.arange(Ttot)[None]
    pads = torch.tensor(pad_steps, dtype=torch.int64)
    mask = (torch.arange(T)[None] >= pads[:, None]).long()
    with torch.no_grad():
        o = model(states=states[:, :T], actions=actions[:, :T], returns_to_go=rtg[:, :T],
                  timesteps=timesteps[:, :T], attention_mask=mask, use_cache=True)
    out = {"seed": seed, "B": B, "T": T, "pad_steps": pads.numpy().astype(np.int32),
           "states_checksum": np.float64(checksum(states.float())),
           "w_checksum": np.float64(sum(checksum(sd[k]) for k in sorted(sd))),
           "actions": actions.numpy(), "rtg": rtg.numpy(), "timesteps": timesteps.numpy(),
           "logits": o.action_logits.numpy(), "values": o.value_preds.numpy(),
           "hidden": o.last_hidden_state.numpy(), "loss": np.float32(o.loss.item()),
           "present0_k": o.past_key_values[0][0].numpy(), "present0_v": o.past_key_values[0][1].numpy()}
    for k, v in cfgd.items():
        out["cfg_" + k] = np.asarray(v)
    if decode_steps:
        # Cached continuation without a mask (the model rejects a [B, T_new] mask
        # on the cached path, :425-428 vs :238-242).
        with torch.no_grad():
            o0 = model(states=states[:, :T], actions=actions[:, :T], returns_to_go=rtg[:, :T],
                       timesteps=timesteps[:, :T], use_cache=True)
            o1 = model(states=states[:, T:], actions=actions[:, T:], returns_to_go=rtg[:, T:],
                       timesteps=timesteps[:, T:], past_key_values=o0.past_key_values, use_cache=True)
        out["nomask_logits"] = o0.action_logits.numpy()
        out["dec_logits"] = o1.action_logits.numpy()
        out["dec_hidden"] = o1.last_hidden_state.numpy()
        out["decode_steps"] = np.int32(decode_steps)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(name, {k: getattr(v, "shape", v) for k, v in out.items() if not k.startswith("cfg_")})


def rmsnorm_case(name, seed):
    x = seeded_normal((4, 10, 256), seed, name + ":x", 2.0)
    mod = RMSNorm(256, eps=1e-5)
    w = seeded_normal((256,), seed, name + ":w", 0.1, 1.0)
    mod.weight.data.copy_(w)
    with torch.no_grad():
        y = mod(x)
    np.savez_compressed(HERE / f"{name}.npz", x_checksum=np.float64(checksum(x)), out=y.numpy())
    print(name)


def rope_case(name):
    cos, sin = precompute_freqs_cis(32, 252, 1e4)
    cos64, sin64 = precompute_freqs_cis(64, 768, 1e4)
    # Every 7th row keeps the fixture small while covering the whole range.
    np.savez_compressed(HERE / f"{name}.npz", cos32=cos.numpy(), sin32=sin.numpy(), rows64=np.arange(0, 768, 7),
                        cos64=cos64[::7].numpy(), sin64=sin64[::7].numpy())
    print(name)


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    attn_case("attn_d32_mask", 256, 8, 2, B=3, S=24, pads=[0, 6, 15], seed=11, decode_new=3)
    attn_case("attn_d32_nomask", 256, 8, 2, B=2, S=24, pads=None, seed=12, decode_new=1)
    attn_case("attn_d32_decmask", 256, 8, 2, B=3, S=21, pads=[0, 3, 12], seed=13, decode_new=3, decode_mask=True)
    attn_case("attn_d64_mask", 768, 12, 4, B=2, S=30, pads=[0, 9], seed=14, decode_new=3)
    attn_case("attn_d32_long", 256, 8, 2, B=2, S=150, pads=[0, 96], seed=15)
    dt_case("dt_small", seed=21,
            cfgd=dict(state_shape=(4, 84, 84), act_dim=7, max_ep_len=4096, context_len=8, hidden_size=128,
                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=1, rms_norm_eps=1e-5,
                      rope_theta=1e4), B=2, T=7, pad_steps=[0, 3], decode_steps=1)
    rmsnorm_case("rmsnorm", seed=31)
    rope_case("rope_tables")


if __name__ == "__main__":
    main()
