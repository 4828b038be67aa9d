"""Generates the golden vectors that pin the oracle to the reference.

Runs the UNMODIFIED reference modules from a checkout of FujiM3/RL_for_Mario
(the directory named by $RL_FOR_MARIO_REF) on the CPU with seeded weights
(oracle/seeded.py) and writes tests/golden/*.npz.  The fixtures store
outputs (and the small inputs); weights and frames are regenerated from their
seeds by the tests, with checksums stored to detect drift.

    RL_FOR_MARIO_REF=<checkout> python tests/golden/make_golden.py [case ...]

The DT-level cases also record the reference's own bfloat16 execution
(``model.to(torch.bfloat16)``) and its float32 execution on the
bfloat16-rounded weights, so bf16 implementations are compared with the same
model the reference would run in bf16.

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
if not os.environ.get("RL_FOR_MARIO_REF"):
    sys.exit("set RL_FOR_MARIO_REF to a checkout of FujiM3/RL_for_Mario (the reference whose outputs are pinned)")
REF = Path(os.environ["RL_FOR_MARIO_REF"])
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF))

from oracle.dt_ref import dt_param_shapes  # noqa: E402
from oracle.seeded import (  # noqa: E402
    checksum,
    dt_synthetic_inputs,
    seeded_normal,
    seeded_state_dict,
    seeded_uniform,
    seeded_uniform_int,
)

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


def _ref_model(cfgd, seed, dtype=torch.float32, round_bf16=False):
    """The reference MarioDecisionTransformer with seeded weights, in eval mode.
    round_bf16: the weights are first rounded to bfloat16 (fp32 arithmetic on
    the bf16 model's weights)."""
    cfg = DecisionTransformerConfig(**cfgd, dropout=0.0)
    model = MarioDecisionTransformer(cfg).eval()
    shapes = dt_param_shapes(cfgd)
    assert sorted(n for n, _ in shapes) == sorted(dict(model.named_parameters())), "param list drift"
    sd = seeded_state_dict(shapes, seed)
    if round_bf16:
        sd = {k: v.bfloat16().float() for k, v in sd.items()}
    model.load_state_dict(sd, strict=True)
    return model.to(dtype), sd


def _ref_forward(model, inp, sl=slice(None), mask=True):
    with torch.no_grad():
        o = model(states=inp["states"][sl], actions=inp["actions"][sl], returns_to_go=inp["rtg"][sl],
                  timesteps=inp["timesteps"][sl], attention_mask=inp["mask"][sl] if mask and "mask" in inp else None)
    return o.action_logits.float(), o.value_preds.float()


def _agree(a, b):
    return float((a.argmax(-1) == b.argmax(-1)).float().mean())


def dt_precision_case(name, seed, cfgd, B, T, pad_max):
    """One DT workload in three executions of the reference: float32, float32 on
    the bf16-rounded weights, and the reference's own bfloat16 (model.to(bf16)).
    Also records how far the reference's bf16 execution moves against itself
    when the same samples run one at a time instead of as one batch (the GEMM
    and convolution blockings, hence the fp32 accumulation orders, change):
    the reproducibility floor of bf16 logits."""
    inp = dt_synthetic_inputs(name, seed, B, T, cfgd["state_shape"], cfgd["act_dim"], pad_max)
    m32, sd = _ref_model(cfgd, seed)
    l32, v32 = _ref_forward(m32, inp)
    m32w, _ = _ref_model(cfgd, seed, round_bf16=True)
    l32w, v32w = _ref_forward(m32w, inp)
    m16, _ = _ref_model(cfgd, seed, dtype=torch.bfloat16)
    l16, v16 = _ref_forward(m16, inp)
    # The same bf16 forward, one sample at a time (batch 1, as a single
    # environment's act() runs it): other GEMM / convolution blockings.
    l16s = torch.cat([_ref_forward(m16, inp, slice(i, i + 1))[0] for i in range(B)])
    out = {"seed": seed, "B": B, "T": T, "pad_max": np.int32(pad_max),
           "states_checksum": np.float64(checksum(inp["states"].float())),
           "w_checksum": np.float64(sum(checksum(sd[k]) for k in sorted(sd))),
           "actions": inp["actions"].numpy(), "rtg": inp["rtg"].numpy(), "timesteps": inp["timesteps"].numpy(),
           "logits": l32.numpy(), "values": v32.numpy(),
           "logits_f32_bf16w": l32w.numpy(), "values_f32_bf16w": v32w.numpy(),
           "logits_bf16": l16.numpy(), "values_bf16": v16.numpy(),
           "bf16_self_maxabs": np.float32((l16 - l16s).abs().max()),
           "bf16_self_meanabs": np.float32((l16 - l16s).abs().mean()),
           "bf16_self_agree": np.float32(_agree(l16, l16s))}
    if "pad_steps" in inp:
        out["pad_steps"] = inp["pad_steps"].numpy().astype(np.int32)
    for k, v in cfgd.items():
        out["cfg_" + k] = np.asarray(v)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    d = lambda a, b: (float((a - b).abs().max()), float((a - b).abs().mean()), _agree(a, b))  # noqa: E731
    print(name, "rows", B * T, "| bf16 vs f32", d(l16, l32), "| bf16 vs f32(bf16 w)", d(l16, l32w),
          "| f32(bf16 w) vs f32", d(l32w, l32), "| bf16 self", d(l16, l16s))


CFG1 = dict(state_shape=(4, 84, 84), act_dim=7, max_ep_len=4096, context_len=64, hidden_size=256,
            num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2, rms_norm_eps=1e-5, rope_theta=1e4)
CFG4 = dict(CFG1, context_len=256, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
            num_key_value_heads=4)
# cfg3's 252-token rollout window needs context_len >= 84.
CFG3 = dict(CFG1, context_len=84)


CASES = {
    "attn": lambda: [
        attn_case("attn_d32_mask", 256, 8, 2, B=3, S=24, pads=[0, 6, 15], seed=11, decode_new=3),
        attn_case("attn_d32_nomask", 256, 8, 2, B=2, S=24, pads=None, seed=12, decode_new=1),
        attn_case("attn_d32_decmask", 256, 8, 2, B=3, S=21, pads=[0, 3, 12], seed=13, decode_new=3,
                  decode_mask=True),
        attn_case("attn_d64_mask", 768, 12, 4, B=2, S=30, pads=[0, 9], seed=14, decode_new=3),
        attn_case("attn_d32_long", 256, 8, 2, B=2, S=150, pads=[0, 96], seed=15)],
    "dt_small": lambda: dt_case(
        "dt_small", seed=21,
        cfgd=dict(state_shape=(4, 84, 84), act_dim=7, max_ep_len=4096, context_len=8, hidden_size=128,
                  num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=1, rms_norm_eps=1e-5,
                  rope_theta=1e4), B=2, T=7, pad_steps=[0, 3], decode_steps=1),
    "rmsnorm": lambda: rmsnorm_case("rmsnorm", seed=31),
    "rope": lambda: rope_case("rope_tables"),
    # Repo-default DT at the cfg1 shapes (hidden 256, 4 layers, 8/2 heads, 64
    # timesteps, left padding U{0..32}), 64 samples = 4096 state-token rows.
    "dt_cfg1": lambda: dt_precision_case("dt_cfg1", seed=0, cfgd=CFG1, B=64, T=64, pad_max=32),
    # The cfg4 model shape (hidden 768, 12 layers, 12/4 heads, head_dim 64,
    # 256 timesteps = 768 tokens, left padding U{0..128}) at 4 samples.
    "dt_cfg4": lambda: dt_precision_case("dt_cfg4", seed=3, cfgd=CFG4, B=4, T=256, pad_max=128),
    # A 252-token rollout trajectory at the cfg3 model shape (no padding): the
    # logits of every state token of the full forward are what a cached
    # rollout must reproduce step by step (teacher-forced actions).
    "dt_rollout": lambda: dt_precision_case("dt_rollout", seed=2, cfgd=CFG3, B=16, T=84, pad_max=-1),
}


def main():
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    names = sys.argv[1:] or list(CASES)
    for n in names:
        CASES[n]()


if __name__ == "__main__":
    main()
