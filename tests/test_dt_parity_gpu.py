"""DT action-logit parity at the workload shapes, against the reference itself.

Fixtures (tests/golden/make_golden.py, run on the unmodified reference):

* ``dt_cfg1``: the repo-default DT (hidden 256, 4 layers, 8/2 heads), 64
  samples x 64 timesteps with left padding U{0..32}: 4,096 state-token rows;
* ``dt_cfg4``: the large DT shape (hidden 768, 12 layers, 12/4 heads,
  head_dim 64), 4 samples x 256 timesteps (768 tokens), padding U{0..128};
* ``dt_rollout``: a 252-token trajectory (84 timesteps, no padding) of the
  repo-default DT for 16 environments: 1,344 rows, replayed step by step
  through the cached rollout with the fixture's actions.

Each fixture holds three executions of the reference: float32, float32 on
the bf16-rounded weights, and the reference's own bfloat16 run
(``model.to(torch.bfloat16)``), plus the distance between that bf16 run and
the same bf16 run done one sample at a time.  That last figure is the
reproducibility floor of bf16 logits: at cfg1 the reference moves by 2.7e-2
max-abs (99.93 % identical argmax) against itself, so no bf16 implementation
can be held to a tighter max-abs bound than that.

Bounds asserted here:
* float32 models (fp32 kernels): max-abs <= 1e-5 against the fp32 reference
  and every argmax identical;
* bfloat16 models (default and fused blocks): against the fp32 reference, as
  close as the reference's own bf16 run is (mean-abs within 10 %, max-abs
  within 25 %, argmax agreement within 0.6 points: these are statistics of
  rounding noise, not identities);
* bfloat16 models at the reference's rounding points
  (``MarioDT.reference_rounding()``): the same bounds; their distance to the
  reference's own bf16 run is reported.
The measured figures are printed on one ``PARITY`` line per case.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.dt_ref import dt_param_shapes
from oracle.seeded import checksum, dt_synthetic_inputs, seeded_state_dict

GOLD = Path(__file__).resolve().parent / "golden"


def _load(name):
    return dict(np.load(GOLD / f"{name}.npz"))


def _cfgd(g):
    return {k[4:]: (tuple(v.tolist()) if v.ndim else v.item()) for k, v in g.items() if k.startswith("cfg_")}


def _model(g, dtype, fused=False, refround=False):
    from rl_for_mario_b200.dt_model import DTConfig, MarioDT

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    cfgd = _cfgd(g)
    model = MarioDT(DTConfig(**cfgd, dropout=0.0))
    sd = seeded_state_dict(dt_param_shapes(cfgd), int(g["seed"]))
    assert abs(sum(checksum(sd[k]) for k in sorted(sd)) - float(g["w_checksum"])) < 1e-6 * abs(float(g["w_checksum"]))
    model.load_state_dict(sd, strict=True)
    model = model.cuda().to(dtype).eval()
    if fused:
        model.fuse_norms()
    if refround:
        model.reference_rounding()
    return model


def _inputs(name, g):
    cfgd = _cfgd(g)
    inp = dt_synthetic_inputs(name, int(g["seed"]), int(g["B"]), int(g["T"]), cfgd["state_shape"], cfgd["act_dim"],
                              int(g["pad_max"]))
    assert checksum(inp["states"].float()) == pytest.approx(float(g["states_checksum"]), rel=1e-12)
    np.testing.assert_array_equal(inp["actions"].numpy(), g["actions"])
    return {k: v.cuda() for k, v in inp.items()}


def _stats(out, ref):
    d = (out - ref).abs()
    return {"maxabs": float(d.max()), "meanabs": float(d.mean()),
            "agree": float((out.argmax(-1) == ref.argmax(-1)).float().mean()), "rows": int(ref[..., 0].numel())}


def _report(case, out, g):
    out = out.float().cpu()
    rep = {"case": case,
           "vs_f32": _stats(out, torch.from_numpy(g["logits"])),
           "vs_f32_bf16w": _stats(out, torch.from_numpy(g["logits_f32_bf16w"])),
           "vs_ref_bf16": _stats(out, torch.from_numpy(g["logits_bf16"])),
           "ref_bf16_vs_f32": _stats(torch.from_numpy(g["logits_bf16"]), torch.from_numpy(g["logits"])),
           "ref_bf16_self": {"maxabs": float(g["bf16_self_maxabs"]), "meanabs": float(g["bf16_self_meanabs"]),
                             "agree": float(g["bf16_self_agree"])}}
    print("PARITY " + json.dumps(rep))
    return rep


def _check_bf16(rep):
    ours, refs = rep["vs_f32"], rep["ref_bf16_vs_f32"]
    assert ours["meanabs"] <= 1.1 * refs["meanabs"], rep
    assert ours["maxabs"] <= 1.25 * refs["maxabs"], rep
    assert ours["agree"] >= refs["agree"] - 0.006, rep


def _check_refround(rep):
    """At the reference's rounding points (RoPE rounded per op, frames / 255 rounded,
    unfused blocks) the bf16 model is as close to fp32 as the reference's bf16 run
    is.  It moves closer to that run (cfg1: 6.7e-3 mean-abs, 99.37 % argmax, against
    8.1e-3 / 99.12 % for the default path) but does not reproduce it: the CPU
    attention kernel the reference's bf16 run uses rounds in an order that is not
    documented (an fp32 softmax with bf16 probabilities matches its outputs on
    92 % of elements only), so no identity is asserted against it."""
    _check_bf16(rep)


def _check_f32(rep):
    assert rep["vs_f32"]["maxabs"] <= 1e-5, rep
    assert rep["vs_f32"]["agree"] == 1.0, rep


def _forward_logits(model, inp, chunk=16):
    outs = []
    B = inp["states"].shape[0]
    with torch.no_grad():
        for b0 in range(0, B, chunk):
            sl = slice(b0, b0 + chunk)
            o = model(inp["states"][sl], inp["actions"][sl], inp["rtg"][sl], inp["timesteps"][sl],
                      attention_mask=inp["mask"][sl] if "mask" in inp else None)
            outs.append(o.action_logits.float())
    return torch.cat(outs)


MODES = ["fp32", "bf16", "bf16_fused", "bf16_refround"]
CHECKS = {"fp32": _check_f32, "bf16": _check_bf16, "bf16_fused": _check_bf16, "bf16_refround": _check_refround}


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["dt_cfg1", "dt_cfg4"])
@pytest.mark.parametrize("mode", MODES)
def test_dt_logits_against_reference(name, mode):
    g = _load(name)
    dtype = torch.float32 if mode == "fp32" else torch.bfloat16
    model = _model(g, dtype, fused=(mode == "bf16_fused"), refround=(mode == "bf16_refround"))
    inp = _inputs(name, g)
    rep = _report(f"{name}/{mode}", _forward_logits(model, inp), g)
    CHECKS[mode](rep)


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
def test_cached_rollout_against_reference(mode):
    """Step t of the cached rollout appends (a_{t-1}, R_t, s_t) and yields the
    logits of s_t; with the fixture's actions fed back, every step must give the
    reference's full-forward logits of that state token."""
    from rl_for_mario_b200.rollout import DTRollout

    g = _load("dt_rollout")
    dtype = torch.float32 if mode == "fp32" else torch.bfloat16
    model = _model(g, dtype, fused=(mode == "bf16_fused"), refround=(mode == "bf16_refround"))
    inp = _inputs("dt_rollout", g)
    B, T = int(g["B"]), int(g["T"])
    ro = DTRollout(model, num_envs=B, max_steps=T, page_size=64)
    logits = torch.empty(B, T, 7, device="cuda")
    for t in range(T):
        _, lg = ro.step(inp["states"][:, t], inp["rtg"][:, t], inp["timesteps"][:, t])
        logits[:, t] = lg
        ro.prev_action = inp["actions"][:, t]  # teacher forcing: the fixture's action a_t
    assert ro.cache.length == 3 * T - 1
    rep = _report(f"dt_rollout/{mode}", logits, g)
    CHECKS[mode](rep)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_swap_into_model_with_reference_attention(dtype):
    """The drop-in path a maintainer gets: a DT whose blocks hold the reference's
    attention module (same parameter names and forward contract) has it replaced
    by FastDTAttention with swap_attention(); the unfused projections, in-kernel
    RoPE and the prefill kernels then run.  fp32: the dt_small and cfg1 logits
    within 1e-5; bf16: cfg1 logits at the bf16 bounds above."""
    from oracle.attention_ref import ReferenceAttention
    from rl_for_mario_b200.attention import FastDTAttention, swap_attention

    for name in (["dt_small", "dt_cfg1"] if dtype == torch.float32 else ["dt_cfg1"]):
        g = _load(name)
        model = _model(g, dtype)
        cfg = model.config
        for layer in model.model.layers:
            ref_attn = ReferenceAttention(cfg).to(device="cuda", dtype=dtype)
            ref_attn.load_state_dict(layer.self_attn.state_dict())
            layer.self_attn = ref_attn
        assert swap_attention(model, cfg) == cfg.num_hidden_layers
        assert all(isinstance(layer.self_attn, FastDTAttention) for layer in model.model.layers)
        if name == "dt_small":
            inp = {k: torch.from_numpy(g[k]).cuda() for k in ("actions", "rtg", "timesteps")}
            from oracle.seeded import seeded_uniform_int

            B, T = int(g["B"]), int(g["T"])
            inp["states"] = seeded_uniform_int((B, T + int(g["decode_steps"]), *cfg.state_shape), 0, 256,
                                               int(g["seed"]), "dt_small:states").to(torch.uint8).cuda()
            inp = {k: v[:, :T] for k, v in inp.items()}
            inp["mask"] = (torch.arange(T)[None] >= torch.from_numpy(g["pad_steps"]).long()[:, None]).long().cuda()
            out = _forward_logits(model, inp).cpu()
            err = (out - torch.from_numpy(g["logits"])).abs().max().item()
            assert err <= 1e-5, err
            continue
        rep = _report(f"{name}/swap_{str(dtype)[6:]}", _forward_logits(model, _inputs(name, g)), g)
        (_check_f32 if dtype == torch.float32 else _check_bf16)(rep)
