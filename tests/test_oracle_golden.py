"""Pins the CPU oracle to golden vectors produced by the reference itself.

The fixtures (tests/golden/*.npz) were written by tests/golden/make_golden.py
running the unmodified reference modules in float32.  Weights and inputs are
regenerated here from their seeds; stored checksums guard against drift.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention_module_ref, precompute_freqs_cis, rmsnorm_ref
from oracle.dt_ref import dt_forward_ref, dt_param_shapes
from oracle.seeded import checksum, seeded_normal, seeded_state_dict, seeded_uniform, seeded_uniform_int

GOLD = Path(__file__).resolve().parent / "golden"
ATOL = 1e-5


def load(name):
    return dict(np.load(GOLD / f"{name}.npz"))


def attn_weights(g):
    H, nh, nkv = int(g["hidden"]), int(g["nh"]), int(g["nkv"])
    D = H // nh
    shapes = [("q_proj.weight", (nh * D, H)), ("k_proj.weight", (nkv * D, H)),
              ("v_proj.weight", (nkv * D, H)), ("o_proj.weight", (H, nh * D))]
    sd = seeded_state_dict(shapes, int(g["seed"]))
    assert sum(checksum(sd[k]) for k in sorted(sd)) == pytest.approx(float(g["w_checksum"]), rel=1e-12)
    return sd


@pytest.mark.parametrize("name", ["attn_d32_mask", "attn_d32_nomask", "attn_d32_decmask", "attn_d64_mask",
                                  "attn_d32_long"])
def test_attention_module_matches_reference(name):
    g = load(name)
    sd = attn_weights(g)
    H, nh, nkv, B, S, seed = (int(g[k]) for k in ("hidden", "nh", "nkv", "B", "S", "seed"))
    D = H // nh
    x = seeded_normal((B, S, H), seed, name + ":x")
    assert checksum(x) == pytest.approx(float(g["x_checksum"]), rel=1e-12)
    cos, sin = precompute_freqs_cis(D, S + 16, 1e4)
    mask = None
    if "pad_len" in g:
        mask = (torch.arange(S)[None] >= torch.from_numpy(g["pad_len"]).long()[:, None]).float()
    w = [sd[k] for k in ("q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight")]
    out, past = attention_module_ref(x, *w, nh, nkv, cos[:S], sin[:S], use_cache=True, attention_mask=mask)
    np.testing.assert_allclose(out.numpy(), g["out"], atol=ATOL, rtol=1e-5)
    np.testing.assert_allclose(past[0].numpy(), g["past_k"], atol=ATOL, rtol=1e-5)
    np.testing.assert_allclose(past[1].numpy(), g["past_v"], atol=ATOL, rtol=1e-5)
    if "dec_out" in g:
        n_new = g["dec_out"].shape[1]
        xn = seeded_normal((B, n_new, H), seed, name + ":xn")
        assert checksum(xn) == pytest.approx(float(g["x_new_checksum"]), rel=1e-12)
        dmask = None
        if int(g["decode_mask"]):
            dmask = (torch.arange(S + n_new)[None] >= torch.from_numpy(g["pad_len"]).long()[:, None]).float()
        dout, dpast = attention_module_ref(xn, *w, nh, nkv, cos[S:S + n_new], sin[S:S + n_new],
                                           past_key_value=past, use_cache=True, attention_mask=dmask)
        np.testing.assert_allclose(dout.numpy(), g["dec_out"], atol=ATOL, rtol=1e-5)
        np.testing.assert_allclose(dpast[0].numpy(), g["dec_k"], atol=ATOL, rtol=1e-5)
        np.testing.assert_allclose(dpast[1].numpy(), g["dec_v"], atol=ATOL, rtol=1e-5)


def test_padded_rows_are_prefix_means():
    """Reference semantics of a left-padded row q < pad: mean(V[0..q]) (fixture attn_d32_long, pad 96)."""
    g = load("attn_d32_long")
    sd = attn_weights(g)
    H, nh, nkv, B, S, seed = (int(g[k]) for k in ("hidden", "nh", "nkv", "B", "S", "seed"))
    x = seeded_normal((B, S, H), seed, "attn_d32_long:x")
    v = (x @ sd["v_proj.weight"].t()).view(B, S, nkv, H // nh)
    pad = int(g["pad_len"][1])
    means = torch.cumsum(v[1], dim=0) / torch.arange(1, S + 1).view(S, 1, 1)
    # out = o_proj(attn); recover attn rows through o_proj's pseudo-inverse is overkill:
    # compare the oracle's pre-o_proj output instead, then check the fixture through o_proj.
    from oracle import attention_prefill_ref
    q = (x @ sd["q_proj.weight"].t()).view(B, S, nh, -1)
    k = (x @ sd["k_proj.weight"].t()).view(B, S, nkv, -1)
    cos, sin = precompute_freqs_cis(H // nh, S, 1e4)
    mask = (torch.arange(S)[None] >= torch.from_numpy(g["pad_len"]).long()[:, None]).float()
    a = attention_prefill_ref(q, k, v, cos, sin, mask)
    r = nh // nkv
    for h in range(nh):
        np.testing.assert_allclose(a[1, :pad, h].numpy(), means[:pad, h // r].numpy(), atol=2e-6)
    y = a.reshape(B, S, -1) @ sd["o_proj.weight"].t()
    np.testing.assert_allclose(y.numpy(), g["out"], atol=ATOL, rtol=1e-5)


def test_rmsnorm_matches_reference():
    g = load("rmsnorm")
    x = seeded_normal((4, 10, 256), 31, "rmsnorm:x", 2.0)
    assert checksum(x) == pytest.approx(float(g["x_checksum"]), rel=1e-12)
    w = seeded_normal((256,), 31, "rmsnorm:w", 0.1, 1.0)
    np.testing.assert_allclose(rmsnorm_ref(x, w).numpy(), g["out"], atol=1e-6, rtol=1e-6)


def test_rope_tables_match_reference():
    g = load("rope_tables")
    c, s = precompute_freqs_cis(32, 252, 1e4)
    np.testing.assert_array_equal(c.numpy(), g["cos32"])
    np.testing.assert_array_equal(s.numpy(), g["sin32"])
    c, s = precompute_freqs_cis(64, 768, 1e4)
    np.testing.assert_array_equal(c[g["rows64"]].numpy(), g["cos64"])
    np.testing.assert_array_equal(s[g["rows64"]].numpy(), g["sin64"])


def _dt_inputs(g, name="dt_small"):
    cfg = {k[4:]: (tuple(v.tolist()) if v.ndim else v.item()) for k, v in g.items() if k.startswith("cfg_")}
    seed, B = int(g["seed"]), int(g["B"])
    T = int(g["T"]) + int(g.get("decode_steps", 0))
    states = seeded_uniform_int((B, T, *cfg["state_shape"]), 0, 256, seed, name + ":states").to(torch.uint8)
    assert checksum(states.float()) == pytest.approx(float(g["states_checksum"]), rel=1e-12)
    sd = seeded_state_dict(dt_param_shapes(cfg), seed)
    assert sum(checksum(sd[k]) for k in sorted(sd)) == pytest.approx(float(g["w_checksum"]), rel=1e-12)
    actions = torch.from_numpy(g["actions"])
    rtg = torch.from_numpy(g["rtg"])
    ts = torch.from_numpy(g["timesteps"])
    np.testing.assert_array_equal(actions.numpy(), seeded_uniform_int((B, T), 0, cfg["act_dim"], seed,
                                                                      name + ":actions").numpy())
    np.testing.assert_array_equal(rtg.numpy(), seeded_uniform((B, T), 0.0, 3000.0, seed, name + ":rtg").numpy())
    return cfg, sd, states, actions, rtg, ts


def test_dt_model_logits_match_reference():
    g = load("dt_small")
    cfg, sd, states, actions, rtg, ts = _dt_inputs(g)
    T = int(g["T"])
    mask = (torch.arange(T)[None] >= torch.from_numpy(g["pad_steps"]).long()[:, None]).long()
    logits, values, hidden, presents = dt_forward_ref(sd, cfg, states[:, :T], actions[:, :T], rtg[:, :T],
                                                      ts[:, :T], attention_mask=mask, use_cache=True)
    np.testing.assert_allclose(logits.numpy(), g["logits"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(values.numpy(), g["values"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(hidden.numpy(), g["hidden"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(presents[0][0].numpy(), g["present0_k"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(presents[0][1].numpy(), g["present0_v"], atol=1e-5, rtol=1e-5)


def test_dt_model_cached_step_matches_reference():
    g = load("dt_small")
    cfg, sd, states, actions, rtg, ts = _dt_inputs(g)
    T = int(g["T"])
    l0, _, _, pres = dt_forward_ref(sd, cfg, states[:, :T], actions[:, :T], rtg[:, :T], ts[:, :T], use_cache=True)
    np.testing.assert_allclose(l0.numpy(), g["nomask_logits"], atol=1e-5, rtol=1e-5)
    l1, _, h1, _ = dt_forward_ref(sd, cfg, states[:, T:], actions[:, T:], rtg[:, T:], ts[:, T:],
                                  past_key_values=pres, use_cache=True)
    np.testing.assert_allclose(l1.numpy(), g["dec_logits"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(h1.numpy(), g["dec_hidden"], atol=1e-5, rtol=1e-5)


def test_oracle_catches_a_planted_mask_error():
    """A mistake planted in the oracle (keys < pad not masked) must break parity with the fixture."""
    g = load("attn_d32_mask")
    sd = attn_weights(g)
    H, nh, nkv, B, S, seed = (int(g[k]) for k in ("hidden", "nh", "nkv", "B", "S", "seed"))
    x = seeded_normal((B, S, H), seed, "attn_d32_mask:x")
    cos, sin = precompute_freqs_cis(H // nh, S, 1e4)
    w = [sd[k] for k in ("q_proj.weight", "k_proj.weight", "v_proj.weight", "o_proj.weight")]
    out, _ = attention_module_ref(x, *w, nh, nkv, cos, sin, attention_mask=None)  # planted: mask dropped
    assert np.abs(out.numpy() - g["out"]).max() > 1e-2


@pytest.mark.parametrize("name,samples", [("dt_cfg1", [0, 17, 63]), ("dt_cfg4", [2]), ("dt_rollout", [0, 15])])
def test_dt_workload_goldens_pin_the_oracle(name, samples):
    """The oracle's DT forward equals the reference's fp32 logits at the workload
    shapes (cfg1: 4/256/8x2, cfg4: 12/768/12x4 at 768 tokens, the 252-token
    rollout trajectory) on a few samples of each fixture (the CPU suite stays fast;
    samples are independent, so a slice of the batch is the same computation)."""
    from oracle.seeded import dt_synthetic_inputs

    g = load(name)
    cfgd = {k[4:]: (tuple(v.tolist()) if v.ndim else v.item()) for k, v in g.items() if k.startswith("cfg_")}
    sd = seeded_state_dict(dt_param_shapes(cfgd), int(g["seed"]))
    assert sum(checksum(sd[k]) for k in sorted(sd)) == pytest.approx(float(g["w_checksum"]), rel=1e-12)
    inp = dt_synthetic_inputs(name, int(g["seed"]), int(g["B"]), int(g["T"]), cfgd["state_shape"], cfgd["act_dim"],
                              int(g["pad_max"]))
    sel = torch.tensor(samples)
    mask = inp["mask"][sel] if "mask" in inp else None
    logits, values, _, _ = dt_forward_ref(sd, cfgd, inp["states"][sel], inp["actions"][sel], inp["rtg"][sel],
                                          inp["timesteps"][sel], mask)
    np.testing.assert_allclose(logits.numpy(), g["logits"][samples], atol=ATOL, rtol=1e-5)
    np.testing.assert_allclose(values.numpy(), g["values"][samples], atol=ATOL, rtol=1e-5)
