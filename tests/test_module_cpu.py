"""Host-side checks of the drop-in module and the DT host model (no GPU).

The reference import is used only when $RL_FOR_MARIO_REF names a checkout
of FujiM3/RL_for_Mario; the test that needs it is skipped otherwise.
"""
import os
import sys
from pathlib import Path

import pytest
import torch

from oracle.dt_ref import dt_param_shapes
from oracle.seeded import seeded_state_dict

REF = Path(os.environ["RL_FOR_MARIO_REF"]) if os.environ.get("RL_FOR_MARIO_REF") else None


def small_cfg():
    from rl_for_mario_b200.dt_model import DTConfig

    return DTConfig(hidden_size=128, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=1,
                    context_len=8, dropout=0.0)


def test_dt_model_param_names_match_reference_layout():
    from rl_for_mario_b200.dt_model import MarioDT

    cfg = small_cfg()
    names = sorted(n for n, _ in MarioDT(cfg).named_parameters())
    cfgd = {k: getattr(cfg, k) for k in ("state_shape", "act_dim", "max_ep_len", "context_len", "hidden_size",
                                         "num_hidden_layers", "num_attention_heads", "num_key_value_heads",
                                         "intermediate_size")}
    assert names == sorted(n for n, _ in dt_param_shapes(cfgd))


def test_seeded_state_dict_loads_strictly():
    from rl_for_mario_b200.dt_model import MarioDT

    cfg = small_cfg()
    m = MarioDT(cfg)
    shapes = [(n, tuple(p.shape)) for n, p in m.named_parameters()]
    m.load_state_dict(seeded_state_dict(shapes, 5), strict=True)


def test_fast_attention_rejects_bad_heads_and_cpu_inputs():
    from rl_for_mario_b200.attention import FastDTAttention

    class C:
        hidden_size, num_attention_heads, num_key_value_heads, dropout, flash_attn = 96, 6, 4, 0.0, True

    with pytest.raises(ValueError, match="divisible"):
        FastDTAttention(C())
    C.num_key_value_heads = 2
    m = FastDTAttention(C())
    x = torch.zeros(1, 3, 96)
    with pytest.raises(ValueError, match="CUDA"):
        m(x, (torch.zeros(3, 16), torch.zeros(3, 16)))


def test_paged_cache_presents_reference_tuple_contract():
    from rl_for_mario_b200.cache import PagedKVCache

    c = PagedKVCache(2, batch=3, num_kv_heads=2, head_dim=32, max_len=100, page_size=16, device="cpu")
    past = c.as_past()
    assert not hasattr(past[0], "layers")
    assert past[0][0].shape[2] == 0
    past[0].advance(7)
    assert past[0][0].shape == torch.Size((3, 2, 7, 32)) and past[1][0].shape[2] == 0
    k, v = past[0].dense()
    assert k.shape == (3, 2, 7, 32)


@pytest.mark.skipif(REF is None or not (REF / "model" / "model_decision_transformer.py").exists(),
                    reason="RL_FOR_MARIO_REF does not name a reference checkout")
def test_swap_into_reference_model_keeps_weights():
    sys.path.insert(0, str(REF))
    from model.model_decision_transformer import DecisionTransformerConfig, MarioDecisionTransformer

    from rl_for_mario_b200.attention import FastDTAttention, swap_attention

    cfg = DecisionTransformerConfig(hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                    num_key_value_heads=1, context_len=8, dropout=0.0)
    ref = MarioDecisionTransformer(cfg)
    before = {k: v.clone() for k, v in ref.state_dict().items()}
    assert swap_attention(ref, cfg) == 2
    assert all(isinstance(l.self_attn, FastDTAttention) for l in ref.model.layers)
    after = ref.state_dict()
    assert before.keys() == after.keys()
    assert all(torch.equal(before[k], after[k]) for k in before)
