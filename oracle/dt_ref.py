"""Float32 functional restatement of MarioDecisionTransformer (oracle; test infrastructure).

``dt_forward_ref(sd, cfg, ...)`` evaluates the reference model
(model/model_decision_transformer.py:348-524) in eval mode from a state_dict
keyed by the reference's own parameter names, so the same weights load into
the reference, this oracle and the CUDA-backed model.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .attention_ref import attention_module_ref, precompute_freqs_cis, rmsnorm_ref

Tensor = torch.Tensor


def dt_param_shapes(cfg: dict) -> List[Tuple[str, Tuple[int, ...]]]:
    """Names and shapes of every parameter of the reference model (:348-477)."""
    H = cfg["hidden_size"]
    nh, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    D = H // nh
    inter = cfg.get("intermediate_size")
    if inter is None:  # FeedForward default width, :259-262
        inter = int(H * 8 / 3)
        inter = 64 * ((inter + 63) // 64)
    c = cfg["state_shape"][0]
    out = [
        ("model.state_encoder.cnn.0.weight", (32, c, 8, 8)), ("model.state_encoder.cnn.0.bias", (32,)),
        ("model.state_encoder.cnn.2.weight", (64, 32, 4, 4)), ("model.state_encoder.cnn.2.bias", (64,)),
        ("model.state_encoder.cnn.4.weight", (64, 64, 3, 3)), ("model.state_encoder.cnn.4.bias", (64,)),
        ("model.state_encoder.cnn.7.weight", (H, 64 * 7 * 7)), ("model.state_encoder.cnn.7.bias", (H,)),
        ("model.embed_return.weight", (H, 1)), ("model.embed_return.bias", (H,)),
        ("model.embed_action.weight", (cfg["act_dim"], H)),
        ("model.embed_timestep.weight", (cfg["max_ep_len"], H)),
        ("model.embed_norm.weight", (H,)),
    ]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (H,)), (p + "post_attention_layernorm.weight", (H,)),
            (p + "self_attn.q_proj.weight", (nh * D, H)), (p + "self_attn.k_proj.weight", (nkv * D, H)),
            (p + "self_attn.v_proj.weight", (nkv * D, H)), (p + "self_attn.o_proj.weight", (H, nh * D)),
            (p + "mlp.gate_proj.weight", (inter, H)), (p + "mlp.up_proj.weight", (inter, H)),
            (p + "mlp.down_proj.weight", (H, inter)),
        ]
    out += [("model.norm.weight", (H,)), ("action_head.weight", (cfg["act_dim"], H)),
            ("value_head.weight", (1, H)), ("value_head.bias", (1,))]
    return out


def state_encoder_ref(sd: Dict[str, Tensor], states: Tensor) -> Tensor:
    """Nature-DQN CNN, :332-341: uint8 -> float, /255 when max > 1, 3 conv+ReLU, Linear."""
    B, T = states.shape[:2]
    x = states.float()
    if x.max() > 1.0:
        x = x / 255.0
    x = x.reshape(B * T, *states.shape[2:])
    p = "model.state_encoder.cnn."
    x = F.relu(F.conv2d(x, sd[p + "0.weight"].float(), sd[p + "0.bias"].float(), stride=4))
    x = F.relu(F.conv2d(x, sd[p + "2.weight"].float(), sd[p + "2.bias"].float(), stride=2))
    x = F.relu(F.conv2d(x, sd[p + "4.weight"].float(), sd[p + "4.bias"].float(), stride=1))
    x = x.flatten(1) @ sd[p + "7.weight"].float().t() + sd[p + "7.bias"].float()
    return x.reshape(B, T, -1)


def embed_tokens_ref(sd, cfg, states, actions, returns_to_go, timesteps) -> Tensor:
    """Embeddings and (R, s, a) interleave, :401-420 -> [B, 3T, H] after embed_norm."""
    B, T = states.shape[:2]
    H = cfg["hidden_size"]
    ts = timesteps.clamp(0, cfg["max_ep_len"] - 1).long()
    te = sd["model.embed_timestep.weight"].float()[ts]
    se = state_encoder_ref(sd, states) + te
    re = returns_to_go.float().unsqueeze(-1) @ sd["model.embed_return.weight"].float().t() \
        + sd["model.embed_return.bias"].float() + te
    ae = sd["model.embed_action.weight"].float()[actions.long().clamp(0, cfg["act_dim"] - 1)] + te
    h = torch.stack((re, se, ae), dim=2).reshape(B, 3 * T, H)
    return rmsnorm_ref(h, sd["model.embed_norm.weight"], cfg["rms_norm_eps"])


def block_ref(sd, cfg, i: int, h: Tensor, cos: Tensor, sin: Tensor, past=None, use_cache=False, mask=None):
    """Pre-norm block, :294-304: attention (+residual) then SwiGLU FFN (+residual)."""
    p = f"model.layers.{i}."
    eps = cfg["rms_norm_eps"]
    a_in = rmsnorm_ref(h, sd[p + "input_layernorm.weight"], eps)
    a, present = attention_module_ref(
        a_in, sd[p + "self_attn.q_proj.weight"], sd[p + "self_attn.k_proj.weight"],
        sd[p + "self_attn.v_proj.weight"], sd[p + "self_attn.o_proj.weight"],
        cfg["num_attention_heads"], cfg["num_key_value_heads"], cos, sin,
        past_key_value=past, use_cache=use_cache, attention_mask=mask)
    h = h + a
    f_in = rmsnorm_ref(h, sd[p + "post_attention_layernorm.weight"], eps)
    gate = f_in @ sd[p + "mlp.gate_proj.weight"].float().t()
    up = f_in @ sd[p + "mlp.up_proj.weight"].float().t()
    h = h + (F.silu(gate) * up) @ sd[p + "mlp.down_proj.weight"].float().t()
    return h, present


def dt_forward_ref(sd: Dict[str, Tensor], cfg: dict, states: Tensor, actions: Tensor, returns_to_go: Tensor,
                   timesteps: Tensor, attention_mask: Optional[Tensor] = None,
                   past_key_values: Optional[list] = None, use_cache: bool = False):
    """MarioDecisionTransformer.forward in eval mode, :479-524 and :371-461.

    Returns (action_logits [B,T,A], value_preds [B,T], hidden [B,T,3,H], presents).
    """
    B, T = states.shape[:2]
    H = cfg["hidden_size"]
    h = embed_tokens_ref(sd, cfg, states, actions, returns_to_go, timesteps)
    mask3 = None
    if attention_mask is not None:  # :424-433
        mask3 = torch.stack((attention_mask,) * 3, dim=2).reshape(B, 3 * T).float()
    L = cfg["num_hidden_layers"]
    past = past_key_values or [None] * L
    start = past[0][0].shape[2] if past[0] is not None else 0  # :439
    cos_t, sin_t = precompute_freqs_cis(H // cfg["num_attention_heads"], 3 * cfg["context_len"],
                                        cfg["rope_theta"])
    cos, sin = cos_t[start:start + 3 * T], sin_t[start:start + 3 * T]
    presents = []
    for i in range(L):
        h, pr = block_ref(sd, cfg, i, h, cos, sin, past[i], use_cache, mask3)
        presents.append(pr)
    h = rmsnorm_ref(h, sd["model.norm.weight"], cfg["rms_norm_eps"]).view(B, T, 3, H)
    st = h[:, :, 1, :]
    logits = st @ sd["action_head.weight"].float().t()
    values = (st @ sd["value_head.weight"].float().t() + sd["value_head.bias"].float()).squeeze(-1)
    return logits, values, h, presents
