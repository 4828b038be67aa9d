"""Float32 CPU restatement of the DT attention path (oracle; test infrastructure).

Each function cites the reference lines it restates
(model/model_decision_transformer.py in FujiM3/RL_for_Mario).  Everything is
computed in float32 on the CPU from whatever inputs are given (callers upcast
bf16 kernel inputs so both sides see identical values).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

Tensor = torch.Tensor


def precompute_freqs_cis(dim: int, end: int, rope_base: float = 1e4) -> Tuple[Tensor, Tensor]:
    """RoPE tables, reference :93-99.

    inv_freq[i] = base^(-2i/dim); angle[t, i] = t * inv_freq[i]; the cos/sin
    tables repeat the dim/2 angles twice along the last axis -> [end, dim].
    """
    inv = 1.0 / (rope_base ** (torch.arange(0, dim, 2).float() / dim))
    t = torch.arange(end, dtype=torch.float32)
    ang = torch.outer(t, inv).float()
    return torch.cat([ang.cos(), ang.cos()], dim=-1), torch.cat([ang.sin(), ang.sin()], dim=-1)


def rotate_half(x: Tensor) -> Tensor:
    """rot(x) = concat(-x[D/2:], x[:D/2]), reference :103-105."""
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rotary_pos_emb(q: Tensor, k: Tensor, cos: Tensor, sin: Tensor) -> Tuple[Tensor, Tensor]:
    """q, k [B, S, H, D]; cos/sin [S, D] broadcast over heads, reference :108-117."""
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    return q * c + rotate_half(q) * s, k * c + rotate_half(k) * s


def repeat_kv(x: Tensor, n_rep: int) -> Tensor:
    """[B, Hkv, L, D] -> [B, Hkv*n_rep, L, D], head h reads KV head h // n_rep, reference :121-130."""
    if n_rep == 1:
        return x
    b, h, l, d = x.shape
    return x[:, :, None].expand(b, h, n_rep, l, d).reshape(b, h * n_rep, l, d)


def mask_from_pad_len(pad_len: Tensor, S: int) -> Tensor:
    """Left-padding mask [B, S] (1 = valid) with pad_len[b] leading zeros."""
    return (torch.arange(S)[None, :] >= pad_len.view(-1, 1).long()).float()


def _softmax_attend(q: Tensor, k: Tensor, v: Tensor, add_mask: Optional[Tensor], scale: float) -> Tensor:
    """softmax(q k^T * scale + mask) v in float32 (the SDPA definition)."""
    s = torch.matmul(q, k.transpose(-2, -1)) * scale
    if add_mask is not None:
        s = s + add_mask
    return torch.matmul(torch.softmax(s, dim=-1), v)


def attention_prefill_ref(q: Tensor, k: Tensor, v: Tensor, cos: Optional[Tensor], sin: Optional[Tensor],
                          attention_mask: Optional[Tensor] = None, rope: bool = True,
                          scale: Optional[float] = None) -> Tensor:
    """Prefill branch, reference :179-224 (after the projections).

    q [B, S, Hq, D], k/v [B, S, Hkv, D]; returns the attention output
    [B, S, Hq, D] (before o_proj).  Without a mask: causal attention
    (is_causal=True, :201-205).  With a [B, S] mask (1 = valid): additive
    triu(-inf, 1) causal mask plus (1 - mask) * -1e9 on key columns (:209-224).
    """
    q, k, v = q.float(), k.float(), v.float()
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    if rope:
        q, k = apply_rotary_pos_emb(q, k, cos.float(), sin.float())
    qh = q.transpose(1, 2)
    kh = repeat_kv(k.transpose(1, 2), Hq // Hkv)
    vh = repeat_kv(v.transpose(1, 2), Hq // Hkv)
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    causal = torch.triu(torch.full((S, S), float("-inf")), diagonal=1)[None, None]
    if attention_mask is None:
        add = causal
    else:
        pad = (1.0 - attention_mask.float()).unsqueeze(1).unsqueeze(2) * -1e9
        add = causal + pad
    out = _softmax_attend(qh, kh, vh, add, sc)
    return out.transpose(1, 2).contiguous()


def attention_decode_ref(q: Tensor, k: Tensor, v: Tensor, past_k: Optional[Tensor], past_v: Optional[Tensor],
                         cos: Optional[Tensor], sin: Optional[Tensor],
                         attention_mask: Optional[Tensor] = None, rope: bool = True,
                         scale: Optional[float] = None) -> Tuple[Tensor, Tensor, Tensor]:
    """Cached ("slow path") branch, reference :179-191 and :225-245.

    q [B, Sn, Hq, D], k/v [B, Sn, Hkv, D] new tokens; past_k/past_v
    [B, Hkv, L, D] (post-RoPE K).  cos/sin [Sn, D] are the rows of the new
    tokens.  attention_mask, if given, is [B, L + Sn] (1 = valid).  Returns
    (out [B, Sn, Hq, D], k_all, v_all) with k_all/v_all [B, Hkv, L + Sn, D].
    """
    q, k, v = q.float(), k.float(), v.float()
    B, Sn, Hq, D = q.shape
    Hkv = k.shape[2]
    if rope:
        q, k = apply_rotary_pos_emb(q, k, cos.float(), sin.float())
    qh = q.transpose(1, 2)
    kc = k.transpose(1, 2)
    vc = v.transpose(1, 2)
    if past_k is not None:
        kc = torch.cat([past_k.float(), kc], dim=2)
        vc = torch.cat([past_v.float(), vc], dim=2)
    kh = repeat_kv(kc, Hq // Hkv)
    vh = repeat_kv(vc, Hq // Hkv)
    sc = 1.0 / math.sqrt(D) if scale is None else scale
    s = torch.matmul(qh, kh.transpose(-2, -1)) * sc
    L = kh.shape[2]
    causal = torch.triu(torch.full((Sn, Sn), float("-inf")), diagonal=1)
    s[:, :, :, L - Sn:] = s[:, :, :, L - Sn:] + causal
    if attention_mask is not None:
        s = s + (1.0 - attention_mask.float()).unsqueeze(1).unsqueeze(2) * -1e9
    p = torch.softmax(s.float(), dim=-1)
    out = torch.matmul(p, vh)
    return out.transpose(1, 2).contiguous(), kc, vc


def rmsnorm_ref(x: Tensor, weight: Tensor, eps: float = 1e-5) -> Tensor:
    """weight * (x * rsqrt(mean(x^2) + eps)), in float32, reference :76-86."""
    xf = x.float()
    return weight.float() * (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps))


def attention_module_ref(x: Tensor, wq: Tensor, wk: Tensor, wv: Tensor, wo: Tensor, n_heads: int,
                         n_kv_heads: int, cos: Tensor, sin: Tensor,
                         past_key_value: Optional[Tuple[Tensor, Tensor]] = None, use_cache: bool = False,
                         attention_mask: Optional[Tensor] = None):
    """Whole DecisionTransformerAttention.forward in eval mode, reference :165-249.

    Dispatches like the reference: the prefill branch when seq_len > 1 and no
    cache is given (:198), the cached branch otherwise.
    """
    x = x.float()
    B, S, H = x.shape
    D = H // n_heads
    xq = (x @ wq.float().t()).view(B, S, n_heads, D)
    xk = (x @ wk.float().t()).view(B, S, n_kv_heads, D)
    xv = (x @ wv.float().t()).view(B, S, n_kv_heads, D)
    if S > 1 and past_key_value is None:
        out = attention_prefill_ref(xq, xk, xv, cos, sin, attention_mask)
        _, kr = apply_rotary_pos_emb(xq, xk, cos.float(), sin.float())
        past = (kr.transpose(1, 2).contiguous(), xv.transpose(1, 2).contiguous()) if use_cache else None
    else:
        pk, pv = past_key_value if past_key_value is not None else (None, None)
        out, kc, vc = attention_decode_ref(xq, xk, xv, pk, pv, cos, sin, attention_mask)
        past = (kc, vc) if use_cache else None
    out = out.reshape(B, S, n_heads * D) @ wo.float().t()
    return out, past


class ReferenceAttention(torch.nn.Module):
    """DecisionTransformerAttention (reference :137-249) as a module with the
    reference's parameter names and forward contract, evaluated by
    ``attention_module_ref`` in float32 on the inputs' device.  Lets a test
    build a model whose attention is the reference's and then swap it for the
    drop-in replacement."""

    def __init__(self, config):
        super().__init__()
        nh = config.num_attention_heads
        nkv = nh if config.num_key_value_heads is None else config.num_key_value_heads
        if nh % nkv:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        self.n_local_heads, self.n_local_kv_heads = nh, nkv
        self.head_dim = config.hidden_size // nh
        H = config.hidden_size
        self.q_proj = torch.nn.Linear(H, nh * self.head_dim, bias=False)
        self.k_proj = torch.nn.Linear(H, nkv * self.head_dim, bias=False)
        self.v_proj = torch.nn.Linear(H, nkv * self.head_dim, bias=False)
        self.o_proj = torch.nn.Linear(nh * self.head_dim, H, bias=False)

    def forward(self, x, position_embeddings, past_key_value=None, use_cache=False, attention_mask=None):
        cos, sin = position_embeddings
        out, past = attention_module_ref(x, self.q_proj.weight, self.k_proj.weight, self.v_proj.weight,
                                         self.o_proj.weight, self.n_local_heads, self.n_local_kv_heads,
                                         cos.float(), sin.float(), past_key_value, use_cache, attention_mask)
        if past is not None:
            past = (past[0].to(x.dtype), past[1].to(x.dtype))
        return out.to(x.dtype), past
