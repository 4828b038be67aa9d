"""Host model around the attention kernels: the Mario Decision Transformer.

A restatement of the reference model (model/model_decision_transformer.py:
config :17-55, RMSNorm :76-86, RoPE tables :93-99, FeedForward :256-271,
block :278-304, state encoder :315-341, backbone :348-461, wrapper :468-548)
whose attention is ``FastDTAttention``.  Parameter names match the reference,
so a reference state_dict loads unchanged (checkpoint compatibility).  With
``fuse_norms()`` a block runs as: RMSNorm + Q/K/V + RoPE kernel, attention
kernel, o_proj GEMM with the residual as accumulator input, RMSNorm + gate/up
+ SwiGLU kernel, down_proj GEMM with the residual (the two residual GEMMs on
the library's CTA-pair GEMM at prefill sizes, on cuBLAS for a rollout step's
small, latency-bound ones); the rest (CNN encoder past its first layer,
embeddings, final norm, heads) runs as PyTorch on the GPU.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from . import kernels
from .attention import FastDTAttention
from .cache import LayerKV, PagedKVCache

Tensor = torch.Tensor


@dataclass
class DTConfig:
    """Fields and defaults of DecisionTransformerConfig (:20-55)."""

    state_shape: Tuple[int, int, int] = (4, 84, 84)
    act_dim: int = 7
    max_ep_len: int = 4096
    context_len: int = 64
    hidden_size: int = 512
    intermediate_size: Optional[int] = None
    num_hidden_layers: int = 6
    num_attention_heads: int = 8
    num_key_value_heads: int = 2
    hidden_act: str = "silu"
    dropout: float = 0.1
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    flash_attn: bool = True
    label_smoothing: float = 0.1
    max_position_embeddings: int = field(init=False)

    def __post_init__(self):
        self.state_shape = tuple(self.state_shape)
        self.max_position_embeddings = self.context_len * 3

    @classmethod
    def from_reference(cls, ref_cfg) -> "DTConfig":
        names = [f for f in cls.__dataclass_fields__ if f != "max_position_embeddings"]
        return cls(**{n: getattr(ref_cfg, n) for n in names})


class RMSNorm(nn.Module):
    """weight * (x * rsqrt(mean(x^2) + eps)) in fp32, cast back (:76-86)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        w = self.weight
        if (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype and x.numel()
                and x.shape[-1] % 8 == 0 and x.stride(-1) == 1 and x.data_ptr() % 16 == 0
                and all(st % 8 == 0 for st in x.stride()[:-1])
                and not (torch.is_grad_enabled() and (x.requires_grad or w.requires_grad))):
            return kernels.rmsnorm(x, w.contiguous(), self.eps)  # one pass, same rounding
        xf = x.float()
        return w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).type_as(x)


def rope_tables(dim: int, end: int, base: float) -> Tuple[Tensor, Tensor]:
    """cos/sin [end, dim] with duplicated halves (:93-99)."""
    inv = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
    ang = torch.outer(torch.arange(end).float(), inv)
    return torch.cat([ang.cos(), ang.cos()], -1), torch.cat([ang.sin(), ang.sin()], -1)


class FeedForward(nn.Module):
    """SwiGLU, width 64 * ceil(8H/3 / 64) by default (:256-271)."""

    def __init__(self, cfg: DTConfig):
        super().__init__()
        inter = cfg.intermediate_size
        if inter is None:
            inter = int(cfg.hidden_size * 8 / 3)
            inter = 64 * ((inter + 63) // 64)
        self.gate_proj = nn.Linear(cfg.hidden_size, inter, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, inter, bias=False)
        self.down_proj = nn.Linear(inter, cfg.hidden_size, bias=False)
        self.dropout = nn.Dropout(cfg.dropout)

    def forward(self, x: Tensor) -> Tensor:
        return self.dropout(self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x)))


class DTBlock(nn.Module):
    """Pre-norm block (:278-304)."""

    def __init__(self, cfg: DTConfig):
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.self_attn = FastDTAttention(cfg)
        self.mlp = FeedForward(cfg)

    def fuse_norm(self, on: bool = True) -> None:
        """Runs input_layernorm inside the attention's fused RMSNorm + QKV kernel,
        the residual adds inside the o_proj / down_proj GEMMs and
        post_attention_layernorm + gate / up + SwiGLU in one kernel (16-bit
        weights, dropout off)."""
        self.self_attn.set_fused_norm(self.input_layernorm if on else None)
        self._swiglu_w = None

    def _swiglu_weight(self, dtype: torch.dtype) -> Tensor:
        ps = (self.mlp.gate_proj.weight, self.mlp.up_proj.weight, self.post_attention_layernorm.weight)
        key = tuple((p.data_ptr(), p._version) for p in ps) + (dtype,)
        if getattr(self, "_swiglu_w", None) is None or self._swiglu_key != key:
            self._swiglu_w = kernels.fold_swiglu_weight(*ps, dtype=dtype)
            self._swiglu_key = key
        return self._swiglu_w

    def _fused_mlp_ok(self, h: Tensor) -> bool:
        mlp = self.mlp
        inter = mlp.gate_proj.weight.shape[0]
        return (h.is_cuda and h.dtype in (torch.bfloat16, torch.float16)
                and mlp.down_proj.weight.dtype == h.dtype and mlp.down_proj.bias is None
                and mlp.gate_proj.bias is None and mlp.up_proj.bias is None
                and (not self.training or mlp.dropout.p == 0) and inter % 64 == 0 and inter >= 128
                and h.shape[-1] % 8 == 0 and not (torch.is_grad_enabled() and h.requires_grad))

    def forward(self, hidden_states, position_embeddings, past_key_value=None, use_cache=False,
                attention_mask=None, _owns_input: bool = False):
        """``_owns_input``: the caller (the backbone's layer loop) owns
        ``hidden_states`` and drops it after this call, so the fused path may
        accumulate the o_proj GEMM into it in place."""
        if self.self_attn._fused_norm is not None:
            h, present = self.self_attn(hidden_states, position_embeddings, past_key_value=past_key_value,
                                        use_cache=use_cache, attention_mask=attention_mask, raw_input=True,
                                        residual=hidden_states,
                                        residual_inplace=_owns_input and not torch.is_grad_enabled())
            if self._fused_mlp_ok(h):
                a = kernels.rmsnorm_swiglu(h, self._swiglu_weight(h.dtype), self.post_attention_layernorm.eps)
                # h is this block's own intermediate: the down projection
                # accumulates into it in place (no copy of the residual), on the
                # library's CTA-pair GEMM at prefill sizes; a rollout step's small
                # GEMM is latency-bound and faster on cuBLAS's addmm_ (measured).
                h2, a2, wd = h.view(-1, h.shape[-1]), a.reshape(-1, a.shape[-1]), self.mlp.down_proj.weight
                if kernels.gemm_residual_on_pairs(a2, wd, h2):
                    kernels.gemm_residual(a2, wd, h2)
                else:
                    h2.addmm_(a2, wd.t())
            else:
                h = h + self.mlp(self.post_attention_layernorm(h))
            return h, present
        else:
            h, present = self.self_attn(self.input_layernorm(hidden_states), position_embeddings,
                                        past_key_value=past_key_value, use_cache=use_cache,
                                        attention_mask=attention_mask)
        h = h + hidden_states
        h = h + self.mlp(self.post_attention_layernorm(h))
        return h, present


class MarioStateEncoder(nn.Module):
    """Nature-DQN CNN (:315-341)."""

    def __init__(self, state_shape, hidden_size: int):
        super().__init__()
        c = state_shape[0]
        self.cnn = nn.Sequential(
            nn.Conv2d(c, 32, 8, 4), nn.ReLU(inplace=True), nn.Conv2d(32, 64, 4, 2), nn.ReLU(inplace=True),
            nn.Conv2d(64, 64, 3, 1), nn.ReLU(inplace=True), nn.Flatten(), nn.Linear(64 * 7 * 7, hidden_size))

    def forward(self, states: Tensor) -> Tensor:
        if states.ndim != 5:
            raise ValueError(f"states must be [B,T,C,H,W], got {tuple(states.shape)}")
        B, T, C, H, W = states.shape
        conv0, conv1, conv2, lin = self.cnn[0], self.cnn[2], self.cnn[4], self.cnn[7]
        dt = conv0.weight.dtype
        s = states.reshape(B * T, C, H, W)
        cl = torch.channels_last
        if (conv0.in_channels == 4 and conv0.out_channels == 32 and conv0.kernel_size == (8, 8)
                and conv0.stride == (4, 4) and conv0.padding == (0, 0) and conv0.bias is not None
                and s.is_cuda and s.dtype == torch.uint8 and dt in (torch.bfloat16, torch.float16)
                and s.is_contiguous() and (H - 8) % 4 == 0 and (W - 8) % 4 == 0
                and s.data_ptr() % 16 == 0 and s.numel() % 16 == 0):
            # One tensor-core kernel from the uint8 frames: the reference's
            # /255 when the max exceeds 1 (:338), the 8 x 8 stride-4
            # convolution, bias and ReLU (device-side decision, no host sync).
            x, _ = kernels.frames_conv1(s, conv0.weight, conv0.bias, round_input=self.round_input)
        elif self.round_input:
            # The reference's own 16-bit evaluation (:336-341) for shapes the
            # first-layer kernel does not take.
            x = s.to(dt)
            x = torch.where(x.amax() > 1.0, x / 255.0, x)
            x = F.relu(F.conv2d(x, conv0.weight, conv0.bias, stride=conv0.stride))
            x = x.contiguous(memory_format=cl)
        else:
            # The reference divides by 255 when the frames' max exceeds 1 (:338).
            # The test stays on the device (no host synchronisation) and the 1/255
            # goes into the first convolution's weight instead of a pass over the
            # frames.
            use_blocks = (conv0.kernel_size == (8, 8) and conv0.stride == (4, 4) and conv0.padding == (0, 0)
                          and H % 4 == 0 and W % 4 == 0 and s.is_cuda and s.dtype == torch.uint8
                          and dt in (torch.bfloat16, torch.float16) and s.is_contiguous())
            if use_blocks:
                # The frame-block kernel also reports the largest byte.
                fmax = torch.zeros(1, dtype=torch.int32, device=s.device)
                xb = kernels.frames_to_blocks(s, dt, fmax)
                big = fmax > 1
            else:
                big = (s.amax() > 1) if s.dtype == torch.uint8 else (s.to(dt).amax() > 1.0)
            w0 = torch.where(big, conv0.weight / 255.0, conv0.weight)
            cl = torch.channels_last
            k0, st0 = conv0.kernel_size[0], conv0.stride[0]
            if (conv0.kernel_size == (k0, k0) and conv0.stride == (st0, st0) and conv0.padding == (0, 0)
                    and k0 % st0 == 0 and H % st0 == 0 and W % st0 == 0):
                # Space-to-depth: a k x k stride-st convolution over C channels is a
                # (k/st) x (k/st) stride-1 convolution over C*st*st channels of the
                # frames cut into st x st blocks (same products, same sums).  With
                # 4 x 8 x 8 / 4 that turns a 4-channel input, which has no
                # tensor-core convolution, into a 64-channel one.  One pass writes
                # the blocked frames in the compute dtype, channels-last.
                f = st0
                if use_blocks:
                    x = xb
                else:
                    x = torch.empty((B * T, C * f * f, H // f, W // f), dtype=dt, device=s.device, memory_format=cl)
                    x.permute(0, 2, 3, 1).view(B * T, H // f, W // f, C, f, f).copy_(
                        s.view(B * T, C, H // f, f, W // f, f).permute(0, 2, 4, 1, 3, 5))
                kb = k0 // f
                w0 = (w0.view(conv0.out_channels, C, kb, f, kb, f).permute(0, 1, 3, 5, 2, 4)
                      .reshape(conv0.out_channels, C * f * f, kb, kb))
                x = self._conv_relu(x, w0.contiguous(memory_format=cl), conv0.bias, (1, 1))
            else:
                # One pass: frames -> compute dtype, channels-last (the layout the
                # convolution kernels run in, so no layout conversions per layer).
                x = torch.empty(s.shape, dtype=dt, device=s.device, memory_format=cl)
                x.copy_(s)
                x = self._conv_relu(x, w0.contiguous(memory_format=cl), conv0.bias, conv0.stride)
        if self._tc_conv23 and self._conv23_shapes(x, conv1, conv2):
            # Layers 2 and 3 (:322-325) in one tensor-core kernel; layer 2's output
            # stays in shared memory.
            _, x = kernels.encoder_conv23(x, conv1.weight, conv1.bias, conv2.weight, conv2.bias, keep_y2=False)
        else:
            x = self._conv_relu(x, conv1.weight.contiguous(memory_format=cl), conv1.bias, conv1.stride)
            x = self._conv_relu(x, conv2.weight.contiguous(memory_format=cl), conv2.bias, conv2.stride)
        if x.dim() == 4 and x.is_contiguous(memory_format=cl):
            # The reference flattens in (C, H, W) order; channels-last
            # activations are (H, W, C) in memory, so the Linear's input
            # columns are permuted instead of the activations (no copy).
            n, c3, h3, w3 = x.shape
            lw = lin.weight.view(lin.out_features, c3, h3, w3).permute(0, 2, 3, 1).reshape(lin.out_features, -1)
            return F.linear(x.permute(0, 2, 3, 1).reshape(n, -1), lw, lin.bias).reshape(B, T, -1)
        return lin(x.contiguous().flatten(1)).reshape(B, T, -1)

    _fused_conv = True
    # True: layers 2 and 3 on the library's fused tensor-core kernel
    # (dt_encoder_conv23) when the shapes are the Nature-DQN ones on 84 x 84
    # frames: 4.3 ms against 4.8 ms for cuDNN's two fused convolutions at
    # 262,144 frames, same fp32 accumulation and single rounding.  Off by
    # default: with it, the cfg1-shape bf16 DT's largest logit error against the
    # fp32 reference measured 1.29x the reference's own bf16 run (0.0566 vs
    # 0.0438), above the 1.25x bound the parity tests hold the default path to,
    # although its mean error and argmax agreement over the bf16 golden cases
    # match cuDNN's.
    _tc_conv23 = False

    @staticmethod
    def _conv23_shapes(x: Tensor, c2: nn.Conv2d, c3: nn.Conv2d) -> bool:
        return (x.is_cuda and x.dim() == 4 and tuple(x.shape[1:]) == (32, 20, 20)
                and x.dtype in (torch.bfloat16, torch.float16) and x.is_contiguous(memory_format=torch.channels_last)
                and x.data_ptr() % 16 == 0
                and c2.in_channels == 32 and c2.out_channels == 64 and c2.kernel_size == (4, 4)
                and c2.stride == (2, 2) and c2.padding == (0, 0) and c2.bias is not None
                and c3.in_channels == 64 and c3.out_channels == 64 and c3.kernel_size == (3, 3)
                and c3.stride == (1, 1) and c3.padding == (0, 0) and c3.bias is not None
                and c2.weight.dtype == x.dtype and c3.weight.dtype == x.dtype)
    # True: frames / 255 rounded to the model dtype before the first convolution,
    # as the reference's 16-bit model does (:338); False: exact pixels, 1/255 on
    # the fp32 accumulator.
    round_input = False

    def _conv_relu(self, x: Tensor, w: Tensor, b: Optional[Tensor], stride) -> Tensor:
        """relu(conv2d(x, w) + b): cuDNN's fused convolution + bias + activation for
        16-bit CUDA inputs (one pass over the output instead of three), else the
        plain sequence."""
        if self._fused_conv and x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and w.dtype == x.dtype:
            try:
                return torch.cudnn_convolution_relu(x, w, b, tuple(stride), (0, 0), (1, 1), 1)
            except torch.cuda.OutOfMemoryError:
                raise
            except RuntimeError:
                type(self)._fused_conv = False  # no fused engine for this build / shape
        return F.relu(F.conv2d(x, w, b, stride=stride), inplace=True)


class DTBackbone(nn.Module):
    """DecisionTransformerModel (:348-461)."""

    def __init__(self, cfg: DTConfig):
        super().__init__()
        self.config = cfg
        self.state_encoder = MarioStateEncoder(cfg.state_shape, cfg.hidden_size)
        self.embed_return = nn.Linear(1, cfg.hidden_size)
        self.embed_action = nn.Embedding(cfg.act_dim, cfg.hidden_size)
        self.embed_timestep = nn.Embedding(cfg.max_ep_len, cfg.hidden_size)
        self.embed_norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.dropout = nn.Dropout(cfg.dropout)
        self.layers = nn.ModuleList([DTBlock(cfg) for _ in range(cfg.num_hidden_layers)])
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        cos, sin = rope_tables(cfg.hidden_size // cfg.num_attention_heads, cfg.max_position_embeddings,
                               cfg.rope_theta)
        self.register_buffer("freqs_cos", cos, persistent=False)
        self.register_buffer("freqs_sin", sin, persistent=False)

    def embed(self, states, actions, returns_to_go, timesteps) -> Tensor:
        """Token embeddings interleaved (R, s, a) -> [B, 3T, H] after embed_norm (:401-420)."""
        cfg = self.config
        B, T = states.shape[0], states.shape[1]
        ts = timesteps.clamp(0, cfg.max_ep_len - 1).long()
        te = self.embed_timestep(ts)
        se = self.state_encoder(states) + te
        re = self.embed_return(returns_to_go.unsqueeze(-1).to(self.embed_return.weight.dtype)) + te
        ae = self.embed_action(actions.long().clamp(0, cfg.act_dim - 1)) + te
        h = torch.stack((re, se, ae), dim=2).reshape(B, 3 * T, cfg.hidden_size)
        return self.dropout(self.embed_norm(h))

    def forward(self, states, actions, returns_to_go, timesteps, attention_mask=None, past_key_values=None,
                use_cache=False):
        cfg = self.config
        B, T = states.shape[0], states.shape[1]
        if states.ndim != 5:
            raise ValueError(f"states must be [B,T,C,H,W], got {tuple(states.shape)}")
        if states.shape[2:] != tuple(cfg.state_shape):
            raise ValueError(f"states spatial shape {tuple(states.shape[2:])} != config {cfg.state_shape}")
        if actions is None or actions.shape[:2] != (B, T):
            raise ValueError("actions must be [B,T]")
        if returns_to_go.shape[:2] != (B, T):
            raise ValueError("returns_to_go must be [B,T]")
        if timesteps.shape[:2] != (B, T):
            raise ValueError("timesteps must be [B,T]")
        if T > cfg.context_len:
            raise ValueError(f"seq_len={T} exceeds context_len={cfg.context_len}")
        h = self.embed(states, actions, returns_to_go, timesteps)
        mask3 = None
        if attention_mask is not None:
            if attention_mask.shape != (B, T):
                raise ValueError(f"attention_mask must be [B,T], got {tuple(attention_mask.shape)}")
            mask3 = torch.stack((attention_mask,) * 3, dim=2).reshape(B, 3 * T).to(h.dtype)
        return self.run_layers(h, mask3, past_key_values, use_cache, _owns_h=True)

    def run_layers(self, h, mask3=None, past_key_values=None, use_cache=False, flat: bool = False,
                   _owns_h: bool = False):
        """Layers + final norm on [B, S, H] token states (:435-461); returns [B, S/3, 3, H]
        (the reference's view) unless ``flat``.  The caller's ``h`` is left as it
        is unless ``_owns_h``; the layers' own intermediates are updated in place."""
        cfg = self.config
        B, S = h.shape[0], h.shape[1]
        if hasattr(past_key_values, "layers") and not isinstance(past_key_values, PagedKVCache):
            past_key_values = None  # the reference drops HF Cache objects (:436-437)
        if isinstance(past_key_values, PagedKVCache):
            past_key_values = past_key_values.as_past()
        past = past_key_values or [None] * len(self.layers)
        start = past[0][0].shape[2] if past[0] is not None else 0
        if start + S > self.freqs_cos.shape[0]:
            raise ValueError(f"positions {start}..{start + S - 1} exceed max_position_embeddings "
                             f"{self.freqs_cos.shape[0]}")
        pe = (self.freqs_cos[start:start + S], self.freqs_sin[start:start + S])
        presents = []
        owns = _owns_h
        for layer, pkv in zip(self.layers, past):
            h, pr = layer(h, pe, past_key_value=pkv, use_cache=use_cache, attention_mask=mask3, _owns_input=owns)
            owns = True
            presents.append(pr)
        h = self.norm(h)
        if not flat:
            h = h.view(B, S // 3, 3, cfg.hidden_size)
        return h, presents


@dataclass
class DTOutput:
    loss: Optional[Tensor] = None
    action_logits: Optional[Tensor] = None
    value_preds: Optional[Tensor] = None
    last_hidden_state: Optional[Tensor] = None
    past_key_values: Optional[List] = None


class MarioDT(nn.Module):
    """MarioDecisionTransformer (:468-548) with FastDTAttention."""

    def __init__(self, cfg: DTConfig):
        super().__init__()
        self.config = cfg
        self.model = DTBackbone(cfg)
        self.action_head = nn.Linear(cfg.hidden_size, cfg.act_dim, bias=False)
        self.value_head = nn.Linear(cfg.hidden_size, 1)

    def fuse_norms(self, on: bool = True) -> "MarioDT":
        """Fuses every block's input RMSNorm into its Q/K/V projection kernel."""
        for layer in self.model.layers:
            layer.fuse_norm(on)
        return self

    def reference_rounding(self, on: bool = True) -> "MarioDT":
        """Evaluates a 16-bit model at the reference's own rounding points, so its
        logits track the reference's 16-bit execution (model.to(torch.bfloat16))
        rather than only its fp32 one: unfused blocks (RMSNorm, projections,
        residual adds and the SwiGLU as separate roundings), RoPE with the
        reference's three roundings inside the attention kernels, and frames /
        255 rounded before the first convolution.  Slower than the fused
        default; off restores RoPE in fp32 and exact encoder inputs (call
        fuse_norms() again for the fused blocks)."""
        if on:
            self.fuse_norms(False)
        for layer in self.model.layers:
            layer.self_attn.rope_rounding = "reference" if on else "fp32"
        self.model.state_encoder.round_input = bool(on)
        return self

    def heads(self, hidden: Tensor) -> Tuple[Tensor, Tensor]:
        st = hidden[:, :, 1, :]  # state tokens predict the action (:505-507)
        return self.action_head(st), self.value_head(st).squeeze(-1)

    def forward(self, states, actions, returns_to_go, timesteps, attention_mask=None, action_targets=None,
                past_key_values=None, use_cache=False, **kw) -> DTOutput:
        hidden, presents = self.model(states, actions, returns_to_go, timesteps, attention_mask,
                                      past_key_values, use_cache)
        logits, values = self.heads(hidden)
        targets = action_targets if action_targets is not None else actions
        loss = F.cross_entropy(logits.reshape(-1, self.config.act_dim).float(), targets.reshape(-1).long(),
                               ignore_index=-100, label_smoothing=self.config.label_smoothing)
        return DTOutput(loss, logits, values, hidden, presents)

    @torch.no_grad()
    def act(self, states, actions, returns_to_go, timesteps, attention_mask=None, deterministic=False):
        """Next action from the last state token; re-prefills the context (:526-548)."""
        out = self.forward(states, actions, returns_to_go, timesteps, attention_mask, use_cache=False)
        logits = out.action_logits[:, -1, :]
        if deterministic:
            return torch.argmax(logits, dim=-1)
        return torch.distributions.Categorical(logits=logits.float()).sample()
