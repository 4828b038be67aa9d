"""Drop-in replacement of DecisionTransformerAttention backed by the sm_100a kernels.

``FastDTAttention`` keeps the reference module's constructor contract
(model/model_decision_transformer.py:137-163: same parameter names
q_proj/k_proj/v_proj/o_proj, ValueError when heads do not divide) and its
forward contract (:165-172, 249):

    forward(x, position_embeddings, past_key_value=None, use_cache=False,
            attention_mask=None) -> (out, past_kv)

Dispatch follows the reference (:198): the prefill kernel when
``flash and seq_len > 1 and past_key_value is None``, the cached decode
kernel otherwise.  ``past_key_value`` may be the reference's tuple of dense
tensors (functional: a new, longer tuple is returned, like torch.cat) or a
``cache.LayerKV`` (paged, appended in place and returned).

Masks: ``attention_mask`` [B, S] (prefill) or [B, kv_len] (decode), 1 =
valid, is taken as left padding (the layout scripts/mario/dt_offline_dataset.py
:228-235 produces); set ``check_masks=True`` to verify that on the host.
Numerics: bf16 / fp16 inputs run on the tensor-core kernels (fp32 softmax and
accumulation); fp32 inputs run on the fp32 kernels (CUDA cores, fp32
throughout) unless ``compute_dtype`` selects bf16/fp16 tensor-core compute, in
which case Q/K/V are cast for the kernels and the result is cast back.  There
is no CPU path: CPU inputs raise.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch import nn

from . import kernels
from .cache import LayerKV, dense_layer

Tensor = torch.Tensor


class FastDTAttention(nn.Module):
    def __init__(self, config, compute_dtype: Optional[torch.dtype] = None, check_masks: bool = False):
        super().__init__()
        self.num_key_value_heads = (config.num_attention_heads if config.num_key_value_heads is None
                                    else config.num_key_value_heads)
        if config.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        self.n_local_heads = config.num_attention_heads
        self.n_local_kv_heads = self.num_key_value_heads
        self.n_rep = self.n_local_heads // self.n_local_kv_heads
        self.head_dim = config.hidden_size // config.num_attention_heads
        self.dropout = getattr(config, "dropout", 0.0)
        self.flash = bool(getattr(config, "flash_attn", True))
        self.q_proj = nn.Linear(config.hidden_size, self.n_local_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(config.hidden_size, self.n_local_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(config.hidden_size, self.n_local_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(self.n_local_heads * self.head_dim, config.hidden_size, bias=False)
        self.attn_dropout = nn.Dropout(self.dropout)
        self.resid_dropout = nn.Dropout(self.dropout)
        self.compute_dtype = compute_dtype
        self.check_masks = check_masks
        # "fp32": RoPE in fp32 inside the kernels, one rounding of the result.
        # "reference": the reference's roundings (q * cos, rotate_half(q) * sin
        # and their sum each rounded to the activation dtype, :113-116).
        self.rope_rounding = "fp32"
        # RMSNorm of the owning block, fused into the projections when set
        # (held outside the module tree so the state_dict is unchanged).
        object.__setattr__(self, "_fused_norm", None)
        object.__setattr__(self, "_fused_w", None)
        object.__setattr__(self, "_fused_key", None)

    @classmethod
    def from_reference(cls, ref_attn: nn.Module, config, **kw) -> "FastDTAttention":
        """Builds the fast module with the weights of a reference DecisionTransformerAttention."""
        m = cls(config, **kw)
        m.load_state_dict(ref_attn.state_dict())
        p = next(ref_attn.parameters())
        return m.to(device=p.device, dtype=p.dtype)

    # ------------------------------------------------------------------ helpers
    def _kernel_dtype(self, x: Tensor) -> torch.dtype:
        kd = self.compute_dtype or x.dtype
        if kd not in (torch.bfloat16, torch.float16, torch.float32):
            raise TypeError(f"unsupported compute dtype {kd}")
        return kd

    def _pad_len(self, mask: Optional[Tensor], length: int) -> Optional[Tensor]:
        if mask is None:
            return None
        if mask.dim() != 2 or mask.shape[1] != length:
            raise ValueError(f"attention_mask must be [B, {length}], got {tuple(mask.shape)}")
        pad = kernels.pad_len_from_mask(mask, length)
        if self.check_masks:
            want = torch.arange(length, device=mask.device)[None] >= pad[:, None]
            if not torch.equal(want, mask != 0):
                raise ValueError("attention_mask is not a left-padding mask (zeros then ones per row)")
        return pad

    def set_fused_norm(self, norm: Optional[nn.Module]) -> None:
        """Fuses ``norm`` (an RMSNorm with ``weight`` and ``eps``) into the Q/K/V
        projections: forward(..., raw_input=True) then takes the un-normalised x."""
        object.__setattr__(self, "_fused_norm", norm)
        object.__setattr__(self, "_fused_w", None)

    def _fused_weight(self, dtype: torch.dtype) -> Tensor:
        ps = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight, self._fused_norm.weight)
        key = tuple((p.data_ptr(), p._version) for p in ps) + (dtype,)
        if self._fused_w is None or self._fused_key != key:
            w = kernels.fold_norm_weight(*ps, dtype=dtype)
            object.__setattr__(self, "_fused_w", w)
            object.__setattr__(self, "_fused_key", key)
        return self._fused_w

    def _qkv_rope_ok(self, x: Tensor) -> bool:
        """The one-GEMM q | k | v + RoPE path: 16-bit x [B, S, H] with a contiguous last
        dimension, no projection biases, head_dim 32 / 64, sizes multiples of 8."""
        H = x.shape[-1]
        return (x.dim() == 3 and x.stride(-1) == 1 and H % 8 == 0 and self.head_dim in (32, 64)
                and self.q_proj.bias is None and self.k_proj.bias is None and self.v_proj.bias is None
                and self.q_proj.weight.dtype == x.dtype and x.data_ptr() % 16 == 0
                and not (torch.is_grad_enabled() and (x.requires_grad or self.q_proj.weight.requires_grad)))

    def _cat_weight(self, dtype: torch.dtype) -> Tensor:
        """[Wq; Wk; Wv] as one contiguous [N, H] weight (cached while the parameters are unchanged)."""
        ps = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        key = tuple((p.data_ptr(), p._version) for p in ps) + (dtype,)
        if getattr(self, "_cat_key", None) != key:
            object.__setattr__(self, "_cat_w", torch.cat([p.to(dtype) for p in ps], dim=0).contiguous())
            object.__setattr__(self, "_cat_key", key)
        return self._cat_w

    def _project(self, x: Tensor, kd: torch.dtype, raw_input: bool, pe: Tuple[Tensor, Tensor]):
        """q, k, v [B, S, H*, D] and whether q / k are already rotated.  With the
        fused norm on 16-bit inputs one kernel does RMSNorm, the three
        projections and the RoPE of q / k (rows s of the position tables)."""
        bsz, seq_len, _ = x.shape
        Hq, Hkv, D = self.n_local_heads, self.n_local_kv_heads, self.head_dim
        if raw_input:
            if self._fused_norm is None:
                raise ValueError("raw_input=True needs set_fused_norm()")
            if x.dtype in (torch.bfloat16, torch.float16) and kd == x.dtype:
                qkv = kernels.rmsnorm_qkv(x, self._fused_weight(x.dtype), self._fused_norm.eps,
                                          rope=(pe[0], pe[1], (Hq + Hkv) * D, D))
                qkv = qkv.view(bsz, seq_len, Hq + 2 * Hkv, D)
                return qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hkv], qkv[:, :, Hq + Hkv:], True
            x = self._fused_norm(x)  # fp32 models: exact RMSNorm, then the projections
        if (x.dtype in (torch.bfloat16, torch.float16) and kd == x.dtype and self.rope_rounding == "fp32"
                and self._qkv_rope_ok(x)):
            # Drop-in path (x already normalised by the caller's block): one GEMM for
            # q | k | v with the RoPE of q and k in its epilogue, so the attention
            # kernels take pre-rotated q / k (their in-kernel RoPE is slower at D = 64).
            qkv = kernels.qkv_rope(x, self._cat_weight(x.dtype), pe[0], pe[1], (Hq + Hkv) * D, D)
            qkv = qkv.view(bsz, seq_len, Hq + 2 * Hkv, D)
            return qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hkv], qkv[:, :, Hq + Hkv:], True
        xq = self.q_proj(x).view(bsz, seq_len, Hq, D).to(kd)
        xk = self.k_proj(x).view(bsz, seq_len, Hkv, D).to(kd)
        xv = self.v_proj(x).view(bsz, seq_len, Hkv, D).to(kd)
        return xq, xk, xv, False

    # ------------------------------------------------------------------ forward
    def forward(self, x: Tensor, position_embeddings: Tuple[Tensor, Tensor],
                past_key_value=None, use_cache: bool = False, attention_mask: Optional[Tensor] = None,
                raw_input: bool = False, residual: Optional[Tensor] = None, residual_inplace: bool = False):
        """``residual`` (the block input, [B, S, H]) is added to the output: one
        GEMM with the residual as its accumulator input when dropout is off;
        with ``residual_inplace`` (a caller that owns the residual and no longer
        needs it) the GEMM accumulates into it instead of a copy."""
        if not x.is_cuda:
            raise ValueError("FastDTAttention runs on CUDA only (no CPU path)")
        bsz, seq_len, _ = x.shape
        kd = self._kernel_dtype(x)
        cos, sin = position_embeddings
        xq, xk, xv, rotated = self._project(x, kd, raw_input, (cos, sin))
        if self.rope_rounding not in ("fp32", "reference"):
            raise ValueError(f"rope_rounding must be 'fp32' or 'reference', got {self.rope_rounding!r}")
        rope = 0 if rotated else (2 if self.rope_rounding == "reference" else 1)

        if (isinstance(past_key_value, LayerKV) and past_key_value.length == 0 and seq_len > 1 and self.flash
                and attention_mask is None):
            # First fill of a paged cache: prefill kernel, then write the rotated
            # keys and values into the pages (same result as the cached branch
            # with an empty cache, :225-245).
            layer = past_key_value
            if layer.k_pages.dtype != kd:
                raise TypeError(f"cache dtype {layer.k_pages.dtype} differs from compute dtype {kd}")
            if seq_len > layer.capacity:
                raise ValueError(f"cache full: {seq_len} > capacity {layer.capacity}")
            out = kernels.attn_prefill(xq, xk, xv, cos, sin, None, apply_rope=rope)
            kernels.kv_write(xk, xv, layer, cos, sin, apply_rope=rope)
            layer.advance(seq_len)
            past_kv = layer if use_cache else None
        elif self.flash and seq_len > 1 and past_key_value is None:
            out = kernels.attn_prefill(xq, xk, xv, cos, sin, self._pad_len(attention_mask, seq_len), apply_rope=rope)
            past_kv = None
            if use_cache:
                kc = torch.empty(bsz, self.n_local_kv_heads, seq_len, self.head_dim, dtype=kd, device=x.device)
                vc = torch.empty_like(kc)
                layer = dense_layer(kc, vc, 0)
                kernels.kv_write(xk, xv, layer, cos, sin, apply_rope=rope)
                past_kv = (kc, vc)
        else:
            if isinstance(past_key_value, LayerKV):
                layer = past_key_value
                if layer.k_pages.dtype != kd:
                    raise TypeError(f"cache dtype {layer.k_pages.dtype} differs from compute dtype {kd}")
                kv_len = layer.length + seq_len
                out = kernels.attn_decode(xq, xk, xv, layer, cos, sin, self._pad_len(attention_mask, kv_len),
                                          apply_rope=rope)
                layer.advance(seq_len)
                past_kv = layer if use_cache else None
            else:
                # Reference tuple (or no cache): functional append into new dense tensors.
                L = 0 if past_key_value is None else past_key_value[0].shape[2]
                kc = torch.empty(bsz, self.n_local_kv_heads, L + seq_len, self.head_dim, dtype=kd,
                                 device=x.device)
                vc = torch.empty_like(kc)
                if L:
                    kc[:, :, :L].copy_(past_key_value[0])
                    vc[:, :, :L].copy_(past_key_value[1])
                layer = dense_layer(kc, vc, L)
                out = kernels.attn_decode(xq, xk, xv, layer, cos, sin,
                                          self._pad_len(attention_mask, L + seq_len), apply_rope=rope)
                past_kv = (kc, vc) if use_cache else None

        out = out.reshape(bsz, seq_len, -1).to(x.dtype)
        if residual is None:
            return self.resid_dropout(self.o_proj(out)), past_kv
        w = self.o_proj.weight
        if ((not self.training or self.resid_dropout.p == 0) and self.o_proj.bias is None
                and residual.dtype == out.dtype == w.dtype):
            r2 = residual.reshape(-1, residual.shape[-1])
            o2 = out.reshape(-1, out.shape[-1])
            if not (residual_inplace and r2.data_ptr() == residual.data_ptr() and r2.is_contiguous()):
                r2 = r2.clone()  # the caller keeps its residual: accumulate into a copy
            # o_proj with the residual as the GEMM's accumulator input: the
            # library's CTA-pair GEMM at prefill sizes, cuBLAS's addmm_ for a
            # rollout step's small, latency-bound GEMM (measured faster there).
            if kernels.gemm_residual_on_pairs(o2, w, r2):
                kernels.gemm_residual(o2, w, r2)
            else:
                r2.addmm_(o2, w.t())
            return r2.view(residual.shape), past_kv
        return residual + self.resid_dropout(self.o_proj(out)), past_kv


def swap_attention(model: nn.Module, config, **kw) -> int:
    """Replaces every ``self_attn`` DecisionTransformerAttention of a reference DT
    (or of dt_model.MarioDT) by FastDTAttention with the same weights; returns
    the number of modules swapped."""
    n = 0
    for name, mod in list(model.named_modules()):
        attn = getattr(mod, "self_attn", None)
        if attn is not None and not isinstance(attn, FastDTAttention) and hasattr(attn, "q_proj"):
            mod.self_attn = FastDTAttention.from_reference(attn, config, **kw)
            n += 1
    return n
