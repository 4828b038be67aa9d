"""Tensor-level wrappers over the C-ABI entry points.

Each wrapper validates device / dtype, allocates its outputs with torch (the
library itself never allocates), and launches on torch's current CUDA stream.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib

Tensor = torch.Tensor

_DTYPES = {torch.bfloat16: _lib.DT_DTYPE_BF16, torch.float16: _lib.DT_DTYPE_FP16,
           torch.float32: _lib.DT_DTYPE_FP32}


def _dtype_code(t: Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: Optional[Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("dt attention kernels take CUDA tensors only (no CPU path)")


def pad_len_from_mask(attention_mask: Tensor, S: int) -> Tensor:
    """Left-padding length per row of a [B, S] 0/1 mask (1 = valid), as int32 on its device.

    The DT dataset left-pads (scripts/mario/dt_offline_dataset.py:228-235), so
    the number of zeros is the index of the first valid token.
    """
    m = attention_mask.reshape(attention_mask.shape[0], -1)
    if m.shape[1] != S:
        raise ValueError(f"attention_mask has {m.shape[1]} columns, expected {S}")
    return (S - (m != 0).sum(dim=1)).to(torch.int32)


def attn_prefill(q: Tensor, k: Tensor, v: Tensor, cos: Optional[Tensor], sin: Optional[Tensor],
                 pad_len: Optional[Tensor] = None, out: Optional[Tensor] = None, apply_rope: bool = True,
                 scale: Optional[float] = None) -> Tensor:
    """Causal GQA prefill: q [B,S,Hq,D], k/v [B,S,Hkv,D] -> out [B,S,Hq,D].

    RoPE (cos/sin [>=S, D] fp32) is applied to q and k inside the kernel when
    apply_rope; pad_len [B] int32 gives per-row left padding (None = no mask).
    """
    _require_cuda(q, k, v, cos, sin, pad_len, out)
    B, S, Hq, D = q.shape
    Hkv = k.shape[2]
    if k.shape != (B, S, Hkv, D) or v.shape != (B, S, Hkv, D):
        raise ValueError(f"k/v shapes {tuple(k.shape)}, {tuple(v.shape)} do not match q {tuple(q.shape)}")
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share a dtype")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(3) != 1:
            raise ValueError(f"{name} must be contiguous in head_dim")
    if out is None:
        out = torch.empty((B, S, Hq, D), dtype=q.dtype, device=q.device)
    if apply_rope:
        if cos is None or sin is None:
            raise ValueError("apply_rope needs cos and sin")
        cos = cos.float().contiguous() if (cos.dtype != torch.float32 or cos.stride(-1) != 1) else cos
        sin = sin.float().contiguous() if (sin.dtype != torch.float32 or sin.stride(-1) != 1) else sin
        if cos.stride(0) != sin.stride(0):
            cos, sin = cos.contiguous(), sin.contiguous()
    if pad_len is not None:
        pad_len = pad_len.to(torch.int32).contiguous()
    lib = _lib.load()
    rc = lib.dt_attn_prefill(
        _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(cos) if apply_rope else None,
        _ptr(sin) if apply_rope else None, cos.shape[0] if apply_rope else 0,
        cos.stride(0) if apply_rope else 0, _ptr(pad_len), B, S, Hq, Hkv, D,
        q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
        v.stride(0), v.stride(1), v.stride(2), out.stride(0), out.stride(1), out.stride(2),
        float(scale) if scale is not None else 0.0, 1 if apply_rope else 0, _dtype_code(q),
        _stream_ptr(q.device))
    _lib.check("dt_attn_prefill", rc)
    return out


def device_status(device: Optional[torch.device] = None) -> int:
    """Synchronises the current stream; returns and clears the kernels' device status word."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    return _lib.load().dt_device_status(_stream_ptr(dev))


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)
