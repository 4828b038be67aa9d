"""Tensor-level wrappers over the C-ABI entry points.

Each wrapper validates device / dtype, allocates its outputs with torch (the
library itself never allocates), and launches on torch's current CUDA stream.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

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


def _rope_mode(apply_rope) -> int:
    """apply_rope of the entry points: False / 0 none, True / 1 RoPE in fp32 with one
    rounding of the result, 2 the reference's roundings in the activation dtype
    (q * cos, rotate_half(q) * sin and their sum each rounded, as on 16-bit tensors)."""
    mode = int(apply_rope)
    if mode not in (0, 1, 2):
        raise ValueError(f"apply_rope must be False/True or 0, 1, 2 (got {apply_rope!r})")
    return mode


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
    apply_rope (2: with the reference's roundings, see _rope_mode); pad_len [B]
    int32 gives per-row left padding (None = no mask).
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
        float(scale) if scale is not None else 0.0, _rope_mode(apply_rope), _dtype_code(q),
        _stream_ptr(q.device))
    _lib.check("dt_attn_prefill", rc)
    return out


_COPY_STREAMS: dict = {}


def _copy_streams(device: torch.device):
    """A host-to-device and a device-to-host stream per device (created once)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    if key not in _COPY_STREAMS:
        _COPY_STREAMS[key] = (torch.cuda.Stream(device=key), torch.cuda.Stream(device=key))
    return _COPY_STREAMS[key]


def attn_prefill_host(hq: Tensor, hk: Tensor, hv: Tensor, cos: Optional[Tensor], sin: Optional[Tensor],
                      hpad: Optional[Tensor], hout: Tensor, device_buffers: Tuple[Tensor, ...],
                      chunks: int = 8, apply_rope: bool = True, scale: Optional[float] = None) -> Tensor:
    """attn_prefill on host tensors: q/k/v (and pad_len) in pinned host memory in,
    out into the pinned host tensor ``hout``.

    The batch is cut into ``chunks`` pieces of whole samples (samples are
    independent) and pipelined over three streams: the copy of chunk i + 1 to
    the device, the kernel on chunk i (current stream) and the copy of chunk
    i - 1 back run at the same time, so the step costs about the larger of the
    two PCIe transfers instead of their sum.  ``device_buffers`` = (q, k, v,
    pad_len or None, out) device tensors of the full batch's shapes.  On return
    the current stream is ordered after every copy (synchronise it, or record an
    event on it, before reading ``hout`` on the host).
    """
    dq, dk, dv, dpad, dout = device_buffers
    for name, h in (("hq", hq), ("hk", hk), ("hv", hv), ("hout", hout), ("hpad", hpad)):
        if h is not None and (h.is_cuda or not h.is_pinned()):
            raise ValueError(f"{name} must be a pinned host tensor")
    _require_cuda(dq, dk, dv, dpad, dout)
    if (hpad is None) != (dpad is None):
        raise ValueError("hpad and the device pad_len buffer go together")
    # Tensor.copy_ would silently cast or broadcast: host and device buffers
    # must match exactly.
    for name, h, d in (("q", hq, dq), ("k", hk, dk), ("v", hv, dv), ("out", hout, dout), ("pad_len", hpad, dpad)):
        if h is not None and (h.dtype != d.dtype or h.shape != d.shape):
            raise ValueError(f"host {name} {tuple(h.shape)} {h.dtype} does not match its device buffer "
                             f"{tuple(d.shape)} {d.dtype}")
    B = hq.shape[0]
    chunks = max(1, min(int(chunks), B))
    bounds = [B * i // chunks for i in range(chunks + 1)]
    dev = dq.device
    cur = torch.cuda.current_stream(dev)
    s_in, s_out = _copy_streams(dev)
    # Earlier work on the current stream (a previous call's kernels reading these
    # buffers) comes before this call's uploads.
    s_in.wait_stream(cur)
    for i in range(chunks):
        b0, b1 = bounds[i], bounds[i + 1]
        if b1 == b0:
            continue
        with torch.cuda.stream(s_in):
            dq[b0:b1].copy_(hq[b0:b1], non_blocking=True)
            dk[b0:b1].copy_(hk[b0:b1], non_blocking=True)
            dv[b0:b1].copy_(hv[b0:b1], non_blocking=True)
            if hpad is not None:
                dpad[b0:b1].copy_(hpad[b0:b1], non_blocking=True)
        cur.wait_stream(s_in)
        attn_prefill(dq[b0:b1], dk[b0:b1], dv[b0:b1], cos, sin, None if dpad is None else dpad[b0:b1],
                     out=dout[b0:b1], apply_rope=apply_rope, scale=scale)
        s_out.wait_stream(cur)
        with torch.cuda.stream(s_out):
            hout[b0:b1].copy_(dout[b0:b1], non_blocking=True)
    cur.wait_stream(s_out)
    return hout


def device_status(device: Optional[torch.device] = None) -> int:
    """Synchronises the current stream; returns and clears the kernels' device status word."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    return _lib.load().dt_device_status(_stream_ptr(dev))


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)


def _prep_tables(cos: Optional[Tensor], sin: Optional[Tensor]):
    if cos is None or sin is None:
        raise ValueError("apply_rope needs cos and sin")
    if cos.dtype != torch.float32 or cos.stride(-1) != 1:
        cos = cos.float().contiguous()
    if sin.dtype != torch.float32 or sin.stride(-1) != 1:
        sin = sin.float().contiguous()
    if cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin


def attn_decode(q: Tensor, k_new: Tensor, v_new: Tensor, layer, cos: Optional[Tensor], sin: Optional[Tensor],
                pad_len: Optional[Tensor] = None, rope_abs: bool = False, out: Optional[Tensor] = None,
                apply_rope: bool = True, scale: Optional[float] = None) -> Tensor:
    """Cached decode step: q [B,Sn,Hq,D], k_new/v_new [B,Sn,Hkv,D] -> out [B,Sn,Hq,D].

    Appends the rotated k_new / v_new to ``layer`` (a cache.LayerKV) at
    positions layer.seq_lens .. +Sn and attends over all cached keys.  Does not
    advance the layer's length (the caller does, once per step).
    """
    _require_cuda(q, k_new, v_new, cos, sin, pad_len, out)
    B, Sn, Hq, D = q.shape
    Hkv = k_new.shape[2]
    if k_new.shape != (B, Sn, Hkv, D) or v_new.shape != (B, Sn, Hkv, D):
        raise ValueError("k_new/v_new shapes do not match q")
    if not (q.dtype == k_new.dtype == v_new.dtype == layer.k_pages.dtype):
        raise TypeError("q, k_new, v_new and the cache must share a dtype")
    if layer.batch != B or layer.num_kv_heads != Hkv or layer.head_dim != D:
        raise ValueError("cache geometry does not match the inputs")
    if layer.length + Sn > layer.capacity:
        raise ValueError(f"cache full: {layer.length} + {Sn} > capacity {layer.capacity}")
    for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new)):
        if t.stride(3) != 1:
            raise ValueError(f"{name} must be contiguous in head_dim")
    if out is None:
        out = torch.empty((B, Sn, Hq, D), dtype=q.dtype, device=q.device)
    if apply_rope:
        cos, sin = _prep_tables(cos, sin)
    if pad_len is not None:
        pad_len = pad_len.to(torch.int32).contiguous()
    lib = _lib.load()
    rc = lib.dt_attn_decode(
        _ptr(q), _ptr(k_new), _ptr(v_new), _ptr(out), _ptr(layer.k_pages), _ptr(layer.v_pages),
        layer.k_pages.shape[0], layer.page_size, _ptr(layer.block_table), layer.block_table.shape[1],
        _ptr(layer.seq_lens), _ptr(pad_len), _ptr(cos) if apply_rope else None, _ptr(sin) if apply_rope else None,
        cos.shape[0] if apply_rope else 0, cos.stride(0) if apply_rope else 0, 1 if rope_abs else 0,
        B, Sn, Hq, Hkv, D, q.stride(0), q.stride(1), q.stride(2), k_new.stride(0), k_new.stride(1),
        k_new.stride(2), v_new.stride(0), v_new.stride(1), v_new.stride(2), out.stride(0), out.stride(1),
        out.stride(2), float(scale) if scale is not None else 0.0, _rope_mode(apply_rope), _dtype_code(q),
        _stream_ptr(q.device))
    _lib.check("dt_attn_decode", rc)
    return out


def kv_write(k: Tensor, v: Tensor, layer, cos: Optional[Tensor], sin: Optional[Tensor],
             start_pos: Optional[Tensor] = None, rope_abs: bool = False, apply_rope: bool = True) -> None:
    """Writes k (rotated) and v [B,S,Hkv,D] into ``layer`` at positions start_pos[b] + s."""
    _require_cuda(k, v, cos, sin, start_pos)
    B, S, Hkv, D = k.shape
    if v.shape != k.shape:
        raise ValueError("k and v shapes differ")
    if k.dtype != layer.k_pages.dtype or v.dtype != k.dtype:
        raise TypeError("k, v and the cache must share a dtype")
    if k.stride(3) != 1 or v.stride(3) != 1:
        raise ValueError("k/v must be contiguous in head_dim")
    if apply_rope:
        cos, sin = _prep_tables(cos, sin)
    if start_pos is not None:
        start_pos = start_pos.to(torch.int32).contiguous()
    lib = _lib.load()
    rc = lib.dt_kv_write(
        _ptr(k), _ptr(v), _ptr(layer.k_pages), _ptr(layer.v_pages), layer.k_pages.shape[0], layer.page_size,
        _ptr(layer.block_table), layer.block_table.shape[1], _ptr(start_pos), _ptr(cos) if apply_rope else None,
        _ptr(sin) if apply_rope else None, cos.shape[0] if apply_rope else 0, cos.stride(0) if apply_rope else 0,
        1 if rope_abs else 0, B, S, Hkv, D, k.stride(0), k.stride(1), k.stride(2), v.stride(0), v.stride(1),
        v.stride(2), _rope_mode(apply_rope), _dtype_code(k), _stream_ptr(k.device))
    _lib.check("dt_kv_write", rc)


def fold_norm_weight(w_q: Tensor, w_k: Tensor, w_v: Tensor, w_norm: Tensor, dtype: torch.dtype) -> Tensor:
    """[Wq; Wk; Wv] * diag(w_norm) in ``dtype``: the weight of rmsnorm_qkv."""
    w = torch.cat([w_q, w_k, w_v], dim=0).float() * w_norm.float()[None, :]
    return w.to(dtype).contiguous()


def frames_to_blocks(frames: Tensor, dtype: torch.dtype, frame_max: Optional[Tensor] = None) -> Tensor:
    """uint8 frames [N, C, H, W] -> ``dtype`` 4 x 4 space-to-depth blocks as a
    channels-last [N, C*16, H/4, W/4] tensor (channel c*16 + dy*4 + dx).
    ``frame_max`` (an int32 [1] device tensor) is raised to the largest byte."""
    _require_cuda(frames, frame_max)
    if frame_max is not None and (frame_max.dtype != torch.int32 or frame_max.numel() != 1):
        raise ValueError("frame_max must be an int32 tensor with one element")
    if frames.dtype != torch.uint8 or frames.dim() != 4 or not frames.is_contiguous():
        raise ValueError("frames must be a contiguous uint8 [N, C, H, W] tensor")
    N, C, H, W = frames.shape
    out = torch.empty((N, C * 16, H // 4, W // 4), dtype=dtype, device=frames.device,
                      memory_format=torch.channels_last)
    rc = _lib.load().dt_frames_to_blocks(_ptr(frames), _ptr(out), N, C, H, W,
                                         None if frame_max is None else _ptr(frame_max), _dtype_code(out),
                                         _stream_ptr(frames.device))
    _lib.check("dt_frames_to_blocks", rc)
    return out


def frames_conv1(frames: Tensor, weight: Tensor, bias: Tensor, round_input: bool = False) -> Tuple[Tensor, Tensor]:
    """relu(conv2d(frames / 255 if max > 1 else frames, weight, bias, stride 4)) from
    uint8 frames [N, 4, H, W] with an 8 x 8 weight [32, 4, 8, 8] (16-bit): returns the
    output as a channels-last [N, 32, OH, OW] tensor of the weight's dtype and an
    int32 [1] device tensor that is > 1 exactly when the frames' max exceeds 1.
    round_input: frames / 255 rounded to the weight's dtype before the
    convolution (the reference's 16-bit rounding) instead of exact pixels."""
    _require_cuda(frames, weight, bias)
    if frames.dtype != torch.uint8 or frames.dim() != 4 or not frames.is_contiguous():
        raise ValueError("frames must be a contiguous uint8 [N, C, H, W] tensor")
    N, C, H, W = frames.shape
    if tuple(weight.shape) != (32, C, 8, 8):
        raise ValueError(f"weight must be [32, {C}, 8, 8]")
    OH, OW = (H - 8) // 4 + 1, (W - 8) // 4 + 1
    w2 = weight.reshape(32, C * 64).contiguous()
    b = bias.float().contiguous()
    out = torch.empty((N, 32, OH, OW), dtype=weight.dtype, device=frames.device, memory_format=torch.channels_last)
    fmax = torch.empty(1, dtype=torch.int32, device=frames.device)
    rc = _lib.load().dt_frames_conv1(_ptr(frames), N, C, H, W, _ptr(w2), _ptr(b), _ptr(fmax), _ptr(out),
                                     1 if round_input else 0, _dtype_code(out), _stream_ptr(frames.device))
    _lib.check("dt_frames_conv1", rc)
    return out, fmax


def encoder_conv23(x1: Tensor, w2: Tensor, b2: Tensor, w3: Tensor, b3: Tensor,
                   keep_y2: bool = True) -> Tuple[Optional[Tensor], Tensor]:
    """relu(conv2d(x1, w2, b2, stride 2)) and relu(conv2d(that, w3, b3)) for the
    state encoder's second and third layers: x1 a channels-last [N, 32, 20, 20]
    16-bit tensor (the first layer's output), w2 [64, 32, 4, 4], w3 [64, 64, 3, 3]
    of x1's dtype.  Returns both outputs as channels-last tensors ([N, 64, 9, 9],
    [N, 64, 7, 7]); with keep_y2=False the second layer's output is not written
    to memory at all (None is returned in its place)."""
    _require_cuda(x1, w2, b2, w3, b3)
    if x1.dim() != 4 or tuple(x1.shape[1:]) != (32, 20, 20) or not x1.is_contiguous(memory_format=torch.channels_last):
        raise ValueError("x1 must be a channels-last [N, 32, 20, 20] tensor")
    if tuple(w2.shape) != (64, 32, 4, 4) or tuple(w3.shape) != (64, 64, 3, 3):
        raise ValueError("w2 must be [64, 32, 4, 4] and w3 [64, 64, 3, 3]")
    if w2.dtype != x1.dtype or w3.dtype != x1.dtype or tuple(b2.shape) != (64,) or tuple(b3.shape) != (64,):
        raise ValueError("weights must have x1's dtype and biases 64 entries")
    N = x1.shape[0]
    w2c, w3c = w2.contiguous(), w3.contiguous()
    b2f, b3f = b2.float().contiguous(), b3.float().contiguous()
    cl = torch.channels_last
    y2 = torch.empty((N, 64, 9, 9), dtype=x1.dtype, device=x1.device, memory_format=cl) if keep_y2 else None
    y3 = torch.empty((N, 64, 7, 7), dtype=x1.dtype, device=x1.device, memory_format=cl)
    rc = _lib.load().dt_encoder_conv23(_ptr(x1), N, _ptr(w2c), _ptr(b2f), _ptr(y2), _ptr(w3c), _ptr(b3f), _ptr(y3),
                                       _dtype_code(x1), _stream_ptr(x1.device))
    _lib.check("dt_encoder_conv23", rc)
    return y2, y3


def rmsnorm(x: Tensor, weight: Tensor, eps: float, out: Optional[Tensor] = None) -> Tensor:
    """weight * cast(x * rsqrt(mean(x^2) + eps)) over the last dim (bf16 / fp16)."""
    _require_cuda(x, weight, out)
    K = x.shape[-1]
    if weight.shape != (K,) or weight.dtype != x.dtype or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous [K] tensor of x's dtype")
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    o2 = out.view(-1, K)
    rc = _lib.load().dt_rmsnorm(_ptr(x2), x2.stride(0), _ptr(weight), _ptr(o2), o2.stride(0), x2.shape[0], K,
                                float(eps), _dtype_code(x), _stream_ptr(x.device))
    _lib.check("dt_rmsnorm", rc)
    return out


def fold_swiglu_weight(w_gate: Tensor, w_up: Tensor, w_norm: Tensor, dtype: torch.dtype) -> Tensor:
    """The weight of rmsnorm_swiglu: gate and up rows scaled by the norm weight,
    interleaved in blocks of 64 rows ([gate 0:64; up 0:64; gate 64:128; ...])."""
    inter, hidden = w_gate.shape
    if w_up.shape != w_gate.shape or inter % 64:
        raise ValueError("gate / up weights must be equal [F, H] with F a multiple of 64")
    nw = w_norm.float()[None, None, :]
    g = w_gate.float().view(inter // 64, 64, hidden) * nw
    u = w_up.float().view(inter // 64, 64, hidden) * nw
    return torch.stack((g, u), dim=1).reshape(2 * inter, hidden).to(dtype).contiguous()


def rmsnorm_swiglu(x: Tensor, w_fused: Tensor, eps: float, out: Optional[Tensor] = None) -> Tensor:
    """silu(g) * u with [g | u] = RMSNorm(x) @ [W_gate; W_up]^T: the post-attention
    norm and the SwiGLU up-projection of the block's MLP in one kernel.

    x [..., K] bf16/fp16 -> y [..., F], ``w_fused`` = fold_swiglu_weight(...) [2F, K].
    """
    _require_cuda(x, w_fused, out)
    K = x.shape[-1]
    F2 = w_fused.shape[0]
    if w_fused.shape[1] != K or w_fused.dtype != x.dtype or not w_fused.is_contiguous() or F2 % 128:
        raise ValueError("w_fused must be a contiguous [2F, K] tensor of x's dtype (F a multiple of 64)")
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty(x.shape[:-1] + (F2 // 2,), dtype=x.dtype, device=x.device)
    o2 = out.view(-1, F2 // 2)
    rc = _lib.load().dt_rmsnorm_swiglu(_ptr(x2), x2.stride(0), _ptr(w_fused), _ptr(o2), o2.stride(0), M, K,
                                       F2 // 2, float(eps), _dtype_code(x), _stream_ptr(x.device))
    _lib.check("dt_rmsnorm_swiglu", rc)
    return out


def qkv_rope(x: Tensor, w_cat: Tensor, cos: Tensor, sin: Tensor, rope_cols: int, head_dim: int,
             out: Optional[Tensor] = None) -> Tensor:
    """[q | k | v] = x @ w_cat^T with the rotate-half RoPE of the q and k heads
    (the first rope_cols columns) in the GEMM epilogue, no norm: x [B, S, K]
    16-bit, w_cat = [Wq; Wk; Wv] [N, K] -> y [B, S, N]; row (b, s) uses table
    row s of cos / sin."""
    _require_cuda(x, w_cat, cos, sin, out)
    if x.dim() != 3:
        raise ValueError("qkv_rope needs x of shape [B, S, K]")
    K = x.shape[-1]
    N = w_cat.shape[0]
    if w_cat.shape[1] != K or w_cat.dtype != x.dtype or not w_cat.is_contiguous():
        raise ValueError("w_cat must be a contiguous [N, K] tensor of x's dtype")
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    if out is None:
        out = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    o2 = out.view(-1, N)
    cos, sin = _prep_tables(cos, sin)
    rc = _lib.load().dt_qkv_rope(_ptr(x2), x2.stride(0), _ptr(w_cat), _ptr(o2), o2.stride(0), x2.shape[0], K, N,
                                 _ptr(cos), _ptr(sin), cos.stride(0), cos.shape[0], x.shape[1], int(rope_cols),
                                 int(head_dim), _dtype_code(x), _stream_ptr(x.device))
    _lib.check("dt_qkv_rope", rc)
    return out


def gemm_residual_ok(x: Tensor, w: Tensor, y: Tensor) -> bool:
    """Whether gemm_residual takes these operands (16-bit CUDA tensors, row-major
    views with 16-byte aligned rows, N a multiple of 64)."""
    if not (x.is_cuda and y.is_cuda and w.is_cuda):
        return False
    if x.dtype not in (torch.bfloat16, torch.float16) or w.dtype != x.dtype or y.dtype != x.dtype:
        return False
    K, N = x.shape[-1], y.shape[-1]
    if w.shape != (N, K) or N % 64 or K % 8 or not w.is_contiguous():
        return False
    for t in (x, y):
        if t.dim() != 2 or t.stride(1) != 1 or t.stride(0) % 8 or t.data_ptr() % 16:
            return False
    return x.shape[0] == y.shape[0]


_NUM_SMS: dict = {}


def gemm_residual_on_pairs(x: Tensor, w: Tensor, y: Tensor) -> bool:
    """Whether gemm_residual runs these operands on CTA pairs: N a multiple of 256 and
    at least four 256 x 256 tiles per pair of SMs, the sizes at which it matches
    cuBLAS's addmm (cfg4's o_proj / down_proj, measured).  Smaller, latency-bound
    problems (a rollout step's GEMMs) fall to the single-CTA kernel, which is slower
    than cuBLAS there."""
    if not gemm_residual_ok(x, w, y):
        return False
    M, N = y.shape
    dev = y.device.index if y.device.index is not None else torch.cuda.current_device()
    if dev not in _NUM_SMS:
        _NUM_SMS[dev] = torch.cuda.get_device_properties(dev).multi_processor_count
    return N % 256 == 0 and ((M + 255) // 256) * (N // 256) >= 2 * _NUM_SMS[dev]


def gemm_residual(x: Tensor, w: Tensor, y: Tensor) -> Tensor:
    """y += x @ w^T in place (fp32 accumulation, one rounding of the sum): the
    block's o_proj / down_proj with its residual add.  x [M, K], w [N, K],
    y [M, N] (2-D row-major views), bf16 / fp16."""
    _require_cuda(x, w, y)
    if not gemm_residual_ok(x, w, y):
        raise ValueError("gemm_residual: x [M, K], w [N, K] contiguous, y [M, N] 16-bit row-major views with "
                         "16-byte aligned rows and N a multiple of 64")
    rc = _lib.load().dt_gemm_residual(_ptr(x), x.stride(0), _ptr(w), _ptr(y), y.stride(0), x.shape[0], x.shape[1],
                                      y.shape[1], _dtype_code(x), _stream_ptr(x.device))
    _lib.check("dt_gemm_residual", rc)
    return y


def rmsnorm_qkv(x: Tensor, w_fused: Tensor, eps: float, out: Optional[Tensor] = None,
                rope: Optional[Tuple[Tensor, Tensor, int, int]] = None) -> Tensor:
    """y = RMSNorm(x) @ [Wq; Wk; Wv]^T with the norm weight folded into ``w_fused`` [N, K].

    x [..., K] bf16/fp16 (last dim contiguous) -> y [..., N] (the fused q|k|v rows).
    ``rope = (cos, sin, rope_cols, head_dim)`` also rotates the first rope_cols
    columns (the q and k heads) in the epilogue; x is then [B, S, K] and row
    (b, s) uses table row s.
    """
    _require_cuda(x, w_fused, out)
    if rope is not None:
        _require_cuda(rope[0], rope[1])
    K = x.shape[-1]
    N = w_fused.shape[0]
    if w_fused.shape[1] != K or w_fused.dtype != x.dtype or not w_fused.is_contiguous():
        raise ValueError("w_fused must be a contiguous [N, K] tensor of x's dtype")
    x2 = x.reshape(-1, K)
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M = x2.shape[0]
    if out is None:
        out = torch.empty(x.shape[:-1] + (N,), dtype=x.dtype, device=x.device)
    o2 = out.view(-1, N)
    if rope is None:
        rc = _lib.load().dt_rmsnorm_qkv(_ptr(x2), x2.stride(0), _ptr(w_fused), _ptr(o2), o2.stride(0), M, K, N,
                                        float(eps), _dtype_code(x), _stream_ptr(x.device))
        _lib.check("dt_rmsnorm_qkv", rc)
        return out
    if x.dim() != 3:
        raise ValueError("rmsnorm_qkv with rope needs x of shape [B, S, K]")
    cos, sin = _prep_tables(rope[0], rope[1])
    rope_cols, head_dim = int(rope[2]), int(rope[3])
    rc = _lib.load().dt_rmsnorm_qkv_rope(_ptr(x2), x2.stride(0), _ptr(w_fused), _ptr(o2), o2.stride(0), M, K, N,
                                         float(eps), _ptr(cos), _ptr(sin), cos.stride(0), cos.shape[0], x.shape[1],
                                         rope_cols, head_dim, _dtype_code(x), _stream_ptr(x.device))
    _lib.check("dt_rmsnorm_qkv_rope", rc)
    return out
