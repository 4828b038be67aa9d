"""GPU parity of the fused prefill kernel (dt_attn_prefill) against the CPU oracle.

Inputs are drawn in float32, rounded to the kernel dtype, and the oracle sees
the same rounded values upcast to float32.  Tolerances (written per dtype
below) cover bf16/fp16 rounding of the rotated q/k, the probabilities and the
output; the mean error bound catches systematic mistakes that a loose
max-abs bound would let through.
"""
import pytest
import torch

from oracle import attention_prefill_ref, mask_from_pad_len, precompute_freqs_cis

TOL = {torch.bfloat16: dict(atol=1.5e-2, rtol=1e-2, mean=2.5e-3),
       torch.float16: dict(atol=4e-3, rtol=4e-3, mean=5e-4),
       torch.float32: dict(atol=1e-5, rtol=1e-5, mean=1e-6)}

CASES = [
    # B, S, Hq, Hkv, D, pads, dtype
    (3, 24, 8, 2, 32, [0, 6, 15], torch.bfloat16),
    (4, 192, 8, 2, 32, [0, 96, 47, 191], torch.bfloat16),
    (6, 21, 8, 2, 32, [0, 1, 20, 21, 7, 16], torch.bfloat16),
    (2, 1, 8, 2, 32, None, torch.bfloat16),
    (2, 7, 8, 2, 32, [0, 3], torch.bfloat16),
    (2, 150, 8, 2, 32, [0, 96], torch.float16),
    (2, 768, 12, 4, 64, [0, 384], torch.bfloat16),
    (3, 100, 12, 4, 64, [0, 5, 50], torch.float16),
    (2, 300, 8, 8, 32, [0, 17], torch.bfloat16),
    (2, 64, 16, 2, 32, [0, 10], torch.bfloat16),
    (1, 255, 8, 2, 32, None, torch.bfloat16),
    (2, 129, 4, 4, 64, [0, 128], torch.bfloat16),
    (3, 100, 4, 4, 32, [0, 50, 99], torch.bfloat16),
    (4, 190, 4, 2, 32, [0, 1, 100, 189], torch.float16),
    (300, 96, 8, 2, 32, "random", torch.bfloat16),
    (150, 192, 8, 2, 32, "random", torch.bfloat16),
    (3, 24, 8, 2, 32, [0, 6, 15], torch.float32),
    (4, 192, 8, 2, 32, [0, 96, 47, 191], torch.float32),
    (2, 300, 12, 4, 64, [0, 100], torch.float32),
    (2, 1, 8, 2, 32, None, torch.float32),
]


def _run_case(B, S, Hq, Hkv, D, pads, dtype, seed=0, fused_layout=False, rope=True):
    from rl_for_mario_b200.kernels import attn_prefill, device_status

    g = torch.Generator().manual_seed(seed)
    if fused_layout:
        # q/k/v as strided views of one [B, S, Hq + 2 Hkv, D] projection output.
        qkv = (torch.randn(B, S, Hq + 2 * Hkv, D, generator=g) * 0.5).to(dtype)
        q32, k32, v32 = qkv.float().split([Hq, Hkv, Hkv], dim=2)
        dev = qkv.cuda()
        q, k, v = dev.split([Hq, Hkv, Hkv], dim=2)
    else:
        q32 = (torch.randn(B, S, Hq, D, generator=g) * 0.5).to(dtype).float()
        k32 = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).to(dtype).float()
        v32 = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).to(dtype).float()
        q, k, v = (t.to(dtype).cuda() for t in (q32, k32, v32))
    cos, sin = precompute_freqs_cis(D, S, 1e4)
    if isinstance(pads, str):
        pads = torch.randint(0, S // 2 + 1, (B,), generator=g).tolist()
    pad_t = None if pads is None else torch.tensor(pads, dtype=torch.int32)
    mask = None if pads is None else mask_from_pad_len(pad_t, S)
    ref = attention_prefill_ref(q32, k32, v32, cos, sin, mask, rope=rope)
    out = attn_prefill(q, k, v, cos.cuda(), sin.cuda(), None if pad_t is None else pad_t.cuda(),
                       apply_rope=rope)
    assert device_status() == 0
    return out.float().cpu(), ref


def _check(out, ref, dtype):
    tol = TOL[dtype]
    assert torch.isfinite(out).all()
    err = (out - ref).abs()
    bound = tol["atol"] + tol["rtol"] * ref.abs()
    worst = (err - bound).max().item()
    assert worst <= 0, f"max err {err.max().item():.3e} exceeds tolerance by {worst:.3e}"
    assert err.mean().item() < tol["mean"], f"mean err {err.mean().item():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}_S{c[1]}_{c[2]}x{c[3]}_D{c[4]}_{str(c[6])[6:]}{'_rp' if c[5] == 'random' else ''}")
def test_prefill_matches_oracle(case):
    out, ref = _run_case(*case)
    _check(out, ref, case[6])


@pytest.mark.gpu
def test_prefill_strided_fused_qkv_layout():
    out, ref = _run_case(3, 50, 8, 2, 32, [0, 9, 30], torch.bfloat16, fused_layout=True)
    _check(out, ref, torch.bfloat16)


@pytest.mark.gpu
def test_prefill_without_rope():
    out, ref = _run_case(2, 40, 8, 2, 32, [0, 12], torch.bfloat16, rope=False)
    _check(out, ref, torch.bfloat16)


@pytest.mark.gpu
def test_prefill_repeatable():
    a, _ = _run_case(2, 192, 8, 2, 32, [0, 50], torch.bfloat16, seed=5)
    b, _ = _run_case(2, 192, 8, 2, 32, [0, 50], torch.bfloat16, seed=5)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_prefill_rejects_bad_arguments():
    from rl_for_mario_b200._lib import DTKernelError
    from rl_for_mario_b200.kernels import attn_prefill

    q = torch.zeros(1, 8, 6, 32, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 8, 4, 32, dtype=torch.bfloat16, device="cuda")
    cos, sin = (t.cuda() for t in precompute_freqs_cis(32, 8))
    with pytest.raises(DTKernelError, match="divisible"):
        attn_prefill(q, k, k.clone(), cos, sin)
    q = torch.zeros(1, 8, 2, 48, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 8, 1, 48, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(DTKernelError, match="head_dim"):
        attn_prefill(q, k, k.clone(), None, None, apply_rope=False)
    q = torch.zeros(1, 16, 2, 32, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 16, 1, 32, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(DTKernelError, match="rows"):
        attn_prefill(q, k, k.clone(), cos, sin)  # cos has 8 rows < S = 16


@pytest.mark.gpu
@pytest.mark.parametrize("direction", ["rising", "falling"])
@pytest.mark.parametrize("D,dtype", [(32, torch.bfloat16), (32, torch.float16), (32, torch.float32),
                                     (64, torch.bfloat16), (64, torch.float32)],
                         ids=["d32_bf16", "d32_fp16", "d32_fp32", "d64_bf16", "d64_fp32"])
def test_prefill_wide_logit_range(direction, D, dtype):
    """Scores that climb (or fall) by ~16 log2 units per 32 keys.  Fully padded
    rows then see their keys in several of the reference's 64-wide -1e9 bands
    (not a plain mean), and a running row maximum has to move along the row."""
    from rl_for_mario_b200.kernels import attn_prefill, device_status

    B, S, Hq, Hkv = 3, 192, 8, 2
    g = torch.Generator().manual_seed(11)
    ramp = torch.arange(S, dtype=torch.float32) * (0.06 * (32 / D) ** 0.5)
    if direction == "falling":
        ramp = ramp.flip(0)
    if dtype == torch.float16:
        ramp = ramp * 0.25  # fp16 keys stay well inside its range
    q32 = (1.0 + 0.1 * torch.randn(B, S, Hq, D, generator=g)).to(dtype).float()
    k32 = (ramp.view(1, S, 1, 1) * (1.0 + 0.1 * torch.randn(B, S, Hkv, D, generator=g))).to(dtype).float()
    v32 = torch.randn(B, S, Hkv, D, generator=g).to(dtype).float()
    pad_t = torch.tensor([0, 37, 100], dtype=torch.int32)
    ref = attention_prefill_ref(q32, k32, v32, None, None, mask_from_pad_len(pad_t, S), rope=False)
    out = attn_prefill(*(t.to(dtype).cuda() for t in (q32, k32, v32)), None, None, pad_t.cuda(), apply_rope=False)
    assert device_status() == 0
    _check(out.float().cpu(), ref, dtype)


LONG_CASES = [
    # B, S, Hq, Hkv, D, pads, dtype  (Q/K pre-rotated: the persistent two-tile kernel)
    (2, 768, 12, 4, 64, [0, 384], torch.bfloat16),
    (3, 300, 12, 4, 64, "random", torch.bfloat16),
    (2, 129, 4, 4, 64, [0, 128], torch.bfloat16),
    (2, 1, 8, 2, 64, None, torch.bfloat16),
    (3, 100, 8, 2, 64, [0, 50, 99], torch.float16),
    (2, 513, 16, 2, 64, [0, 200], torch.bfloat16),
    (4, 256, 12, 4, 64, [0, 1, 255, 256], torch.bfloat16),
    (1, 1024, 12, 4, 64, [100], torch.bfloat16),
    (40, 200, 12, 4, 64, "random", torch.bfloat16),
    (300, 64, 12, 4, 64, "random", torch.bfloat16),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", LONG_CASES,
                         ids=lambda c: f"B{c[0]}_S{c[1]}_{c[2]}x{c[3]}_D{c[4]}_{str(c[6])[6:]}{'_rp' if c[5] == 'random' else ''}")
def test_prefill_prerotated_matches_oracle(case):
    out, ref = _run_case(*case, rope=False)
    _check(out, ref, case[6])


@pytest.mark.gpu
@pytest.mark.parametrize("B,chunks", [(37, 8), (5, 2), (3, 8), (1, 1)])
def test_prefill_host_pipeline_matches_device_call(B, chunks):
    """The host-buffer entry point (chunked, pipelined copies) gives the device call's result bit for bit,
    twice in a row on the same buffers."""
    from rl_for_mario_b200.kernels import attn_prefill, attn_prefill_host, device_status

    S, Hq, Hkv, D = 192, 8, 2, 32
    g = torch.Generator().manual_seed(B * 10 + chunks)
    q = (torch.randn(B, S, Hq, D, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).to(torch.bfloat16)
    pad = torch.randint(0, 97, (B,), generator=g, dtype=torch.int32)
    cos, sin = (t.cuda() for t in precompute_freqs_cis(D, S))
    ref = attn_prefill(q.cuda(), k.cuda(), v.cuda(), cos, sin, pad.cuda()).cpu()
    hq, hk, hv, hpad = (t.pin_memory() for t in (q, k, v, pad))
    ho = torch.empty(B, S, Hq, D, dtype=torch.bfloat16).pin_memory()
    bufs = tuple(torch.empty(t.shape, dtype=t.dtype, device="cuda") for t in (q, k, v, pad, ho))
    for _ in range(2):
        ho.zero_()
        attn_prefill_host(hq, hk, hv, cos, sin, hpad, ho, bufs, chunks=chunks)
        torch.cuda.current_stream().synchronize()
        assert device_status() == 0
        assert torch.equal(ho, ref)


@pytest.mark.gpu
def test_prefill_host_rejects_pageable_buffers():
    from rl_for_mario_b200.kernels import attn_prefill_host

    t = torch.zeros(2, 8, 2, 32, dtype=torch.bfloat16)
    bufs = tuple(torch.zeros(2, 8, 2, 32, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    with pytest.raises(ValueError):
        attn_prefill_host(t, t, t, None, None, None, t.pin_memory(), bufs + (None, bufs[0]), apply_rope=False)


@pytest.mark.gpu
def test_prefill_host_rejects_mismatched_buffers():
    """A host tensor whose dtype or batch differs from its device buffer is an error
    (a copy would cast or fill only part of the buffer)."""
    from rl_for_mario_b200.kernels import attn_prefill_host

    dev = tuple(torch.zeros(2, 8, 2, 32, dtype=torch.bfloat16, device="cuda") for _ in range(4))
    bufs = dev[:3] + (None, dev[3])
    ok = torch.zeros(2, 8, 2, 32, dtype=torch.bfloat16).pin_memory()
    f32 = torch.zeros(2, 8, 2, 32, dtype=torch.float32).pin_memory()
    short = torch.zeros(1, 8, 2, 32, dtype=torch.bfloat16).pin_memory()
    with pytest.raises(ValueError):
        attn_prefill_host(f32, ok, ok, None, None, None, ok, bufs, apply_rope=False)
    with pytest.raises(ValueError):
        attn_prefill_host(ok, ok, short, None, None, None, ok, bufs, apply_rope=False)
    attn_prefill_host(ok, ok, ok, None, None, None, ok, bufs, apply_rope=False)
    torch.cuda.synchronize()
