"""Kernel parity at the full workload sizes that the bench times.

The persistent kernels schedule work per CTA (units or tile pairs over 148
SMs, heaviest first); small cases never reach the wave counts of the timed
workloads.  Each test here runs a kernel at full size, checks a spread of
samples against the CPU oracle (including the first and last samples, i.e.
the first and last waves of the schedule), and checks size-independent
properties over the whole batch: every output finite, and the outputs of a
batch run in another sample order equal, bit for bit, to the original run
(no result depends on where the schedule put a sample).

Tolerance for bf16 attention outputs against the fp32 oracle on the same
bf16-rounded inputs: 2e-3 absolute on top of the output's own bf16 rounding
(half an ulp, 2^-8 relative), and 2e-4 mean-abs.
"""
import pytest
import torch

from oracle import (apply_rotary_pos_emb, attention_decode_ref, attention_prefill_ref, mask_from_pad_len,
                    precompute_freqs_cis)

ATOL, RTOL, MEAN = 2e-3, 2.0 ** -8, 2e-4


def _spread(B, n):
    idx = torch.linspace(0, B - 1, n).round().long()
    return torch.unique(idx)


def _close(out, ref):
    err = (out - ref).abs()
    assert torch.isfinite(out).all()
    print(f"FULLSIZE max {err.max().item():.3e} mean {err.mean().item():.3e} "
          f"excess {(err - RTOL * ref.abs()).max().item():.3e}")
    worst = (err - ATOL - RTOL * ref.abs()).max().item()
    assert worst <= 0, f"max err {err.max().item():.3e} exceeds the bound by {worst:.3e}"
    assert err.mean().item() <= MEAN, f"mean err {err.mean().item():.3e}"


def _qkv(B, S, Hq, Hkv, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(B, S, Hq, D, generator=g, device="cuda") * 0.5).bfloat16()
    k = (torch.randn(B, S, Hkv, D, generator=g, device="cuda") * 0.5).bfloat16()
    v = (torch.randn(B, S, Hkv, D, generator=g, device="cuda") * 0.5).bfloat16()
    return q, k, v


@pytest.mark.gpu
@pytest.mark.parametrize("shape", ["cfg2", "cfg4"])
def test_prefill_full_size(shape):
    """cfg2: B=4096, S=192, 8/2 heads, D=32, left pads U{0..96} tokens, RoPE in the
    kernel.  cfg4: B=1024, S=768, 12/4 heads, D=64, pads U{0..128} timesteps
    (x3 tokens), q/k pre-rotated as the model path feeds the long kernel."""
    from rl_for_mario_b200.kernels import attn_prefill, device_status

    if shape == "cfg2":
        B, S, Hq, Hkv, D, rope = 4096, 192, 8, 2, 32, True
        pads = torch.randint(0, 97, (B,), generator=torch.Generator().manual_seed(1), dtype=torch.int32)
    else:
        B, S, Hq, Hkv, D, rope = 1024, 768, 12, 4, 64, False
        pads = 3 * torch.randint(0, 129, (B,), generator=torch.Generator().manual_seed(3), dtype=torch.int32)
    q, k, v = _qkv(B, S, Hq, Hkv, D, seed=5)
    cos, sin = precompute_freqs_cis(D, S)
    dpads = pads.cuda()
    out = attn_prefill(q, k, v, cos.cuda(), sin.cuda(), dpads, apply_rope=rope)
    assert device_status() == 0
    assert torch.isfinite(out).all()
    # Oracle on a spread of samples.
    sel = _spread(B, 24 if shape == "cfg2" else 8)
    ref = attention_prefill_ref(q[sel].float().cpu(), k[sel].float().cpu(), v[sel].float().cpu(),
                                cos, sin, mask_from_pad_len(pads[sel], S), rope=rope)
    _close(out[sel].float().cpu(), ref)
    # The whole batch in a permuted sample order gives the same bits per sample.
    perm = torch.randperm(B, generator=torch.Generator().manual_seed(9)).cuda()
    out_p = attn_prefill(q[perm].contiguous(), k[perm].contiguous(), v[perm].contiguous(), cos.cuda(), sin.cuda(),
                         dpads[perm].contiguous(), apply_rope=rope)
    assert device_status() == 0
    assert torch.equal(out_p, out[perm])


@pytest.mark.gpu
def test_decode_full_size():
    """cfg3's decode at its mid-episode length: 16,384 environments, 219 cached
    positions + 3 new tokens (kv 222), 8/2 heads, D=32, 64-position pages."""
    from rl_for_mario_b200.cache import LayerKV
    from rl_for_mario_b200.kernels import attn_decode, device_status, kv_write

    B, L, Sn, Hq, Hkv, D, page = 16384, 219, 3, 8, 2, 32, 64
    cap = 256
    pps = cap // page
    g = torch.Generator(device="cuda").manual_seed(11)
    # A permuted page table: sample b's pages are scattered over the pool.
    ids = torch.randperm(B * pps, generator=torch.Generator().manual_seed(12)).view(B, pps).to(torch.int32).cuda()
    kp = torch.zeros(B * pps, Hkv, page, D, dtype=torch.bfloat16, device="cuda")
    layer = LayerKV(kp, torch.zeros_like(kp), ids, torch.zeros(B, dtype=torch.int32, device="cuda"), 0)
    k_pre = (torch.randn(B, L, Hkv, D, generator=g, device="cuda") * 0.5).bfloat16()
    v_pre = (torch.randn(B, L, Hkv, D, generator=g, device="cuda") * 0.5).bfloat16()
    cos, sin = precompute_freqs_cis(D, cap)
    kv_write(k_pre, v_pre, layer, cos.cuda(), sin.cuda())
    layer.advance(L)
    q = (torch.randn(B, Sn, Hq, D, generator=g, device="cuda") * 0.5).bfloat16()
    kn = (torch.randn(B, Sn, Hkv, D, generator=g, device="cuda") * 0.5).bfloat16()
    vn = (torch.randn(B, Sn, Hkv, D, generator=g, device="cuda") * 0.5).bfloat16()
    out = attn_decode(q, kn, vn, layer, cos.cuda(), sin.cuda(), None, rope_abs=True)
    assert device_status() == 0
    assert torch.isfinite(out).all()
    sel = _spread(B, 32)
    kp_ = k_pre[sel].float().cpu()
    _, k_rot = apply_rotary_pos_emb(kp_, kp_, cos[:L], sin[:L])
    past_k = k_rot.transpose(1, 2).bfloat16().float()  # the cache holds bf16 rotated keys
    past_v = v_pre[sel].float().cpu().transpose(1, 2)
    ref, _, _ = attention_decode_ref(q[sel].float().cpu(), kn[sel].float().cpu(), vn[sel].float().cpu(), past_k,
                                     past_v, cos[L:L + Sn], sin[L:L + Sn], None)
    _close(out[sel].float().cpu(), ref)
