"""RoPE with the reference's roundings (apply_rope = 2) and the encoder's
rounded-input mode: bit-exact against the reference's own 16-bit arithmetic.

On 16-bit tensors the reference evaluates q * cos + rotate_half(q) * sin
(model/model_decision_transformer.py:113-116) as three ops, each rounded to
the tensor dtype; the oracle's apply_rotary_pos_emb is the same expression, so
running it on CPU bf16 / fp16 tensors gives the reference's rotated values
bit for bit.  A kernel that rotates with apply_rope = 2 must therefore give
exactly the output it gives on the oracle-rotated inputs with apply_rope = 0,
and write exactly the oracle-rotated keys into the cache.
"""
import pytest
import torch

from oracle import apply_rotary_pos_emb, mask_from_pad_len, precompute_freqs_cis  # noqa: F401


def _tables(D, n, dtype):
    cos, sin = precompute_freqs_cis(D, n)
    # The reference's 16-bit model holds its tables in the model dtype.
    return cos.to(dtype), sin.to(dtype)


def _qkv(B, S, Hq, Hkv, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return tuple((torch.randn(B, S, h, D, generator=g) * 0.5).to(dtype) for h in (Hq, Hkv, Hkv))


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,Hq,Hkv,D,dtype", [
    (3, 24, 8, 2, 32, torch.bfloat16),    # persistent short kernel
    (2, 192, 8, 2, 32, torch.float16),
    (2, 300, 12, 4, 64, torch.bfloat16),  # long kernel (its RoPE warp)
    (2, 300, 8, 2, 32, torch.bfloat16),   # streaming kernel (S > 192, D = 32)
])
def test_prefill_reference_rounded_rope_is_bit_exact(B, S, Hq, Hkv, D, dtype):
    from rl_for_mario_b200.kernels import attn_prefill, device_status

    q, k, v = _qkv(B, S, Hq, Hkv, D, dtype, seed=S + D)
    cos, sin = _tables(D, S, dtype)
    pads = torch.tensor([0] + [S // 3] * (B - 1), dtype=torch.int32).cuda()
    out = attn_prefill(q.cuda(), k.cuda(), v.cuda(), cos.float().cuda(), sin.float().cuda(), pads, apply_rope=2)
    qr, kr = apply_rotary_pos_emb(q, k, cos, sin)  # the reference's 16-bit RoPE on CPU
    assert qr.dtype == dtype
    ref = attn_prefill(qr.cuda(), kr.cuda(), v.cuda(), None, None, pads, apply_rope=False)
    assert device_status() == 0
    assert torch.equal(out, ref)
    # The default mode differs (one fp32 rounding instead of three): the test has teeth.
    out1 = attn_prefill(q.cuda(), k.cuda(), v.cuda(), cos.float().cuda(), sin.float().cuda(), pads, apply_rope=True)
    assert not torch.equal(out1, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cache_writes_and_decode_with_reference_rounded_rope(dtype):
    """kv_write and the decode append store exactly the reference's rotated keys;
    the decode output equals the one on oracle-rotated inputs."""
    from rl_for_mario_b200.cache import LayerKV
    from rl_for_mario_b200.kernels import attn_decode, device_status, kv_write

    B, L, Sn, Hq, Hkv, D, page = 3, 40, 3, 8, 2, 32, 16
    cap = 48
    pps = cap // page
    cos, sin = _tables(D, cap, dtype)
    k_pre = (torch.randn(B, L, Hkv, D, generator=torch.Generator().manual_seed(1)) * 0.5).to(dtype)
    v_pre = (torch.randn(B, L, Hkv, D, generator=torch.Generator().manual_seed(2)) * 0.5).to(dtype)
    q, kn, vn = _qkv(B, Sn, Hq, Hkv, D, dtype, seed=3)

    def fresh():
        kp = torch.zeros(B * pps, Hkv, page, D, dtype=dtype, device="cuda")
        bt = torch.arange(B * pps, dtype=torch.int32).view(B, pps).cuda()
        return LayerKV(kp, torch.zeros_like(kp), bt, torch.zeros(B, dtype=torch.int32, device="cuda"), 0)

    _, k_rot = apply_rotary_pos_emb(k_pre, k_pre, cos[:L], sin[:L])
    qn_rot, kn_rot = apply_rotary_pos_emb(q, kn, cos[L:L + Sn], sin[L:L + Sn])
    # Rotated in the kernels, reference rounding.
    a = fresh()
    kv_write(k_pre.cuda(), v_pre.cuda(), a, cos.float().cuda(), sin.float().cuda(), apply_rope=2)
    a.advance(L)
    cn, sn = cos[L:L + Sn].float().cuda(), sin[L:L + Sn].float().cuda()
    out_a = attn_decode(q.cuda(), kn.cuda(), vn.cuda(), a, cn, sn, None, apply_rope=2)
    a.advance(Sn)
    # Rotated by the oracle on CPU, kernels without RoPE.
    b = fresh()
    kv_write(k_rot.cuda(), v_pre.cuda(), b, None, None, apply_rope=False)
    b.advance(L)
    out_b = attn_decode(qn_rot.cuda(), kn_rot.cuda(), vn.cuda(), b, None, None, None, apply_rope=False)
    b.advance(Sn)
    assert device_status() == 0
    ka, va = a.dense()
    kb, vb = b.dense()
    assert torch.equal(ka, kb) and torch.equal(va, vb)
    assert torch.equal(ka[:, :, :L].cpu(), k_rot.transpose(1, 2))
    assert torch.equal(out_a, out_b)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_frames_conv1_rounded_input(dtype):
    """round_input: frames / 255 rounded to the dtype first (the reference's 16-bit x / 255,
    :338), then the convolution in fp32 and one output rounding."""
    import torch.nn.functional as Fn
    from rl_for_mario_b200.kernels import device_status, frames_conv1

    g = torch.Generator().manual_seed(4)
    fr = torch.randint(0, 256, (300, 4, 84, 84), generator=g, dtype=torch.uint8).cuda()
    w = (torch.randn(32, 4, 8, 8, generator=g) * 0.05).to(dtype).cuda()
    b = (torch.randn(32, generator=g) * 0.1).to(dtype).cuda()
    out, _ = frames_conv1(fr, w, b, round_input=True)
    assert device_status() == 0
    torch.backends.cudnn.allow_tf32 = False
    x16 = fr.to(dtype) / 255.0  # the reference's 16-bit division, rounded
    ref = Fn.relu(Fn.conv2d(x16.float(), w.float(), b.float(), stride=4))
    err = (out.float() - ref).abs()
    rel = 2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11
    assert (err <= rel * ref.abs() + 1e-5).all(), (err - rel * ref.abs()).max().item()
    # The exact-input mode differs from it (the input rounding is visible).
    out0, _ = frames_conv1(fr, w, b, round_input=False)
    assert not torch.equal(out0, out)
