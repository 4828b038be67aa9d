"""GPU parity of the paged-cache decode kernel (dt_attn_decode) and the cache
writer (dt_kv_write) against the CPU oracle's cached branch."""
import pytest
import torch

from oracle import apply_rotary_pos_emb, attention_decode_ref, mask_from_pad_len, precompute_freqs_cis

TOL = {torch.bfloat16: dict(atol=1.5e-2, rtol=1e-2, mean=2.5e-3),
       torch.float16: dict(atol=4e-3, rtol=4e-3, mean=5e-4),
       torch.float32: dict(atol=1e-5, rtol=1e-5, mean=1e-6)}

CASES = [
    # B, L, Sn, Hq, Hkv, D, page, pads, dtype, permute
    (3, 24, 3, 8, 2, 32, 16, [0, 6, 15], torch.bfloat16, False),
    (4, 189, 3, 8, 2, 32, 64, None, torch.bfloat16, False),
    (2, 0, 3, 8, 2, 32, 64, None, torch.bfloat16, False),
    (2, 300, 3, 8, 2, 32, 64, [0, 120], torch.bfloat16, True),
    (3, 40, 1, 8, 2, 32, 16, [0, 1, 40], torch.bfloat16, True),
    (2, 30, 3, 12, 4, 64, 32, [0, 9], torch.float16, False),
    (2, 50, 8, 8, 2, 32, 64, [0, 20], torch.bfloat16, False),
    (2, 60, 12, 8, 2, 32, 64, [0, 30], torch.bfloat16, True),   # new tokens re-read from the cache
    (3, 70, 20, 8, 2, 32, 32, "random", torch.bfloat16, False),
    (5, 253, 3, 8, 2, 32, 64, "random", torch.bfloat16, True),
    (2, 100, 3, 4, 4, 64, 64, None, torch.bfloat16, True),
    (3, 24, 3, 8, 2, 32, 16, [0, 6, 15], torch.float32, True),
    (2, 300, 3, 12, 4, 64, 64, [0, 120], torch.float32, False),
    (2, 40, 130, 8, 2, 32, 64, [0, 50], torch.float32, False),
]


def _check(out, ref, dtype):
    tol = TOL[dtype]
    assert torch.isfinite(out).all()
    err = (out - ref).abs()
    worst = (err - (tol["atol"] + tol["rtol"] * ref.abs())).max().item()
    assert worst <= 0, f"max err {err.max().item():.3e}"
    assert err.mean().item() < tol["mean"], f"mean err {err.mean().item():.3e}"


def _make_cache(B, Hkv, D, cap, page, dtype, permute, g):
    from rl_for_mario_b200.cache import LayerKV

    pps = (cap + page - 1) // page
    n_pages = B * pps + 3  # spare pages so a permuted table exercises real indirection
    ids = torch.randperm(n_pages, generator=g)[: B * pps] if permute else torch.arange(B * pps)
    bt = ids.view(B, pps).to(torch.int32).cuda()
    kp = torch.zeros(n_pages, Hkv, page, D, dtype=dtype, device="cuda")
    return LayerKV(kp, torch.zeros_like(kp), bt, torch.zeros(B, dtype=torch.int32, device="cuda"), 0)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"B{c[0]}_L{c[1]}_Sn{c[2]}_{c[3]}x{c[4]}_D{c[5]}_p{c[6]}")
@pytest.mark.parametrize("rope_abs", [False, True])
def test_decode_matches_oracle(case, rope_abs):
    from rl_for_mario_b200.kernels import attn_decode, device_status, kv_write

    B, L, Sn, Hq, Hkv, D, page, pads, dtype, permute = case
    g = torch.Generator().manual_seed(7)
    cap = L + Sn + 5
    layer = _make_cache(B, Hkv, D, cap, page, dtype, permute, g)
    cos_t, sin_t = precompute_freqs_cis(D, cap + 4)
    # Prefix: pre-RoPE keys rotated by the cache writer (absolute positions 0..L-1).
    k_pre = (torch.randn(B, max(L, 1), Hkv, D, generator=g) * 0.5).to(dtype)
    v_pre = (torch.randn(B, max(L, 1), Hkv, D, generator=g) * 0.5).to(dtype)
    if L > 0:
        kv_write(k_pre[:, :L].cuda(), v_pre[:, :L].cuda(), layer, cos_t.cuda(), sin_t.cuda())
        layer.advance(L)
    _, k_rot = apply_rotary_pos_emb(k_pre[:, :L].float(), k_pre[:, :L].float(), cos_t[:L], sin_t[:L])
    past_k = k_rot.transpose(1, 2).to(dtype).float()
    past_v = v_pre[:, :L].float().transpose(1, 2)
    q = (torch.randn(B, Sn, Hq, D, generator=g) * 0.5).to(dtype)
    kn = (torch.randn(B, Sn, Hkv, D, generator=g) * 0.5).to(dtype)
    vn = (torch.randn(B, Sn, Hkv, D, generator=g) * 0.5).to(dtype)
    if isinstance(pads, str):
        pads = torch.randint(0, L + Sn + 1, (B,), generator=g).tolist()
    pad_t = None if pads is None else torch.tensor(pads, dtype=torch.int32)
    mask = None if pad_t is None else mask_from_pad_len(pad_t, L + Sn)
    cn, sn = cos_t[L:L + Sn], sin_t[L:L + Sn]
    ref, k_all, v_all = attention_decode_ref(q.float(), kn.float(), vn.float(), past_k, past_v, cn, sn, mask)
    if rope_abs:
        out = attn_decode(q.cuda(), kn.cuda(), vn.cuda(), layer, cos_t.cuda(), sin_t.cuda(),
                          None if pad_t is None else pad_t.cuda(), rope_abs=True)
    else:
        out = attn_decode(q.cuda(), kn.cuda(), vn.cuda(), layer, cn.cuda(), sn.cuda(),
                          None if pad_t is None else pad_t.cuda(), rope_abs=False)
    assert device_status() == 0
    _check(out.float().cpu(), ref, dtype)
    layer.advance(Sn)
    dk, dv = layer.dense()
    torch.testing.assert_close(dv.float().cpu(), v_all, atol=0, rtol=0)
    ktol = 1e-5 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(dk.float().cpu(), k_all, atol=ktol, rtol=ktol)


@pytest.mark.gpu
def test_decode_steps_accumulate_like_the_reference_cat():
    """Three consecutive 3-token steps through one cache equal the oracle's cat-based steps."""
    from rl_for_mario_b200.kernels import attn_decode, device_status

    B, Hq, Hkv, D, dtype = 4, 8, 2, 32, torch.bfloat16
    g = torch.Generator().manual_seed(3)
    layer = _make_cache(B, Hkv, D, 64, 16, dtype, True, g)
    cos_t, sin_t = precompute_freqs_cis(D, 64)
    pk = pv = None
    for step in range(3):
        L = 3 * step
        q, kn, vn = ((torch.randn(B, 3, h, D, generator=g) * 0.5).to(dtype) for h in (Hq, Hkv, Hkv))
        ref, pk, pv = attention_decode_ref(q.float(), kn.float(), vn.float(), pk, pv, cos_t[L:L + 3], sin_t[L:L + 3])
        pk = pk.to(dtype).float()
        out = attn_decode(q.cuda(), kn.cuda(), vn.cuda(), layer, cos_t[L:L + 3].cuda(), sin_t[L:L + 3].cuda())
        layer.advance(3)
        _check(out.float().cpu(), ref, dtype)
    assert device_status() == 0


@pytest.mark.gpu
def test_decode_rejects_full_cache():
    from rl_for_mario_b200.kernels import attn_decode

    B, Hq, Hkv, D = 2, 8, 2, 32
    layer = _make_cache(B, Hkv, D, 16, 16, torch.bfloat16, False, torch.Generator().manual_seed(0))
    layer.advance(15)
    x = torch.zeros(B, 3, Hq, D, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(B, 3, Hkv, D, dtype=torch.bfloat16, device="cuda")
    cos, sin = (t.cuda() for t in precompute_freqs_cis(D, 32))
    with pytest.raises(ValueError, match="cache full"):
        attn_decode(x, kv, kv, layer, cos, sin)


@pytest.mark.gpu
def test_decode_device_check_flags_bad_page_ids():
    """A block table holding an out-of-range page id is refused on the device (no access)."""
    from rl_for_mario_b200.cache import LayerKV
    from rl_for_mario_b200.kernels import attn_decode, device_status

    B, Hq, Hkv, D = 1, 8, 2, 32
    kp = torch.zeros(2, Hkv, 16, D, dtype=torch.bfloat16, device="cuda")
    bt = torch.tensor([[0, 7]], dtype=torch.int32, device="cuda")  # page 7 does not exist
    layer = LayerKV(kp, torch.zeros_like(kp), bt, torch.tensor([14], dtype=torch.int32, device="cuda"), 14)
    x = torch.zeros(B, 3, Hq, D, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(B, 3, Hkv, D, dtype=torch.bfloat16, device="cuda")
    cos, sin = (t.cuda() for t in precompute_freqs_cis(D, 3))
    attn_decode(x, kv, kv, layer, cos, sin)
    assert device_status() != 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_wide_logit_range(dtype):
    """Cached keys whose scores climb by ~16 log2 units per 32 positions: new
    tokens inside the left padding weigh their keys in the reference's 64-wide
    -1e9 bands, the others need a moving running maximum."""
    from rl_for_mario_b200.kernels import attn_decode, device_status, kv_write

    B, L, Sn, Hq, Hkv, D = 3, 150, 3, 8, 2, 32
    g = torch.Generator().manual_seed(5)
    layer = _make_cache(B, Hkv, D, L + Sn, 64, dtype, True, g)
    ramp = torch.arange(L + Sn, dtype=torch.float32) * 0.06
    k_all = (ramp.view(1, -1, 1, 1) * (1.0 + 0.1 * torch.randn(B, L + Sn, Hkv, D, generator=g))).to(dtype)
    v_all = torch.randn(B, L + Sn, Hkv, D, generator=g).to(dtype)
    q = (1.0 + 0.1 * torch.randn(B, Sn, Hq, D, generator=g)).to(dtype)
    kv_write(k_all[:, :L].cuda(), v_all[:, :L].cuda(), layer, None, None, apply_rope=False)
    layer.advance(L)
    pads = torch.tensor([0, 60, L + 2], dtype=torch.int32)  # last sample: two new tokens still padded
    mask = mask_from_pad_len(pads, L + Sn)
    past_k = k_all[:, :L].float().transpose(1, 2)
    past_v = v_all[:, :L].float().transpose(1, 2)
    ref, _, _ = attention_decode_ref(q.float(), k_all[:, L:].float(), v_all[:, L:].float(), past_k, past_v,
                                     None, None, mask, rope=False)
    out = attn_decode(q.cuda(), k_all[:, L:].cuda(), v_all[:, L:].cuda(), layer, None, None, pads.cuda(),
                      apply_rope=False)
    assert device_status() == 0
    _check(out.float().cpu(), ref, dtype)
