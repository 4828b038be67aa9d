"""GPU parity of the fused RMSNorm + QKV projection kernel (dt_rmsnorm_qkv)."""
import pytest
import torch

from oracle import rmsnorm_ref


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(1, 256, 384), (300, 256, 384), (4096, 256, 384), (777, 768, 1280),
                                   (130, 128, 192), (64, 64, 128), (257, 512, 512), (1000, 256, 96),
                                   (200, 256, 520), (130, 128, 776), (1, 64, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm_qkv_matches_reference(M, K, N, dtype):
    from rl_for_mario_b200.kernels import device_status, fold_norm_weight, rmsnorm_qkv

    g = torch.Generator().manual_seed(M + K + N)
    x = (torch.randn(M, K, generator=g) * 2).to(dtype)
    wn = (1 + 0.1 * torch.randn(K, generator=g))
    w = torch.randn(N, K, generator=g) / K ** 0.5
    nq = N // 2
    nk = (N - nq) // 2
    wq, wk, wv = w[:nq], w[nq:nq + nk], w[nq + nk:]
    wf = fold_norm_weight(wq, wk, wv, wn, dtype).cuda()
    y = rmsnorm_qkv(x.cuda(), wf, 1e-5)
    assert device_status() == 0
    ref = rmsnorm_ref(x.float(), wn) @ w.t()
    err = (y.float().cpu() - ref).abs()
    tol = 2e-2 if dtype == torch.bfloat16 else 4e-3
    assert (err <= tol + tol * ref.abs()).all(), f"max err {err.max().item():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("N", [384, 1280])
def test_rmsnorm_qkv_strided_rows(N):
    """x rows with a padded stride (a column slice of a wider buffer)."""
    from rl_for_mario_b200.kernels import device_status, rmsnorm_qkv

    g = torch.Generator().manual_seed(N)
    M, K = 300, 256
    xb = (torch.randn(M, K + 64, generator=g) * 2).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    x = xb.cuda()[:, :K]
    assert x.stride(0) == K + 64
    y = rmsnorm_qkv(x, w.cuda(), 1e-5)
    assert device_status() == 0
    ref = rmsnorm_ref(xb[:, :K].float(), torch.ones(K)) @ w.float().t()
    err = (y.float().cpu() - ref).abs()
    assert (err <= 2e-2 + 2e-2 * ref.abs()).all(), f"max err {err.max().item():.3e}"


@pytest.mark.gpu
def test_fused_block_matches_unfused_block():
    from rl_for_mario_b200.dt_model import DTConfig, DTBlock, rope_tables

    cfg = DTConfig(hidden_size=256, num_attention_heads=8, num_key_value_heads=2, context_len=64, dropout=0.0)
    torch.manual_seed(0)
    blk = DTBlock(cfg).cuda().to(torch.bfloat16).eval()
    x = torch.randn(4, 96, 256, device="cuda").to(torch.bfloat16)
    cos, sin = (t.cuda() for t in rope_tables(32, 96, 1e4))
    mask = (torch.arange(96, device="cuda")[None] >= torch.tensor([0, 3, 30, 95], device="cuda")[:, None]).float()
    with torch.no_grad():
        ref, _ = blk(x, (cos, sin), attention_mask=mask)
        blk.fuse_norm(True)
        out, _ = blk(x, (cos, sin), attention_mask=mask)
    err = (out.float() - ref.float()).abs().max().item()
    assert err < 6e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,K,Hq,Hkv,D", [(2, 96, 256, 8, 2, 32), (3, 50, 768, 12, 4, 64), (1, 7, 128, 4, 4, 32),
                                            (2, 130, 512, 8, 8, 64), (2, 21, 128, 4, 1, 32), (3, 40, 256, 19, 2, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("tables", ["rotate_half", "arbitrary"])
def test_rmsnorm_qkv_rope_matches_reference(B, S, K, Hq, Hkv, D, dtype, tables):
    """RMSNorm -> q/k/v projections -> rotate-half RoPE of q and k, fused in one kernel.

    "rotate_half" tables repeat their halves (the reference's cat([cos, cos]));
    "arbitrary" tables do not, and take the kernels' general table path."""
    from oracle import apply_rotary_pos_emb, precompute_freqs_cis
    from rl_for_mario_b200.kernels import device_status, fold_norm_weight, rmsnorm_qkv

    g = torch.Generator().manual_seed(B * S + K + D)
    x = (torch.randn(B, S, K, generator=g) * 2).to(dtype)
    wn = 1 + 0.1 * torch.randn(K, generator=g)
    wq, wk, wv = (torch.randn(h * D, K, generator=g) / K ** 0.5 for h in (Hq, Hkv, Hkv))
    wf = fold_norm_weight(wq, wk, wv, wn, dtype).cuda()
    cos, sin = precompute_freqs_cis(D, S + 5)
    if tables == "arbitrary":
        cos, sin = (torch.rand(S + 5, D, generator=g) * 2 - 1 for _ in range(2))
    y = rmsnorm_qkv(x.cuda(), wf, 1e-5, rope=(cos[:S].cuda(), sin[:S].cuda(), (Hq + Hkv) * D, D))
    assert device_status() == 0
    xn = rmsnorm_ref(x.float(), wn)
    q = (xn @ wq.t()).view(B, S, Hq, D)
    k = (xn @ wk.t()).view(B, S, Hkv, D)
    v = (xn @ wv.t()).view(B, S, Hkv, D)
    q, k = apply_rotary_pos_emb(q, k, cos[:S], sin[:S])
    ref = torch.cat([q, k, v], dim=2).reshape(B, S, -1)
    err = (y.float().cpu() - ref).abs()
    tol = 2e-2 if dtype == torch.bfloat16 else 4e-3
    assert (err <= tol + tol * ref.abs()).all(), f"max err {err.max().item():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("hidden,heads,kv_heads,S", [(256, 8, 2, 96), (768, 12, 4, 300)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_block_with_rope_epilogue_matches_unfused_block(hidden, heads, kv_heads, S, dtype):
    """A block whose RMSNorm + QKV + RoPE run in one kernel and whose attention
    takes pre-rotated q / k (short and long prefill kernels), with the fused
    RMSNorm + SwiGLU MLP and residual GEMMs, equals the unfused block."""
    from rl_for_mario_b200.dt_model import DTConfig, DTBlock, rope_tables

    cfg = DTConfig(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
                   context_len=(S + 2) // 3, dropout=0.0)
    torch.manual_seed(1)
    blk = DTBlock(cfg).cuda().to(dtype).eval()
    x = torch.randn(3, S, hidden, device="cuda").to(dtype)
    cos, sin = (t.cuda() for t in rope_tables(hidden // heads, S, 1e4))
    mask = (torch.arange(S, device="cuda")[None] >= torch.tensor([0, 5, S // 2], device="cuda")[:, None]).float()
    with torch.no_grad():
        ref, _ = blk(x, (cos, sin), attention_mask=mask)
        blk.fuse_norm(True)
        out, _ = blk(x, (cos, sin), attention_mask=mask)
    err = (out.float() - ref.float()).abs().max().item()
    assert err < 6e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,F", [(1, 256, 704), (300, 256, 704), (777, 768, 2048), (130, 128, 128),
                                   (4096, 512, 192)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm_swiglu_matches_reference(M, K, F, dtype):
    """post_attention_layernorm -> silu(gate_proj) * up_proj (FeedForward before down_proj)."""
    import torch.nn.functional as Fn
    from rl_for_mario_b200.kernels import device_status, fold_swiglu_weight, rmsnorm_swiglu

    g = torch.Generator().manual_seed(M + K + F)
    x = (torch.randn(M, K, generator=g) * 2).to(dtype)
    wn = 1 + 0.1 * torch.randn(K, generator=g)
    wg, wu = (torch.randn(F, K, generator=g) / K ** 0.5 for _ in range(2))
    wf = fold_swiglu_weight(wg, wu, wn, dtype).cuda()
    y = rmsnorm_swiglu(x.cuda(), wf, 1e-5)
    assert device_status() == 0
    xn = rmsnorm_ref(x.float(), wn)
    ref = Fn.silu(xn @ wg.t()) * (xn @ wu.t())
    err = (y.float().cpu() - ref).abs()
    tol = 2e-2 if dtype == torch.bfloat16 else 4e-3
    assert (err <= tol + tol * ref.abs()).all(), f"max err {err.max().item():.3e}"


@pytest.mark.gpu
def test_rmsnorm_swiglu_rejects_bad_widths():
    from rl_for_mario_b200.kernels import rmsnorm_swiglu

    x = torch.zeros(4, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        rmsnorm_swiglu(x, torch.zeros(2 * 96, 64, dtype=torch.bfloat16, device="cuda"), 1e-5)
    with pytest.raises(RuntimeError):
        rmsnorm_swiglu(x, torch.zeros(2 * 64, 64, dtype=torch.bfloat16, device="cuda"), 1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(300, 256, 256), (1000, 768, 768), (777, 2048, 768), (130, 704, 256),
                                   (5000, 256, 256), (3000, 512, 512), (65536, 768, 768), (65536, 2048, 768),
                                   (70000, 256, 512)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_residual_matches_fp32(M, K, N, dtype):
    """y += x @ w^T in place (the block's o_proj / down_proj with the residual add):
    within one output rounding of the fp32 result.  N a multiple of 256 with at least
    four 256 x 256 tiles per CTA pair runs on CTA pairs (the three large cases: each
    pair gets about ten tiles, so its stage ring and both accumulators wrap; 70,000
    rows end in a partial 256-row block); the others run on the single-CTA kernel."""
    from rl_for_mario_b200.kernels import device_status, gemm_residual

    g = torch.Generator(device="cuda").manual_seed(M + K + N)
    x = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(dtype)
    y0 = torch.randn(M, N, device="cuda", generator=g).to(dtype)
    ref = y0.float() + x.float() @ w.float().t()
    y = y0.clone()
    out = gemm_residual(x, w, y)
    assert out.data_ptr() == y.data_ptr()
    assert device_status() == 0
    rel = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    err = (y.float() - ref).abs()
    assert (err <= rel * ref.abs() + 1e-3).all(), (err - rel * ref.abs()).max().item()


@pytest.mark.gpu
def test_gemm_residual_rejects_bad_shapes():
    from rl_for_mario_b200.kernels import gemm_residual

    x = torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        gemm_residual(x, torch.zeros(100, 64, dtype=torch.bfloat16, device="cuda"),
                      torch.zeros(8, 100, dtype=torch.bfloat16, device="cuda"))  # N not a multiple of 64


@pytest.mark.gpu
@pytest.mark.parametrize("B,S,K,Hq,Hkv,D", [(3, 48, 256, 8, 2, 32), (2, 300, 768, 12, 4, 64), (5, 21, 128, 4, 1, 32)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_qkv_rope_matches_projections_then_rope(B, S, K, Hq, Hkv, D, dtype):
    """q | k | v projections with the RoPE of q and k in the GEMM epilogue, no norm
    (the drop-in module's path on an already-normalised input)."""
    from oracle import apply_rotary_pos_emb, precompute_freqs_cis
    from rl_for_mario_b200.kernels import device_status, qkv_rope

    g = torch.Generator().manual_seed(B * S + K + D)
    x = torch.randn(B, S, K, generator=g).to(dtype)
    wq, wk, wv = ((torch.randn(h * D, K, generator=g) / K ** 0.5).to(dtype) for h in (Hq, Hkv, Hkv))
    cos, sin = precompute_freqs_cis(D, S + 3)
    y = qkv_rope(x.cuda(), torch.cat([wq, wk, wv]).cuda(), cos[:S].cuda(), sin[:S].cuda(), (Hq + Hkv) * D, D)
    assert device_status() == 0
    xf = x.float()
    q = (xf @ wq.float().t()).view(B, S, Hq, D)
    k = (xf @ wk.float().t()).view(B, S, Hkv, D)
    v = (xf @ wv.float().t()).view(B, S, Hkv, D)
    q, k = apply_rotary_pos_emb(q, k, cos[:S], sin[:S])
    ref = torch.cat([q, k, v], dim=2).reshape(B, S, -1)
    err = (y.float().cpu() - ref).abs()
    rel = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10  # one output rounding + fp32 accumulation
    assert (err <= rel * ref.abs() + 1e-3).all(), f"max err {err.max().item():.3e}"


@pytest.mark.gpu
def test_dropin_module_uses_one_gemm_path_and_matches_unfused():
    """FastDTAttention on 16-bit inputs takes the one-GEMM q | k | v + RoPE path; its output
    matches the separate projections + in-kernel RoPE path within bf16 noise, at D = 32 and 64."""
    from rl_for_mario_b200.attention import FastDTAttention
    from rl_for_mario_b200.dt_model import rope_tables

    for H, nh, nkv, S in ((256, 8, 2, 60), (768, 12, 4, 200)):
        class _Cfg:
            hidden_size, num_attention_heads, num_key_value_heads = H, nh, nkv
            dropout, flash_attn = 0.0, True

        torch.manual_seed(3)
        m = FastDTAttention(_Cfg()).cuda().to(torch.bfloat16).eval()
        with torch.no_grad():  # the one-GEMM path has no autograd: inference only
            assert m._qkv_rope_ok(torch.zeros(2, S, H, dtype=torch.bfloat16, device="cuda"))
        x = torch.randn(2, S, H, device="cuda").to(torch.bfloat16)
        cos, sin = (t.cuda().to(torch.bfloat16) for t in rope_tables(H // nh, S, 1e4))
        mask = (torch.arange(S, device="cuda")[None] >= torch.tensor([0, S // 3], device="cuda")[:, None]).float()
        with torch.no_grad():
            y1, _ = m(x, (cos, sin), attention_mask=mask)
            m.rope_rounding = "reference"  # separate projections, RoPE inside the attention kernel
            y2, _ = m(x, (cos, sin), attention_mask=mask)
        assert (y1.float() - y2.float()).abs().max().item() < 5e-2


# Whole-size rows (38,227 rows: an odd number of 128-row blocks, the last one
# mostly past the end; 65,536 rows: cfg4's per-layer batch of 128 x 512 rows
# over the persistent CTAs, several blocks each).  A row's result depends on its
# block only through its row index modulo 32 (the lane that sums its squares
# starts at a lane-dependent 16-byte piece), so the first 16 sequences and the
# last ones from a sequence whose first row is a multiple of 32, run alone, must
# come out bit-identical; the whole output is also checked against fp32.
@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["qkv", "qkv_rope", "swiglu", "nonorm_rope"])
@pytest.mark.parametrize("B,S", [(127, 301), (128, 512)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_large_row_counts_match_reference(mode, B, S, dtype):
    import torch.nn.functional as Fn
    from oracle import apply_rotary_pos_emb, precompute_freqs_cis
    from rl_for_mario_b200.kernels import (device_status, fold_norm_weight, fold_swiglu_weight, qkv_rope,
                                           rmsnorm_qkv, rmsnorm_swiglu)

    M, K, Hq, Hkv, D, F = B * S, 768, 12, 4, 64, 2048
    b_tail = 32 * ((B - 16) // 32)  # b_tail * S is a multiple of 32
    g = torch.Generator(device="cuda").manual_seed(M + len(mode))
    x = (torch.randn(B, S, K, generator=g, device="cuda") * 2).to(dtype)
    wn = 1 + 0.1 * torch.randn(K, generator=g, device="cuda")
    xn = x.float() if mode == "nonorm_rope" else rmsnorm_ref(x.float(), wn)
    cos, sin = (t.cuda() for t in precompute_freqs_cis(D, S))
    tab = 0.0
    if mode == "swiglu":
        wg, wu = (torch.randn(F, K, generator=g, device="cuda") / K ** 0.5 for _ in range(2))
        wf = fold_swiglu_weight(wg, wu, wn, dtype)
        run = lambda xs: rmsnorm_swiglu(xs.reshape(-1, K), wf, 1e-5)
        ref = (Fn.silu(xn @ wg.t()) * (xn @ wu.t())).view(M, F)
    else:
        wq, wk, wv = ((torch.randn(h * D, K, generator=g, device="cuda") / K ** 0.5).to(dtype)
                      for h in (Hq, Hkv, Hkv))
        rope = (cos, sin, (Hq + Hkv) * D, D)
        if mode == "qkv":
            wf = fold_norm_weight(wq, wk, wv, wn, dtype)
            run = lambda xs: rmsnorm_qkv(xs.reshape(-1, K), wf, 1e-5)
        elif mode == "qkv_rope":
            wf = fold_norm_weight(wq, wk, wv, wn, dtype)
            run = lambda xs: rmsnorm_qkv(xs, wf, 1e-5, rope=rope)
        else:
            wc = torch.cat([wq, wk, wv])
            run = lambda xs: qkv_rope(xs, wc, *rope)
        q, k, v = (xn @ w.float().t() for w in (wq, wk, wv))
        if mode != "qkv":
            # the kernel holds cos / sin as fp16 (relative rounding 2^-11): that
            # moves a rotated value by at most 2^-11 (|x[d]| + |x[d +- D/2]|)
            qk = torch.cat([q.reshape(M, -1), k.reshape(M, -1)], dim=1).view(M, -1, D).abs()
            tab = 2.0 ** -11 * (qk + torch.cat([qk[..., D // 2:], qk[..., :D // 2]], dim=-1)).view(M, -1)
            tab = torch.cat([tab, torch.zeros(M, Hkv * D, device="cuda")], dim=1)
            q, k = apply_rotary_pos_emb(q.view(B, S, Hq, D), k.view(B, S, Hkv, D), cos, sin)
        ref = torch.cat([t.reshape(M, -1) for t in (q, k, v)], dim=1)
    y = run(x).reshape(B, S, -1)
    assert device_status() == 0
    for part in (slice(0, 16), slice(b_tail, B)):
        assert torch.equal(y[part], run(x[part].contiguous()).reshape(part.stop - part.start, S, -1))
    err = (y.float().reshape(M, -1) - ref).abs()
    if mode == "nonorm_rope":
        rel = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
        bound = rel * ref.abs() + 1e-3 + tab
    else:
        # SwiGLU multiplies two projections, each with the folded norm weight
        # rounded to 16 bits, so its relative error is about twice the others'
        # (134 M outputs at 128 x 512 rows reach past the 2e-2 bf16 bound).
        tol = (3e-2 if mode == "swiglu" else 2e-2) if dtype == torch.bfloat16 else 4e-3
        bound = tol + tol * ref.abs()
    assert bool((err <= bound).all()), f"max excess {(err - bound).max().item():.3e}"
