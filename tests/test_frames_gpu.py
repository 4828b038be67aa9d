"""GPU parity of the state-encoder input kernel (dt_frames_to_blocks) and of the
space-to-depth first convolution against the reference encoder's direct one."""
import pytest
import torch


@pytest.mark.gpu
@pytest.mark.parametrize("N,C,H,W", [(1, 4, 84, 84), (37, 4, 84, 84), (5, 1, 8, 12), (3, 3, 16, 4)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_frames_to_blocks_exact(N, C, H, W, dtype):
    from rl_for_mario_b200.kernels import device_status, frames_to_blocks

    g = torch.Generator().manual_seed(N * C + H)
    fr = torch.randint(0, 256, (N, C, H, W), generator=g, dtype=torch.uint8)
    out = frames_to_blocks(fr.cuda(), dtype)
    assert device_status() == 0
    assert out.shape == (N, C * 16, H // 4, W // 4) and out.is_contiguous(memory_format=torch.channels_last)
    ref = fr.view(N, C, H // 4, 4, W // 4, 4).permute(0, 1, 3, 5, 2, 4).reshape(N, C * 16, H // 4, W // 4)
    assert torch.equal(out.cpu().to(torch.int32), ref.to(torch.int32))


@pytest.mark.gpu
@pytest.mark.parametrize("N,C,H,W,offset", [(7, 4, 84, 84, 4), (3, 4, 128, 128, 0), (5, 3, 8, 8, 4)])
def test_frames_to_blocks_other_layouts(N, C, H, W, offset):
    """Frames that are only 4-byte aligned, or larger than one CTA's shared memory,
    take the per-position kernels; same result."""
    from rl_for_mario_b200.kernels import device_status, frames_to_blocks

    g = torch.Generator().manual_seed(N + C + H + offset)
    fr = torch.randint(0, 256, (N, C, H, W), generator=g, dtype=torch.uint8)
    buf = torch.zeros(fr.numel() + 16, dtype=torch.uint8, device="cuda")
    view = buf[offset:offset + fr.numel()].view(N, C, H, W)
    view.copy_(fr.cuda())
    fm = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = frames_to_blocks(view, torch.bfloat16, fm)
    assert device_status() == 0
    ref = fr.view(N, C, H // 4, 4, W // 4, 4).permute(0, 1, 3, 5, 2, 4).reshape(N, C * 16, H // 4, W // 4)
    assert torch.equal(out.cpu().to(torch.int32), ref.to(torch.int32))
    assert int(fm.item()) == int(fr.max())


@pytest.mark.gpu
def test_frames_to_blocks_rejects_bad_shapes():
    from rl_for_mario_b200.kernels import frames_to_blocks

    with pytest.raises(RuntimeError):
        frames_to_blocks(torch.zeros(2, 4, 10, 84, dtype=torch.uint8, device="cuda"), torch.bfloat16)
    with pytest.raises(ValueError):
        frames_to_blocks(torch.zeros(2, 4, 84, 84, dtype=torch.float32, device="cuda"), torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_state_encoder_matches_direct_convolution(dtype):
    """16-bit encoder (frame blocks + 2 x 2 convolution, fused convolution + bias +
    ReLU, permuted Linear) vs the reference's direct 8 x 8 stride-4 convolution of
    frames / 255, in fp32."""
    from rl_for_mario_b200.dt_model import MarioStateEncoder

    torch.manual_seed(0)
    enc = MarioStateEncoder((4, 84, 84), 256).eval()
    s = torch.randint(0, 256, (3, 5, 4, 84, 84), dtype=torch.uint8)
    with torch.no_grad():
        ref = enc.cnn(s.reshape(15, 4, 84, 84).float() / 255.0).reshape(3, 5, -1)
        out = enc.cuda().to(dtype)(s.cuda())
    err = (out.float().cpu() - ref).abs().max().item()
    assert err < 3e-2 * max(1.0, ref.abs().max().item()), err


@pytest.mark.gpu
@pytest.mark.parametrize("hi", [1, 2, 255])
def test_frames_to_blocks_reports_max(hi):
    from rl_for_mario_b200.kernels import frames_to_blocks

    g = torch.Generator().manual_seed(hi)
    fr = torch.randint(0, hi + 1, (9, 4, 84, 84), generator=g, dtype=torch.uint8)
    fm = torch.zeros(1, dtype=torch.int32, device="cuda")
    frames_to_blocks(fr.cuda(), torch.bfloat16, fm)
    assert int(fm.item()) == int(fr.max())


@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(1, 768), (1000, 768), (77, 256), (5, 8), (33, 2048), (300, 1032)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm_kernel_matches_reference(M, K, dtype):
    """Row RMSNorm with the reference's rounding (normalised row cast before the weight product)."""
    from rl_for_mario_b200.kernels import device_status, rmsnorm

    g = torch.Generator().manual_seed(M * 7 + K)
    x = (torch.randn(M, K, generator=g) * 3).to(dtype)
    w = (1 + 0.2 * torch.randn(K, generator=g)).to(dtype)
    y = rmsnorm(x.cuda(), w.cuda(), 1e-5)
    assert device_status() == 0
    xf = x.float()
    ref = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(dtype)
    err = (y.cpu().float() - ref.float()).abs()
    ulp = 2.0 ** (-7 if dtype == torch.bfloat16 else -10)
    # a different summation order may move the normalised value across a rounding boundary
    assert (err <= 2 * ulp * ref.float().abs() + 1e-6).all(), err.max().item()
    assert (err == 0).float().mean().item() > 0.95


@pytest.mark.gpu
def test_rmsnorm_module_unaligned_view_uses_reference_formula():
    """A row view that is not 16-byte aligned takes the PyTorch formula instead of the kernel."""
    from rl_for_mario_b200.dt_model import RMSNorm

    g = torch.Generator().manual_seed(3)
    big = (torch.randn(6, 10, 72, generator=g) * 2).to(torch.bfloat16).cuda()
    x = big[..., 3:67]  # 64 columns starting 6 bytes into each row
    norm = RMSNorm(64).cuda().to(torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.1 * torch.randn(64, generator=g)).to(torch.bfloat16))
        y = norm(x)
    xf = x.float()
    ref = norm.weight * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + norm.eps)).to(torch.bfloat16)
    assert torch.equal(y, ref)


# Output rounding bound: the kernel forms the convolution of the frames / 255
# in fp32 (exact 16-bit pixel values, fp32 accumulation, the 1/255 applied to
# the accumulator) and rounds once to the output dtype, so it is within half an
# output ulp (2^-8 relative for bf16, 2^-11 for fp16) plus fp32 summation
# error of the fp32 convolution of frames / 255.  (The reference's bf16 model
# rounds frames / 255 to bf16 before its convolution; this kernel does not.)
CONV1_REL = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


@pytest.mark.gpu
@pytest.mark.parametrize("N,H,W,hi", [(1, 84, 84, 255), (37, 84, 84, 255), (3, 12, 20, 255), (5, 84, 84, 1),
                                      (256, 84, 84, 255), (1024, 84, 84, 255)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_frames_conv1_matches_reference(N, H, W, hi, dtype):
    """relu(conv2d(frames / 255 when their max exceeds 1, w, b, stride 4)) from uint8 frames in one kernel.
    256 and 1,024 frames of 84 x 84 give 800 and 3,200 tiles of 128 positions over the
    persistent CTAs (5 and 21 per CTA), so both A buffers and TMEM accumulators wrap."""
    import torch.nn.functional as Fn
    from rl_for_mario_b200.kernels import device_status, frames_conv1

    g = torch.Generator().manual_seed(N * 3 + H + hi)
    fr = torch.randint(0, hi + 1, (N, 4, H, W), generator=g, dtype=torch.uint8)
    w = (torch.randn(32, 4, 8, 8, generator=g) * 0.05).to(dtype)
    b = (torch.randn(32, generator=g) * 0.1).to(dtype)
    out, fmax = frames_conv1(fr.cuda(), w.cuda(), b.cuda())
    assert device_status() == 0
    assert (int(fmax.item()) > 1) == (int(fr.max()) > 1)
    # fp32 reference convolution on the GPU (TF32 off), exact inputs.
    torch.backends.cudnn.allow_tf32 = False
    frc = fr.cuda()
    x = frc.float() / 255.0 if int(fr.max()) > 1 else frc.float()
    ref = Fn.relu(Fn.conv2d(x, w.cuda().float(), b.cuda().float(), stride=4))
    assert out.shape == ref.shape and out.is_contiguous(memory_format=torch.channels_last)
    err = (out.float() - ref).abs()
    bound = CONV1_REL[dtype] * ref.abs() + 1e-5
    assert (err <= bound).all(), (err - bound).max().item()


@pytest.mark.gpu
def test_frames_conv1_scale_from_a_single_byte():
    """Frames of 0 / 1 with one byte of 2 in the last frame still take the 1/255 scale."""
    import torch.nn.functional as Fn
    from rl_for_mario_b200.kernels import frames_conv1

    g = torch.Generator().manual_seed(11)
    fr = torch.randint(0, 2, (50, 4, 84, 84), generator=g, dtype=torch.uint8)
    fr[-1, 3, 83, 83] = 2
    w = (torch.randn(32, 4, 8, 8, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(32, generator=g) * 0.1).to(torch.bfloat16)
    out, fmax = frames_conv1(fr.cuda(), w.cuda(), b.cuda())
    assert int(fmax.item()) > 1
    ref = Fn.relu(Fn.conv2d(fr.float() / 255.0, w.float(), b.float(), stride=4))
    err = (out.float().cpu() - ref).abs()
    assert (err <= 1e-2 * (1 + ref.abs())).all(), err.max().item()
