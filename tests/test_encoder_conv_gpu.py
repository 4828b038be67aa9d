"""The state encoder's second and third layers on the tensor cores
(dt_encoder_conv23) against PyTorch's fp32 convolution of the same 16-bit
values (reference model/model_decision_transformer.py:322-325).

Frame counts cover one frame, counts below and above the number of SMs (the
persistent CTAs take one frame at a time, loading the next one into the other
input buffer, so 300 and 1001 frames wrap both buffers and the accumulator
barrier's phase many times).  Tolerance: the output's own 16-bit rounding
(2^-8 relative) plus 2e-3 absolute for fp32 accumulation order.
"""
import pytest
import torch
import torch.nn.functional as F

RTOL, ATOL = 2.0 ** -8, 2e-3


def _inputs(N, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x1 = torch.relu(torch.randn(N, 32, 20, 20, generator=g, device="cuda")).to(dtype)
    x1 = x1.contiguous(memory_format=torch.channels_last)
    w2 = (torch.randn(64, 32, 4, 4, generator=g, device="cuda") * 0.05).to(dtype)
    b2 = (torch.randn(64, generator=g, device="cuda") * 0.1).to(dtype)
    w3 = (torch.randn(64, 64, 3, 3, generator=g, device="cuda") * 0.05).to(dtype)
    b3 = (torch.randn(64, generator=g, device="cuda") * 0.1).to(dtype)
    return x1, w2, b2, w3, b3


def _ref(x, w, b, stride):
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        return torch.relu(F.conv2d(x.float(), w.float(), b.float(), stride=stride))
    finally:
        torch.backends.cudnn.allow_tf32 = prev


def _close(out, ref, what):
    err = (out.float() - ref).abs()
    worst = (err - ATOL - RTOL * ref.abs()).max().item()
    assert worst <= 0, f"{what}: max err {err.max().item():.3e} exceeds the bound by {worst:.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("N", [1, 2, 3, 7, 300, 1001])
def test_encoder_conv23_matches_fp32(N, dtype):
    from rl_for_mario_b200.kernels import device_status, encoder_conv23

    x1, w2, b2, w3, b3 = _inputs(N, dtype, seed=N)
    y2, y3 = encoder_conv23(x1, w2, b2, w3, b3)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert y2.shape == (N, 64, 9, 9) and y3.shape == (N, 64, 7, 7)
    assert y2.is_contiguous(memory_format=torch.channels_last)
    _close(y2, _ref(x1, w2, b2, 2), "conv2")
    # The third layer against fp32 on its actual (16-bit) input.
    _close(y3, _ref(y2, w3, b3, 1), "conv3")


@pytest.mark.gpu
def test_encoder_conv23_repeatable_and_order_free():
    """Same bits for a frame whatever its place in the batch (the persistent
    schedule and the frame pairing of the third layer do not change results)."""
    from rl_for_mario_b200.kernels import encoder_conv23

    x1, w2, b2, w3, b3 = _inputs(517, torch.bfloat16, seed=7)
    y2, y3 = encoder_conv23(x1, w2, b2, w3, b3)
    perm = torch.randperm(517, generator=torch.Generator().manual_seed(3)).cuda()
    y2p, y3p = encoder_conv23(x1[perm].contiguous(memory_format=torch.channels_last), w2, b2, w3, b3)
    assert torch.equal(y2p, y2[perm])
    assert torch.equal(y3p, y3[perm])


@pytest.mark.gpu
def test_encoder_conv23_rejects_bad_arguments():
    from rl_for_mario_b200.kernels import encoder_conv23

    x1, w2, b2, w3, b3 = _inputs(2, torch.bfloat16, seed=1)
    with pytest.raises(ValueError):
        encoder_conv23(x1.contiguous(), w2, b2, w3, b3)  # not channels-last
    with pytest.raises(ValueError):
        encoder_conv23(x1, w2.float(), b2, w3, b3)
    with pytest.raises(ValueError):
        encoder_conv23(x1, w3, b2, w2, b3)


@pytest.mark.gpu
def test_encoder_conv23_in_the_model_encoder():
    """The DT's state encoder with layers 2 and 3 routed through dt_encoder_conv23
    equals its default path (cuDNN's fused convolution) within the 16-bit bound."""
    from rl_for_mario_b200.dt_model import MarioStateEncoder

    torch.manual_seed(0)
    enc = MarioStateEncoder((4, 84, 84), 256).cuda().to(torch.bfloat16).eval()
    g = torch.Generator(device="cuda").manual_seed(2)
    frames = torch.randint(0, 256, (3, 5, 4, 84, 84), device="cuda", generator=g, dtype=torch.uint8)
    with torch.no_grad():
        base = enc(frames)
        MarioStateEncoder._tc_conv23 = True
        try:
            ours = enc(frames)
        finally:
            MarioStateEncoder._tc_conv23 = False
    err = (ours.float() - base.float()).abs()
    assert (err - 2e-2 - 2.0 ** -7 * base.float().abs()).max().item() <= 0, f"max err {err.max().item():.3e}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_encoder_conv23_without_storing_y2(dtype):
    """keep_y2=False: the second layer's output stays in shared memory; the
    third layer's output is bit-identical to the run that also stores y2."""
    from rl_for_mario_b200.kernels import device_status, encoder_conv23

    x1, w2, b2, w3, b3 = _inputs(333, dtype, seed=5)
    y2, y3 = encoder_conv23(x1, w2, b2, w3, b3)
    none, y3b = encoder_conv23(x1, w2, b2, w3, b3, keep_y2=False)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert none is None and torch.equal(y3, y3b)
