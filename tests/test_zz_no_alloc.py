"""The allocation-free variant of the encoder's first-layer entry point.

dt_frames_conv1_noalloc serves callers that cannot allocate device memory (an
environment host in C or C++ that owns no allocator, a process whose memory
pool has reserved the GPU): it keeps its frame-maximum word in a static device
array of the library instead of a caller buffer.  Called through the C ABI,
it must give what dt_frames_conv1 gives on the same frames (bit for bit: the
same kernels run; any tolerance the conv1 tests use is therefore met), on two
calls in a row whose frames need different scaling, so a word left over from
the first call would show in the second.

This file is named to be collected last: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes

import pytest
import torch

from rl_for_mario_b200 import _lib


def _frames(seed, hi, n=64):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, hi + 1, (n, 4, 84, 84), generator=g, dtype=torch.uint8).cuda()


def _conv1(lib, frames, w2, bias, noalloc):
    N, C, H, W = frames.shape
    y = torch.empty((N, 20, 20, 32), dtype=w2.dtype, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = lib.dt_frames_conv1_noalloc(frames.data_ptr(), N, C, H, W, w2.data_ptr(), bias.data_ptr(),
                                         y.data_ptr(), 0, _lib.DT_DTYPE_BF16, stream)
    else:
        fmax = torch.empty(1, dtype=torch.int32, device="cuda")
        rc = lib.dt_frames_conv1(frames.data_ptr(), N, C, H, W, w2.data_ptr(), bias.data_ptr(), fmax.data_ptr(),
                                 y.data_ptr(), 0, _lib.DT_DTYPE_BF16, stream)
    _lib.check("dt_frames_conv1_noalloc" if noalloc else "dt_frames_conv1", rc)
    return y


@pytest.mark.gpu
def test_noalloc_conv1_matches_the_allocating_entry_point():
    lib = _lib.load()
    g = torch.Generator().manual_seed(5)
    w2 = (torch.randn(32, 256, generator=g) * 0.05).to(torch.bfloat16).cuda()
    bias = (torch.randn(32, generator=g) * 0.1).cuda()
    # First call: pixels up to 255, so the 1/255 scale applies and the scratch
    # word ends at a value > 1.  Second call: 0 / 1 pixels, no scale; a stale
    # word would wrongly scale them.
    for frames in (_frames(1, 255), _frames(2, 1)):
        ref = _conv1(lib, frames, w2, bias, noalloc=False)
        out = _conv1(lib, frames, w2, bias, noalloc=True)
        torch.cuda.synchronize()
        assert lib.dt_device_status(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        assert torch.equal(out, ref)
    # The unscaled second call differs from the scaled first one (the test has teeth).
    assert _conv1(lib, _frames(2, 1), w2, bias, True).float().abs().max() > 0.5


@pytest.mark.gpu
def test_noalloc_conv1_rejects_bad_arguments():
    lib = _lib.load()
    frames = _frames(3, 255, n=2)
    w2 = torch.zeros(32, 256, dtype=torch.bfloat16, device="cuda")
    bias = torch.zeros(32, device="cuda")
    y = torch.empty((2, 20, 20, 32), dtype=torch.bfloat16, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.dt_frames_conv1_noalloc(frames.data_ptr(), 2, 3, 84, 84, w2.data_ptr(), bias.data_ptr(), y.data_ptr(),
                                       0, _lib.DT_DTYPE_BF16, s) == _lib.DT_ERR_UNSUPPORTED
    assert lib.dt_frames_conv1_noalloc(None, 2, 4, 84, 84, w2.data_ptr(), bias.data_ptr(), y.data_ptr(),
                                       0, _lib.DT_DTYPE_BF16, s) == _lib.DT_ERR_INVALID
    assert lib.dt_frames_conv1_noalloc(frames.data_ptr(), 2, 4, 83, 84, w2.data_ptr(), bias.data_ptr(),
                                       y.data_ptr(), 0, _lib.DT_DTYPE_BF16, s) == _lib.DT_ERR_INVALID
