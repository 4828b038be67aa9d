"""CPU-side checks of the C-ABI library: it loads, exports every symbol the
public header declares, and the host wrappers reject bad input before any
device work (no GPU needed)."""
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?\w+\s*\*?\s*(dt_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "dt_attn_prefill" in names and "dt_last_error" in names


def test_library_exports_every_declared_symbol():
    from rl_for_mario_b200 import _lib

    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string():
    from rl_for_mario_b200 import _lib

    lib = _lib.load()
    assert lib.dt_version() >= 1
    assert isinstance(lib.dt_last_error(), bytes)


def test_null_pointer_rejected_without_gpu():
    from rl_for_mario_b200 import _lib

    lib = _lib.load()
    rc = lib.dt_attn_prefill(None, None, None, None, None, None, 0, 0, None, 1, 1, 8, 2, 32,
                             *([8] * 12), 0.0, 1, 0, None)
    assert rc == _lib.DT_ERR_INVALID
    assert b"null" in lib.dt_last_error()


def test_wrapper_refuses_cpu_tensors():
    from rl_for_mario_b200.kernels import attn_prefill

    q = torch.zeros(1, 4, 8, 32, dtype=torch.bfloat16)
    k = torch.zeros(1, 4, 2, 32, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        attn_prefill(q, k, k, None, None, apply_rope=False)


def test_pad_len_from_mask():
    from rl_for_mario_b200.kernels import pad_len_from_mask

    m = torch.tensor([[1, 1, 1, 1], [0, 0, 1, 1], [0, 0, 0, 0]])
    assert pad_len_from_mask(m, 4).tolist() == [0, 2, 4]
