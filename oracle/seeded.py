"""Deterministic synthetic weights and inputs (test infrastructure).

Parameters are drawn per name from numpy's PCG64 stream seeded with
(seed, crc32(name)), so a state_dict is reproducible from (seed, names,
shapes) alone on any machine with the same numpy.  Used to build identical
weights for the reference module (golden generation), the oracle and the CUDA
path without shipping weight files.
"""
from __future__ import annotations

import zlib
from typing import Dict, Iterable, Tuple

import numpy as np
import torch


def _rng(seed: int, tag: str) -> np.random.Generator:
    return np.random.default_rng([int(seed), zlib.crc32(tag.encode())])


def seeded_normal(shape, seed: int, tag: str, scale: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    a = _rng(seed, tag).standard_normal(tuple(shape), dtype=np.float32)
    return torch.from_numpy(a * np.float32(scale) + np.float32(mean))


def seeded_uniform_int(shape, low: int, high: int, seed: int, tag: str) -> torch.Tensor:
    return torch.from_numpy(_rng(seed, tag).integers(low, high, size=tuple(shape), dtype=np.int64))


def seeded_uniform(shape, low: float, high: float, seed: int, tag: str) -> torch.Tensor:
    return torch.from_numpy(_rng(seed, tag).uniform(low, high, size=tuple(shape)).astype(np.float32))


def param_init(name: str, shape: Tuple[int, ...], seed: int) -> torch.Tensor:
    """One parameter: norm weights ~ 1 + 0.1 N, biases ~ 0.02 N, embeddings ~ 0.5 N,
    linear / conv weights ~ N / sqrt(fan_in)."""
    if name.endswith("norm.weight") or name.endswith("layernorm.weight"):
        return seeded_normal(shape, seed, name, 0.1, 1.0)
    if name.endswith(".bias"):
        return seeded_normal(shape, seed, name, 0.02)
    if "embed_action" in name or "embed_timestep" in name:
        return seeded_normal(shape, seed, name, 0.5)
    fan_in = int(np.prod(shape[1:])) if len(shape) > 1 else int(shape[0])
    return seeded_normal(shape, seed, name, 1.0 / np.sqrt(fan_in))


def seeded_state_dict(named_shapes: Iterable[Tuple[str, Tuple[int, ...]]], seed: int) -> Dict[str, torch.Tensor]:
    return {n: param_init(n, tuple(s), seed) for n, s in named_shapes}


def checksum(t: torch.Tensor) -> float:
    """Order-sensitive float64 checksum used to detect stream drift."""
    a = t.detach().double().reshape(-1)
    w = torch.arange(1, a.numel() + 1, dtype=torch.float64)
    return float((a * (1.0 + (w % 97) / 97.0)).sum())


def dt_synthetic_inputs(tag: str, seed: int, B: int, T: int, state_shape, act_dim: int,
                        pad_max: int = -1):
    """Seeded DT inputs with the shapes and distributions of the repo-default
    workload: uint8 frames U[0, 255], actions U{0..act_dim-1}, returns-to-go
    U[0, 3000], timesteps start + arange(T) with start U{0..3999}, and (when
    pad_max >= 0) left padding U{0..pad_max} timesteps per sample with the
    matching [B, T] attention mask (1 = valid).  Returns a dict of CPU tensors."""
    states = seeded_uniform_int((B, T, *state_shape), 0, 256, seed, tag + ":states").to(torch.uint8)
    actions = seeded_uniform_int((B, T), 0, act_dim, seed, tag + ":actions")
    rtg = seeded_uniform((B, T), 0.0, 3000.0, seed, tag + ":rtg")
    start = seeded_uniform_int((B, 1), 0, 4000, seed, tag + ":start")
    out = {"states": states, "actions": actions, "rtg": rtg, "timesteps": start + torch.arange(T)[None]}
    if pad_max >= 0:
        pads = seeded_uniform_int((B,), 0, pad_max + 1, seed, tag + ":pads")
        out["pad_steps"] = pads
        out["mask"] = (torch.arange(T)[None] >= pads[:, None]).long()
    return out
