"""Paged KV cache of the decode path.

The reference keeps, per layer, a pair of post-RoPE tensors (K, V) of shape
[B, Hkv, L, D] and grows them with torch.cat every step
(model/model_decision_transformer.py:188-191).  Here each layer owns a pool of
pages ``k_pages / v_pages [num_pages, Hkv, page_size, D]`` written in place
by the kernels; ``block_table [B, max_pages]`` maps positions to pages and
``seq_lens [B]`` counts the cached positions of every sample.

``LayerKV`` is what a decoder layer receives as ``past_key_value``: it
indexes like the reference's tuple (``cache[0].shape[2] == L``, which the
backbone reads to slice RoPE tables, :439) and has no ``layers`` attribute
(the backbone drops such objects, :436-437).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Tuple

import torch

Tensor = torch.Tensor


class _ShapeView:
    """Stands in for the reference's cached K (or V) tensor: exposes its shape."""

    def __init__(self, layer: "LayerKV", which: int):
        self._layer, self._which = layer, which

    @property
    def shape(self) -> torch.Size:
        c = self._layer
        return torch.Size((c.batch, c.num_kv_heads, c.length, c.head_dim))

    def size(self, dim: Optional[int] = None):
        return self.shape if dim is None else self.shape[dim]

    @property
    def dtype(self):
        return self._layer.k_pages.dtype

    @property
    def device(self):
        return self._layer.k_pages.device

    def materialize(self) -> Tensor:
        return self._layer.dense()[self._which]


@dataclass
class LayerKV:
    """One layer's paged cache plus the host mirror of its (uniform) length."""

    k_pages: Tensor          # [num_pages, Hkv, page_size, D]
    v_pages: Tensor
    block_table: Tensor      # [B, max_pages] int32
    seq_lens: Tensor         # [B] int32, device
    length: int              # cached positions (all samples advance together)

    @property
    def batch(self) -> int:
        return self.block_table.shape[0]

    @property
    def num_kv_heads(self) -> int:
        return self.k_pages.shape[1]

    @property
    def page_size(self) -> int:
        return self.k_pages.shape[2]

    @property
    def head_dim(self) -> int:
        return self.k_pages.shape[3]

    @property
    def capacity(self) -> int:
        return self.block_table.shape[1] * self.page_size

    def __getitem__(self, i: int):
        if i not in (0, 1):
            raise IndexError(i)
        return _ShapeView(self, i)

    def __len__(self) -> int:
        return 2

    def __iter__(self):
        return iter((self[0], self[1]))

    def advance(self, n: int) -> None:
        """Counts n appended positions (on the device and in the host mirror)."""
        self.seq_lens.add_(n)
        self.length += n

    def reset(self) -> None:
        self.seq_lens.zero_()
        self.length = 0

    def dense(self) -> Tuple[Tensor, Tensor]:
        """Gathers the cached positions into the reference's [B, Hkv, L, D] tensors."""
        B, L, P = self.batch, self.length, self.page_size
        pos = torch.arange(L, device=self.k_pages.device)
        pages = self.block_table[:, pos // P].long()              # [B, L]
        slot = (pos % P).view(1, L).expand(B, L)
        k = self.k_pages[pages, :, slot]                          # [B, L, Hkv, D]
        v = self.v_pages[pages, :, slot]
        return k.permute(0, 2, 1, 3).contiguous(), v.permute(0, 2, 1, 3).contiguous()


class PagedKVCache:
    """Per-layer paged caches for B sequences of up to max_len positions.

    Pages are assigned statically: sample b owns pages
    [b * pages_per_seq, (b + 1) * pages_per_seq).  The block table is shared by
    all layers; each layer has its own pool and length counter, so a layer's
    append is visible to later layers of the same step only through their own
    counters (as with the reference's per-layer presents).
    """

    def __init__(self, num_layers: int, batch: int, num_kv_heads: int, head_dim: int, max_len: int,
                 page_size: int = 64, dtype: torch.dtype = torch.bfloat16, device="cuda"):
        if max_len < 1 or page_size < 1:
            raise ValueError("max_len and page_size must be positive")
        self.pages_per_seq = (max_len + page_size - 1) // page_size
        num_pages = batch * self.pages_per_seq
        self.block_table = torch.arange(num_pages, dtype=torch.int32, device=device).view(batch,
                                                                                         self.pages_per_seq)
        self.layers: List[LayerKV] = []
        for _ in range(num_layers):
            kp = torch.zeros(num_pages, num_kv_heads, page_size, head_dim, dtype=dtype, device=device)
            vp = torch.zeros_like(kp)
            self.layers.append(LayerKV(kp, vp, self.block_table, torch.zeros(batch, dtype=torch.int32,
                                                                            device=device), 0))

    def __getitem__(self, i: int) -> LayerKV:
        return self.layers[i]

    def __len__(self) -> int:
        return len(self.layers)

    def as_past(self) -> list:
        """The list the backbone takes as past_key_values (one LayerKV per layer)."""
        return list(self.layers)

    def reset(self) -> None:
        for l in self.layers:
            l.reset()

    @property
    def length(self) -> int:
        return self.layers[0].length if self.layers else 0


def dense_layer(k: Tensor, v: Tensor, length: int) -> LayerKV:
    """Wraps dense [B, Hkv, cap, D] tensors as a one-page-per-sample cache of `length` positions."""
    B, Hkv, cap, D = k.shape
    bt = torch.arange(B, dtype=torch.int32, device=k.device).view(B, 1)
    # [B, Hkv, cap, D] is exactly [num_pages=B, Hkv, page_size=cap, D].
    return LayerKV(k, v, bt, torch.full((B,), length, dtype=torch.int32, device=k.device), length)
