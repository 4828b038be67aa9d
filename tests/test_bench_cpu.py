"""Roofline arithmetic of bench.py, checked on the CPU.

The prefill rooflines count FLOPs and exponentials from bench._attended_pairs;
that count is held here to the (query, key) pairs the oracle's masked softmax
(causal triangle plus the reference's -1e9 band on padded key columns) gives
weight to.  The headline byte count and the fused encoder kernel's operand
floor are checked against their definitions.
"""
import torch

import bench
from oracle.attention_ref import attention_prefill_ref, mask_from_pad_len


def test_attended_pairs_match_the_oracle_softmax():
    # q = k = 0 makes every score 0, and v = identity makes the output rows the
    # softmax weights themselves: the pairs with weight > 0 are the attended ones
    # (a fully padded row spreads its weight over keys 0..q).
    S, pads = 24, [0, 1, 5, 12, 23, 24]
    B = len(pads)
    q = torch.zeros(B, S, 1, S)
    k = torch.zeros(B, S, 1, S)
    v = torch.eye(S).expand(B, S, S).reshape(B, S, 1, S).contiguous()
    w = attention_prefill_ref(q, k, v, None, None, mask_from_pad_len(torch.tensor(pads), S), rope=False)
    assert torch.allclose(w.sum(-1), torch.ones(B, S, 1))
    assert int((w > 0).sum()) == bench._attended_pairs(S, pads)


def test_headline_algorithmic_bytes():
    # Q and O: 4096 x 192 x 8 heads x 32 x 2 bytes each; K and V: 2 heads each.
    B, S, Hq, Hkv, D = 4096, 192, 8, 2, 32
    q_or_o = B * S * Hq * D * 2
    k_or_v = B * S * Hkv * D * 2
    assert bench._algorithmic_bytes(B, S, Hq, Hkv, D) == 2 * q_or_o + 2 * k_or_v == 1_006_632_960


def test_conv23_operand_floor():
    # Per frame: conv2 2 (dy) x 8 (K steps) MMAs of M = 128, N = 128, K = 16;
    # conv3 3 (ky) x 4 MMAs of M = 128, N = 192; A and B read once per MMA, 2 bytes each.
    per_frame = 2 * 8 * (128 * 16 + 128 * 16) * 2 + 3 * 4 * (128 * 16 + 192 * 16) * 2
    assert bench.CONV23_OPERAND_BYTES_PER_FRAME == per_frame
    r = bench.conv23_bound(262144, 4.0, 1965.0, 148)
    floor_ms = 262144 * per_frame / (128 * 148 * 1965e6) * 1e3
    assert abs(r["lower_bound_ms"] - floor_ms) < 1e-9
    assert abs(r["frac"] - floor_ms / 4.0) < 1e-12
