"""Seeded input recipes shared by the golden generator and the tests.

The golden files store outputs (and small inputs); the larger acceptance
inputs are rebuilt from these recipes, which use only the CPU torch
generator and are therefore identical wherever the same torch runs.
"""

from __future__ import annotations

import torch


def acceptance_inputs(B: int, K: int, V: int, seed: int, temperature: float):
    """Config-4-shaped acceptance inputs at a chosen size.

    Target logits ``2 N(0, 1)`` in bf16 (B, K+1, V).  Greedy: row b's draft
    matches the target argmax on its first ``b mod (K+1)`` slots, then
    misses.  Sampled: draft tokens uniform, draft probabilities
    ``softmax(N(0, 1))`` fp32, and the target logits raised by 3 at the
    drafted tokens so that some drafts are accepted.
    """
    g = torch.Generator().manual_seed(seed)
    target = (2.0 * torch.randn(B, K + 1, V, generator=g))
    if temperature <= 0:
        tt = target.to(torch.bfloat16).argmax(-1)
        draft = torch.randint(0, V, (B, K), generator=g)
        for b in range(B):
            a = b % (K + 1)
            draft[b, :a] = tt[b, :a]
            if a < K:
                draft[b, a] = (tt[b, a] + 1) % V
        return target.to(torch.bfloat16), draft, None
    draft = torch.randint(0, V, (B, K), generator=g)
    q = torch.randn(B, K, V, generator=g).softmax(-1)
    rows = torch.arange(B)[:, None]
    cols = torch.arange(K)[None, :]
    target[rows, cols, draft] += 3.0
    return target.to(torch.bfloat16), draft, q
