"""The verify tree of a multi-candidate draft (flashmap/sglang/tree.py) on
this library's kernel: ``build_tree_abi`` under the reference's name and
contract (``fm_tree_build``)."""

from __future__ import annotations

import torch

from . import _lib
from .serving_ops import _need, _p, _stream

__all__ = ["build_tree_abi"]


def build_tree_abi(candidates: torch.Tensor, width: int):
    """The verify tree from N candidate blocks per request, in EAGLE's encoding
    (tree.py:9-78): ``candidates (bs, N, K)`` int64 drafts after each request's
    root; returns ``tokens (bs, width - 1)``, ``ids (bs, width - 1)`` = parent *
    width + index, and ``stats (bs, 2)`` = (trie nodes, distinct candidates).
    The kept nodes are the width - 1 with the most candidates through them
    (ties: shallower, then lower candidate), listed by depth then candidate; a
    smaller trie is padded with copies of the first node under the root.  On
    device, fixed shapes, no host synchronization."""
    _need(candidates.is_cuda and candidates.dim() == 3, "candidates must be a CUDA (bs, N, K) tensor")
    _need(width >= 2, "width must be at least 2")
    bs, n, k = candidates.shape
    c = candidates.to(torch.int64).contiguous()
    tokens = torch.empty(bs, width - 1, dtype=torch.int64, device=c.device)
    ids = torch.empty(bs, width - 1, dtype=torch.int64, device=c.device)
    stats = torch.empty(bs, 2, dtype=torch.int64, device=c.device)
    _lib.call("fm_tree_build", _p(c), bs, n, k, int(width), _p(tokens), _p(ids), _p(stats), _stream())
    return tokens.to(candidates.dtype), ids, stats
