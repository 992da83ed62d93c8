"""The tree-drafting oracle (oracle/tree_oracle.py) against golden vectors of
the reference's build_tree_abi (flashmap/sglang/tree.py) and tree_commit
(flashmap/sglang/kernels.py, run by Triton's CPU interpreter), made by
tests/golden/make_tree_golden.py: identical results."""

import os

import pytest
import torch

from oracle import tree_oracle as TO

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "tree_cases.pt")
CASES = torch.load(GOLDEN)


@pytest.mark.parametrize("i", range(len(CASES["builds"])))
def test_build_tree(i):
    c = CASES["builds"][i]
    tokens, ids, stats = TO.build_tree(c["candidates"], c["width"])
    assert torch.equal(tokens, c["tokens"]) and torch.equal(ids, c["ids"]) and torch.equal(stats, c["stats"])


@pytest.mark.parametrize("i", range(len(CASES["commits"])))
def test_tree_commit(i):
    c = CASES["commits"][i]
    table = c["req_to_token_before"].clone()
    out = TO.tree_commit(c["accept"], c["num_correct"], c["window"], c["predict"], c["req_pool"], c["prefix"], table)
    assert torch.equal(table, c["req_to_token_after"])
    for got, name in zip(out, ("out_tokens", "bonus", "commit", "new_seq_lens", "inject_locs")):
        assert torch.equal(got, c[name]), name
