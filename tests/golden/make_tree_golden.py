"""Generate the golden vectors that pin the tree-drafting oracle
(``oracle/tree_oracle.py``) to the reference: ``build_tree_abi``
(flashmap/sglang/tree.py, pure torch) and ``tree_commit``
(flashmap/sglang/kernels.py, a Triton kernel, run here by Triton's CPU
interpreter), al-jshen/flashmap v0.2.1 imported from a checkout given by
``--reference``.  Saves ``tests/golden/tree_cases.pt``.

    python tests/golden/make_tree_golden.py --reference /path/to/flashmap
"""

from __future__ import annotations

import argparse
import importlib.util
import os

os.environ.setdefault("TRITON_INTERPRET", "1")  # before triton is imported

import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def load(reference: str, name: str):
    spec = importlib.util.spec_from_file_location(f"ref_{name}", os.path.join(reference, "flashmap", "sglang",
                                                                              f"{name}.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def candidates_with_prefixes(g, bs, n, k, vocab):
    """Candidate blocks sharing prefixes: each candidate copies a random prefix
    of an earlier one, then draws the rest."""
    c = torch.randint(0, vocab, (bs, n, k), generator=g)
    for b in range(bs):
        for i in range(1, n):
            j = int(torch.randint(0, i, (1,), generator=g))
            p = int(torch.randint(0, k + 1, (1,), generator=g))
            c[b, i, :p] = c[b, j, :p]
    return c


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a checkout of al-jshen/flashmap (the directory holding flashmap/)")
    args = ap.parse_args()
    tree = load(args.reference, "tree")
    kernels = load(args.reference, "kernels")
    g = torch.Generator().manual_seed(5)

    builds = []
    for bs, n, k, width, vocab in [(3, 6, 5, 12, 7), (2, 8, 4, 40, 3), (2, 4, 3, 64, 50), (1, 16, 8, 32, 2),
                                   (2, 5, 6, 8, 1000)]:
        cand = candidates_with_prefixes(g, bs, n, k, vocab)
        tokens, ids, stats = tree.build_tree_abi(cand, width)
        builds.append(dict(candidates=cand, width=width, tokens=tokens, ids=ids, stats=stats))

    commits = []
    for bs, W, D1 in [(3, 8, 5), (2, 12, 4), (1, 5, 6)]:
        rows, stride = bs + 2, 64
        req_to_token = torch.randint(0, 10**6, (rows, stride), generator=g, dtype=torch.int32)
        req_pool = torch.randperm(rows, generator=g)[:bs].to(torch.int64)
        prefix = torch.randint(0, stride - W - 1, (bs,), generator=g).to(torch.int64)
        window = torch.randint(1, 10**6, (bs, W), generator=g, dtype=torch.int64)
        predict = torch.randint(0, 50000, (bs * W,), generator=g, dtype=torch.int32)
        accept = torch.full((bs, D1), -1, dtype=torch.int32)
        correct = torch.zeros(bs, dtype=torch.int32)
        for b in range(bs):
            depth = int(torch.randint(0, D1, (1,), generator=g))
            nodes = [0] + sorted(torch.randperm(W - 1, generator=g)[:depth].add(1).tolist())
            accept[b, : len(nodes)] = torch.tensor(nodes, dtype=torch.int32) + b * W
            correct[b] = len(nodes) - 1
        before = req_to_token.clone()
        out = kernels.tree_commit(accept, correct, window, predict, req_pool, prefix, req_to_token)
        commits.append(dict(accept=accept, num_correct=correct, window=window, predict=predict, req_pool=req_pool,
                            prefix=prefix, req_to_token_before=before, req_to_token_after=req_to_token.clone(),
                            out_tokens=out[0], bonus=out[1], commit=out[2], new_seq_lens=out[3],
                            inject_locs=out[4]))
    path = os.path.join(HERE, "tree_cases.pt")
    torch.save(dict(builds=builds, commits=commits), path)
    print("wrote", path)


if __name__ == "__main__":
    main()
