"""CPU restatement of tree drafting's index work, test infrastructure only:
the trie that merges a request's candidate blocks into a verify tree in
EAGLE's encoding (flashmap/sglang/tree.py:9-78) and the commit of the
accepted tree path (flashmap/sglang/kernels.py:363-454).  Pinned by
tests/golden/tree_cases.pt (made by tests/golden/make_tree_golden.py from the
reference itself).  Written as plain loops over one request at a time.
"""

from __future__ import annotations

import torch


def build_tree(candidates: torch.Tensor, width: int):
    """``(tokens, ids, stats)`` of the verify trees of ``candidates (bs, N, K)``.

    A trie node is a distinct prefix (candidate i, depth d) — represented by
    the lowest candidate holding that prefix; its vote is how many candidates
    hold it.  The ``width - 1`` nodes with the most votes are kept (ties: the
    shallower, then the lower candidate), listed by depth then candidate; a
    node's id is ``parent * width + index`` (root 0, indices from 1).  With
    fewer nodes, the rest are copies of the first node (parent the root).
    ``stats``: the trie's node count and its number of distinct candidates."""
    bs, n, k = candidates.shape
    m = width - 1
    tokens = torch.zeros(bs, m, dtype=candidates.dtype)
    ids = torch.zeros(bs, m, dtype=torch.int64)
    stats = torch.zeros(bs, 2, dtype=torch.int64)
    for b in range(bs):
        c = candidates[b].tolist()
        # common prefix length of every pair of candidates
        common = [[0] * n for _ in range(n)]
        for i in range(n):
            for j in range(n):
                length = 0
                while length < k and c[i][length] == c[j][length]:
                    length += 1
                common[i][j] = length
        first = [[min(j for j in range(n) if common[i][j] > d) for d in range(k)] for i in range(n)]
        nodes = []  # (key, i, d) of every trie node
        for i in range(n):
            for d in range(k):
                if first[i][d] == i:
                    votes = sum(1 for j in range(n) if common[i][j] > d)
                    nodes.append((votes * n * k + (k - 1 - d) * n + (n - 1 - i), i, d))
        kept = sorted(nodes, reverse=True)[:m]
        kept.sort(key=lambda node: node[2] * n + node[1])  # depth, then candidate
        index = {(i, d): pos + 1 for pos, (_, i, d) in enumerate(kept)}
        for pos, (_, i, d) in enumerate(kept):
            parent = 0 if d == 0 else index[(first[i][d - 1], d - 1)]
            tokens[b, pos] = c[i][d]
            ids[b, pos] = parent * width + pos + 1
        for pos in range(len(kept), m):
            tokens[b, pos] = tokens[b, 0]
            ids[b, pos] = pos + 1
        stats[b, 0] = len(nodes)
        stats[b, 1] = sum(1 for (_, i, d) in nodes if d == k - 1)
    return tokens, ids, stats


def tree_commit(accept, num_correct, window, predict, req_pool, prefix, req_to_token):
    """Commit each request's accepted tree path (kernels.py:363-454): the path's
    KV slots move to the front of its verify window in ``req_to_token``
    (updated in place; the other nodes follow in index order), and the path's
    tokens (the target's token after each node), the bonus token, the commit
    length, the new sequence length and the context-injection slots (the
    path's own, 0 elsewhere) are returned."""
    bs, d1 = accept.shape
    w = window.shape[1]
    out_tokens = torch.zeros(bs, d1, dtype=torch.int64)
    bonus = torch.zeros(bs, dtype=torch.int64)
    commit = torch.zeros(bs, dtype=torch.int32)
    new_seq_lens = torch.zeros(bs, dtype=prefix.dtype)
    inject = torch.zeros(bs * w, dtype=torch.int64)
    for b in range(bs):
        n = int(num_correct[b])
        path = [int(accept[b, j]) - b * w for j in range(min(n + 1, d1))]
        path = [node for node in path if node >= 0]
        row, base = int(req_pool[b]), int(prefix[b])
        for j, node in enumerate(path):
            req_to_token[row, base + j] = int(window[b, node])
            out_tokens[b, j] = int(predict[b * w + node])
        on_path = set(path)
        rest = [i for i in range(w) if i not in on_path]
        for r, i in enumerate(rest):
            req_to_token[row, base + n + 1 + r] = int(window[b, i])
        bonus[b] = out_tokens[b, n] if n < d1 else 0
        commit[b] = n + 1
        new_seq_lens[b] = base + n + 1
        for i in range(w):
            inject[b * w + i] = int(window[b, i]) if i in on_path else 0
    return out_tokens, bonus, commit, new_seq_lens, inject
