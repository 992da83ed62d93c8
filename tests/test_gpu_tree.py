"""Tree drafting on the GPU: the trie kernel (fm_tree_build) and the path
commit (fm_tree_commit) against golden vectors of the reference's
build_tree_abi and tree_commit (tests/golden/tree_cases.pt, exact), and the
sglang plugin's tree mode: N candidate blocks per request in one pass, the
tree buffers equal to the oracle's trie of the candidates' greedy tokens,
those tokens agreeing with the oracle's drafts of the same noise (tie-aware,
no disagreement at a decisive position: one whose reference top-1/top-2
gap exceeds twice the first candidate's largest logit difference), the first candidate's logits within 2e-2."""

import os
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import serving_ops as S  # noqa: E402
from flashmap_b200 import sglang_model as SG  # noqa: E402
from flashmap_b200.tree import build_tree_abi  # noqa: E402
from oracle import tree_oracle as TO  # noqa: E402
from oracle.flashmap_oracle import OracleCache  # noqa: E402
from tests.helpers import CONFIG1, CONFIG5S, LOGITS_RTOL, Emb, Head, build, decisive_disagreements  # noqa: E402

DEV = "cuda"
CASES = torch.load(os.path.join(os.path.dirname(__file__), "golden", "tree_cases.pt"))


@pytest.mark.parametrize("i", range(len(CASES["builds"])))
def test_tree_build_matches_reference(i):
    c = CASES["builds"][i]
    tokens, ids, stats = build_tree_abi(c["candidates"].to(DEV), c["width"])
    assert torch.equal(tokens.cpu(), c["tokens"]) and torch.equal(ids.cpu(), c["ids"])
    assert torch.equal(stats.cpu(), c["stats"])


@pytest.mark.parametrize("i", range(len(CASES["commits"])))
def test_tree_commit_matches_reference(i):
    c = CASES["commits"][i]
    table = c["req_to_token_before"].to(DEV)
    out = S.tree_commit(c["accept"].to(DEV), c["num_correct"].to(DEV), c["window"].to(DEV), c["predict"].to(DEV),
                        c["req_pool"].to(DEV), c["prefix"].to(DEV), table)
    assert torch.equal(table.cpu(), c["req_to_token_after"])
    for got, name in zip(out, ("out_tokens", "bonus", "commit", "new_seq_lens", "inject_locs")):
        assert torch.equal(got.cpu(), c[name]), name


def test_tree_build_random_against_oracle():
    g = torch.Generator().manual_seed(3)
    for bs, n, k, width, vocab in [(4, 8, 16, 17, 3), (2, 32, 16, 17, 2), (3, 64, 16, 17, 5), (2, 16, 8, 200, 4)]:
        cand = torch.randint(0, vocab, (bs, n, k), generator=g)
        cand[:, 1:, :2] = cand[:, :1, :2]  # a shared prefix
        got = build_tree_abi(cand.to(DEV), width)
        want = TO.build_tree(cand, width)
        for a, b in zip(got, want):
            assert torch.equal(a.cpu(), b)


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
def test_sglang_tree_mode(cfg):
    config, model, oracle, emb, head = build(cfg, seed=31)
    K, H, hd, L = config.block_size, config.num_attention_heads, config.hidden_size // config.num_attention_heads, \
        config.num_hidden_layers
    sm = SG.FlashMapDraftModel(config).to(DEV, torch.bfloat16)
    sm.load_weights(model.state_dict().items())
    sm.tree_max_n, sm.tree_mode = 3, True  # FLASHMAP_TREE_N, read at construction
    sm.attach_shared_modules(embed_tokens=Emb(emb.to(DEV)), lm_head=Head(head.to(DEV)))
    core = sm._core
    rows_pool = 1024
    kb = [torch.zeros(rows_pool, H, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    vb = [torch.zeros(rows_pool, H, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    pool = SimpleNamespace(get_key_buffer=lambda i: kb[i], get_value_buffer=lambda i: vb[i])
    lengths = [29, 75]
    bsz, n_cand = len(lengths), sm.tree_n_for(len(lengths))
    assert n_cand == 3
    g = torch.Generator().manual_seed(32)
    req_to_token = torch.randperm(rows_pool, generator=g)[: 2 * 200].view(2, 200).int().to(DEV)
    sm.token_to_kv_pool = lambda: pool
    sm.req_to_token = lambda: req_to_token
    width = len(config.target_layer_ids) * config.target_hidden_size
    hiddens = [torch.randn(n, width, generator=g).to(torch.bfloat16) for n in lengths]
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        sm.write_target_hidden_kv(target_hidden=h.to(DEV), pool=pool, positions=torch.arange(n, device=DEV),
                                  cache_loc=req_to_token[r, :n].long())
    z = torch.randn(bsz * n_cand * K, config.target_hidden_size, generator=g).to(torch.bfloat16)
    core.noise = lambda *args, **kwargs: z.to(DEV)
    recorded = []
    top = core.top_predictions

    def record(*args, **kwargs):
        out = top(*args, **kwargs)
        recorded.append(out[0].clone())
        return out

    core.top_predictions = record
    anchors = torch.randint(0, config.vocab_size, (bsz,), generator=g)
    input_ids = torch.stack([torch.cat([a[None], torch.zeros(K - 1, dtype=torch.long)]) for a in anchors]).view(-1)
    positions = torch.cat([n + torch.arange(K) for n in lengths]).to(DEV)
    out_cache_loc = torch.cat([req_to_token[r, n:n + K].long() for r, n in enumerate(lengths)])
    batch = SimpleNamespace(batch_size=bsz, seq_lens=torch.tensor(lengths, device=DEV), out_cache_loc=out_cache_loc,
                            req_pool_indices=torch.arange(bsz, device=DEV))
    out = sm.forward(input_ids.to(DEV), positions, batch)
    logits, _ = sm.compute_base_logits(out.hidden_states)
    node_tokens, node_ids, parents, stats = (t.cpu() for t in sm.tree_outputs(bsz))
    torch.cuda.synchronize()
    assert len(recorded) == 1
    cand = recorded[0].cpu().view(bsz, n_cand, K)
    want = TO.build_tree(cand, sm.tree_width)
    assert torch.equal(node_tokens, want[0]) and torch.equal(node_ids, want[1]) and torch.equal(stats, want[2])
    assert torch.equal(parents[:, 1:node_ids.shape[1] + 1], node_ids)
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        oc = OracleCache(config, 1, n + K + 2, torch.bfloat16)
        oracle.extend_context(oc, h[None])
        refs = []
        for c in range(n_cand):
            zc = z[(r * n_cand + c) * K:(r * n_cand + c + 1) * K]
            refs.append(oracle.draft(torch.tensor([int(anchors[r])]), oc, emb, head, num_steps=1, z=zc[None],
                                     folded=True)[0])
        # the first candidate's logits give the block's logit error; it is the
        # margin of every candidate's argmax (same kernels, same request)
        cols = refs[0] if config.state_vocab_size is None else refs[0][:, oracle.p["draft_ids"].long()]
        got = logits[r * K:(r + 1) * K].float().cpu()
        rel = float((got - cols.float()).abs().max() / cols.float().abs().max())
        assert rel <= LOGITS_RTOL, f"request {r}: first-candidate logits relative error {rel}"
        thr = float((got - cols.float()).abs().max())
        for c, ref in enumerate(refs):
            bad = decisive_disagreements(cand[r, c], ref, ref, drift=thr)[0]
            assert bad == 0, f"request {r} candidate {c}: {bad} argmax disagreements at decisive positions"
