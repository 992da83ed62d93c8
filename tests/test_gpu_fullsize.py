"""Batched drafting at the full BASELINE sizes against the per-sequence CPU
oracle (modeling_flashmap.py:422-479): config 3 (the Qwen3-8B-sized drafter,
12 of the 64 ragged sequences, contexts from U[512, 4096], one and two jumps:
192 token rows, so the GEMMs run 256-wide CTA-pair tiles with a ragged tail)
and config 5 (the Qwen3.8-27B-sized drafter with its 32768-of-248320 state
vocabulary, 4 of the 512 requests, contexts from U[1024, 8192], one jump),
each drafted in one batched plan and compared sequence by sequence with the
oracle drafting it alone at batch 1.

Tolerances are those of every draft parity test: logits within 2e-2 of the
reference's largest magnitude, and no argmax disagreement at a position whose
reference top-1/top-2 margin exceeds twice the block's largest logit error.

The weights and target rows are drawn on the device (the synthetic law at
these sizes takes minutes on the host) and copied to the host for the oracle.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import FlashMapCache, FlashMapConfig, FlashMapDraftModel  # noqa: E402
from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head  # noqa: E402
from oracle.flashmap_oracle import Oracle, OracleCache  # noqa: E402
from tests.helpers import (CONFIG2, CONFIG5, LOGITS_RTOL, Emb, Head, decisive_disagreements,  # noqa: E402
                           logits_rel_error)

DEV = "cuda"


def _build_on_device(cfg, seed):
    config = FlashMapConfig(**cfg)
    sd = synthetic_state_dict(config, seed=seed, dtype=torch.bfloat16, device=DEV)
    with torch.device(DEV):
        model = FlashMapDraftModel(config).to(torch.bfloat16).eval()
    model.load_state_dict(sd, strict=True)
    emb, head = synthetic_target_head(config, seed=seed, dtype=torch.bfloat16, device=DEV)
    oracle = Oracle(config, {k: v.cpu() for k, v in sd.items()}, torch.bfloat16)
    return config, model, oracle, emb, head


def _batched_vs_oracle(cfg, lengths, steps_list, seed):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    config, model, oracle, emb, head = _build_on_device(cfg, seed)
    E, W = Emb(emb), Head(head)
    emb_c, head_c = emb.cpu(), head.cpu()
    K, B = config.block_size, len(lengths)
    width = len(config.target_layer_ids) * config.target_hidden_size
    g = torch.Generator().manual_seed(seed + 1)
    ctx = [torch.randn(n, width, generator=g).to(torch.bfloat16) for n in lengths]
    cache = FlashMapCache(config, B, max(lengths) + K + 2, device=DEV, dtype=torch.bfloat16)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lengths), 0)), dtype=torch.int32)
    model.extend_context_varlen(cache, torch.cat(ctx).to(DEV), cu.to(DEV), E, W)
    assert cache.lengths.cpu().tolist() == list(lengths)
    caches = []
    for b, n in enumerate(lengths):
        oc = OracleCache(config, 1, n + K + 2, torch.bfloat16)
        oracle.extend_context(oc, ctx[b][None])
        caches.append(oc)
    report = []
    for steps in steps_list:
        anchors = torch.randint(0, config.vocab_size, (B,), generator=g)
        if steps == 1:  # a one-jump draft starts from z (B, K, Ht), a multi-jump one from noise (B, K, S)
            draw = dict(z=torch.randn(B, K, config.target_hidden_size, generator=g).to(torch.bfloat16))
        else:
            draw = dict(noise=torch.randn(B, K, config.state_vocab_size or config.vocab_size, generator=g))
        got, tok = model.draft(anchors.to(DEV), cache, E, W, num_steps=steps, return_tokens=True,
                               **{k: v.to(DEV) for k, v in draw.items()})
        torch.cuda.synchronize()
        # the fused argmax is the argmax of the returned logits
        assert torch.equal(tok.cpu(), got.float().argmax(-1).cpu())
        for b in range(B):
            ref = oracle.draft(anchors[b:b + 1], caches[b], emb_c, head_c, num_steps=steps,
                               **{k: v[b:b + 1] for k, v in draw.items()})
            err = logits_rel_error(got[b:b + 1], ref)
            bad, under, _ = decisive_disagreements(tok[b:b + 1], got[b:b + 1], ref)
            report.append((steps, b, lengths[b], err, bad, under))
            assert err <= LOGITS_RTOL, report[-1]
            assert bad == 0, report[-1]
    plan = model._plan(model._pack(cache.kv.device, E, W), cache, B, steps_list[-1])
    assert int(plan.err.item()) == 0
    return report


def test_config3_twelve_ragged_sequences_one_and_two_jumps():
    g = torch.Generator().manual_seed(5)
    lengths = torch.randint(512, 4097, (64,), generator=g)[:12].tolist()
    _batched_vs_oracle(CONFIG2, lengths, (1, 2), seed=21)


def test_config5_four_requests_state_vocabulary():
    g = torch.Generator().manual_seed(5)
    lengths = torch.randint(1024, 8193, (512,), generator=g)[:4].tolist()
    _batched_vs_oracle(CONFIG5, lengths, (1,), seed=31)
