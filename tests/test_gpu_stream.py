"""The streamed single-launch draft pass (launch_mode "stream") on the GPU.

Its drafts are held to the CPU oracle with the tolerances of the kernel
sequence (logits within 2e-2 of the reference's scale, no argmax
disagreement at a decisive position) and to the kernel sequence itself:
both compute the same GEMM partial sums, epilogues and attention, and differ
only in the summation order of the LayerNorm / RMSNorm statistics (per
128-feature tile, then over tiles), so their logits agree far more closely
than either agrees with the CPU.  Drafts repeat bit for bit (the pass's
counters return to zero after every launch), and a CUDA-graph DraftSession
replays the pass.
"""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import DraftSession, FlashMapCache  # noqa: E402
from oracle.flashmap_oracle import OracleCache  # noqa: E402
from tests.helpers import (CONFIG1, CONFIG2, CONFIG5S, LOGITS_RTOL, Emb, Head, build,  # noqa: E402
                           decisive_disagreements, logits_rel_error)

DEV = "cuda"
# head_dim 128 at test size (the Qwen3-8B map's head size)
CONFIG_HD128 = dict(target_hidden_size=256, vocab_size=2048, target_layer_ids=[0], block_size=16, hidden_size=256,
                    num_hidden_layers=2, num_attention_heads=2, intermediate_size=1024, mlp_type="gelu")


def _context(config, ctx_len, seed):
    g = torch.Generator().manual_seed(1000 + seed)
    hidden = torch.randn(1, ctx_len, len(config.target_layer_ids) * config.target_hidden_size, generator=g)
    return hidden.to(torch.bfloat16)


def _draft(model, mode, anchor, cache, E, W, z):
    model.launch_mode = mode
    try:
        return model.draft(anchor, cache, E, W, num_steps=1, z=z, return_tokens=True)
    finally:
        model.launch_mode = "auto"


@pytest.mark.parametrize("cfg,ctx_len", [(CONFIG1, 40), (CONFIG1, 300), (CONFIG_HD128, 129), (CONFIG5S, 29),
                                         (CONFIG5S, 64)])
def test_stream_draft_matches_oracle_and_kernel_sequence(cfg, ctx_len):
    config, model, oracle, emb, head = build(cfg, seed=3)
    E, W = Emb(emb.to(DEV)), Head(head.to(DEV))
    K = config.block_size
    hidden = _context(config, ctx_len, 3)
    cache = FlashMapCache(config, 1, ctx_len + K + 2, device=DEV, dtype=torch.bfloat16)
    model.extend_context(cache, hidden.to(DEV), E, W)
    ocache = OracleCache(config, 1, ctx_len + K + 2, torch.bfloat16)
    oracle.extend_context(ocache, hidden)
    for seed in range(4):
        g = torch.Generator().manual_seed(seed)
        anchor = torch.randint(0, config.vocab_size, (1,), generator=g)
        z = torch.randn(1, K, config.target_hidden_size, generator=g).to(torch.bfloat16)
        got, tok = _draft(model, "stream", anchor.to(DEV), cache, E, W, z.to(DEV))
        seq, _ = _draft(model, "kernels", anchor.to(DEV), cache, E, W, z.to(DEV))
        torch.cuda.synchronize()
        ref = oracle.draft(anchor, ocache, emb, head, num_steps=1, z=z)
        assert torch.equal(tok.cpu(), got.float().argmax(-1).cpu()), "fused argmax is not the logits' argmax"
        assert logits_rel_error(got, ref) <= LOGITS_RTOL
        assert decisive_disagreements(tok, got, ref)[0] == 0
        # against the kernel sequence: the same arithmetic up to the normalisation statistics' order
        assert logits_rel_error(got, seq) <= 5e-3, f"seed {seed}: stream vs kernel sequence"
    plan = model._plan(model._pack(cache.kv.device, E, W), cache, 1, 1)
    assert int(plan.err.item()) == 0


def test_stream_draft_is_deterministic_and_counts_one_launch():
    config, model, _, emb, head = build(CONFIG_HD128, seed=5, with_oracle=False)
    E, W = Emb(emb.to(DEV)), Head(head.to(DEV))
    K = config.block_size
    cache = FlashMapCache(config, 1, 100, device=DEV, dtype=torch.bfloat16)
    model.extend_context(cache, _context(config, 77, 5).to(DEV), E, W)
    z = torch.randn(1, K, config.target_hidden_size, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    outs = [_draft(model, "stream", torch.tensor([17], device=DEV), cache, E, W, z.to(DEV))[0] for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    model.launch_mode = "stream"
    try:
        plan = model._plan(model._pack(cache.kv.device, E, W), cache, 1, 1)
    finally:
        model.launch_mode = "auto"
    assert plan.last_launches() == 1
    assert int(plan.err.item()) == 0


def test_stream_session_replays_the_pass():
    """DraftSession over the streamed pass: CUDA-graph replays with fresh
    Philox noise per replay give the kernel sequence's logits for the same
    noise (same seed, same per-draft counter)."""
    config, model, _, emb, head = build(CONFIG_HD128, seed=6, with_oracle=False)
    E, W = Emb(emb.to(DEV)), Head(head.to(DEV))
    cache = FlashMapCache(config, 1, 200, device=DEV, dtype=torch.bfloat16)
    model.extend_context(cache, _context(config, 150, 6).to(DEV), E, W)
    logits = {}
    for mode in ("kernels", "stream"):
        model.launch_mode = mode
        try:
            sess = DraftSession(model, cache, E, W, with_logits=True, seed=99)
        finally:
            model.launch_mode = "auto"
        rows = []
        for anchor in (3, 1000, 2047):
            sess.draft([anchor])
            rows.append(sess.logits.clone())
        logits[mode] = torch.stack(rows)
    torch.cuda.synchronize()
    assert logits_rel_error(logits["stream"], logits["kernels"]) <= 5e-3


@pytest.mark.skipif(os.environ.get("FM_SKIP_CONFIG2") == "1", reason="config-2 parity skipped by request")
def test_stream_config2_matches_kernel_sequence_and_oracle():
    """BASELINE config 2 (Qwen3-8B sizing, 2048-token context): a few
    streamed drafts against the kernel sequence and the CPU reference."""
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    config, model, oracle, emb, head = build(CONFIG2, seed=0)
    E, W = Emb(emb.to(DEV)), Head(head.to(DEV))
    K, ctx_len = config.block_size, 2048
    hidden = torch.randn(1, ctx_len, config.target_hidden_size, generator=torch.Generator().manual_seed(2))
    hidden = hidden.to(torch.bfloat16)
    cache = FlashMapCache(config, 1, ctx_len + K + 2, device=DEV, dtype=torch.bfloat16)
    model.extend_context(cache, hidden.to(DEV), E, W)
    ocache = OracleCache(config, 1, ctx_len + K + 2, torch.bfloat16)
    oracle.extend_context(ocache, hidden)
    for seed in range(3):
        g = torch.Generator().manual_seed(seed)
        anchor = torch.randint(0, config.vocab_size, (1,), generator=g)
        z = torch.randn(1, K, config.target_hidden_size, generator=g).to(torch.bfloat16)
        got, tok = _draft(model, "stream", anchor.to(DEV), cache, E, W, z.to(DEV))
        seq, _ = _draft(model, "kernels", anchor.to(DEV), cache, E, W, z.to(DEV))
        ref = oracle.draft(anchor, ocache, emb, head, num_steps=1, z=z)
        assert logits_rel_error(got, ref) <= LOGITS_RTOL
        assert decisive_disagreements(tok, got, ref)[0] == 0
        assert logits_rel_error(got, seq) <= 1e-2
