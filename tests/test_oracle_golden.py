"""The CPU oracle reproduces the reference's own outputs bit for bit.

The golden files were produced by running the reference FlashMap code on the
CPU (``tests/golden/make_golden.py``); here the oracle replays the same
inputs and must give identical tensors, sequences and acceptance decisions.
"""

import hashlib
import os

import pytest
import torch

from flashmap_b200.configuration_flashmap import FlashMapConfig
from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
from oracle import accept
from oracle.flashmap_oracle import Oracle, OracleCache, greedy_accept_batch, spec_generate
from tests.golden.inputs import acceptance_inputs

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DTYPES = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16}


def sha(t):
    t = t.detach().contiguous()
    raw = t.view(torch.int16) if t.dtype == torch.bfloat16 else t
    return hashlib.sha256(raw.numpy().tobytes()).hexdigest()


def draft_cases():
    return torch.load(os.path.join(GOLDEN, "draft_cases.pt"))


@pytest.mark.parametrize("name", ["c1_fp32_1step", "c1_bf16_1step", "c1_fp32_2step", "c5s_bf16_1step",
                                  "c5s_bf16_2step"])
def test_oracle_draft_matches_reference(name):
    case = draft_cases()[name]
    dtype = DTYPES[case["dtype"]]
    config = FlashMapConfig(**case["config"])
    params = synthetic_state_dict(config, seed=case["seed"], dtype=torch.float32)
    oracle = Oracle(config, params, dtype)
    emb, head = synthetic_target_head(config, seed=case["seed"], dtype=dtype)
    cache = OracleCache(config, 1, case["ctx_len"] + config.block_size + 2, dtype)
    oracle.extend_context(cache, case["hidden"])
    assert sha(cache.kv[:, :, :, :, : case["ctx_len"]]) == case["kv_after_extend_sha"]
    logits = oracle.draft(case["anchor"], cache, emb, head, num_steps=case["num_steps"],
                          z=case.get("z"), noise=case.get("noise"))
    assert sha(cache.kv[:, :, :, :, case["ctx_len"]]) == case["anchor_kv_sha"]
    assert logits.dtype == case["logits"].dtype
    assert torch.equal(logits, case["logits"])


def _tiny_target():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from tests.golden.make_golden import TARGET1

    torch.manual_seed(0)
    return Qwen3ForCausalLM(Qwen3Config(**TARGET1)).eval()


@pytest.mark.parametrize("which", ["greedy", "t1"])
def test_oracle_spec_generate_matches_reference(which):
    from tests.golden.make_golden import CONFIG1

    case = torch.load(os.path.join(GOLDEN, "spec_cases.pt"))[which]
    config = FlashMapConfig(**CONFIG1)
    oracle = Oracle(config, synthetic_state_dict(config, seed=0), torch.float32)
    target = _tiny_target()
    zg = torch.Generator().manual_seed(77)
    draws = []

    def z_source(r):
        while len(draws) <= r:
            draws.append(torch.randn((1, 16, 256), generator=zg))
        return draws[r]

    seqs, lengths = spec_generate(oracle, target, case["prompt"], max_new_tokens=case["max_new_tokens"],
                                  temperature=case["temperature"], z_source=z_source, rng_seed=case["rng_seed"],
                                  softmax_mode="torch")
    assert torch.equal(seqs, case["sequences"])
    assert lengths == case["acceptance_lengths"]


def test_oracle_spec_generate_fixed_softmax_same_decisions():
    """The fixed-order softmax (what the CUDA kernels compute) leads to the
    same sampled sequence as torch's softmax on the golden T=1 run."""
    from tests.golden.make_golden import CONFIG1

    case = torch.load(os.path.join(GOLDEN, "spec_cases.pt"))["t1"]
    config = FlashMapConfig(**CONFIG1)
    oracle = Oracle(config, synthetic_state_dict(config, seed=0), torch.float32)
    zg = torch.Generator().manual_seed(77)
    draws = []

    def z_source(r):
        while len(draws) <= r:
            draws.append(torch.randn((1, 16, 256), generator=zg))
        return draws[r]

    seqs, lengths = spec_generate(oracle, _tiny_target(), case["prompt"], max_new_tokens=case["max_new_tokens"],
                                  temperature=1.0, z_source=z_source, rng_seed=case["rng_seed"],
                                  softmax_mode="fixed")
    assert torch.equal(seqs, case["sequences"])
    assert lengths == case["acceptance_lengths"]


@pytest.mark.parametrize("which", ["greedy", "t1", "t07"])
def test_acceptance_oracle_matches_reference_block(which):
    case = torch.load(os.path.join(GOLDEN, "acceptance_cases.pt"))[which]
    target, draft, q = acceptance_inputs(case["B"], case["K"], case["V"], case["seed"], case["temperature"])
    if case["temperature"] <= 0:
        acc, bonus = accept.accept_greedy(target, draft)
        acc2, bonus2 = greedy_accept_batch(draft, target)
        assert acc.tolist() == acc2.tolist() and bonus.tolist() == bonus2.tolist()
    else:
        acc, bonus = accept.accept_rejection(target, draft, q, case["temperature"], seed=case["rng_seed"], offset=0)
    assert acc.tolist() == case["accepted"]
    assert bonus.tolist() == case["bonus"]
