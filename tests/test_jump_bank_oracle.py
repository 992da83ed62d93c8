"""The banked multi-jump oracle (oracle/jump_bank_oracle.py) against golden
vectors of the reference's flashmap/sglang/jump_bank.py run on the CPU
(tests/golden/make_jump_bank_golden.py): bit for bit."""

import os

import pytest
import torch

from oracle import jump_bank_oracle as JB

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "jump_bank_cases.pt")


@pytest.fixture(scope="module")
def case():
    return torch.load(GOLDEN)


def test_token_normals(case):
    assert torch.equal(JB.token_normals(case["seeds"], case["ids"]), case["normals"])


def test_jump_coefficients(case):
    for grid, want in case["coefficients"].items():
        got = JB.jump_coefficients(eval(grid))  # noqa: S307 - a list literal written by the generator
        assert len(got) == len(want)
        for (ga, gb), (wa, wb) in zip(got, want):
            assert ga == wa and gb == wb


def test_bank(case):
    noise_embed, mean_embed, log_mass = JB.build_bank(case["embedding"], case["z"], case["grid"])
    assert torch.equal(noise_embed, case["noise_embed"])
    assert torch.equal(mean_embed, case["mean_embed"])
    assert torch.equal(log_mass, case["log_mass"])
    _, evidence, slopes = JB.bank_constants(case["grid"])
    assert evidence == case["evidence"] and slopes == case["slopes"]


def test_top_predictions(case):
    ids, probs = JB.top_predictions(case["topk_logits"], case["k"], case["topk_rows"])
    assert torch.equal(ids, case["topk_ids"]) and torch.equal(probs, case["topk_probs"])


def _gate(case, n):
    grid = case["grid"]
    return (torch.tensor(case["noise_gate"]).to(torch.bfloat16).float() * (grid[n + 1] - grid[n])).to(torch.bfloat16)


@pytest.mark.parametrize("n", [0, 1, 2])
def test_jump_inputs(case, n):
    bank = (case["noise_embed"], case["mean_embed"], case["log_mass"])
    E, rows = case["embedding"], case["rows"]
    if n == 0:
        noise = JB.first_rows(case["noise_embed"], rows)
        got = case["uniform"] + _gate(case, 0) * JB.rms_norm(noise, case["w_noise"], case["eps"])
        want = case["first"]
    else:
        post, noise = JB.jump_rows(bank, case["grid"], n, rows, case["slot_seeds"], case["supports"][:n], E,
                                   case["temperature"])
        got = JB.embed_rows(post, noise, case["w_state"], case["w_noise"], case["eps"], _gate(case, n))
        want = case[f"jump{n}"]
    assert torch.equal(got, want)
