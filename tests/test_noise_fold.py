"""CPU checks of the oracle's eigen-folded noise (vllm/fold.py:44-73,
sglang/model.py:576-595), the checker of the library's ``fold_noise`` mode.

The fold's weight depends on the eigenbasis the decomposition returns (signs,
degenerate subspaces), so the checks use basis-free identities of
``weight = W_x diag(w) Q diag(sqrt lam)`` with ``E^T E = Q diag(lam) Q^T``:
``weight weight^T = W_x diag(w) E^T E diag(w) W_x^T`` and ``sum(var) = tr(E^T E)
/ H``, plus the algebra the reference states — the folded first-layer input
equals ``x_embed(state_norm(u) + gate * noise_norm(y))`` for the eigenbasis
noise ``y = (z * sqrt(lam)) Q^T``."""

import pytest
import torch

from flashmap_b200 import FlashMapConfig
from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
from oracle.flashmap_oracle import Oracle, linear, rms_norm
from tests.helpers import CONFIG1, CONFIG5S


def _setup(cfg, dtype):
    config = FlashMapConfig(**cfg)
    sd = synthetic_state_dict(config, seed=3, dtype=torch.float32)
    emb, _ = synthetic_target_head(config, seed=3, dtype=dtype)
    return config, Oracle(config, sd, dtype), emb


def _state_rows(config, oracle, emb):
    return emb if config.state_vocab_size is None else emb[oracle.p["draft_ids"]]


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
def test_fold_is_basis_free_identity(cfg):
    config, oracle, emb = _setup(cfg, torch.float32)
    (weight, var, x0), lam, basis = oracle.fold_noise(emb, return_basis=True)
    e = _state_rows(config, oracle, emb).double()
    gram = e.T @ e
    wx = oracle.p["x_embed.weight"].double() * oracle.p["noise_norm.weight"].double()[None, :]
    want = wx @ gram @ wx.T
    got = weight.double() @ weight.double().T
    assert float((got - want).abs().max() / want.abs().max()) < 1e-5
    assert abs(float(var.double().sum()) - float(torch.trace(gram)) / config.target_hidden_size) < 1e-4 * float(
        torch.trace(gram)) / config.target_hidden_size
    assert weight.shape == (config.hidden_size, config.target_hidden_size) and x0.shape == (config.hidden_size,)
    assert bool((lam >= 0).all()) and var.dtype == torch.float32


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 3e-2)])
def test_folded_input_equals_unfolded_formula(cfg, dtype, tol):
    """sglang/model.py:581-589: x_embed(u + gate * noise_norm(y)) ==
    x_embed(u) + gate * r * (z @ M) for y = (z * sqrt(lam)) Q^T."""
    config, oracle, emb = _setup(cfg, dtype)
    fold, lam, basis = oracle.fold_noise(emb, return_basis=True)
    g = torch.Generator().manual_seed(5)
    z = torch.randn(2, config.block_size, config.target_hidden_size, generator=g).to(dtype)
    gate = torch.tensor(0.75).to(dtype)
    got = oracle.folded_noise_input(z, fold, gate).double()
    p = oracle.p
    y = (z.double() * lam.sqrt()) @ basis.T
    u = rms_norm(oracle.target_constants(_state_rows(config, oracle, emb))[0].double(), p["state_norm.weight"].double(),
                 config.rms_norm_eps)
    n = rms_norm(y, p["noise_norm.weight"].double(), config.rms_norm_eps)
    want = linear(u + gate.double() * n, p["x_embed.weight"].double(), p["x_embed.bias"].double())
    assert float((got - want).abs().max() / want.abs().max()) < tol


def test_fold_noise_ignored_by_multi_step_oracle_draft():
    """A multi-step draft starts from the vocabulary-sized state, not from z: the
    folded noise does not apply (the reference folds one-jump drafts only)."""
    from oracle.flashmap_oracle import OracleCache

    config, oracle, emb = _setup(CONFIG1, torch.bfloat16)
    _, head = synthetic_target_head(config, seed=3, dtype=torch.bfloat16)
    steps = next(int(k) for k in config.jump_grids if int(k) > 1)
    cache = OracleCache(config, 1, 64, torch.bfloat16)
    g = torch.Generator().manual_seed(6)
    oracle.extend_context(cache, torch.randn(1, 20, config.target_hidden_size, generator=g).to(torch.bfloat16))
    noise = torch.randn(1, config.block_size, config.vocab_size, generator=g)
    anchor = torch.tensor([7])
    a = oracle.draft(anchor, cache, emb, head, num_steps=steps, noise=noise)
    b = oracle.draft(anchor, cache, emb, head, num_steps=steps, noise=noise, noise_fold=oracle.fold_noise(emb))
    assert torch.equal(a, b)
