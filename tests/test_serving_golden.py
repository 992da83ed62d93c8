"""The serving operators' CPU restatement (oracle/serving_ops.py) and the
oracle's folds against the reference's own code: golden vectors of the
Triton kernels of flashmap/vllm/kernels.py and flashmap/sglang/kernels.py
(run by Triton's CPU interpreter) and of flashmap/vllm/fold.py, made by
tests/golden/make_serving_golden.py.

The restatement matches the kernels bit for bit on these cases (both round
every stage to bf16 at the same points), and so does greedy sampling (first
index on ties) and the folded head (one fp32 product per row).  The folded
noise is held to one bf16 rounding step (2^-8 relative): it multiplies the
same float64 eigen-decomposition in a different association order.
"""

import os

import pytest
import torch

from oracle import serving_ops as O
from oracle.flashmap_oracle import Oracle
from tests.helpers import CONFIG1, CONFIG5S

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = torch.load(os.path.join(HERE, "golden", "serving_cases.pt"), weights_only=False)
ULP = 2.0 ** -8  # one bf16 rounding step, relative


def close_bf16(got, ref, steps=1.0, floor=1e-2):
    """|got - ref| <= steps bf16 rounding steps of max(|ref|, floor), elementwise."""
    got, ref = got.float(), ref.float()
    bound = steps * ULP * torch.maximum(ref.abs(), torch.full_like(ref, floor)) * 2
    bad = (got - ref).abs() > bound
    return int(bad.sum()), float((got - ref).abs().max())


def test_vllm_rms_norm_rope():
    for c in CASES["vllm_rms_norm_rope"]:
        got = O.rms_norm_rope_vllm(c["x"], c["weight"], c["cos_sin"], c["positions"], c["eps"])
        assert torch.equal(got, c["out"])


def test_sglang_rms_norm_rope():
    for c in CASES["sglang_rms_norm_rope"]:
        got = O.rms_norm_rope_sglang(c["x"], c["weight"], c["freqs"], c["eps"])
        assert torch.equal(got, c["out"])


def _cos_sin(table, positions, blocks, T):
    cs = table[positions.long()].reshape(blocks, T, -1, 2)
    return cs[..., 0], cs[..., 1]


def test_vllm_block_self_attention():
    for c in CASES["vllm_block_self_attention"]:
        blocks, T, _, H, hd = c["qkv"].shape
        cos, sin = _cos_sin(c["cos_sin"], c["positions"], blocks, T)
        got = O.block_self_attention(c["qkv"], c["q_norm"], c["k_norm"], cos, sin, c["eps"]).reshape(blocks * T, -1)
        assert torch.equal(got, c["out"])


def test_sglang_block_self_attention():
    for c in CASES["sglang_block_self_attention"]:
        f = c["freqs"]
        got = O.block_self_attention(c["qkv"], c["q_norm"], c["k_norm"], f[..., 0], f[..., 1], c["eps"])
        assert torch.equal(got, c["out"])


def test_vllm_write_context_kv():
    for c in CASES["vllm_write_context_kv"]:
        caches = [torch.zeros(c["cache_shape"], dtype=torch.bfloat16).reshape(-1) for _ in c["caches"]]
        O.write_context_kv(c["kv"], c["positions"], c["slots"], c["k_norm"], c["cos_sin"], caches, c["strides"],
                           c["block_size"], c["eps"], heads_per_cache=c["heads_per_cache"])
        for got, ref in zip(caches, c["caches"]):
            assert torch.equal(got, ref.reshape(-1))


def test_sglang_sample_rows_greedy_first_index():
    for c in CASES["sglang_sample_rows_greedy"]:
        assert torch.equal(c["logits"].float().argmax(-1), c["out"])


@pytest.mark.parametrize("idx,cfg", [(0, CONFIG1), (1, CONFIG5S)])
def test_folds_match_reference_fold_py(idx, cfg):
    from flashmap_b200 import FlashMapConfig
    from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head

    config = FlashMapConfig(**cfg)
    sd = synthetic_state_dict(config, seed=0, dtype=torch.bfloat16)
    emb, head = synthetic_target_head(config, seed=0, dtype=torch.bfloat16)
    oracle = Oracle(config, sd, torch.bfloat16)
    fh, fn = CASES["fold_head"][idx], CASES["fold_noise"][idx]
    w, b = oracle.fold_head(head)
    assert torch.equal(w, fh["weight"]) and torch.equal(b, fh["bias"])
    weight, var, _ = oracle.fold_noise(emb)
    assert torch.allclose(var, fn["var"], rtol=1e-6, atol=0)
    bad, err = close_bf16(weight, fn["M"], floor=1e-3)
    assert bad == 0, err
