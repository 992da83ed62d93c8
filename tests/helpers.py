"""Shared helpers of the GPU parity tests: model construction from the seeded
synthetic weights, and the draft-logit parity criteria of the north star:

* logits: ``max |got - ref| / max |ref| <= 2e-2`` over the finite entries
  (outside a state vocabulary both are ``-inf``);
* argmax: the fraction of block positions whose drafted token agrees with the
  reference, counting a position as agreeing when the kernel's token has the
  reference's maximal logit (bf16 logits have exact ties).
"""

from __future__ import annotations

import torch
from torch import nn

from flashmap_b200 import FlashMapConfig, FlashMapDraftModel
from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
from oracle.flashmap_oracle import Oracle

LOGITS_RTOL = 2e-2

CONFIG1 = dict(target_hidden_size=256, vocab_size=2048, target_layer_ids=[0], block_size=16, hidden_size=256,
               num_hidden_layers=2, num_attention_heads=4, intermediate_size=1024, mlp_type="gelu")
CONFIG5S = dict(target_hidden_size=320, vocab_size=3000, state_vocab_size=1024, target_layer_ids=[0, 1],
                block_size=16, hidden_size=256, num_hidden_layers=2, num_attention_heads=4, intermediate_size=384,
                mlp_type="swiglu")
# Qwen3-8B sizing of BASELINE config 2 (one target layer feeds fc: [1, 2048, 4096] conditioning)
CONFIG2 = dict(target_hidden_size=4096, vocab_size=151936, target_layer_ids=[1], block_size=16, hidden_size=2048,
               num_hidden_layers=8, num_attention_heads=16, intermediate_size=8192, mlp_type="gelu")
# Qwen3.8-27B drafter sizing of BASELINE config 5
CONFIG5 = dict(target_hidden_size=5120, vocab_size=248320, state_vocab_size=32768, target_layer_ids=[1],
               block_size=16, hidden_size=2560, num_hidden_layers=10, num_attention_heads=20, intermediate_size=6912,
               mlp_type="swiglu")


class Emb(nn.Module):
    def __init__(self, w):
        super().__init__()
        self.weight = nn.Parameter(w, requires_grad=False)

    def forward(self, ids):
        return nn.functional.embedding(ids, self.weight)


class Head(nn.Module):
    def __init__(self, w):
        super().__init__()
        self.weight = nn.Parameter(w, requires_grad=False)
        self.bias = None


def build(cfg_kwargs: dict, seed: int = 0, with_oracle: bool = True):
    """(config, CUDA model, oracle, CPU embedding, CPU lm_head) from the synthetic law."""
    config = FlashMapConfig(**cfg_kwargs)
    sd = synthetic_state_dict(config, seed=seed, dtype=torch.float32)
    model = FlashMapDraftModel(config)
    model.load_state_dict(sd, strict=True)
    model = model.to("cuda", torch.bfloat16).eval()
    emb, head = synthetic_target_head(config, seed=seed, dtype=torch.bfloat16)
    oracle = Oracle(config, sd, torch.bfloat16) if with_oracle else None
    return config, model, oracle, emb, head


def logits_rel_error(got: torch.Tensor, ref: torch.Tensor) -> float:
    got, ref = got.float().cpu(), ref.float().cpu()
    fin = torch.isfinite(ref)
    assert torch.equal(fin, torch.isfinite(got)), "-inf pattern differs"
    return float((got[fin] - ref[fin]).abs().max() / ref[fin].abs().max())


def decisive_disagreements(got_tokens: torch.Tensor, got_logits: torch.Tensor, ref_logits: torch.Tensor,
                            drift: float = 0.0) -> tuple:
    """Argmax disagreements where the reference's decision is clear.

    The margin of a position is its reference top-1 minus top-2 logit.  The
    logit error of a block is the larger of its largest absolute logit
    difference (CUDA vs reference, over all its positions and columns) and
    ``drift`` (the same measure for another faithful execution of the
    reference, e.g. PyTorch on the GPU).  Picking another token than the
    reference's top-1 moves the two logits involved by at most the error
    each, so a disagreement needs a margin of at most twice the error; a
    position whose margin exceeds that is decisive, and there the drafted
    token must be the reference's (tie-aware: its reference logit equals the
    maximum).  The tokens must be the argmax of ``got_logits`` for the bound
    to hold; the callers check that.

    Returns (disagreements at decisive positions, positions under the
    margin, the block's logit error)."""
    ref = ref_logits.float().cpu()
    got = got_logits.float().cpu()
    fin = torch.isfinite(ref)
    err = max(float((got[fin] - ref[fin]).abs().max()), float(drift))
    top2 = ref.topk(2, dim=-1).values
    margin = top2[..., 0] - top2[..., 1]
    tok = got_tokens.cpu().reshape(ref.shape[:-1])
    picked = ref.gather(-1, tok[..., None])[..., 0]
    agree = picked == top2[..., 0]
    decisive = margin > 2.0 * err
    return int((decisive & ~agree).sum()), int((~decisive).sum()), err


def argmax_agreement(got_tokens: torch.Tensor, ref_logits: torch.Tensor) -> tuple:
    """(tie-aware agreement, strict agreement) of drafted tokens vs reference logits."""
    ref = ref_logits.float().cpu()
    tok = got_tokens.cpu().reshape(ref.shape[:-1])
    ref_max = ref.max(-1).values
    picked = ref.gather(-1, tok[..., None])[..., 0]
    tie_aware = (picked == ref_max).float().mean().item()
    strict = (tok == ref.argmax(-1)).float().mean().item()
    return tie_aware, strict
