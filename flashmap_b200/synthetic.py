"""Seeded random-init drafter weights and target embedding/lm_head.

There is no checkpoint on the measurement box, so the parity tests and the
benchmark draw every weight from a documented seeded law.  The default
``torch.nn.Linear`` init of a transformers model is not used: it leaves the
AdaLN gates near 0.0065, so every DiT branch is close to the identity and a
parity check would pass trivially.  The law used instead:

* ``nn.Linear`` weight and bias: ``U(-1/sqrt(fan_in), 1/sqrt(fan_in))``;
* AdaLN modulation bias: ``N(0, 0.5^2)`` (scale, shift and gate of order 0.5);
* RMSNorm weights: ``1 + N(0, 0.1^2)``; ``noise_gate``: 1;
* target embedding ``E``: ``N(0, 1)``; target lm_head: ``U(+-1/sqrt(H))``.

Every tensor has its own generator, seeded from ``(seed, crc32(name))``, so a
tensor's values do not depend on which other tensors are drawn or in which
order, and CPU draws are reproducible across machines for one torch version.
Names are the reference's ``state_dict`` keys (``modeling_flashmap.py:245-269``).
"""

from __future__ import annotations

import math
import zlib

import torch

from .configuration_flashmap import FlashMapConfig


def parameter_shapes(config: FlashMapConfig) -> dict[str, tuple]:
    """Name -> shape of every drafter parameter, in ``state_dict`` order."""
    d, ht, c = config.hidden_size, config.target_hidden_size, config.cond_dim
    hd = d // config.num_attention_heads
    inter = config.intermediate_size
    shapes = {
        "noise_gate": (1,),
        "fc.weight": (d, len(config.target_layer_ids) * ht),
        "hidden_norm.weight": (d,),
        "anchor_proj.weight": (d, ht),
        "anchor_proj.bias": (d,),
        "anchor_norm.weight": (d,),
        "state_norm.weight": (ht,),
        "noise_norm.weight": (ht,),
        "x_embed.weight": (d, ht),
        "x_embed.bias": (d,),
    }
    for emb in ("time_embed", "jump_embed"):
        shapes[f"{emb}.linear_1.weight"] = (c, config.time_embed_dim)
        shapes[f"{emb}.linear_1.bias"] = (c,)
        shapes[f"{emb}.linear_2.weight"] = (c, c)
        shapes[f"{emb}.linear_2.bias"] = (c,)
    for i in range(config.num_hidden_layers):
        p = f"layers.{i}"
        for norm, attn in (("self_attn_adaln", "self_attn"), ("cross_attn_adaln", "cross_attn")):
            shapes[f"{p}.{norm}.linear.weight"] = (3 * d, c)
            shapes[f"{p}.{norm}.linear.bias"] = (3 * d,)
            for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
                shapes[f"{p}.{attn}.{proj}.weight"] = (d, d)
            shapes[f"{p}.{attn}.q_norm.weight"] = (hd,)
            shapes[f"{p}.{attn}.k_norm.weight"] = (hd,)
        shapes[f"{p}.mlp_adaln.linear.weight"] = (3 * d, c)
        shapes[f"{p}.mlp_adaln.linear.bias"] = (3 * d,)
        if config.mlp_type == "swiglu":
            shapes[f"{p}.mlp.gate_up_proj.weight"] = (2 * inter, d)
            shapes[f"{p}.mlp.down_proj.weight"] = (d, inter)
        else:
            shapes[f"{p}.mlp.fc1.weight"] = (inter, d)
            shapes[f"{p}.mlp.fc1.bias"] = (inter,)
            shapes[f"{p}.mlp.fc2.weight"] = (d, inter)
            shapes[f"{p}.mlp.fc2.bias"] = (d,)
    shapes["final_adaln.linear.weight"] = (3 * d, c)
    shapes["final_adaln.linear.bias"] = (3 * d,)
    shapes["head.weight"] = (ht, d)
    shapes["head.bias"] = (ht,)
    return shapes


def _generator(seed: int, name: str, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed((int(seed) * 0x9E3779B1 + zlib.crc32(name.encode())) & 0x7FFFFFFFFFFFFFFF)
    return g


def _uniform(shape, bound, g, device):
    return (torch.rand(shape, generator=g, device=device) * 2.0 - 1.0) * bound


def draw_parameter(name: str, shape: tuple, fan_in: int, seed: int, device="cpu") -> torch.Tensor:
    """One parameter, float32, by the law in the module docstring."""
    g = _generator(seed, name, device)
    if name == "noise_gate":
        return torch.ones(shape, device=device)
    if name.endswith("norm.weight"):
        return 1.0 + 0.1 * torch.randn(shape, generator=g, device=device)
    if "adaln.linear.bias" in name:
        return 0.5 * torch.randn(shape, generator=g, device=device)
    return _uniform(shape, 1.0 / math.sqrt(fan_in), g, device)


def synthetic_state_dict(config: FlashMapConfig, seed: int = 0, dtype=torch.float32, device="cpu") -> dict:
    """Every drafter parameter (reference ``state_dict`` names) in ``dtype``."""
    shapes = parameter_shapes(config)
    out = {}
    for name, shape in shapes.items():
        if name.endswith(".bias"):
            fan_in = shapes[name[: -len("bias")] + "weight"][1]
        else:
            fan_in = shape[-1]
        out[name] = draw_parameter(name, shape, fan_in, seed, device).to(dtype)
    if config.state_vocab_size is not None:
        out["draft_ids"] = synthetic_draft_ids(config, seed).to(device)
    return out


def synthetic_draft_ids(config: FlashMapConfig, seed: int = 0) -> torch.Tensor:
    """A fixed random subset of the vocabulary, in id order (the order
    ``draft_ids`` must have, configuration_flashmap.py:48-53)."""
    g = _generator(seed, "draft_ids", "cpu")
    perm = torch.randperm(config.vocab_size, generator=g)
    return perm[: config.state_vocab_size].sort().values


def synthetic_target_head(config: FlashMapConfig, seed: int = 0, dtype=torch.bfloat16, device="cpu"):
    """``(E, W_lm)``: the target's token embedding ``N(0, 1)`` and lm_head
    ``U(+-1/sqrt(H))``, both ``(vocab_size, target_hidden_size)``."""
    shape = (config.vocab_size, config.target_hidden_size)
    emb = torch.randn(shape, generator=_generator(seed, "target.embed_tokens", device), device=device).to(dtype)
    head = _uniform(shape, 1.0 / math.sqrt(shape[1]), _generator(seed, "target.lm_head", device), device).to(dtype)
    return emb, head


__all__ = [
    "draw_parameter",
    "parameter_shapes",
    "synthetic_draft_ids",
    "synthetic_state_dict",
    "synthetic_target_head",
]
