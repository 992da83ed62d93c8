"""CPU restatement of the banked multi-jump draft (flashmap/sglang/jump_bank.py),
test infrastructure only: the checker of the library's bank kernels and of the
sglang plugin's banked drafts.  Pinned by tests/golden/jump_bank_cases.pt (made
by tests/golden/make_jump_bank_golden.py from the reference itself).

The state of jump n >= 1, ``x_n = alpha_n z + sum_m beta_nm delta_m``, is
embedded without vocabulary-sized products: everything over the whole
vocabulary depends on the noise z alone and is precomputed per bank row
(``z @ E``; per later jump ``softmax(a_n z) @ E`` and ``logsumexp(a_n z)``), and a
draft reads the embedding rows of the earlier predictions' top-k support,
where the noise values are re-drawn from a hash of (slot seed, token).
"""

from __future__ import annotations

import math

import torch

MASK32 = 0xFFFFFFFF
_MIX = 0x45D9F3B            # the multiply of each hash round (jump_bank.py:52-59)
_ID_SALT = 0x9E3779B9       # xor-ed into token ids before hashing (:67)
_SECOND_SALT = 0x68E31DA4   # xor-ed into the first hash for the second uniform (:69)


def hash32(x: torch.Tensor) -> torch.Tensor:
    """Two multiply-xorshift rounds on int64 values in [0, 2^32) (jump_bank.py:52-59);
    every product stays below 2^59, so the int64 arithmetic is exact."""
    for _ in range(2):
        x = x ^ (x >> 16)
        x = (x * _MIX) & MASK32
    return x ^ (x >> 16)


def token_normals(seeds: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
    """A standard normal per (slot seed, token id) (jump_bank.py:62-73): two
    hashed uniforms through Box-Muller in float32; ``seeds (R,)``, ``ids (R, L)``."""
    h_id = hash32((ids & MASK32) ^ _ID_SALT)
    h1 = hash32(h_id ^ (seeds[:, None] & MASK32))
    h2 = hash32(h1 ^ _SECOND_SALT)
    u1 = (h1.float() + 1.0) / 4294967297.0
    u2 = h2.float() / 4294967296.0
    radius = torch.sqrt(-2.0 * torch.log(u1))
    return radius * torch.cos(2.0 * math.pi * u2)


def jump_coefficients(grid) -> list:
    """Per jump n: (alpha_n, [beta_n1 .. beta_nn]), the coefficients of z and of
    each earlier prediction in the state x_n, from the update
    x <- ((1 - t) x + (t - s) delta) / (1 - s) (jump_bank.py:76-86)."""
    out = [(1.0, [])]
    alpha, betas = 1.0, []
    for start, end in zip(grid[:-2], grid[1:-1]):
        start, end = float(start), float(end)
        keep = (1.0 - end) / (1.0 - start)
        alpha *= keep
        betas = [b * keep for b in betas] + [(end - start) / (1.0 - start)]
        out.append((alpha, list(betas)))
    return out


def bank_constants(grid):
    """(coefficients, evidence e_n, slopes a_n) of the jumps after the first:
    e_n = t_n / (1 - t_n)^2 at the jump's start time, a_n = e_n alpha_n
    (jump_bank.py:117-123)."""
    grid = [float(t) for t in grid]
    coefficients = jump_coefficients(grid)
    starts = grid[1:len(grid) - 1]
    evidence = [t / (1.0 - t) ** 2 for t in starts]
    slopes = [e * coefficients[n + 1][0] for n, e in enumerate(evidence)]
    return coefficients, evidence, slopes


def build_bank(embedding: torch.Tensor, z: torch.Tensor, grid):
    """The bank for draws ``z (M, V)`` fp32 (temperature applied):
    ``noise_embed = z @ E`` in the embedding's dtype, and per later jump
    ``mean_embed = softmax(a_n z) @ E`` and ``log_mass = logsumexp(a_n z)``
    (jump_bank.py:124-150)."""
    _, _, slopes = bank_constants(grid)
    noise_embed = z.to(embedding.dtype) @ embedding
    mean_embed, log_mass = [], []
    for slope in slopes:
        logits = slope * z
        log_mass.append(logits.logsumexp(-1))
        mean_embed.append(logits.softmax(dim=-1).to(embedding.dtype) @ embedding)
    hidden = embedding.shape[1]
    if not slopes:
        return noise_embed, embedding.new_empty(0, z.shape[0], hidden), torch.empty(0, z.shape[0])
    return noise_embed, torch.stack(mean_embed), torch.stack(log_mass)


def top_predictions(logits: torch.Tensor, topk: int, rows=None):
    """A jump's prediction cut to its top-k (jump_bank.py:89-92): the ids
    (mapped through ``rows`` when the logits' indices are not state rows) and
    their probabilities under the full softmax."""
    probs, index = logits.float().softmax(dim=-1).topk(topk, dim=-1)
    return (index if rows is None else rows[index]), probs


def first_rows(noise_embed, rows):
    """Jump 0's state rows: the bank rows' noise embeddings (jump_bank.py:164-169;
    the posterior term is the uniform one, embedded once)."""
    return noise_embed[rows]


def jump_rows(bank, grid, n: int, rows, seeds, supports, embedding, temperature: float):
    """The two bf16 rows jump ``n >= 1`` embeds (jump_bank.py:171-205), before
    the norms: the posterior ``(mean_embed + sum_v r_v E_v) / (1 + sum_v r_v / Z)``
    and the noise term ``alpha z @ E + sum_m beta_m delta_m @ E``, each rounded to
    the embedding's dtype.  ``supports``: per earlier prediction (ids (R, k),
    probs (R, k))."""
    noise_embed, mean_embed, log_mass = bank
    coefficients, evidence, slopes = bank_constants(grid)
    alpha, betas = coefficients[n]
    ids = torch.cat([sid for sid, _ in supports], dim=1)
    linear = torch.cat([beta * probs.float() for beta, (_, probs) in zip(betas, supports)], dim=1)
    # c_v: the summed weight of every prediction on token v (a repeated token counts each time)
    same = ids[:, :, None] == ids[:, None, :]
    shift = evidence[n - 1] * (same.float() @ linear[:, :, None])[..., 0]
    # r_v once per distinct token: its first occurrence in the support
    width = ids.shape[1]
    before = torch.ones(width, width, dtype=torch.bool).tril(-1)
    first = ~(same & before).any(dim=-1)
    z = temperature * token_normals(seeds, ids)
    weight = torch.exp(slopes[n - 1] * z - log_mass[n - 1][rows][:, None]) * torch.expm1(shift) * first
    operands = torch.stack([weight, linear], dim=1).to(embedding.dtype)  # (R, 2, L)
    sums = torch.bmm(operands, embedding[ids]).float()
    posterior = (mean_embed[n - 1][rows].float() + sums[:, 0]) / (1.0 + weight.sum(dim=1, keepdim=True))
    noise = alpha * noise_embed[rows].float() + sums[:, 1]
    return posterior.to(embedding.dtype), noise.to(embedding.dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference RMSNorm: the scale weight / rms(x) rounded to x's dtype,
    then times x (modeling_flashmap.py:69-80)."""
    rms = torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + eps)
    return x * (weight.float() * rms).to(x.dtype)


def embed_rows(posterior, noise, w_state, w_noise, eps: float, gate: torch.Tensor):
    """``state_norm(posterior) + gate * noise_norm(noise)`` with the reference's
    bf16 rounding points (jump_bank.py:166-169, 200-205)."""
    return rms_norm(posterior, w_state, eps) + gate * rms_norm(noise, w_noise, eps)
