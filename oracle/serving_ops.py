"""CPU restatement of the serving plugins' operators (test infrastructure only).

The reference implements these as Triton kernels (flashmap/vllm/kernels.py,
flashmap/sglang/kernels.py) and FlashAttention calls (flashmap/vllm/model.py:93,
flashmap/sglang/model.py:127-175); none of them runs on a CPU.  This module
states what each computes, in torch fp32 on the CPU, from the same building
blocks as the HF-path oracle (``flashmap_oracle.rms_norm`` / ``apply_rope``,
which are pinned to the reference by golden vectors); ``tests/`` compares the
CUDA operators with it.  Parity for the serving paths is pinned only through
those shared primitives: the reference ships no tests or fixtures for them.
"""

from __future__ import annotations

import torch

from .flashmap_oracle import apply_rope, rms_norm

FP8 = torch.float8_e4m3fn


def _pairs(table: torch.Tensor):
    """(cos, sin) of a ``(..., hd/2, [cos, sin])`` table."""
    return table[..., 0], table[..., 1]


def norm_rope(x: torch.Tensor, weight: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, eps: float,
              fused: bool = False) -> torch.Tensor:
    """RMSNorm then interleaved RoPE of bf16 rows ``x (..., hd)`` with per-row
    ``cos, sin (..., hd/2)``; returns the fp32 rotation (before rounding).
    DiT rounding (vllm/kernels.py:82-96): ``x * bf16(w * rsqrt(mean(x^2) + eps))``;
    ``fused`` (sglang/kernels.py:307-313): ``bf16(x * rsqrt(...) * w)``."""
    xf = x.float()
    if fused:
        inv = 1.0 / torch.sqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
        xn = (xf * inv * weight.float()).to(torch.bfloat16).float()
    else:
        xn = rms_norm(x, weight, eps).float()
    even, odd = xn.unflatten(-1, (-1, 2)).unbind(-1)
    return torch.stack([even * cos - odd * sin, odd * cos + even * sin], dim=-1).flatten(-2)


def rms_norm_rope_vllm(x, weight, cos_sin, positions, eps):
    """flashmap_vllm::rms_norm_rope (vllm/kernels.py:100-119): x (tokens, heads, hd)."""
    cos, sin = _pairs(cos_sin[positions.long()])
    return norm_rope(x, weight, cos[:, None], sin[:, None], eps).to(torch.bfloat16)


def rms_norm_rope_sglang(x, weight, freqs, eps):
    """flashmap_sglang::rms_norm_rope (sglang/kernels.py:170-183): freqs per token."""
    cos, sin = _pairs(freqs)
    return norm_rope(x, weight, cos[..., None, :], sin[..., None, :], eps).to(torch.bfloat16)


def attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> torch.Tensor:
    """Softmax attention of fp32 ``q (rows, hd)`` onto ``k, v (n, hd)``: scores in
    fp32, numerators exp(s - m) rounded to bf16 for P V, the fp32 sum dividing at
    the end (the FlashAttention numerics of the reference's serving paths and of
    the CPU SDPA the HF path uses)."""
    if k.shape[0] == 0:
        return torch.zeros(q.shape[0], v.shape[1])
    s = (q @ k.T) * scale
    p = torch.exp(s - s.max(dim=-1, keepdim=True).values)
    return (p.to(torch.bfloat16).float() @ v) / p.sum(dim=-1, keepdim=True)


def block_self_attention(qkv, q_norm, k_norm, cos, sin, eps):
    """vllm/kernels.py:123-190 and sglang/kernels.py:18-81: qkv (blocks, T, 3, H, hd);
    ``cos, sin`` (blocks, T, hd/2).  Returns (blocks, T, H, hd) bf16."""
    blocks, T, _, H, hd = qkv.shape
    q = norm_rope(qkv[:, :, 0], q_norm, cos[:, :, None], sin[:, :, None], eps).to(torch.bfloat16).float()
    k = norm_rope(qkv[:, :, 1], k_norm, cos[:, :, None], sin[:, :, None], eps).to(torch.bfloat16).float()
    v = qkv[:, :, 2].float()
    out = torch.empty(blocks, T, H, hd)
    for b in range(blocks):
        for h in range(H):
            out[b, :, h] = attend(q[b, :, h], k[b, :, h], v[b, :, h], hd ** -0.5)
    return out.to(torch.bfloat16)


def paged_attention(q_rows, heads_kv_at, lengths, q_ranges, scale):
    """Cross-attention of each request's query rows onto its first ``lengths[r]``
    positions: ``heads_kv_at(r, n) -> (k (n, H, hd), v (n, H, hd))`` fp32 gathers
    the request's context through its page table; ``q_rows (rows, H, hd)`` fp32,
    rows of request r in ``q_ranges[r]``.  Returns (rows, H, hd) fp32."""
    rows, H, hd = q_rows.shape
    out = torch.zeros(rows, H, hd)
    for r, (a, b) in enumerate(q_ranges):
        k, v = heads_kv_at(r, int(lengths[r]))
        for h in range(H):
            out[a:b, h] = attend(q_rows[a:b, h], k[:, h], v[:, h], scale)
    return out


def gather_vllm(kv_cache: torch.Tensor, block_table: torch.Tensor, hd: int, descale=None):
    """``heads_kv_at`` for the FlashAttention cache (blocks, H, page, 2 hd)
    (vllm/model.py:118): position p of request r at page block_table[r, p // page]."""
    page = kv_cache.shape[2]

    def at(r, n):
        p = torch.arange(n)
        blk = block_table[r, p // page].long()
        rows = kv_cache[blk, :, p % page].float()  # (n, H, 2 hd)
        k, v = rows[..., :hd], rows[..., hd:]
        if descale is not None:
            k = k * descale[1][r][None, :, None]
            v = v * descale[2][r][None, :, None]
        return k, v

    return at


def gather_pool(key_buffer: torch.Tensor, value_buffer: torch.Tensor, page_table: torch.Tensor):
    """``heads_kv_at`` for sglang's pools (rows, H, hd), page size 1 (sglang/model.py:136-144)."""

    def at(r, n):
        rows = page_table[r, :n].long()
        return key_buffer[rows].float(), value_buffer[rows].float()

    return at


def quantize_query_fp8(query: torch.Tensor):
    """sglang/model.py:164-166: per (request, head) scale amax / 448 and the e4m3
    query, widened back to fp32 and descaled."""
    q_scale = query.float().abs().amax(dim=(1, 3)).clamp_min(1e-12) / 448.0
    q8 = (query.float() / q_scale[:, None, :, None]).to(FP8)
    return q8.float() * q_scale[:, None, :, None]


def write_context_kv(kv, positions, slots, k_norm, cos_sin, caches, strides, block_size, eps, scales=None,
                     heads_per_cache=None):
    """vllm/kernels.py:240-307 on flat CPU caches: every (token, layer, head)
    key k-normed (DiT rounding), rotated, bf16 or key / k_scale in e4m3, and its
    value, at the slot's (block, head slot, row); heads layer-major,
    ``heads_per_cache`` to a cache.  ``caches`` are flat tensors, updated in place."""
    tokens, L, _, H, hd = kv.shape
    hpc = heads_per_cache or H
    sb, sh, st, voff = strides
    cos, sin = _pairs(cos_sin)
    for t in range(tokens):
        slot = int(slots[t])
        if slot < 0:
            continue
        pos = int(positions[t])
        for g in range(L * H):
            layer, h = divmod(g, H)
            c, s = divmod(g, hpc)
            key = norm_rope(kv[t, layer, 0, h], k_norm[layer], cos[pos], sin[pos], eps)
            val = kv[t, layer, 1, h].float()
            off = (slot // block_size) * sb + s * sh + (slot % block_size) * st
            if scales is None:
                caches[c][off:off + hd] = key.to(torch.bfloat16)
                caches[c][off + voff:off + voff + hd] = val.to(torch.bfloat16)
            else:
                caches[c][off:off + hd] = (key / scales[layer, 0]).to(FP8)
                caches[c][off + voff:off + voff + hd] = (val / scales[layer, 1]).to(FP8)


def kv_norm_rope_write_pool(kv, k_pools, v_pools, k_norm, cos_sin, positions, locs, L, kv_size, hd, eps, fp8,
                            k_scale=1.0, v_scale=1.0, commit_lens=None, row_width=1):
    """sglang/kernels.py:269-316: kv (tokens, L * 2 * kv_size); keys k-normed
    (the e4m3 writer's fused rounding; a bf16 pool takes the HF path's k_norm,
    modeling_flashmap.py:76-80), rotated with the ``(positions, [cos | sin])``
    table; bf16, or e4m3 of key / k_scale and value / v_scale; pools (rows, kv_size)."""
    half = hd // 2
    for t in range(kv.shape[0]):
        if commit_lens is not None and t % row_width >= int(commit_lens[t // row_width]):
            continue
        loc = int(locs[t])
        if loc < 0:
            continue
        pos = int(positions[t])
        cos, sin = cos_sin[pos, :half], cos_sin[pos, half:]
        row = kv[t].view(L, 2, kv_size)
        for layer in range(L):
            for h in range(kv_size // hd):
                key = norm_rope(row[layer, 0, h * hd:(h + 1) * hd], k_norm[layer], cos, sin, eps, fused=fp8)
                val = row[layer, 1, h * hd:(h + 1) * hd].float()
                if fp8:
                    k_pools[layer][loc, h * hd:(h + 1) * hd] = (key / k_scale).to(FP8)
                    v_pools[layer][loc, h * hd:(h + 1) * hd] = (val / v_scale).to(FP8)
                else:
                    k_pools[layer][loc, h * hd:(h + 1) * hd] = key.to(torch.bfloat16)
                    v_pools[layer][loc, h * hd:(h + 1) * hd] = val.to(torch.bfloat16)


def rope_pairs(max_pos: int, head_dim: int, theta: float) -> torch.Tensor:
    """vllm/kernels.py:27-35: (max_pos, hd/2, [cos, sin]) fp32."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    angles = torch.arange(max_pos).float()[:, None] * inv_freq
    return torch.stack([angles.cos(), angles.sin()], dim=-1).contiguous()


def check_apply_rope_agrees(x: torch.Tensor, weight: torch.Tensor, table: torch.Tensor, positions, eps: float) -> bool:
    """The restated op equals the HF path's RMSNorm + apply_rope (the pinned oracle)."""
    cos, sin = _pairs(table[positions.long()])
    ref = apply_rope(rms_norm(x, weight, eps), (cos[:, None], sin[:, None]))
    return torch.equal(ref, rms_norm_rope_vllm(x, weight, table, positions, eps))
