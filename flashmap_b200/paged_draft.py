"""One FlashMap jump over a context that lives in a serving engine's paged KV
cache, on this library's kernels.  The vLLM and sglang plugin models
(``vllm_model``, ``sglang_model``) drive it; each engine supplies how the
query rows are rotated and how they attend to its cache.

Unfolded, the arithmetic is the HF path's (modeling_flashmap.py:302-313,
378-420, 459-475): noise ``z @ L^T`` through the Cholesky factor of ``E^T E``,
``state_norm(uniform) + bf16(gate * noise_norm(.))``, ``x_embed``, the DiT
layers, the final AdaLN, and for logits the DiT head followed by the target's
LM head.  The reference plugins fold both ends into single projections
(vllm/fold.py:44-100, sglang/model.py:515-595, 945-958), which changes the
rounding: ``fold_head`` maps the final AdaLN output straight to logits through
the LM-head rows times the DiT head, ``fold_noise`` forms the first layer's
input from the noise's eigenbasis projection.  The plugin models choose the
folds their reference counterparts use.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch

from . import _lib, ops
from .configuration_flashmap import jump_times

Rotate = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
Attend = Callable[[torch.Tensor, int], torch.Tensor]


class PagedDraft:
    """The drafter's weights in kernel layout (the HF model's pack) and the
    per-jump constants, with the passes the plugin models compose."""

    def __init__(self, model, device, fold_head: bool = False, fold_noise: bool = False):
        self.model = model
        self.fold_head, self.fold_noise = fold_head, fold_noise
        self.cfg = cfg = model.config
        self.pack = model._pack(torch.device(device))
        self.D, self.H = cfg.hidden_size, cfg.num_attention_heads
        self.hd = self.D // self.H
        self.L, self.K = cfg.num_hidden_layers, cfg.block_size
        self.Ht = cfg.target_hidden_size
        self._tables = {}

    # -------------------------------------------------------------- target side
    def attach(self, embedding: torch.Tensor, lm_head_weight: torch.Tensor, lm_head_bias=None) -> None:
        """The target's embedding and LM head (modeling_flashmap.py:355-368, 401-420)."""
        self.pack.attach_target(embedding, lm_head_weight, lm_head_bias)

    def restrict_lm_rows(self, rows: torch.Tensor) -> None:
        """Cut the LM head to ``rows`` of the attached head (a draft vocabulary
        over the full state vocabulary), always from the full head so that a
        repeated ``prepare`` cuts once; the folded head is rebuilt from it."""
        p = self.pack
        w, b = p.lm_rows_full
        p.lm_w = w[rows].contiguous()
        p.lm_b = None if b is None else b[rows].contiguous()
        p.lm_fold_w = p.lm_fold_b = None

    @property
    def attached(self) -> bool:
        return self.pack.target_key is not None

    def rope_pairs(self, max_pos: int) -> torch.Tensor:
        """``(max_pos, hd/2, [cos, sin])`` fp32, the vLLM table layout
        (vllm/kernels.py:27-35), from the library's table kernel."""
        self.pack.ensure_rope(self.cfg, max_pos)
        n = self.pack.rope_len
        table = self._tables.get(n)
        if table is None:
            table = torch.stack([self.pack.rope_cos, self.pack.rope_sin], dim=-1).contiguous()
            self._tables = {n: table}
        return table

    def jump(self, num_steps: int = 1):
        grid = self.cfg.jump_grids[str(num_steps)]
        return jump_times(grid)

    def modulations(self, s: float, t: float) -> torch.Tensor:
        return self.pack.modulations(self.cfg, s, t)

    # -------------------------------------------------------------- several jumps
    def state_noise(self, tokens: int, seeds=None, rows=None, positions=None, scale: float = 1.0,
                    seed: int = 0, offset: int = 0) -> torch.Tensor:
        """The starting state ``(tokens, S)`` fp32 of a multi-jump draft: keyed
        per row like ``noise`` (vllm/model.py:968-975), else one Philox stream
        (seed, counter offset + row)."""
        dev, S = self.pack.device, self.pack.S
        out = torch.empty(tokens, S, device=dev, dtype=torch.float32)
        if seeds is None:
            seeds = torch.tensor([seed], device=dev, dtype=torch.int64)
            rows = torch.zeros(tokens, device=dev, dtype=torch.int64)
            positions = offset + torch.arange(tokens, device=dev, dtype=torch.int64)
        s64 = seeds.to(torch.int64).contiguous()
        r64 = rows[:tokens].to(torch.int64).contiguous()
        p64 = positions[:tokens].to(torch.int64).contiguous()
        _lib.call("fm_philox_normal_rows_f32", ops._p(out), tokens, S, ops._p(s64), ops._p(r64), ops._p(p64),
                  float(scale), ops._stream())
        return out

    def embed_state(self, state: torch.Tensor, s: float, t: float) -> torch.Tensor:
        """``x_embed(state_norm(softmax(e state) @ E) + bf16(gate * noise_norm(state @
        E)))`` of the fp32 state at jump (s, t), ``e = s / max(1 - s, 1e-3)^2``;
        at s = 0 the posterior is uniform (modeling_flashmap.py:378-420,
        vllm/model.py:944-956)."""
        p = self.pack
        T, S = state.shape
        with_post = s != 0.0
        evidence = s / max(1.0 - s, 1e-3) ** 2 if with_post else 0.0
        rows = torch.empty(2 * T if with_post else T, S, device=p.device, dtype=torch.bfloat16)
        _lib.call("fm_state_rows", ops._p(state.contiguous()), ops._p(rows), T, S, float(evidence),
                  1 if with_post else 0, ops._stream())
        semb = ops.gemm(p.embed_state_t, rows)  # [2T or T, Ht]
        if with_post:
            post, stride, st = semb[:T], self.Ht, semb[T:]
        else:
            post, stride, st = p.uniform_embeds, 0, semb
        inputs = torch.empty(T, self.Ht, device=p.device, dtype=torch.bfloat16)
        _lib.call("fm_mix_state", ops._p(post), stride, ops._p(st), ops._p(p.g["state_norm.weight"]),
                  ops._p(p.g["noise_norm.weight"]), ops._p(inputs), float(p.noise_gate_value(self.cfg, s, t)),
                  float(self.cfg.rms_norm_eps), T, self.Ht, ops._stream())
        return ops.gemm(p.g["x_embed.weight"], inputs, bias=p.g["x_embed.bias"])

    def jump_logits(self, final: torch.Tensor) -> torch.Tensor:
        """A jump's prediction logits over every state row (the jump head: the
        LM head folded with the DiT head with ``fold_head``, vllm/model.py:578-585;
        else the DiT head then the LM head), whatever draft vocabulary cut the
        drafting head."""
        p = self.pack
        full_w, full_b = p.lm_rows_full
        if self.fold_head:
            if p.lm_w is full_w:
                w, b = p.ensure_fold()
            else:
                if getattr(self, "_jump_fold", None) is None or self._jump_fold[0] is not full_w:
                    self._jump_fold = (full_w, p.fold_rows(full_w))
                w, b = self._jump_fold[1]
            return ops.gemm(w, final.contiguous(), bias=b)
        return ops.gemm(full_w, self.head(final), bias=full_b)

    def state_update(self, state: torch.Tensor, logits: torch.Tensor, s: float, nxt: float) -> None:
        """``state = ((1 - next) state + (next - s) softmax(logits)) / (1 - s)`` in
        place (modeling_flashmap.py:470-472)."""
        T, S = state.shape
        _lib.call("fm_state_update", ops._p(state), ops._p(logits), logits.stride(0), T, S, float(1.0 - nxt),
                  float(nxt - s), float(1.0 - s), ops._stream())

    # -------------------------------------------------------------- context rows
    def combine(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """``fc`` of the target's features (modeling_flashmap.py:322-340)."""
        return ops.gemm(self.pack.g["fc.weight"], hidden_states.reshape(-1, hidden_states.shape[-1]).contiguous())

    def context_kv(self, states: torch.Tensor) -> torch.Tensor:
        """Every layer's context (k, v) rows ``(n, L * 2 * D)`` of fc outputs:
        ``hidden_norm`` then the stacked k/v projections (:342-351)."""
        normed = ops.rmsnorm(states.contiguous(), self.pack.g["hidden_norm.weight"], self.cfg.rms_norm_eps)
        return ops.gemm(self.pack.cross_kv_w, normed)

    def anchor_kv(self, anchor_ids: torch.Tensor) -> torch.Tensor:
        """The anchors' context rows: ``anchor_norm(anchor_proj(embed(anchor)))``
        through the k/v projections (modeling_flashmap.py:452-457)."""
        rows = self.pack.embed[anchor_ids.long()].contiguous()
        proj = ops.gemm(self.pack.g["anchor_proj.weight"], rows, bias=self.pack.g["anchor_proj.bias"])
        normed = ops.rmsnorm(proj, self.pack.g["anchor_norm.weight"], self.cfg.rms_norm_eps)
        return ops.gemm(self.pack.cross_kv_w, normed)

    # -------------------------------------------------------------- the jump
    def noise(self, tokens: int, seeds=None, rows=None, positions=None, scale: float = 1.0,
              seed: int = 0, offset: int = 0) -> torch.Tensor:
        """``z (tokens, Ht)`` bf16: per-row keyed noise when ``seeds``/``rows``/
        ``positions`` are given (a seeded request draws the same noise whatever
        is batched with it), else one Philox stream (seed, offset)."""
        dev = self.pack.device
        if scale == 0.0:
            return torch.zeros(tokens, self.Ht, device=dev, dtype=torch.bfloat16)
        if seeds is not None:
            z = torch.empty(tokens, self.Ht, device=dev, dtype=torch.bfloat16)
            s64 = seeds.to(torch.int64).contiguous()
            r64 = rows[:tokens].to(torch.int64).contiguous()
            p64 = positions[:tokens].to(torch.int64).contiguous()
            _lib.call("fm_philox_normal_rows", ops._p(z), tokens, self.Ht, ops._p(s64), ops._p(r64), ops._p(p64),
                      float(scale), ops._stream())
            return z
        z = ops.philox_normal((tokens, self.Ht), seed, offset, device=dev)
        return z if scale == 1.0 else (z.float() * scale).to(torch.bfloat16)

    def first_hidden(self, z: torch.Tensor, s: float, t: float) -> torch.Tensor:
        """``x_embed(state_norm(uniform) + bf16(gate * noise_norm(z @ L^T)))``
        (modeling_flashmap.py:393-399, 459-468); with ``fold_noise``,
        ``x0 + bf16(gate * rsqrt(sum(var z^2) + eps) * (z @ M))``
        (sglang/model.py:945-958)."""
        p, T = self.pack, z.shape[0]
        if self.fold_noise:
            weight, var, x0 = p.ensure_noise_fold(self.cfg)
            proj = ops.gemm(weight, z.contiguous())
            out = torch.empty(T, self.D, device=p.device, dtype=torch.bfloat16)
            _lib.call("fm_noise_fold", ops._p(proj), ops._p(z.contiguous()), ops._p(var), ops._p(x0), ops._p(out),
                      float(p.noise_gate_value(self.cfg, s, t)), float(self.cfg.rms_norm_eps), T, self.D, self.Ht,
                      ops._stream())
            return out
        zl = ops.gemm(p.chol, z.contiguous())
        inputs = torch.empty(T, self.Ht, device=p.device, dtype=torch.bfloat16)
        gate = p.noise_gate_value(self.cfg, s, t)
        _lib.call("fm_mix_state", ops._p(p.uniform_embeds), 0, ops._p(zl), ops._p(p.g["state_norm.weight"]),
                  ops._p(p.g["noise_norm.weight"]), ops._p(inputs), float(gate), float(self.cfg.rms_norm_eps), T,
                  self.Ht, ops._stream())
        return ops.gemm(p.g["x_embed.weight"], inputs, bias=p.g["x_embed.bias"])

    def dit(self, x: torch.Tensor, mods: torch.Tensor, self_attention: Callable[[torch.Tensor, int], torch.Tensor],
            rotate_query: Callable[[torch.Tensor, int], torch.Tensor], attend: Attend) -> torch.Tensor:
        """The DiT layers on ``x (T, D)`` (updated in place) and the final AdaLN
        (modeling_flashmap.py:185-192, 302-313).  ``self_attention(qkv, layer)``
        maps projected ``qkv (T, 3D)`` to ``(T, D)``; ``rotate_query(q, layer)``
        q-norms and rotates ``q (T, H, hd)``; ``attend(query, layer)`` returns
        the cross-attention ``(T, H, hd)`` onto the engine's cache."""
        p, D, eps = self.pack, self.D, self.cfg.layer_norm_eps
        T = x.shape[0]
        n3 = 3 * D

        def mod(n):
            return mods[n * n3:(n + 1) * n3]

        for layer in range(self.L):
            w = p.layers[layer]
            m = mod(3 * layer)
            h = ops.adaln(x, m, eps)
            attn = self_attention(ops.gemm(w["self_qkv_w"], h), layer)
            ops.gemm(w["self_o_w"], attn.reshape(T, D), ops.RESID, gate=m[2 * D:], out=x)
            m = mod(3 * layer + 1)
            h = ops.adaln(x, m, eps)
            q = rotate_query(ops.gemm(w["cross_q_w"], h).view(T, self.H, self.hd), layer)
            ctx = attend(q, layer)
            ops.gemm(w["cross_o_w"], ctx.reshape(T, D).contiguous(), ops.RESID, gate=m[2 * D:], out=x)
            m = mod(3 * layer + 2)
            h = ops.adaln(x, m, eps)
            if p.swiglu:
                u = ops.gemm(w["mlp_w1"], h, ops.SWIGLU)
            else:
                u = ops.gemm(w["mlp_w1"], h, ops.GELU, bias=w["mlp_b1"])
            ops.gemm(w["mlp_w2"], u, ops.RESID, bias=w["mlp_b2"], gate=m[2 * D:], out=x)
        return ops.adaln(x, mod(3 * self.L), eps)

    def head(self, final: torch.Tensor) -> torch.Tensor:
        """The DiT head ``(T, Ht)`` (modeling_flashmap.py:313)."""
        return ops.gemm(self.pack.g["head.weight"], final.contiguous(), bias=self.pack.g["head.bias"])

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """``F.linear(hidden, lm_head)`` over the draft vocabulary (:474-475)."""
        return ops.gemm(self.pack.lm_w, hidden.contiguous(), bias=self.pack.lm_b)

    def draft_logits(self, final: torch.Tensor) -> torch.Tensor:
        """Draft-vocabulary logits from the final AdaLN output: the DiT head then
        the LM head, or with ``fold_head`` their product (vllm/fold.py:76-100)."""
        if self.fold_head:
            weight, bias = self.pack.ensure_fold()
            return ops.gemm(weight, final.contiguous(), bias=bias)
        return self.logits(self.head(final))


def unsupported_steps(num_steps: int) -> Optional[str]:
    if num_steps != 1:
        return ("the plugin models draft one jump per block on this library (multi-jump drafting runs "
                "through FlashMapDraftModel.draft)")
    return None
