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

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import ctypes

import torch

from . import _lib, ops
from .configuration_flashmap import jump_times

Rotate = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def bank_coefficients(grid) -> list:
    """Per jump n: (alpha_n, [beta_n1 .. beta_nn]), the coefficients of the
    starting noise and of each earlier prediction in the state x_n, from the
    jump update x <- ((1 - t) x + (t - s) delta) / (1 - s) (jump_bank.py:76-86)."""
    out, alpha, betas = [(1.0, [])], 1.0, []
    for start, end in zip(grid[:-2], grid[1:-1]):
        keep = (1.0 - float(end)) / (1.0 - float(start))
        alpha *= keep
        betas = [b * keep for b in betas] + [(float(end) - float(start)) / (1.0 - float(start))]
        out.append((alpha, list(betas)))
    return out


@dataclass
class JumpBank:
    """A noise bank (jump_bank.py:95-150): ``size`` draws z over the state
    vocabulary with what the later jumps read of them — ``noise_embed`` [size,
    Ht] = z @ E, and per later jump n ``mean_embed[n-1]`` [size, Ht] =
    softmax(a_n z) @ E and ``log_mass[n-1]`` [size] = logsumexp(a_n z) —
    with the per-jump constants (coefficients, e_n, a_n)."""
    grid: list
    size: int
    temperature: float
    coefficients: list
    evidence: list
    slopes: list
    noise_embed: torch.Tensor
    mean_embed: torch.Tensor
    log_mass: torch.Tensor

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.noise_embed, self.mean_embed, self.log_mass))
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
        state_c = state.contiguous()  # referenced until the launch below
        _lib.call("fm_state_rows", ops._p(state_c), ops._p(rows), T, S, float(evidence),
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

    # -------------------------------------------------------------- banked jumps
    def build_bank(self, grid, size: int, temperature: float, seed: int = 0, chunk: int = 128) -> JumpBank:
        """The noise bank of a banked multi-jump draft (jump_bank.py:104-150):
        bank row i draws z = temperature * N(0, I_S) from the Philox stream of
        (seed, i), so a row does not depend on the chunking; z @ E and the per
        jump softmax(a_n z) @ E are GEMMs against E_S^T."""
        p, S, Ht = self.pack, self.pack.S, self.Ht
        grid = [float(t) for t in grid]
        coefficients = bank_coefficients(grid)
        evidence = [t / (1.0 - t) ** 2 for t in grid[1:len(grid) - 1]]
        slopes = [e * coefficients[n + 1][0] for n, e in enumerate(evidence)]
        nj = len(slopes)
        if nj > 8:
            raise ValueError("a banked draft takes at most 9 jumps")
        dev = p.device
        noise_embed = torch.empty(size, Ht, device=dev, dtype=torch.bfloat16)
        mean_embed = torch.empty(nj, size, Ht, device=dev, dtype=torch.bfloat16)
        log_mass = torch.empty(nj, size, device=dev, dtype=torch.float32)
        slope_arr = (ctypes.c_float * 8)(*slopes)
        seeds = torch.tensor([seed], device=dev, dtype=torch.int64)
        for start in range(0, size, chunk):
            rows = min(chunk, size - start)
            z = torch.empty(rows, S, device=dev, dtype=torch.float32)
            zeros = torch.zeros(rows, device=dev, dtype=torch.int64)
            index = start + torch.arange(rows, device=dev, dtype=torch.int64)
            _lib.call("fm_philox_normal_rows_f32", ops._p(z), rows, S, ops._p(seeds), ops._p(zeros), ops._p(index),
                      float(temperature), ops._stream())
            zb = torch.empty(rows, S, device=dev, dtype=torch.bfloat16)
            probs = torch.empty(max(nj, 1), rows, S, device=dev, dtype=torch.bfloat16)
            mass = torch.empty(max(nj, 1), rows, device=dev, dtype=torch.float32)
            _lib.call("fm_bank_rows", ops._p(z), ops._p(zb), ops._p(probs), ops._p(mass), rows, S,
                      ctypes.cast(slope_arr, ctypes.c_void_p), nj, ops._stream())
            ops.gemm(p.embed_state_t, zb, out=noise_embed[start:start + rows])
            for j in range(nj):
                ops.gemm(p.embed_state_t, probs[j], out=mean_embed[j, start:start + rows])
                log_mass[j, start:start + rows] = mass[j]
        return JumpBank(grid, int(size), float(temperature), coefficients, evidence, slopes, noise_embed, mean_embed,
                        log_mass)

    def bank_draw(self, slots: int, bank: JumpBank, seed: int, offset: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """A bank row and a slot seed per slot (jump_bank.py:157-161), from the
        Philox stream (seed, offset)."""
        dev = self.pack.device
        rows = torch.empty(slots, device=dev, dtype=torch.int64)
        seeds = torch.empty(slots, device=dev, dtype=torch.int64)
        _lib.call("fm_philox_randint", ops._p(rows), slots, bank.size, seed, offset & 0xFFFFFFFF, 5, ops._stream())
        _lib.call("fm_philox_randint", ops._p(seeds), slots, 2 ** 31 - 1, seed, offset & 0xFFFFFFFF, 6,
                  ops._stream())
        return rows, seeds

    def _embed_rows(self, post, post_stride: int, state, s: float, t: float) -> torch.Tensor:
        p, T = self.pack, state.shape[0]
        inputs = torch.empty(T, self.Ht, device=p.device, dtype=torch.bfloat16)
        _lib.call("fm_mix_state", ops._p(post), post_stride, ops._p(state), ops._p(p.g["state_norm.weight"]),
                  ops._p(p.g["noise_norm.weight"]), ops._p(inputs), float(p.noise_gate_value(self.cfg, s, t)),
                  float(self.cfg.rms_norm_eps), T, self.Ht, ops._stream())
        return ops.gemm(p.g["x_embed.weight"], inputs, bias=p.g["x_embed.bias"])

    def bank_first_input(self, bank: JumpBank, rows: torch.Tensor, s: float, t: float) -> torch.Tensor:
        """``x_embed(state_norm(uniform) + gate * noise_norm(noise_embed[rows]))``
        (jump_bank.py:164-169): jump 0 from the bank rows' noise."""
        p, R = self.pack, rows.shape[0]
        rows = rows.contiguous()
        noise = torch.empty(R, self.Ht, device=p.device, dtype=torch.bfloat16)
        _lib.call("fm_bank_gather", ops._p(bank.noise_embed), bank.size, self.Ht, ops._p(rows), R, ops._p(noise),
                  None, ops._stream())
        return self._embed_rows(p.uniform_embeds, 0, noise, s, t)

    def bank_jump_rows(self, bank: JumpBank, n: int, rows: torch.Tensor, seeds: torch.Tensor,
                       supports: List[Tuple[torch.Tensor, torch.Tensor]]) -> torch.Tensor:
        """Jump n's posterior and noise rows [2R, Ht] before the norms
        (jump_bank.py:171-205) over the earlier predictions' supports."""
        p, R = self.pack, rows.shape[0]
        rows, seeds = rows.contiguous(), seeds.contiguous()  # referenced until the launch below
        ids = torch.cat([i for i, _ in supports], dim=1).to(torch.int64).contiguous()
        probs = torch.cat([q for _, q in supports], dim=1).float().contiguous()
        alpha, betas = bank.coefficients[n]
        beta_t = torch.tensor(betas, device=p.device, dtype=torch.float32)
        out = torch.empty(2 * R, self.Ht, device=p.device, dtype=torch.bfloat16)
        a = _lib.BankJump()
        a.noise_embed, a.mean_embed = bank.noise_embed.data_ptr(), bank.mean_embed[n - 1].data_ptr()
        a.log_mass, a.embed = bank.log_mass[n - 1].data_ptr(), p.embed.data_ptr()
        a.state_map = None if p.draft_ids is None else p.draft_ids.data_ptr()
        a.bank_rows, a.state_rows, a.hidden, a.slots = bank.size, p.S, self.Ht, R
        a.rows, a.seeds = rows.data_ptr(), seeds.data_ptr()
        a.ids, a.probs, a.betas = ids.data_ptr(), probs.data_ptr(), beta_t.data_ptr()
        a.support, a.topk = ids.shape[1], supports[0][0].shape[1]
        a.alpha, a.evidence, a.slope = alpha, bank.evidence[n - 1], bank.slopes[n - 1]
        a.temperature, a.out, a.err = bank.temperature, out.data_ptr(), None
        _lib.call("fm_bank_jump_rows", ctypes.byref(a), ops._stream())
        return out

    def bank_jump_input(self, bank: JumpBank, n: int, rows, seeds, supports, s: float, t: float) -> torch.Tensor:
        """``x_embed(state_norm(posterior) + gate * noise_norm(noise))`` of jump n >= 1."""
        R = rows.shape[0]
        both = self.bank_jump_rows(bank, n, rows, seeds, supports)
        return self._embed_rows(both[:R], self.Ht, both[R:], s, t)

    def top_predictions(self, logits: torch.Tensor, k: int, row_map: Optional[torch.Tensor] = None):
        """A jump's prediction cut to its top k (jump_bank.py:89-92): (ids, probs),
        ids mapped through ``row_map`` to state rows when given."""
        R, V = logits.shape
        ids = torch.empty(R, k, device=logits.device, dtype=torch.int64)
        probs = torch.empty(R, k, device=logits.device, dtype=torch.float32)
        rm = None if row_map is None else row_map.to(torch.int64).contiguous()
        _lib.call("fm_topk_rows", ops._p(logits), logits.stride(0), R, V, k, None if rm is None else ops._p(rm),
                  0 if rm is None else rm.numel(), ops._p(ids), ops._p(probs), None, ops._stream())
        return ids, probs

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
            z = z.contiguous()  # one tensor, referenced until the launch below
            proj = ops.gemm(weight, z)
            out = torch.empty(T, self.D, device=p.device, dtype=torch.bfloat16)
            _lib.call("fm_noise_fold", ops._p(proj), ops._p(z), ops._p(var), ops._p(x0), ops._p(out),
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
