"""CPU restatement of the FlashMap drafter (test infrastructure: the checker).

Each function restates one step of the reference
``flashmap/modeling_flashmap.py`` (al-jshen/flashmap v0.2.1) with plain torch
CPU ops, in the same order and dtypes, so that on the CPU it reproduces the
reference bit for bit (pinned by ``tests/test_oracle_golden.py`` against
vectors the reference itself produced).  Weights are a plain ``dict`` keyed by
the reference's ``state_dict`` names; nothing here is an ``nn.Module``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may use this module.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# ---------------------------------------------------------------- primitives


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float):
    """fp32 ``cos, sin`` of shape (B, T, 1, head_dim/2) — modeling_flashmap.py:53-58."""
    exponent = torch.arange(0, head_dim, 2, device=positions.device).float() / head_dim
    inv_freq = 1.0 / theta**exponent
    angle = positions.float()[..., None, None] * inv_freq
    return angle.cos(), angle.sin()


def apply_rope(x: torch.Tensor, rope) -> torch.Tensor:
    """Rotate interleaved pairs (2i, 2i+1) in fp32, round back — :61-66."""
    cos, sin = rope
    even, odd = x.float().unflatten(-1, (-1, 2)).unbind(-1)
    rotated = torch.stack([even * cos - odd * sin, odd * cos + even * sin], dim=-1)
    return rotated.flatten(-2).type_as(x)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``x * dtype(w * rsqrt(mean(x^2) + eps))`` — the scale is rounded to the
    input dtype before it multiplies (:69-80)."""
    inv = torch.rsqrt(x.float().pow(2).mean(dim=-1, keepdim=True) + eps)
    return x * (weight.float() * inv).to(x.dtype)


def linear(x, w, b=None):
    return F.linear(x, w, b)


def time_embedding(p: dict, prefix: str, t: torch.Tensor, dim: int, scale: float) -> torch.Tensor:
    """Sinusoid of ``t * scale`` -> linear_1 -> SiLU -> linear_2 (:83-97)."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device).float() / half)
    args = (t.float() * scale)[..., None] * freqs
    w1 = p[f"{prefix}.linear_1.weight"]
    feats = torch.cat([args.cos(), args.sin()], dim=-1).to(w1.dtype)
    hidden = F.silu(linear(feats, w1, p[f"{prefix}.linear_1.bias"]))
    return linear(hidden, p[f"{prefix}.linear_2.weight"], p[f"{prefix}.linear_2.bias"])


def modulation(p: dict, prefix: str, cond: torch.Tensor):
    """``(scale, shift, gate)`` = chunk3(linear(silu(cond))) (:108-110)."""
    return linear(F.silu(cond), p[f"{prefix}.linear.weight"], p[f"{prefix}.linear.bias"]).chunk(3, dim=-1)


def ada_layer_norm(x: torch.Tensor, mod, eps: float):
    """``layer_norm(x) * (1 + scale) + shift`` and the gate (:112-115)."""
    scale, shift, gate = mod
    return F.layer_norm(x, x.shape[-1:], eps=eps) * (1 + scale) + shift, gate


def split_heads(x: torch.Tensor, heads: int) -> torch.Tensor:
    return x.view(*x.shape[:2], heads, x.shape[-1] // heads)


def project_kv(p: dict, prefix: str, x, rope, heads: int, qk_eps: float):
    """Keys ``RoPE(k_norm(k_proj x))`` and values ``v_proj x`` as (B, H, T, hd) (:139-142)."""
    keys = apply_rope(rms_norm(split_heads(linear(x, p[f"{prefix}.k_proj.weight"]), heads),
                               p[f"{prefix}.k_norm.weight"], qk_eps), rope)
    values = split_heads(linear(x, p[f"{prefix}.v_proj.weight"]), heads)
    return keys.transpose(1, 2), values.transpose(1, 2)


def attention(p: dict, prefix: str, x, rope, keys, values, heads: int, qk_eps: float):
    """Queries ``RoPE(q_norm(q_proj x))``, unmasked SDPA, ``o_proj`` (:144-147)."""
    queries = apply_rope(rms_norm(split_heads(linear(x, p[f"{prefix}.q_proj.weight"]), heads),
                                  p[f"{prefix}.q_norm.weight"], qk_eps), rope)
    out = F.scaled_dot_product_attention(queries.transpose(1, 2), keys, values)
    return linear(out.transpose(1, 2).flatten(2), p[f"{prefix}.o_proj.weight"])


def mlp(p: dict, prefix: str, x, mlp_type: str):
    """GELU: ``fc2(gelu(fc1 x))``; SwiGLU: ``down(silu(gate) * up)`` (:150-169)."""
    if mlp_type == "swiglu":
        gate, up = linear(x, p[f"{prefix}.gate_up_proj.weight"]).chunk(2, dim=-1)
        return linear(F.silu(gate) * up, p[f"{prefix}.down_proj.weight"])
    hidden = F.gelu(linear(x, p[f"{prefix}.fc1.weight"], p[f"{prefix}.fc1.bias"]))
    return linear(hidden, p[f"{prefix}.fc2.weight"], p[f"{prefix}.fc2.bias"])


# ---------------------------------------------------------------- the model


class OracleCache:
    """Dense context cache (L, 2, B, H, T, hd) and its length (:195-219)."""

    def __init__(self, config, batch_size: int, max_length: int, dtype, device="cpu"):
        hd = config.hidden_size // config.num_attention_heads
        shape = (config.num_hidden_layers, 2, batch_size, config.num_attention_heads, max_length, hd)
        self.kv = torch.zeros(shape, dtype=dtype, device=device)
        self.length = 0

    def write(self, layer: int, start: int, keys, values) -> None:
        end = start + keys.shape[2]
        if end > self.kv.shape[4]:
            raise ValueError(f"cache holds {self.kv.shape[4]} positions, writing up to {end}")
        self.kv[layer, 0, :, :, start:end] = keys
        self.kv[layer, 1, :, :, start:end] = values

    def context(self, end: int):
        return [(kv[0, :, :, :end], kv[1, :, :, :end]) for kv in self.kv]


class Oracle:
    """The drafter of ``modeling_flashmap.py`` as plain functions over a weight dict.

    ``params`` holds the drafter weights in the model dtype (``dtype``);
    ``embedding``/``lm_head`` are the target's (V, H) matrices.
    """

    def __init__(self, config, params: dict, dtype=torch.float32):
        self.config = config
        self.p = {k: (v if k == "draft_ids" else v.to(dtype)) for k, v in params.items()}
        self.dtype = dtype
        self.heads = config.num_attention_heads
        self.head_dim = config.hidden_size // self.heads
        self._time_cache = {}
        self._target_cache = {}

    # -- time conditioning, :287-300
    @torch.no_grad()
    def time_conditioning(self, s: float, t: float):
        if (s, t) not in self._time_cache:
            cfg, p = self.config, self.p
            times = torch.tensor([s, t], device=p["noise_gate"].device)
            cond = (time_embedding(p, "time_embed", times[:1], cfg.time_embed_dim, cfg.time_scale)
                    + time_embedding(p, "jump_embed", times[1:], cfg.time_embed_dim, cfg.time_scale))[None]
            layers = [
                [modulation(p, f"layers.{i}.{n}", cond) for n in ("self_attn_adaln", "cross_attn_adaln", "mlp_adaln")]
                for i in range(cfg.num_hidden_layers)
            ]
            self._time_cache[(s, t)] = (layers, modulation(p, "final_adaln", cond))
        return self._time_cache[(s, t)]

    # -- one DiT block, :185-192
    def layer(self, i: int, x, mods, rope, context):
        cfg, p = self.config, self.p
        eps, qk = cfg.layer_norm_eps, cfg.qk_norm_eps
        pre = f"layers.{i}"
        h, gate = ada_layer_norm(x, mods[0], eps)
        keys, values = project_kv(p, f"{pre}.self_attn", h, rope, self.heads, qk)
        x = x + gate * attention(p, f"{pre}.self_attn", h, rope, keys, values, self.heads, qk)
        h, gate = ada_layer_norm(x, mods[1], eps)
        x = x + gate * attention(p, f"{pre}.cross_attn", h, rope, *context, self.heads, qk)
        h, gate = ada_layer_norm(x, mods[2], eps)
        return x + gate * mlp(p, f"{pre}.mlp", h, cfg.mlp_type)

    # -- forward, :302-313
    @torch.no_grad()
    def forward(self, inputs_embeds, s: float, t: float, position_ids, context, head=None, embedded=None):
        """``head`` = (weight, bias) replaces the DiT head (the folded head);
        ``embedded`` is the first layer's input when it is formed outside
        x_embed (the folded noise)."""
        layer_mods, final_mod = self.time_conditioning(s, t)
        rope = rope_tables(position_ids, self.head_dim, self.config.rope_theta)
        if embedded is not None:
            h = embedded.to(self.dtype)
        else:
            h = linear(inputs_embeds, self.p["x_embed.weight"], self.p["x_embed.bias"])
        for i in range(self.config.num_hidden_layers):
            h = self.layer(i, h, layer_mods[i], rope, context[i])
        h, _ = ada_layer_norm(h, final_mod, self.config.layer_norm_eps)
        if head is not None:
            return linear(h, *head)
        return linear(h, self.p["head.weight"], self.p["head.bias"])

    def fold_head(self, lm_head_w):
        """The serving plugins' folded head (vllm/fold.py:76-100): the state-vocab
        rows of the LM head times the DiT head, and times its bias, in fp32,
        rounded to the LM head's dtype."""
        rows = lm_head_w if self.config.state_vocab_size is None else lm_head_w[self.p["draft_ids"]]
        w = (rows.float() @ self.p["head.weight"].float()).to(lm_head_w.dtype)
        b = (rows.float() @ self.p["head.bias"].float()).to(lm_head_w.dtype)
        return w, b

    def fold_noise(self, embedding, return_basis=False):
        """The serving plugins' eigen-folded noise (vllm/fold.py:44-73,
        sglang/model.py:576-595) for the state vocabulary's rows ``E`` of the
        target embedding: ``E^T E = Q diag(lam) Q^T`` (the Gram matrix in fp32
        as noise_factor accumulates it, eigh in float64, negative round-off
        eigenvalues clamped to 0); ``weight = W_x diag(w_noise) Q diag(sqrt
        lam)`` [D, H] in the embedding's dtype (the transpose of the
        reference's ``M``), ``var = lam / H`` in fp32 and ``x0 =
        x_embed(state_norm(uniform @ E))``."""
        cfg, p = self.config, self.p
        emb_s = embedding if cfg.state_vocab_size is None else embedding[p["draft_ids"]]
        gram = sum(rows.float().T @ rows.float() for rows in emb_s.split(16384))
        lam, basis = torch.linalg.eigh(gram.double())
        lam = lam.clamp_min(0)
        wx = p["x_embed.weight"].double() * p["noise_norm.weight"].double()[None, :]
        weight = (wx @ (basis * lam.sqrt()[None, :])).to(embedding.dtype)
        var = (lam / cfg.target_hidden_size).float()
        uniform = rms_norm(self.target_constants(emb_s)[0].to(self.dtype), p["state_norm.weight"], cfg.rms_norm_eps)
        x0 = linear(uniform, p["x_embed.weight"], p["x_embed.bias"]).reshape(-1).to(embedding.dtype)
        fold = (weight, var, x0)
        return (fold, lam, basis) if return_basis else fold

    def folded_noise_input(self, z, fold, gate):
        """The first layer's input from the folded noise (sglang/model.py:945-958):
        ``x0 + (scale * (z @ M)).to(dtype)``, ``scale = gate * rsqrt(sum(var z^2)
        + eps)`` per token in fp32, ``z @ M`` a matmul in the weight's dtype."""
        weight, var, x0 = fold
        mean_square = (z.float().square() * var).sum(-1, keepdim=True)
        scale = gate.float() * torch.rsqrt(mean_square + self.config.rms_norm_eps)
        proj = z.to(weight.dtype) @ weight.T
        return x0 + (scale * proj.float()).to(weight.dtype)

    # -- extend_context, :342-351
    @torch.no_grad()
    def extend_context(self, cache: OracleCache, target_hidden) -> None:
        cfg, p = self.config, self.p
        start, n = cache.length, target_hidden.shape[1]
        context = rms_norm(linear(target_hidden.to(self.dtype), p["fc.weight"]), p["hidden_norm.weight"], cfg.rms_norm_eps)
        positions = torch.arange(start, start + n, device=context.device).expand(context.shape[0], -1)
        rope = rope_tables(positions, self.head_dim, cfg.rope_theta)
        for i in range(cfg.num_hidden_layers):
            cache.write(i, start, *project_kv(p, f"layers.{i}.cross_attn", context, rope, self.heads, cfg.qk_norm_eps))
        cache.length += n

    # -- state vocabulary, :355-376
    def state_vocab(self, embedding, lm_head_w, lm_head_b=None):
        if self.config.state_vocab_size is None:
            return embedding, lm_head_w, lm_head_b
        ids = self.p["draft_ids"]
        return embedding[ids], lm_head_w[ids], None if lm_head_b is None else lm_head_b[ids]

    def token_logits(self, logits):
        if self.config.state_vocab_size is None:
            return logits
        full = logits.new_full((*logits.shape[:-1], self.config.vocab_size), float("-inf"))
        full[..., self.p["draft_ids"]] = logits
        return full

    # -- state featurisation, :378-399
    def mix_state(self, posterior_embeds, state_embeds, s: float, t: float):
        p, cfg = self.p, self.config
        jump = 1.0 if cfg.noise_gate == "constant" else t - s
        gate = (p["noise_gate"].float() * jump).to(self.dtype)
        noise_term = gate * rms_norm(state_embeds.to(self.dtype), p["noise_norm.weight"], cfg.rms_norm_eps)
        return rms_norm(posterior_embeds.to(self.dtype), p["state_norm.weight"], cfg.rms_norm_eps) + noise_term

    def embed_state(self, state, s: float, t: float, embedding):
        if s == 0:
            posterior_embeds = self.target_constants(embedding)[0]
        else:
            posterior = (state.float() * (s / max(1.0 - s, 1e-3) ** 2)).softmax(dim=-1)
            posterior_embeds = posterior.to(embedding.dtype) @ embedding
        return self.mix_state(posterior_embeds, state.to(embedding.dtype) @ embedding, s, t)

    # -- target constants, :401-420
    @torch.no_grad()
    def target_constants(self, embedding):
        key = (embedding.data_ptr(), tuple(embedding.shape), embedding.dtype)
        if key not in self._target_cache:
            vocab = embedding.shape[0]
            uniform = torch.full((1, vocab), 1.0 / vocab, device=embedding.device)
            gram = sum(rows.float().T @ rows.float() for rows in embedding.split(16384))
            factor = torch.linalg.cholesky(gram.cpu().double()).to(embedding.device)
            uniform_embeds = uniform.to(embedding.dtype) @ embedding
            self._target_cache = {key: (uniform_embeds, factor.to(self.dtype))}
        return self._target_cache[key]

    def anchor_context(self, cache: OracleCache, anchor_ids, embedding):
        """Write the anchor row's keys/values at position ``cache.length`` (:451-457)."""
        cfg, p = self.config, self.p
        anchor = cache.length
        rows = embedding[anchor_ids[:, None]].to(self.dtype)
        ctx = rms_norm(linear(rows, p["anchor_proj.weight"], p["anchor_proj.bias"]), p["anchor_norm.weight"], cfg.rms_norm_eps)
        pos = torch.full((anchor_ids.shape[0], 1), anchor, device=anchor_ids.device)
        rope = rope_tables(pos, self.head_dim, cfg.rope_theta)
        for i in range(cfg.num_hidden_layers):
            cache.write(i, anchor, *project_kv(p, f"layers.{i}.cross_attn", ctx, rope, self.heads, cfg.qk_norm_eps))

    # -- draft, :422-479
    @torch.no_grad()
    def draft(self, anchor_ids, cache: OracleCache, embedding, lm_head_w, lm_head_b=None,
              num_steps=None, z=None, noise=None, return_hidden=False, folded=False, noise_fold=None):
        """Draft logits (B, K, V).  The random draws are inputs: ``z`` (B, K, H)
        for a one-step draft (what ``torch.randn`` gives at :465), ``noise``
        (B, K, S) fp32 for a multi-step draft (:469).  ``noise_fold`` (the
        tuple ``fold_noise`` returns) forms a one-step draft's first layer
        input by the folded noise instead."""
        cfg = self.config
        num_steps = num_steps or cfg.num_steps
        if str(num_steps) not in cfg.jump_grids:
            raise ValueError(f"num_steps must be one of {sorted(cfg.jump_grids, key=int)}, got {num_steps}")
        grid = cfg.jump_grids[str(num_steps)]
        batch, block = anchor_ids.shape[0], cfg.block_size
        emb_s, head_w, head_b = self.state_vocab(embedding, lm_head_w, lm_head_b)

        self.anchor_context(cache, anchor_ids, embedding)
        anchor = cache.length
        context = cache.context(anchor + 1)
        positions = anchor + 1 + torch.arange(block, device=anchor_ids.device).expand(batch, -1)

        state = noise
        embedded = None
        if state is None and num_steps == 1 and noise_fold is not None:
            jump = 1.0 if cfg.noise_gate == "constant" else grid[1] - grid[0]
            gate = (self.p["noise_gate"].float() * jump).to(self.dtype)
            embedded, inputs = self.folded_noise_input(z, noise_fold, gate), None
        elif state is None and num_steps == 1:
            uniform_embeds, factor = self.target_constants(emb_s)
            inputs = self.mix_state(uniform_embeds, z.to(factor.dtype) @ factor.T, 0.0, grid[1])
        elif state is None:
            raise ValueError("a multi-step oracle draft needs its starting state as noise=")

        hidden = None
        for s, t, nxt in [(a, b, b) for a, b in zip(grid[:-1], grid[1:])]:
            if state is not None:
                inputs = self.embed_state(state, s, t, emb_s)
            if folded:  # the serving plugins' folded head (no lm_head bias there)
                logits = self.forward(inputs, s, t, positions, context, head=self.fold_head(lm_head_w),
                                      embedded=embedded)
                hidden = None
            else:
                hidden = self.forward(inputs, s, t, positions, context, embedded=embedded).to(head_w.dtype)
                logits = F.linear(hidden, head_w, head_b)
            if nxt < 1.0:
                state = ((1.0 - nxt) * state + (nxt - s) * logits.float().softmax(dim=-1)) / (1.0 - s)
        out = self.token_logits(logits)
        return (out, hidden) if return_hidden else out


# ---------------------------------------------------------------- sampling / acceptance


def greedy_accept(draft_tokens: torch.Tensor, target_logits: torch.Tensor):
    """Greedy acceptance of one row (:579-582): ``draft (1, K)``, ``target_logits
    (1, K+1, V)`` -> (accepted, bonus token)."""
    target_tokens = target_logits.argmax(dim=-1)
    accepted = int((draft_tokens == target_tokens[:, :-1]).cumprod(dim=1).sum())
    return accepted, int(target_tokens[0, accepted])


def greedy_accept_batch(draft_tokens: torch.Tensor, target_logits: torch.Tensor):
    """Row loop of :579-582 over a batch: (B, K), (B, K+1, V) -> accepted (B,), bonus (B,)."""
    acc, bonus = [], []
    for b in range(draft_tokens.shape[0]):
        a, t = greedy_accept(draft_tokens[b : b + 1], target_logits[b : b + 1])
        acc.append(a)
        bonus.append(t)
    return torch.tensor(acc, dtype=torch.int64), torch.tensor(bonus, dtype=torch.int64)


def softmax_probs(logits: torch.Tensor, temperature: float, mode: str) -> torch.Tensor:
    """``softmax(logits.float() / T)`` over the last axis (:556, :584).

    ``mode="torch"`` is the reference's own op; ``mode="fixed"`` is the
    fixed-order ``fm_exp`` softmax of the C oracle, which the CUDA kernels
    reproduce bit for bit.  bf16 and fp32 logits are read as they are (the
    CUDA path reads both natively); other floats widen to fp32."""
    if mode == "torch":
        return (logits.float() / temperature).softmax(dim=-1)
    from . import accept

    native = logits if logits.dtype in (torch.bfloat16, torch.float32) else logits.float()
    return accept.softmax_rows(native, temperature)


# Philox round word of the first target token's draw (sampled from the
# prefill logits): a counter of its own that no decoding round reaches.
PREFILL_ROUND = 0xFFFFFFFF


@torch.no_grad()
def spec_generate(oracle: Oracle, target, input_ids, max_new_tokens=256, temperature=0.0, num_steps=None,
                  stop_token_ids=None, z_source=None, rng_seed=1234, softmax_mode="torch", draft_fn=None):
    """Speculative decoding loop of :514-612 with injected randomness.

    ``z_source(r)`` gives round r's one-step noise (B=1, K, H).  At T > 0 the
    draws are Philox uniforms: draft slot k of round r (k, 0, r, 3) — the
    first target token, sampled from the prefill, has a counter of its own,
    (0, 0, PREFILL_ROUND, 3), which no round reaches — acceptance (k, 0, r, 1)
    and the bonus (0, 0, r, 2), each turned into a token by the oracle's
    categorical sampler (its sliced form for the bonus).  ``draft_fn(anchor,
    r)``, when given, supplies round r's draft logits instead of the oracle's
    drafter (replaying another implementation's drafts through this loop).
    The target may sit on any device; the oracle's arithmetic runs on the CPU.
    Returns ``(sequences, acceptance_lengths)``.""",
    from transformers import DynamicCache

    from . import accept

    cfg = oracle.config
    if input_ids.shape[0] != 1:
        raise ValueError("spec_generate decodes one sequence at a time")
    if stop_token_ids is None:
        eos = target.generation_config.eos_token_id
        stop_token_ids = [] if eos is None else [eos] if isinstance(eos, int) else list(eos)
    stop = torch.tensor(stop_token_ids, dtype=torch.long)
    embedding = target.get_input_embeddings().weight.detach().cpu()
    head = target.get_output_embeddings()
    head_w = head.weight.detach().cpu()
    head_b = None if getattr(head, "bias", None) is None else head.bias.detach().cpu()
    dev = input_ids.device
    K, P = cfg.block_size, input_ids.shape[1]
    rounds = 0

    def sample(logits, r):
        if temperature <= 0:
            return logits.argmax(dim=-1), None
        probs = softmax_probs(logits, temperature, softmax_mode)
        toks = [accept.categorical(probs[0, k].numpy(), accept.uniform(rng_seed, k, 0, r, 3))
                for k in range(probs.shape[1])]
        return torch.tensor(toks, dtype=torch.int64)[None], probs

    layers, feats = target.get_decoder().layers, {}
    hooks = [layers[i].register_forward_hook(
        (lambda i: lambda m, a, o: feats.__setitem__(i, o[0] if isinstance(o, tuple) else o))(i))
        for i in cfg.target_layer_ids]
    features = lambda: torch.cat([feats[i] for i in cfg.target_layer_ids], dim=-1).cpu()  # noqa: E731
    try:
        target_cache = DynamicCache()
        out = target(input_ids, past_key_values=target_cache, use_cache=True, logits_to_keep=1)
        tokens = sample(out.logits[:, -1:].cpu(), PREFILL_ROUND)[0].to(dev)
        cache = OracleCache(cfg, 1, P + max_new_tokens + K + 1, oracle.dtype)
        oracle.extend_context(cache, features())
        lengths = []
        while tokens.shape[1] < max_new_tokens and not torch.isin(tokens[0, -1].cpu(), stop):
            anchor = tokens[:, -1]
            if draft_fn is not None:
                logits = draft_fn(anchor, rounds).cpu()
            else:
                logits = oracle.draft(anchor.cpu(), cache, embedding, head_w, head_b, num_steps=num_steps,
                                      z=z_source(rounds))
            draft, draft_probs = sample(logits, rounds)
            draft = draft.to(dev)
            position = P + tokens.shape[1] - 1
            out = target(torch.cat([anchor[:, None], draft], dim=1),
                         position_ids=torch.arange(position, position + K + 1, device=dev)[None],
                         past_key_values=target_cache, use_cache=True)
            draft = draft.cpu()
            if temperature <= 0:
                tt = out.logits.cpu().argmax(dim=-1)
                accepted = int((draft == tt[:, :-1]).cumprod(dim=1).sum())
                bonus = tt[:, accepted]
            else:
                tp = softmax_probs(out.logits.cpu(), temperature, softmax_mode)[0]
                p = tp[:-1].gather(-1, draft[0, :, None])[:, 0]
                q = draft_probs[0].gather(-1, draft[0, :, None])[:, 0]
                u = torch.tensor([accept.uniform(rng_seed, k, 0, rounds, 1) for k in range(K)])
                accepted = int((u * q < p).cumprod(dim=0).sum())
                residual = tp[accepted]
                if accepted < K:
                    residual = (residual - draft_probs[0, accepted]).clamp_min(0)
                    if residual.sum() <= 0:
                        residual = tp[accepted]
                bonus = torch.tensor([accept.categorical_sliced(residual.numpy(),
                                                                accept.uniform(rng_seed, 0, 0, rounds, 2))])
            rounds += 1
            new = torch.cat([draft[:, :accepted], bonus.view(1, 1)], dim=1).to(dev)
            hits = torch.isin(new[0].cpu(), stop).nonzero()
            if len(hits):
                new = new[:, : int(hits[0]) + 1]
            tokens = torch.cat([tokens, new], dim=1)
            lengths.append(new.shape[1])
            excess = target_cache.get_seq_length() - (position + accepted + 1)
            if excess > 0:
                target_cache.crop(-excess)
            oracle.extend_context(cache, features()[:, : accepted + 1])
    finally:
        for h in hooks:
            h.remove()
    tokens = tokens[:, :max_new_tokens]
    return torch.cat([input_ids, tokens], dim=1), lengths


__all__ = [
    "Oracle",
    "softmax_probs",
    "spec_generate",
    "OracleCache",
    "apply_rope",
    "greedy_accept",
    "greedy_accept_batch",
    "rms_norm",
    "rope_tables",
]
