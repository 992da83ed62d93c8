"""The sglang (DSPARK) draft-model entry point (flashmap/sglang/model.py) on
this library.

``FlashMapDraftModel`` is the HF-path model (its modules and weights, loaded
from a release folder as they are) with sglang's draft protocol: the
constructor ``(config, quant_config=None, prefix="")``, ``load_weights``,
``attach_shared_modules``, ``prepare``, ``head_logits``, ``forward_embed``,
``compute_base_logits``, ``write_target_hidden_kv`` and ``forward``, and the
attributes DSPARK reads (``flashmap``, ``sample_from_anchor``,
``markov_head``, ``gamma``, ``lm_head``, ``hot_ids``, ``folded_head``).  The
draft step runs on the library's kernels (``paged_draft``): the pool writer,
block self-attention, q-norm + RoPE and page-size-1 cross-attention of
``serving_ops``.

sglang is not imported: the KV pool, the request-to-token table and the
forward batch are read by attribute, through the hooks ``token_to_kv_pool``
and ``req_to_token`` (callables; by default sglang's own getters), so the
model runs inside sglang or against stand-ins.

Like the reference plugin, the DiT head is folded into the LM-head rows
(``folded_head`` = (weight, bias), ``lm_head`` holds them and ``head_logits``
applies them to the final AdaLN output; sglang/model.py:449-513), and
``FLASHMAP_FOLDED_NOISE=1`` draws the noise in the embedding's eigenbasis
through one projection (``folded_noise``; sglang/model.py:576-595, 945-958).
Several jumps (``FLASHMAP_NUM_STEPS``) run banked as the reference plugin
does (``jump_bank.py``): a bank of ``FLASHMAP_JUMP_BANK`` noise draws built at
``prepare`` and the earlier predictions cut to their ``FLASHMAP_JUMP_TOPK``
tokens.  ``FLASHMAP_TREE_N`` >= 1 drafts that many candidate blocks per request in
one pass and merges them into the verify tree (``tree_outputs``; the trie in
EAGLE's encoding by ``flashmap_b200.tree.build_tree_abi``; the accepted path's
commit is ``serving_ops.tree_commit``).  Differences from the reference
plugin: the bank's draws and the slots' bank rows and seeds come from Philox
streams, not torch's generator; no FP8 weights; the ``FLASHMAP_COMPILE`` settings are accepted
and have no effect.
"""

from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from typing import Callable, Iterable, Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from . import serving_ops as S
from .modeling_flashmap import FlashMapDraftModel as FlashMapDiT
from .paged_draft import PagedDraft
from .tree import build_tree_abi

logger = logging.getLogger(__name__)

__all__ = ["FlashMapDraftModel", "IdentityMarkov", "LogitsProcessorOutput", "EntryClass"]


@dataclass
class LogitsProcessorOutput:
    """The fields of sglang's ``LogitsProcessorOutput`` the draft step fills."""

    next_token_logits: Optional[torch.Tensor]
    hidden_states: Optional[torch.Tensor]


class IdentityMarkov(nn.Module):
    """DSPARK's Markov head slot: FlashMap drafts every position at once and
    keeps none (sglang/sampler.py's ``IdentityMarkov``)."""

    def __init__(self, vocab_size: int):
        super().__init__()
        self.vocab_size = int(vocab_size)
        self.hot_ids = None


class _Head(nn.Module):
    """What DSPARK reads as the draft's head: rows over the draft vocabulary
    and the full vocabulary size its sampling buffers take."""

    def __init__(self, weight: torch.Tensor, bias, vocab_size: int):
        super().__init__()
        self.register_buffer("weight", weight, persistent=False)
        self.register_buffer("bias", bias, persistent=False)
        self.org_vocab_size = int(vocab_size)


def _default_pool():
    from sglang.srt.model_executor.forward_context import get_token_to_kv_pool

    return get_token_to_kv_pool()


def _default_req_to_token():
    from sglang.srt.model_executor.forward_context import get_req_to_token_pool

    return get_req_to_token_pool().req_to_token


def _env_int(name: str, default) -> int:
    value = os.environ.get(name)
    return int(value) if value not in (None, "") else int(default)


@dataclass(frozen=True)
class _ServeSettings:
    """The sglang plugin's FLASHMAP_* switches (the reference plugin's
    variables and defaults, sglang/model.py:277-312), read once per model."""

    num_steps: int
    folded_noise: bool
    jump_bank: int
    jump_topk: int
    tree_n: int
    tree_budget: int
    draft_vocab: int

    @classmethod
    def read(cls, fm, config) -> "_ServeSettings":
        return cls(num_steps=_env_int("FLASHMAP_NUM_STEPS", fm.num_steps),
                   folded_noise=os.environ.get("FLASHMAP_FOLDED_NOISE", "0") == "1",
                   jump_bank=_env_int("FLASHMAP_JUMP_BANK", 8192),
                   jump_topk=_env_int("FLASHMAP_JUMP_TOPK", 16),
                   tree_n=_env_int("FLASHMAP_TREE_N", 0),
                   tree_budget=_env_int("FLASHMAP_TREE_BUDGET", 32),
                   draft_vocab=_env_int("FLASHMAP_DRAFT_VOCAB", getattr(config, "draft_vocab_size", 0) or 0))


class FlashMapDraftModel(FlashMapDiT):
    # attributes the DSPARK worker reads
    flashmap = True
    uses_own_vocab_modules = False
    supports_pre_gather_target_hidden_projection = False

    def __init__(self, config, quant_config=None, prefix: str = "") -> None:
        del quant_config, prefix
        if getattr(config, "flow_map", True) is False:
            raise ValueError("flow_map is false in this checkpoint: it holds the stage-1 flow, which needs many "
                             "integration steps per block; the plugin serves the distilled flow map")
        super().__init__(config)
        fm = self.config
        opts = _ServeSettings.read(fm, config)
        if str(opts.num_steps) not in fm.jump_grids:
            raise ValueError(f"FLASHMAP_NUM_STEPS={opts.num_steps} has no jump grid in this checkpoint "
                             f"(grids for {', '.join(sorted(fm.jump_grids, key=int))} steps)")
        if opts.tree_n >= 1 and opts.num_steps != 1:
            raise NotImplementedError(f"tree drafting (FLASHMAP_TREE_N={opts.tree_n}) drafts with one jump, "
                                      f"not {opts.num_steps}")
        # the model's shape, as the worker and the draft step read it
        self.block_size = self.gamma = int(fm.block_size)
        self.vocab_size, self.target_hidden_size = fm.vocab_size, fm.target_hidden_size
        self.dim, self.num_heads, self.num_stages = fm.hidden_size, fm.num_attention_heads, fm.num_hidden_layers
        self.rope_theta = fm.rope_theta
        self.rms_norm_eps, self.qk_norm_eps, self.layer_norm_eps = fm.rms_norm_eps, fm.qk_norm_eps, fm.layer_norm_eps
        # DSPARK's protocol: drafts start from the anchor, no Markov or confidence
        # head of their own, no muP logit scaling; the target's modules arrive later
        self.sample_from_anchor = True
        self.markov_head = IdentityMarkov(self.vocab_size)
        self.confidence_head = None
        self.logits_mup_width_multiplier = None
        self.lm_head = self.embedding = self.hot_ids = self.folded_head = None
        # the switches
        self.num_steps = opts.num_steps
        self.folded_noise = opts.folded_noise
        self.jump_bank_size, self.jump_topk = opts.jump_bank, opts.jump_topk
        self.jump_bank = self.head_to_state = None
        self.tree_max_n, self.tree_budget = opts.tree_n, opts.tree_budget
        self.tree_mode = opts.tree_n >= 1
        self.tree_width = self.block_size + 1  # the block and its root
        self._tree_buffers = self._tree_scratch = None
        # the vocabulary the state lives on: the drafter's own (state_vocab_size),
        # else a ranked draft vocabulary of FLASHMAP_DRAFT_VOCAB tokens, else all
        self.state_vocab_size = getattr(fm, "state_vocab_size", None)
        size = self.state_vocab_size or opts.draft_vocab
        self.draft_vocab_size = size if 0 < size < self.vocab_size else 0
        self._vocab_ranking = None
        self.noise_temperature = 1.0  # scales the starting noise (0: deterministic drafts)
        self._core: Optional[PagedDraft] = None
        self._fused_write = None
        self._kv_fp8 = False
        self._noise_offset = 0
        self.token_to_kv_pool: Callable = _default_pool
        self.req_to_token: Callable = _default_req_to_token

    # --- loading -----------------------------------------------------------
    # tensors of a release folder that are not module weights: the draft
    # vocabulary's ranking (kept) and its counts (unused)
    _RANKING_NAMES = ("ids", "draft_vocab_ids")
    _IGNORED_NAMES = ("counts",)

    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> None:
        """Every tensor of the release folder (sglang/model.py:344-403): module
        weights by name, and ``draft_vocab.safetensors``'s token ranking (most
        frequent first).  Unknown names and absent weights raise KeyError."""
        targets = dict(self.named_parameters())
        targets.update(self.named_buffers())
        seen = set()
        for name, tensor in weights:
            if name in self._RANKING_NAMES:
                self._vocab_ranking = tensor
            elif name in self._IGNORED_NAMES:
                pass
            elif name in targets:
                with torch.no_grad():
                    targets[name].copy_(tensor.to(targets[name].dtype))
                seen.add(name)
            else:
                raise KeyError(f"the checkpoint holds {name!r}, which is no FlashMap weight")
        # the Markov head is the plugin's own stand-in and the LM head the target's
        absent = sorted(set(targets) - seen - {n for n in targets if n.split(".")[0] in ("markov_head", "lm_head")})
        if absent:
            raise KeyError(f"the checkpoint lacks FlashMap weights: {absent}")
        self._clear_caches()

    def attach_shared_modules(self, *, embed_tokens: nn.Module, lm_head: nn.Module):
        """The target's embedding and LM head (sglang/model.py:405-425).  A
        head without a weight of its own (tied embeddings) reads the
        embedding.  Both must be the whole (V, target_hidden) matrix."""
        if self.logits_mup_width_multiplier:
            raise NotImplementedError("muP-scaled target logits are not supported by the FlashMap draft")
        emb = embed_tokens.weight.detach()
        head_w = getattr(lm_head, "weight", None)
        head_w = emb if head_w is None else head_w.detach()
        want = (self.vocab_size, self.target_hidden_size)
        for what, w in (("embedding", emb), ("LM head", head_w)):
            if tuple(w.shape) != want:
                raise ValueError(f"the target's {what} has shape {tuple(w.shape)} but the drafter needs {want}: a "
                                 "vocabulary padded or sharded across tensor-parallel ranks cannot be drafted over")
        self.embedding = emb
        self.prepare(head_w)

    @torch.no_grad()
    def prepare(self, lm_head_weight: torch.Tensor) -> None:
        """The draft vocabulary, kernel-layout weights and the jump's constants
        (sglang/model.py:427-473)."""
        state_vocab = bool(self.state_vocab_size and self.draft_vocab_size)
        device = self.embedding.device
        if state_vocab:
            self.hot_ids = self.draft_ids.to(device)
        elif self.draft_vocab_size and self._vocab_ranking is None:
            logger.warning("FlashMap: no draft_vocab.safetensors next to the weights; drafting over the full "
                           "vocabulary")
            self.draft_vocab_size = 0
        elif self.draft_vocab_size:
            ranking = self._vocab_ranking[: self.draft_vocab_size].to(device=device, dtype=torch.int64)
            self.hot_ids = ranking.sort().values
        self._core = core = PagedDraft(self, device, fold_head=True, fold_noise=self.folded_noise)
        core.attach(self.embedding, lm_head_weight)
        if self.hot_ids is not None and not state_vocab:
            core.restrict_lm_rows(self.hot_ids)
        self.folded_head = core.pack.ensure_fold()
        self.lm_head = _Head(*self.folded_head, self.vocab_size)
        self.markov_head.hot_ids = self.hot_ids
        # the drafting head's columns as state rows (a head cut to a draft
        # vocabulary over the full state vocabulary)
        self.head_to_state = self.hot_ids if (self.hot_ids is not None and not state_vocab) else None
        self._jumps = core.jump(self.num_steps)
        self._mods = [core.modulations(s, t) for s, t, _ in self._jumps]
        if self.tree_mode:
            self._tree_buffers = self._alloc_tree_buffers(self._graph_max_bs())
        if self.num_steps > 1:
            grid = self.config.jump_grids[str(self.num_steps)]
            self.jump_bank = core.build_bank(grid, self.jump_bank_size, self.noise_temperature)
            logger.info("FlashMap: %d jumps from a bank of %d noise draws (%.0f MB), predictions cut to %d tokens",
                        self.num_steps, self.jump_bank_size, self.jump_bank.nbytes() / 2**20, self.jump_topk)

    @staticmethod
    def _graph_max_bs() -> int:
        """The largest batch the engine captures draft graphs for (sglang's
        decode CUDA-graph setting when sglang is importable, else 64)."""
        try:
            from sglang.srt.server_args import get_global_server_args

            return int(get_global_server_args().cuda_graph_max_bs or 64)
        except Exception:  # sglang absent or not configured: its default
            return 64

    def _alloc_tree_buffers(self, max_bs: int):
        """The tree a draft step hands to verification, in EAGLE's encoding
        (build_tree_kernel_efficient): per request its W - 1 non-root nodes'
        tokens and ids ``parent * W + index``, the parent list, and (trie nodes,
        distinct candidates) (sglang/model.py:603-620)."""
        width, device = self.tree_width, self._require_core().pack.device

        def zeros(*shape):
            return torch.zeros(*shape, dtype=torch.int64, device=device)

        return zeros(max_bs, width - 1), zeros(max_bs, width - 1), zeros(max_bs, width * (self.block_size - 1) + 1), \
            zeros(max_bs, 2)

    def tree_outputs(self, bsz: int):
        """The tree buffers for a batch of ``bsz``: the persistent ones, or
        (an eager batch above them) scratch ones."""
        buffers = self._tree_buffers
        if bsz > buffers[0].shape[0]:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"capturing a draft graph for {bsz} requests, above the tree buffers")
            if self._tree_scratch is None or self._tree_scratch[0].shape[0] < bsz:
                self._tree_scratch = self._alloc_tree_buffers(bsz)
            buffers = self._tree_scratch
        return tuple(buffer[:bsz] for buffer in buffers)

    def tree_n_for(self, bsz: int) -> int:
        """Candidates per request in a batch of ``bsz``."""
        return max(1, min(self.tree_max_n, self.tree_budget // max(bsz, 1)))

    def _draft_tree(self, hidden: torch.Tensor, bsz: int, n_cand: int) -> None:
        """Greedy tokens of every candidate (the first index of each row's
        maximum), merged into a trie cut to the verify width, written to the
        tree buffers (sglang/model.py:642-659)."""
        core = self._require_core()
        ids, _ = core.top_predictions(core.draft_logits(hidden), 1, self.hot_ids)
        out_tokens, out_ids, out_parents, out_stats = self.tree_outputs(bsz)
        node_tokens, node_ids, stats = build_tree_abi(ids.view(bsz, n_cand, self.block_size), self.tree_width)
        out_tokens.copy_(node_tokens)
        out_ids.copy_(node_ids)
        out_parents[:, 1:node_ids.shape[1] + 1].copy_(node_ids)
        out_stats.copy_(stats)

    def _require_core(self) -> PagedDraft:
        if self._core is None:
            raise RuntimeError("attach_shared_modules() / prepare() has not run")
        return self._core

    def head_logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """The draft-vocabulary logits of the DiT's final AdaLN output through
        the folded head (the target's LM-head rows times the DiT head)."""
        return self._require_core().draft_logits(hidden.reshape(-1, self.dim))

    # --- DSPARK protocol ------------------------------------------------------
    def forward_embed(self, input_ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(input_ids, self.embedding)

    def prune_to_ctx_kv_injection(self) -> None:
        pass

    def compute_base_logits(self, hidden: torch.Tensor):
        return self.head_logits(hidden), None

    def _write_args(self, pool):
        """The pool's per-layer (key, value, strides) table, the stacked k-norm
        weights and the rotary table (sglang/model.py:768-820)."""
        if self._fused_write is not None and self._fused_write[0] == id(pool):
            return self._fused_write[1]
        buffers = [(pool.get_key_buffer(i), pool.get_value_buffer(i)) for i in range(self.num_stages)]
        hd = self.dim // self.num_heads
        for buf in (b for pair in buffers for b in pair):
            if not buf.is_cuda or buf.dtype not in (torch.bfloat16, torch.float8_e4m3fn):
                raise ValueError(f"the FlashMap draft KV pool must be bf16 or fp8_e4m3 on CUDA, got {buf.dtype} "
                                 "(--speculative-draft-kv-cache-dtype)")
            assert buf.shape[1:] == (self.num_heads, hd), buf.shape
            assert buf.stride(1) == hd and buf.stride(2) == 1
        self._kv_fp8 = buffers[0][0].dtype == torch.float8_e4m3fn
        core = self._require_core()
        device = core.pack.device
        meta = torch.tensor([[k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0)] for k, v in buffers],
                            dtype=torch.int64, device=device)
        k_norm = core.pack.cross_k_norm
        rows = max(int(buffers[0][0].shape[0]), int(getattr(self.config, "max_position_embeddings", 0) or 0))
        pairs = core.rope_pairs(rows + self.block_size + 1)
        cos_sin = torch.cat([pairs[..., 0], pairs[..., 1]], dim=-1).contiguous()
        args = (meta, k_norm, cos_sin, self.num_heads * hd, buffers)
        self._fused_write = (id(pool), args)
        return args

    def _kv_write(self, kv, args, positions, locs, **commit) -> None:
        meta, k_norm, cos_sin, kv_size, _ = args
        hd = self.dim // self.num_heads
        write = S.kv_norm_rope_write_fp8 if self._kv_fp8 else S.kv_norm_rope_write
        write(kv, meta, k_norm, cos_sin, positions, locs, self.num_stages, kv_size, hd, self.qk_norm_eps, **commit)

    @torch.no_grad()
    def write_target_hidden_kv(self, *, target_hidden: torch.Tensor, pool, positions: torch.Tensor,
                               cache_loc: torch.Tensor, cache_loc_2d: Optional[torch.Tensor] = None,
                               commit_lens: Optional[torch.Tensor] = None,
                               target_hidden_is_projected: bool = False) -> None:
        """Every layer's context keys/values of the target's features at the
        pool rows ``cache_loc`` (verify windows: only the committed columns of
        ``cache_loc_2d``) (sglang/model.py:687-733)."""
        assert not target_hidden_is_projected
        if target_hidden.shape[0] == 0:
            return
        core = self._require_core()
        args = self._write_args(pool)
        kv = core.context_kv(core.combine(target_hidden))
        if cache_loc_2d is not None and commit_lens is not None:
            self._kv_write(kv, args, positions, cache_loc_2d.reshape(-1), commit_lens=commit_lens,
                           locs_row_width=cache_loc_2d.shape[1])
            return
        self._kv_write(kv, args, positions, cache_loc)

    @torch.no_grad()
    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor, forward_batch,
                input_embeds: Optional[torch.Tensor] = None, get_embedding: bool = False,
                pp_proxy_tensors=None) -> LogitsProcessorOutput:
        """A block for every request; returns the DiT's final hidden states
        (``compute_base_logits`` maps them to logits), the first ``gamma`` of
        each block (sglang/model.py:822-895)."""
        del input_embeds, get_embedding, pp_proxy_tensors
        core = self._require_core()
        bsz, K = forward_batch.batch_size, self.block_size
        gamma = positions.numel() // bsz
        assert gamma <= K, f"--speculative-dspark-block-size {gamma} exceeds the map's block of {K} drafts"
        pool = self.token_to_kv_pool()
        args = self._write_args(pool)
        anchor_positions = positions.view(bsz, gamma)[:, 0]
        block_positions = anchor_positions[:, None] + torch.arange(K, device=positions.device)
        # tree drafting: a request's candidate blocks side by side in the
        # cross-attention's query axis, so its context is read once
        n_cand = self.tree_n_for(bsz) if self.tree_mode else 1
        if self.tree_mode:
            assert gamma == K, "tree drafting verifies the whole block"
        self._kv_write(core.anchor_kv(input_ids.view(bsz, gamma)[:, 0]), args, anchor_positions,
                       forward_batch.out_cache_loc.view(bsz, gamma)[:, 0])
        page_table = self.req_to_token()[forward_batch.req_pool_indices].to(torch.int32)
        cache_seqlens = (forward_batch.seq_lens + 1).to(torch.int32)
        freqs = S.rope_freqs(block_positions + 1, core.hd, self.rope_theta)
        if n_cand > 1:
            freqs = freqs.repeat_interleave(n_cand, dim=0)
        freqs = freqs.contiguous()
        blocks = bsz * n_cand
        keys = [b[0] for b in args[4]]
        values = [b[1] for b in args[4]]
        p = core.pack
        T = blocks * K
        self._noise_offset += 1
        seed = int(torch.initial_seed()) & (2**63 - 1)
        cross = S.sglang_paged_cross_attention_fp8 if self._kv_fp8 else S.sglang_paged_cross_attention

        def self_attention(qkv, layer):
            w = p.layers[layer]
            return S.sglang_block_self_attention(qkv.view(blocks, K, 3, core.H, core.hd), w["self_q_norm"],
                                                 w["self_k_norm"], freqs, self.qk_norm_eps)

        def rotate(q, layer):
            return S.sglang_rms_norm_rope(q.view(blocks, K, core.H, core.hd), p.layers[layer]["cross_q_norm"],
                                          freqs, self.qk_norm_eps)

        def attend(query, layer):
            out = cross(query.view(bsz, n_cand * K, core.H, core.hd), keys[layer], values[layer], cache_seqlens,
                        page_table, cache_seqlens)
            return out.view(blocks, K, core.H, core.hd) if n_cand > 1 else out

        if self.num_steps == 1:
            (s, t, _), = self._jumps
            z = core.noise(T, scale=self.noise_temperature, seed=seed, offset=self._noise_offset)
            hidden = core.dit(core.first_hidden(z, s, t), self._mods[0], self_attention, rotate, attend)
        else:
            # banked jumps (jump_bank.py; sglang/model.py:958-976): no vocabulary-sized
            # state, the predictions between jumps from the drafting head's top-k
            bank = self.jump_bank
            rows, seeds = core.bank_draw(T, bank, seed, self._noise_offset)
            supports = []
            for step, (s, t, _) in enumerate(self._jumps):
                x = (core.bank_first_input(bank, rows, s, t) if step == 0
                     else core.bank_jump_input(bank, step, rows, seeds, supports, s, t))
                hidden = core.dit(x, self._mods[step], self_attention, rotate, attend)
                if step + 1 < self.num_steps:
                    supports.append(core.top_predictions(core.draft_logits(hidden), self.jump_topk,
                                                         self.head_to_state))
        if self.tree_mode:
            self._draft_tree(hidden, bsz, n_cand)
            # the proposer takes one block per request: the first candidate's
            hidden = hidden.view(bsz, n_cand, K, -1)[:, 0].reshape(bsz * K, -1)
        if gamma < K:
            hidden = hidden.view(bsz, K, -1)[:, :gamma].reshape(bsz * gamma, -1)
        return LogitsProcessorOutput(next_token_logits=None, hidden_states=hidden)


EntryClass = [FlashMapDraftModel]
