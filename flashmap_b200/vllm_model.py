"""The vLLM draft-model entry point (flashmap/vllm/model.py) on this library.

``FlashMapDraftModel`` keeps the reference plugin's constructor, attributes
and methods (``load_weights``, ``prepare``, ``set_noise_keys``,
``combine_hidden_states``, ``precompute_and_store_context_kv``,
``defer_context_kv``, ``forward``, ``compute_draft_logits``; ``hot_ids``,
``noise_scale``, ``compile``), reads the same engine objects (the vLLM config,
the forward context's attention metadata, the context-cache attention layers
with their paged ``kv_cache`` tensors) and draws every block with the
library's kernels: the context writer and paged cross-attention of
``serving_ops`` and the GEMM / AdaLN / norm kernels of ``ops`` (``paged_draft``).

vLLM itself is not imported: the engine's objects are read by attribute, so
the model runs inside vLLM or against stand-ins.  ``forward_context`` may be
set to a callable returning the forward context; by default it is vLLM's
``get_forward_context``.  The cache layers are the attention layers of the
context cache; vLLM binds them (``bind_cache_layers``) once it has allocated
the KV cache.

Like the reference plugin, the draft folds both ends (vllm/fold.py:44-100):
the noise is drawn in the embedding's eigenbasis and reaches the first layer
through one projection, and the DiT head is folded into the LM-head rows, so
a draft equals ``FlashMapDraftModel.draft`` with ``fold_noise`` and
``fold_head`` set, of the same context and noise.  Differences from the
reference plugin: ``compile`` is accepted and has no effect (the kernels are already whole; CUDA
graphs capture them); FP8 weights (``FLASHMAP_FP8``) are not built.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable, Iterable, List, NamedTuple, Optional, Sequence, Tuple

import torch
from torch import nn

from . import serving_ops as S
from .modeling_flashmap import FlashMapDraftModel as _HFModel
from .paged_draft import PagedDraft

__all__ = ["ContextLayout", "FlashMapDraftModel", "HeadRun", "attend_runs", "context_layout"]

# FLASHMAP_CONTEXT_CACHE (the reference plugin's switch): "auto" packs on hybrid
# targets only, "layers" never packs, "virtual" packs whenever the target allows.
LAYOUT_MODES = ("auto", "layers", "virtual")


class HeadRun(NamedTuple):
    """Consecutive heads of one DiT layer stored side by side in one cache:
    ``count`` heads from ``head`` on, at head slots ``slot`` .. of cache ``cache``."""

    cache: int
    slot: int
    count: int
    head: int


@dataclass(frozen=True)
class ContextLayout:
    """Placement of the DiT's context keys/values in vLLM's paged caches.

    The DiT's ``layers`` x ``heads`` heads are numbered layer-major (head h of
    layer l is head number l * heads + h) and stored ``per_cache`` to an
    attention cache, in that order, over ``caches`` caches.  Unpacked, each DiT
    layer is its own cache (``per_cache == heads``); packed (``packed``), every
    cache has the page size of the target's full-attention layers and a DiT
    layer's heads may straddle two or more caches (the layout
    flashmap/vllm/context_cache.py describes).  ``why`` says why this layout
    was chosen."""

    layers: int
    heads: int
    caches: int
    per_cache: int
    packed: bool
    why: str

    def where(self, layer: int, head: int) -> Tuple[int, int]:
        """(cache, head slot) of head ``head`` of DiT layer ``layer``."""
        n = layer * self.heads + head
        return n // self.per_cache, n % self.per_cache

    def runs(self, layer: int) -> List[HeadRun]:
        """Layer ``layer``'s heads cut at cache boundaries, in head order."""
        out: List[HeadRun] = []
        first, end = layer * self.heads, (layer + 1) * self.heads
        while first < end:
            cache, slot = divmod(first, self.per_cache)
            count = min(self.per_cache - slot, end - first)
            out.append(HeadRun(cache, slot, count, first - layer * self.heads))
            first += count
        return out


def context_layout(num_layers: int, heads: int, head_dim: int, *, hybrid: bool, target_attention_layers: int,
                   target_kv_heads: int, target_head_size: int, bf16_cache: bool,
                   mode: Optional[str] = None) -> ContextLayout:
    """The context layout for a DiT of ``num_layers`` layers of ``heads``
    heads of ``head_dim``, beside a target with ``target_attention_layers``
    full-attention layers of ``target_kv_heads`` heads of ``target_head_size``.

    Packing pays off on hybrid targets (linear-attention or Mamba layers beside
    full attention), where vLLM sizes every layer's page to the largest one;
    it needs a bf16 cache, a target page that holds whole DiT heads, and
    enough target layers for all the DiT's heads.  Otherwise each DiT layer
    keeps a cache of its own."""
    mode = mode or os.environ.get("FLASHMAP_CONTEXT_CACHE", "auto")
    if mode not in LAYOUT_MODES:
        raise ValueError(f"FLASHMAP_CONTEXT_CACHE is {mode!r}; expected one of {', '.join(LAYOUT_MODES)}")
    page = target_kv_heads * target_head_size  # elements per token of one target attention layer
    fits = page // head_dim if head_dim > 0 and page > 0 and page % head_dim == 0 else 0
    if mode == "layers":
        why = "per-layer caches requested (FLASHMAP_CONTEXT_CACHE=layers)"
    elif mode == "auto" and not hybrid:
        why = "the target has full attention only, so per-layer caches cost no padding"
    elif not bf16_cache:
        why = "packed caches need a bf16 KV cache; per-layer caches hold fp8"
    elif target_attention_layers <= 0 or fits == 0:
        why = (f"a target attention page ({target_kv_heads} x {target_head_size}) holds no whole number of "
               f"DiT heads of size {head_dim}")
    elif target_attention_layers * fits < num_layers * heads:
        why = (f"{num_layers * heads} DiT heads do not fit in {target_attention_layers} target-sized caches of "
               f"{fits} heads")
    else:
        return ContextLayout(num_layers, heads, target_attention_layers, fits, True,
                             f"packed: {num_layers * heads} DiT heads in {target_attention_layers} caches of "
                             f"{fits} heads (the target attention's page)")
    return ContextLayout(num_layers, heads, num_layers, heads, False, why)


def attend_runs(query: torch.Tensor, caches: Sequence[torch.Tensor], runs: Sequence[HeadRun], attend) -> torch.Tensor:
    """A DiT layer's cross-attention over a layout's head runs.

    ``query`` is (tokens, heads, head_dim) and ``caches`` vLLM's paged
    tensors (blocks, heads, block_size, 2 * head_dim).  ``attend(q, c, n)``
    attends ``n`` query heads to the same ``n`` cache heads; it is called once
    per run on views of the run's heads (the whole tensors when the run covers
    both), and the outputs are joined along the heads in run order."""
    heads = query.shape[1]
    outs = []
    for run in runs:
        cache = caches[run.cache]
        q = query if run.count == heads else query[:, run.head:run.head + run.count].contiguous()
        c = cache if run.count == cache.shape[1] else cache[:, run.slot:run.slot + run.count]
        outs.append(attend(q, c, run.count))
    return outs[0] if len(outs) == 1 else torch.cat(outs, dim=1)


def _default_forward_context():
    from vllm.forward_context import get_forward_context  # the engine's, when it runs us

    return get_forward_context()


class FlashMapDraftModel(nn.Module):
    # Scales the starting noise; tests set 0 to compare deterministic drafts.
    noise_scale = 1.0
    # Accepted for the reference's interface; the draft step is already whole kernels.
    compile = True

    def __init__(self, *, vllm_config, prefix: str = "") -> None:
        super().__init__()
        parallel = getattr(vllm_config, "parallel_config", None)
        if int(getattr(parallel, "tensor_parallel_size", 1) or 1) != 1:
            raise ValueError("FlashMap drafting supports tensor parallel size 1 only (its load-time folds read the "
                             "whole target embedding and LM head).")
        if not getattr(vllm_config, "use_v2_model_runner", True):
            raise ValueError("FlashMap drafting needs vLLM's V2 model runner; unset VLLM_USE_V2_MODEL_RUNNER=0.")
        speculative_config = vllm_config.speculative_config
        assert speculative_config is not None
        self.config = config = speculative_config.draft_model_config.hf_config
        self.dtype = vllm_config.model_config.dtype
        if self.dtype != torch.bfloat16:
            raise ValueError(f"FlashMap drafting runs in bfloat16, not {self.dtype}")
        self.max_model_len = int(vllm_config.model_config.max_model_len)
        self.block_size = int(config.block_size)
        self.num_steps = int(os.environ.get("FLASHMAP_NUM_STEPS", config.num_steps))
        why = None if str(self.num_steps) in config.jump_grids else (
            f"no jump grid for {self.num_steps} steps (the checkpoint has {sorted(config.jump_grids, key=int)})")
        if why:
            raise ValueError(why)
        self.cache_plan = self._context_plan(config, vllm_config)
        self.model = _HFModel(config)
        self.vocab_size = int(config.vocab_size)
        self.state_vocab_size = getattr(config, "state_vocab_size", None)
        draft_vocab_size = int(self.state_vocab_size or getattr(config, "draft_vocab_size", None) or self.vocab_size)
        self.d2t: Optional[nn.Parameter] = None
        if draft_vocab_size != self.vocab_size:
            self.d2t = nn.Parameter(torch.zeros(draft_vocab_size, dtype=torch.long), requires_grad=False)
        self.hot_ids: Optional[torch.Tensor] = None
        self.lm_head: Optional[nn.Module] = None  # the target's, attached by the engine
        self.forward_context: Callable = _default_forward_context
        self._cache_layers: Optional[list] = None
        self._pending_context = None
        self._cache_args = None
        self._noise_keys = None
        self._core: Optional[PagedDraft] = None
        self.kv_fp8 = False
        self.kv_scales: Optional[torch.Tensor] = None

    @staticmethod
    def _context_plan(config, vllm_config) -> ContextLayout:
        heads = int(config.num_attention_heads)
        head_dim = int(config.hidden_size) // heads
        model_config = vllm_config.model_config
        hybrid = bool(getattr(model_config, "is_hybrid", False))
        cache_config = getattr(vllm_config, "cache_config", None)
        bf16 = str(getattr(cache_config, "cache_dtype", "auto")) in ("auto", "bfloat16")
        return context_layout(
            int(config.num_hidden_layers), heads, head_dim, hybrid=hybrid,
            target_attention_layers=int(getattr(model_config, "num_attention_layers", 0) or 0),
            target_kv_heads=int(getattr(model_config, "num_kv_heads", 0) or 0),
            target_head_size=int(getattr(model_config, "head_size", 0) or 0), bf16_cache=bf16)

    @property
    def layers(self) -> nn.ModuleList:
        return self.model.layers

    def bind_cache_layers(self, layers: list) -> None:
        """The attention layers (objects with ``kv_cache``, ``layer_name`` and
        ``kv_cache_dtype``) that hold the context, in cache order."""
        if len(layers) != self.cache_plan.caches:
            raise ValueError(f"the context layout has {self.cache_plan.caches} caches, got {len(layers)} layers")
        self._cache_layers = list(layers)
        self._cache_args = None

    @property
    def cache_layers(self) -> list:
        if self._cache_layers is None:
            raise RuntimeError("the context cache layers are not bound yet (bind_cache_layers)")
        return self._cache_layers

    # ------------------------------------------------------------------ loading
    def load_weights(self, weights: Iterable[Tuple[str, torch.Tensor]]) -> set:
        """The checkpoint's weights (vllm/model.py:407-455): the target's
        embedding and head are skipped, ``draft_ids`` or a draft-vocabulary
        ranking (``ids``) set ``d2t``, every other name must match."""
        params = dict(self.named_parameters())
        buffers = dict(self.named_buffers())
        loaded = set()
        for name, tensor in weights:
            if name in ("embed_tokens.weight", "lm_head.weight", "t2d"):
                continue
            if name == "draft_ids":
                if "model.draft_ids" in buffers:
                    buffers["model.draft_ids"].copy_(tensor.to(torch.int64))
                if self.d2t is not None:
                    size = self.d2t.shape[0]
                    ids = tensor.to(torch.int64)
                    self.d2t.data.copy_(ids - torch.arange(size, device=ids.device))
                    loaded.add("d2t")
                continue
            if name in ("ids", "counts"):
                if name == "ids" and self.d2t is not None and not self.state_vocab_size:
                    size = self.d2t.shape[0]
                    hot = tensor[:size].to(torch.int64).sort().values
                    self.d2t.data.copy_(hot - torch.arange(size, device=hot.device))
                    loaded.add("d2t")
                continue
            key = name if name == "d2t" else "model." + name
            param = params.get(key)
            if param is None:
                raise ValueError(f"unexpected FlashMap weight {name!r}")
            if param.shape != tensor.shape:
                raise ValueError(f"FlashMap weight {name!r} has shape {tuple(tensor.shape)}, expected "
                                 f"{tuple(param.shape)}")
            with torch.no_grad():
                param.data.copy_(tensor)
            loaded.add(key)
        shared = ("model.embed_tokens.", "lm_head.")  # the target's, attached by the engine
        missing = {n for n in params if not n.startswith(shared)} - loaded
        if missing:
            raise ValueError(f"FlashMap checkpoint is missing {sorted(missing)}")
        self.model._clear_caches()
        return set(params)

    @torch.no_grad()
    def prepare(self) -> None:
        """Precompute what the draft step needs once the target's embedding
        (``model.embed_tokens``) and LM head (``lm_head``) are attached
        (vllm/model.py:457-607): kernel-layout weights, the jump's AdaLN
        modulations, the rotary table, the noise factor, the draft vocabulary."""
        embed = self.model.embed_tokens.weight[: self.vocab_size]
        head = self.lm_head.weight[: self.vocab_size]
        device = embed.device
        self.hot_ids = None
        if self.d2t is not None:
            self.hot_ids = torch.arange(self.d2t.shape[0], device=device) + self.d2t.to(device)
        self._core = core = PagedDraft(self.model, device, fold_head=True, fold_noise=True)
        core.attach(embed, head, getattr(self.lm_head, "bias", None))
        if self.hot_ids is not None and not self.state_vocab_size:
            # a restricted head over the full state vocabulary: only the LM-head rows are cut
            core.restrict_lm_rows(self.hot_ids)
        self.num_heads, self.head_dim = core.H, core.hd
        self.dim = core.D
        self.softmax_scale = self.head_dim ** -0.5
        self._check_attention()
        self.segments = [self.cache_plan.runs(layer) for layer in range(self.cache_plan.layers)]
        self._jumps = core.jump(self.num_steps)
        self.modulations = [core.modulations(s, t) for s, t, _ in self._jumps]
        self.cos_sin = core.rope_pairs(self.max_model_len + self.block_size + 1)
        self.context_k_norm = core.pack.cross_k_norm

    def _check_attention(self) -> None:
        """bf16 or e4m3 context caches; e4m3 scales from the layers (vllm/model.py:637-676)."""
        if self._cache_layers is None:
            return
        fp8 = set()
        for attn in self._cache_layers:
            kv_dtype = str(getattr(attn, "kv_cache_dtype", "auto"))
            if kv_dtype in ("fp8", "fp8_e4m3"):
                fp8.add(True)
            elif kv_dtype in ("auto", "bfloat16"):
                fp8.add(False)
            else:
                raise ValueError("FlashMap drafting supports a bf16 or fp8_e4m3 draft KV cache, got "
                                 f"kv_cache_dtype={kv_dtype!r}")
        if len(fp8) > 1:
            raise ValueError("the context caches mix bf16 and fp8")
        self.kv_fp8 = fp8 == {True}
        if self.kv_fp8:
            assert not self.cache_plan.packed, "packed context caches need a bf16 cache"
            device = self._core.pack.device

            def scale(attn, name):
                return float(torch.as_tensor(getattr(attn, name, 1.0)).float().reshape(()))

            self.kv_scales = torch.tensor([[scale(a, "_k_scale"), scale(a, "_v_scale")] for a in self._cache_layers],
                                          dtype=torch.float32, device=device)
            self.q_scales = [scale(a, "_q_scale") for a in self._cache_layers]

    def set_noise_keys(self, seeds: torch.Tensor, rows: torch.Tensor) -> None:
        """Key each query row's noise by ``seeds[rows[i]]`` and its position."""
        self._noise_keys = (seeds, rows)

    # ------------------------------------------------------------------ context
    def combine_hidden_states(self, hidden_states: torch.Tensor) -> torch.Tensor:
        return self._require_core().combine(hidden_states)

    def _require_core(self) -> PagedDraft:
        if self._core is None:
            raise RuntimeError("prepare() has not run")
        return self._core

    def cache_layout(self):
        """(pointers, device pointer tensor, (block, head, token, value offset)
        strides, page size) of the context caches, or None before they exist."""
        caches = [attn.kv_cache for attn in self.cache_layers]
        if not all(isinstance(c, torch.Tensor) and c.numel() for c in caches):
            return None
        ptrs = [c.data_ptr() for c in caches]
        if self._cache_args is None or self._cache_args[0] != ptrs:
            expected = (torch.uint8, torch.float8_e4m3fn) if self.kv_fp8 else (torch.bfloat16,)
            if caches[0].dtype not in expected:
                raise ValueError(f"unexpected FlashMap draft KV cache dtype {caches[0].dtype}")
            c0 = caches[0]
            assert c0.stride(3) == 1 and all(c.stride() == c0.stride() for c in caches)
            strides = (c0.stride(0), c0.stride(1), c0.stride(2), self.head_dim)
            ptr_tensor = torch.tensor(ptrs, dtype=torch.int64, device=c0.device)
            self._cache_args = (ptrs, ptr_tensor, strides, c0.shape[2])
        return self._cache_args

    def _write(self, kv: torch.Tensor, positions, slots) -> None:
        layout = self.cache_layout()
        if layout is None:
            return
        _, ptrs, strides, block_size = layout
        S.write_context_kv(kv.view(-1, len(self.layers), 2, self.num_heads, self.head_dim), positions, slots,
                           self.context_k_norm, self.cos_sin, ptrs, strides, block_size, self.config.qk_norm_eps,
                           self.kv_scales, self.cache_plan.per_cache)

    def precompute_and_store_context_kv(self, context_states: torch.Tensor, context_positions: torch.Tensor,
                                        context_slot_mapping: Optional[torch.Tensor] = None) -> None:
        """Context keys/values of ``combine_hidden_states`` rows, written at
        their slots (vllm/model.py:754-763)."""
        kv = self._require_core().context_kv(context_states)
        if context_slot_mapping is not None:
            self._write(kv, context_positions, context_slot_mapping)

    def defer_context_kv(self, context_states: torch.Tensor, context_positions: torch.Tensor,
                         context_slot_mapping: torch.Tensor) -> None:
        """Written by the next ``forward`` together with its anchors."""
        self._pending_context = (context_states, context_positions, context_slot_mapping)

    # ------------------------------------------------------------------ drafting
    def _attend(self, metadata, seqused_k, caches):
        K, core = self.block_size, self._core

        def attend(query: torch.Tensor, layer: int) -> torch.Tensor:
            descales = None
            if self.kv_fp8:
                q_scale = self.q_scales[layer]
                query = (query.float() / q_scale).to(torch.float8_e4m3fn)
                d = torch.stack([self.kv_scales.new_full((), q_scale), self.kv_scales[layer, 0],
                                 self.kv_scales[layer, 1]])
                descales = d[:, None, None].expand(3, seqused_k.shape[0], core.H).contiguous()

            def one(part_query, part_cache, count):
                return S.vllm_paged_cross_attention(part_query, part_cache, metadata.query_start_loc, seqused_k,
                                                    metadata.block_table, None,
                                                    None if descales is None else descales[..., :count].contiguous(),
                                                    K, self.max_model_len, self.softmax_scale, 3)

            return attend_runs(query, caches, self.segments[layer], one)

        return attend

    def forward(self, input_ids: torch.Tensor, positions: torch.Tensor,
                inputs_embeds: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Blocks of ``block_size`` rows, each opened by its request's anchor
        (vllm/model.py:991-1041): the anchors' (and any deferred) context rows
        are written, then the jumps of the DiT over the paged context; returns
        the final AdaLN output ``(tokens, dim)``."""
        del inputs_embeds
        core = self._require_core()
        tokens = input_ids.shape[0]
        K = self.block_size
        blocks = tokens // K
        pending, self._pending_context = self._pending_context, None
        context = self.forward_context()
        metadata = getattr(context, "attn_metadata", None)
        caches = [attn.kv_cache for attn in self.cache_layers]
        slot_positions = positions + 1
        attend = None
        if metadata is not None:
            metadata = metadata[self.cache_layers[0].layer_name]
            anchors = input_ids.view(blocks, K)[:, 0]
            anchor_positions = positions.view(blocks, K)[:, 0]
            slots = metadata.slot_mapping[:tokens].view(blocks, K)[:, 0]
            kv = core.anchor_kv(anchors)
            write_positions = anchor_positions
            if pending is not None:
                states, ctx_positions, ctx_slots = pending
                kv = torch.cat([core.context_kv(states), kv])
                write_positions = torch.cat([ctx_positions, anchor_positions])
                slots = torch.cat([ctx_slots, slots])
            self._write(kv, write_positions, slots)
            seq_lens = metadata.seq_lens
            seqused_k = torch.where(seq_lens > 0, anchor_positions.to(seq_lens.dtype) + 1, 0).to(torch.int32)
            attend = self._attend(metadata, seqused_k, caches)
        if attend is None:  # profiling run: no KV cache yet
            def attend(query, layer):
                return torch.zeros_like(query)

        seeds = rows = None
        if self._noise_keys is not None:
            seeds, rows = self._noise_keys
        p = core.pack

        def self_attention(qkv, layer):
            w = p.layers[layer]
            return S.vllm_block_self_attention(qkv.view(blocks, K, 3, core.H, core.hd), w["self_q_norm"],
                                               w["self_k_norm"], self.cos_sin, slot_positions,
                                               self.config.qk_norm_eps)

        def rotate(q, layer):
            return S.vllm_rms_norm_rope(q, p.layers[layer]["cross_q_norm"], self.cos_sin, slot_positions,
                                        self.config.qk_norm_eps)

        if self.num_steps == 1:
            (s, t, _), = self._jumps
            z = core.noise(tokens, seeds, rows, positions, self.noise_scale)
            return core.dit(core.first_hidden(z, s, t), self.modulations[0], self_attention, rotate, attend)
        # several jumps (the reference algorithm, a vocabulary-sized state;
        # vllm/model.py:1020-1040): the state moves to the next grid time between them
        state = core.state_noise(tokens, seeds, rows, positions, self.noise_scale)
        for step, (s, t, nxt) in enumerate(self._jumps):
            hidden = core.dit(core.embed_state(state, s, t), self.modulations[step], self_attention, rotate, attend)
            if step + 1 < len(self._jumps):
                core.state_update(state, core.jump_logits(hidden), s, nxt)
        return hidden

    def compute_draft_logits(self, hidden_states: torch.Tensor) -> torch.Tensor:
        """Logits over the draft vocabulary (``hot_ids`` when restricted): the
        final AdaLN output times the target's LM-head rows folded with the DiT
        head (vllm/fold.py:76-100)."""
        return self._require_core().draft_logits(hidden_states)
