"""FlashMap drafter on the B200 CUDA path, behind the reference's API.

``FlashMapDraftModel`` keeps the parameters, module names and public methods
of the reference (``flashmap/modeling_flashmap.py``: ``forward`` :302,
``extend_context`` :342, ``draft`` :422, ``spec_generate`` :514), so a release
folder or ``state_dict`` loads unchanged.  Its modules only hold weights:
every computation runs in ``libflashmap_b200.so`` (tcgen05 GEMMs with fused
epilogues, TMA flash cross-attention, Philox sampling and acceptance), with
no PyTorch or CPU fallback.  Weights are served in bf16 on a B200.

Randomness: the one-step draft noise, draft sampling and rejection sampling
use Philox4x32-10 streams instead of torch's generator; the distributions are
the reference's.  The draft noise is keyed by ``generator.initial_seed()`` (or
``torch.initial_seed()``) and a per-call counter; ``spec_generate``'s
sampling and acceptance draws by a key it draws from the generator once per
call (``philox_key``), with one counter word per decoding round and one for
the prefill's token.
"""

from __future__ import annotations

import ctypes
import warnings
import weakref
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch
from torch import nn
from transformers import DynamicCache, PreTrainedModel

from . import _lib, ops
from .configuration_flashmap import FlashMapConfig, jump_times


# ---------------------------------------------------------------- weight holders (no compute)


class FlashMapRMSNorm(nn.Module):
    """Holds the RMSNorm weight of modeling_flashmap.py:69-80."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps


class FlashMapTimeEmbedding(nn.Module):
    """Holds the time-embedding MLP of modeling_flashmap.py:83-97."""

    def __init__(self, config: FlashMapConfig):
        super().__init__()
        self.dim, self.scale = config.time_embed_dim, config.time_scale
        self.linear_1 = nn.Linear(config.time_embed_dim, config.cond_dim)
        self.linear_2 = nn.Linear(config.cond_dim, config.cond_dim)


class FlashMapAdaLayerNorm(nn.Module):
    """Holds the AdaLN modulation linear of modeling_flashmap.py:100-115."""

    def __init__(self, config: FlashMapConfig):
        super().__init__()
        self.linear = nn.Linear(config.cond_dim, 3 * config.hidden_size)
        self.eps = config.layer_norm_eps


class FlashMapAttention(nn.Module):
    """Holds the attention projections and q/k norms of modeling_flashmap.py:118-147."""

    def __init__(self, config: FlashMapConfig):
        super().__init__()
        dim = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = dim // self.num_heads
        self.q_proj = nn.Linear(dim, dim, bias=False)
        self.k_proj = nn.Linear(dim, dim, bias=False)
        self.v_proj = nn.Linear(dim, dim, bias=False)
        self.o_proj = nn.Linear(dim, dim, bias=False)
        self.q_norm = FlashMapRMSNorm(self.head_dim, config.qk_norm_eps)
        self.k_norm = FlashMapRMSNorm(self.head_dim, config.qk_norm_eps)


class FlashMapMLP(nn.Module):
    """Holds the GELU or SwiGLU MLP weights of modeling_flashmap.py:150-169."""

    def __init__(self, config: FlashMapConfig):
        super().__init__()
        self.mlp_type = getattr(config, "mlp_type", "gelu")
        dim, hidden = config.hidden_size, config.intermediate_size
        if self.mlp_type == "swiglu":
            self.gate_up_proj = nn.Linear(dim, 2 * hidden, bias=False)
            self.down_proj = nn.Linear(hidden, dim, bias=False)
        else:
            self.fc1 = nn.Linear(dim, hidden)
            self.fc2 = nn.Linear(hidden, dim)


class FlashMapLayer(nn.Module):
    """Holds one DiT block (modeling_flashmap.py:172-192)."""

    def __init__(self, config: FlashMapConfig):
        super().__init__()
        self.self_attn_adaln = FlashMapAdaLayerNorm(config)
        self.self_attn = FlashMapAttention(config)
        self.cross_attn_adaln = FlashMapAdaLayerNorm(config)
        self.cross_attn = FlashMapAttention(config)
        self.mlp_adaln = FlashMapAdaLayerNorm(config)
        self.mlp = FlashMapMLP(config)


# ---------------------------------------------------------------- cache and outputs


class FlashMapCache:
    """Cross-attention keys and values of the drafter's context for every layer
    (modeling_flashmap.py:195-219): ``kv`` (L, 2, B, heads, max_length, head_dim).

    ``length`` is the number of verified positions (a host int, as in the
    reference); ``lengths`` is its per-sequence device mirror that the CUDA
    kernels read, so sequences of one cache may also have ragged lengths.
    Position ``length`` is the anchor's: drafting writes it, the next
    ``extend_context`` overwrites it."""

    def __init__(self, config: FlashMapConfig, batch_size: int, max_length: int, device=None, dtype=None):
        head_dim = config.hidden_size // config.num_attention_heads
        shape = (config.num_hidden_layers, 2, batch_size, config.num_attention_heads, max_length, head_dim)
        self.kv = torch.zeros(shape, device=device, dtype=dtype)
        self.lengths = torch.zeros(batch_size, device=self.kv.device, dtype=torch.int32)
        self._length = 0

    @property
    def length(self) -> int:
        return self._length

    @length.setter
    def length(self, value: int) -> None:
        self._length = int(value)
        self.lengths.fill_(self._length)

    @property
    def max_length(self) -> int:
        return self.kv.shape[4]

    def write(self, layer: int, start: int, keys: torch.Tensor, values: torch.Tensor) -> None:
        end = start + keys.shape[2]
        if end > self.kv.shape[4]:
            raise ValueError(f"FlashMapCache holds {self.kv.shape[4]} positions, writing up to {end}")
        self.kv[layer, 0, :, :, start:end] = keys
        self.kv[layer, 1, :, :, start:end] = values

    def context(self, end: int) -> list:
        return [(kv[0, :, :, :end], kv[1, :, :, :end]) for kv in self.kv]


@dataclass
class FlashMapGenerateOutput:
    """``sequences`` (1, length): prompt and generated tokens; ``acceptance_lengths``:
    tokens committed per target forward (modeling_flashmap.py:222-236)."""

    sequences: torch.LongTensor
    num_new_tokens: int
    acceptance_lengths: list = field(default_factory=list)

    @property
    def acceptance_length(self) -> float:
        return sum(self.acceptance_lengths) / max(len(self.acceptance_lengths), 1)


# ---------------------------------------------------------------- device packs and plans


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_handle():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class _Pack:
    """Weights in the kernels' layout on one device; the target's constants
    (embedding, lm_head rows, Cholesky factor) are attached separately."""

    def __init__(self, model: "FlashMapDraftModel", device: torch.device):
        cfg = model.config
        if device.type != "cuda":
            raise ValueError("the FlashMap CUDA path runs on a CUDA device")
        _lib.require_device()
        bf = torch.bfloat16
        sd = {k: v.detach() for k, v in model.state_dict().items()}

        def w(name):
            return sd[name].to(device, bf).contiguous()

        D, L = cfg.hidden_size, cfg.num_hidden_layers
        I = cfg.intermediate_size
        self.swiglu = cfg.mlp_type == "swiglu"
        self.layers = []
        for i in range(L):
            p = f"layers.{i}"
            lw = {
                "self_qkv_w": torch.cat([w(f"{p}.self_attn.{n}_proj.weight") for n in "qkv"]).contiguous(),
                "self_o_w": w(f"{p}.self_attn.o_proj.weight"),
                "self_q_norm": w(f"{p}.self_attn.q_norm.weight"),
                "self_k_norm": w(f"{p}.self_attn.k_norm.weight"),
                "cross_q_w": w(f"{p}.cross_attn.q_proj.weight"),
                "cross_o_w": w(f"{p}.cross_attn.o_proj.weight"),
                "cross_q_norm": w(f"{p}.cross_attn.q_norm.weight"),
            }
            if self.swiglu:
                gu = w(f"{p}.mlp.gate_up_proj.weight")
                # 64 gate rows then the matching 64 up rows in every 128-row tile
                lw["mlp_w1"] = torch.stack([gu[:I].view(I // 64, 64, D), gu[I:].view(I // 64, 64, D)], dim=1)
                lw["mlp_w1"] = lw["mlp_w1"].reshape(2 * I, D).contiguous()
                lw["mlp_b1"] = None
                lw["mlp_w2"] = w(f"{p}.mlp.down_proj.weight")
                lw["mlp_b2"] = None
            else:
                lw["mlp_w1"] = w(f"{p}.mlp.fc1.weight")
                lw["mlp_b1"] = w(f"{p}.mlp.fc1.bias")
                lw["mlp_w2"] = w(f"{p}.mlp.fc2.weight")
                lw["mlp_b2"] = w(f"{p}.mlp.fc2.bias")
            self.layers.append(lw)
        self.g = {n: w(n) for n in ("fc.weight", "hidden_norm.weight", "anchor_proj.weight", "anchor_proj.bias",
                                    "anchor_norm.weight", "state_norm.weight", "noise_norm.weight", "x_embed.weight",
                                    "x_embed.bias", "head.weight", "head.bias")}
        self.cross_kv_w = torch.cat(
            [torch.cat([w(f"layers.{i}.cross_attn.k_proj.weight"), w(f"layers.{i}.cross_attn.v_proj.weight")])
             for i in range(L)]).contiguous()
        self.cross_k_norm = torch.stack([w(f"layers.{i}.cross_attn.k_norm.weight") for i in range(L)]).contiguous()
        self.noise_gate = float(sd["noise_gate"].float().reshape(-1)[0])
        self.time = {n: w(n) for n in sd if n.startswith(("time_embed.", "jump_embed."))}
        norms = [f"layers.{i}.{n}" for i in range(L) for n in ("self_attn_adaln", "cross_attn_adaln", "mlp_adaln")]
        norms.append("final_adaln")
        self.mod_w = torch.cat([w(f"{n}.linear.weight") for n in norms]).contiguous()
        self.mod_b = torch.cat([w(f"{n}.linear.bias") for n in norms]).contiguous()
        self.draft_ids_param = sd.get("draft_ids")
        self.S = cfg.state_vocab_size or cfg.vocab_size
        self.target_key = None
        self.embed = self.lm_w = self.lm_b = self.draft_ids = None
        self.lm_fold_w = self.lm_fold_b = None
        self.noise_fold = None
        self.embed_state_t = self.uniform_embeds = self.chol = None
        self.rope_len = 0
        self.rope_cos = self.rope_sin = None
        self.mods = {}
        self.device = device

    def attach_target(self, embedding: torch.Tensor, head_w: torch.Tensor, head_b) -> bool:
        """The target's side (modeling_flashmap.py:355-368, 401-420); True when it changed."""
        key = (embedding.data_ptr(), head_w.data_ptr(), None if head_b is None else head_b.data_ptr(),
               tuple(embedding.shape), embedding.device)
        if key == self.target_key:
            return False
        dev, bf = self.device, torch.bfloat16
        self.embed = embedding.detach().to(dev, bf).contiguous()
        if self.draft_ids_param is not None:
            self.draft_ids = self.draft_ids_param.to(dev, torch.int64).contiguous()
            e_s = self.embed[self.draft_ids].contiguous()
            self.lm_w = head_w.detach().to(dev, bf)[self.draft_ids].contiguous()
            self.lm_b = None if head_b is None else head_b.detach().to(dev, bf)[self.draft_ids].contiguous()
        else:
            e_s = self.embed
            self.lm_w = head_w.detach().to(dev, bf).contiguous()
            self.lm_b = None if head_b is None else head_b.detach().to(dev, bf).contiguous()
        self.S = e_s.shape[0]
        self.lm_rows_full = (self.lm_w, self.lm_b)  # before any plugin cuts the head to a draft vocabulary
        self.lm_fold_w = self.lm_fold_b = None
        self.noise_fold = None
        self.embed_state_t = ops.transpose(e_s)  # E_S^T [H, S]
        uniform = torch.full((1, self.S), 1.0 / self.S, device=dev).to(bf)
        self.uniform_embeds = ops.gemm(self.embed_state_t, uniform).reshape(-1).contiguous()
        gram = ops.gemm(self.embed_state_t, self.embed_state_t, ops.F32)  # E_S^T E_S, fp32 accumulation
        # the (H, H) factor in float64 on the host, as the reference does (:416-419)
        factor = torch.linalg.cholesky(gram.cpu().double())
        self.chol = factor.to(dev, bf).contiguous()
        self.target_key = key
        return True

    def ensure_fold(self):
        """The folded head of the serving plugins (vllm/fold.py:76-100,
        sglang/model.py:515-531): ``lm_w @ head_w`` [S, D] and ``lm_w @ head_b``
        [S], fp32 accumulation rounded to bf16, once per attached target."""
        if self.lm_fold_w is None:
            self.lm_fold_w, self.lm_fold_b = self.fold_rows(self.lm_w)
        return self.lm_fold_w, self.lm_fold_b

    def fold_rows(self, rows_w: torch.Tensor):
        """``rows_w @ head_w`` [R, D] and ``rows_w @ head_b`` [R] (fp32
        accumulation, bf16) for LM-head rows ``rows_w`` [R, Ht]."""
        head_t = ops.transpose(self.g["head.weight"])  # [D, Ht]
        w = ops.gemm(head_t, rows_w).contiguous()
        b = ops.gemm(self.g["head.bias"].view(1, -1).contiguous(), rows_w)  # [R, 1]
        return w, b.reshape(-1).contiguous()

    def ensure_noise_fold(self, cfg):
        """The serving plugins' eigen-folded noise (vllm/fold.py:44-73,
        sglang/model.py:576-595), once per attached target: with
        ``E_S^T E_S = Q diag(lam) Q^T`` (the Gram matrix in fp32 accumulation,
        its eigen-decomposition in float64 on the device, negative round-off
        eigenvalues clamped to 0), the weight ``W_x diag(w_noise) Q diag(sqrt
        lam)`` [D, Ht] (float64 product rounded to bf16), ``lam / Ht`` [Ht]
        (fp32) and ``x_embed(state_norm(uniform_embeds))`` [D] (bf16, the
        reference's bf16 norm and linear)."""
        if self.noise_fold is None:
            g = self.g
            gram = ops.gemm(self.embed_state_t, self.embed_state_t, ops.F32)  # E_S^T E_S
            lam, basis = torch.linalg.eigh(gram.double())
            lam = lam.clamp_min(0)
            wx = g["x_embed.weight"].double() * g["noise_norm.weight"].double()[None, :]
            weight = (wx @ (basis * lam.sqrt()[None, :])).to(torch.bfloat16).contiguous()
            var = (lam / cfg.target_hidden_size).float().contiguous()
            uniform = ops.rmsnorm(self.uniform_embeds.view(1, -1), g["state_norm.weight"], cfg.rms_norm_eps)
            x0 = ops.gemm(g["x_embed.weight"], uniform, ops.STORE, bias=g["x_embed.bias"]).reshape(-1).contiguous()
            self.noise_fold = (weight, var, x0)
        return self.noise_fold

    def ensure_rope(self, cfg, max_pos: int):
        if max_pos > self.rope_len:
            n = max(max_pos, 2 * self.rope_len, 4096)
            self.rope_cos, self.rope_sin = ops.rope_table(n, cfg.hidden_size // cfg.num_attention_heads,
                                                          cfg.rope_theta, self.device)
            self.rope_len = n
            return True
        return False

    def modulations(self, cfg, s: float, t: float) -> torch.Tensor:
        """AdaLN (scale, shift, gate) rows of every norm for the jump s -> t
        (modeling_flashmap.py:287-300), cached per (s, t)."""
        key = (float(s), float(t))
        if key not in self.mods:
            sin = ops.time_sinusoid(cfg.time_embed_dim, s, t, cfg.time_scale, self.device)
            embs = []
            for row, name in ((0, "time_embed"), (1, "jump_embed")):
                h = ops.gemm(self.time[f"{name}.linear_1.weight"], sin[row : row + 1].contiguous(),
                             bias=self.time[f"{name}.linear_1.bias"])
                h = ops.gemm(self.time[f"{name}.linear_2.weight"], ops.silu(h), bias=self.time[f"{name}.linear_2.bias"])
                embs.append(h)
            cond = ops.silu(ops.add(embs[0], embs[1]))
            self.mods[key] = ops.gemm(self.mod_w, cond, bias=self.mod_b).reshape(-1).contiguous()
        return self.mods[key]

    def noise_gate_value(self, cfg, s: float, t: float) -> float:
        """``bf16(noise_gate * (t - s))`` in fp32 arithmetic (modeling_flashmap.py:396-397)."""
        jump = 1.0 if cfg.noise_gate == "constant" else t - s
        g = np.float32(self.noise_gate) * np.float32(jump)
        return float(torch.tensor(float(g), dtype=torch.float32).to(torch.bfloat16).float())


class _Plan:
    """A ``fm_plan`` over one cache, batch and number of jumps, with its workspace."""

    def __init__(self, model: "FlashMapDraftModel", pack: _Pack, cache: FlashMapCache, batch: int, num_steps: int,
                 max_extend_rows: int, launch_mode: int = _lib.LAUNCH_AUTO):
        cfg = model.config
        lib = _lib.load()
        grid = cfg.jump_grids[str(num_steps)]
        self.jumps_py = jump_times(grid)
        self.mods = [pack.modulations(cfg, s, t) for s, t, _ in self.jumps_py]
        jumps = (_lib.Jump * num_steps)()
        for i, ((s, t, nxt), mods) in enumerate(zip(self.jumps_py, self.mods)):
            jumps[i].mods = mods.data_ptr()
            jumps[i].noise_gate = pack.noise_gate_value(cfg, s, t)
            jumps[i].s = s
            jumps[i].next = nxt
        self._jumps = jumps
        L = cfg.num_hidden_layers
        layers = (_lib.LayerWeights * L)()
        for i, lw in enumerate(pack.layers):
            for name, t in lw.items():
                setattr(layers[i], name, None if t is None else t.data_ptr())
        self._layers = layers
        d = _lib.ModelDesc()
        d.hidden, d.heads = cfg.hidden_size, cfg.num_attention_heads
        d.head_dim = cfg.hidden_size // cfg.num_attention_heads
        d.inter, d.layers = cfg.intermediate_size, L
        d.target_hidden, d.n_target_layers = cfg.target_hidden_size, len(cfg.target_layer_ids)
        d.block, d.vocab, d.state_vocab = cfg.block_size, cfg.vocab_size, pack.S
        d.swiglu = 1 if pack.swiglu else 0
        d.rms_eps, d.qk_eps, d.ln_eps = cfg.rms_norm_eps, cfg.qk_norm_eps, cfg.layer_norm_eps
        g = pack.g
        d.fc_w, d.hidden_norm_w = g["fc.weight"].data_ptr(), g["hidden_norm.weight"].data_ptr()
        d.anchor_proj_w, d.anchor_proj_b = g["anchor_proj.weight"].data_ptr(), g["anchor_proj.bias"].data_ptr()
        d.anchor_norm_w, d.noise_norm_w = g["anchor_norm.weight"].data_ptr(), g["noise_norm.weight"].data_ptr()
        d.x_embed_w, d.x_embed_b = g["x_embed.weight"].data_ptr(), g["x_embed.bias"].data_ptr()
        d.head_w, d.head_b = g["head.weight"].data_ptr(), g["head.bias"].data_ptr()
        d.cross_kv_w, d.cross_k_norm = pack.cross_kv_w.data_ptr(), pack.cross_k_norm.data_ptr()
        d.layer = layers
        ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        d.embed, d.lm_w, d.lm_b, d.draft_ids = ptr(pack.embed), ptr(pack.lm_w), ptr(pack.lm_b), ptr(pack.draft_ids)
        d.embed_state_t, d.chol, d.uniform_embeds = ptr(pack.embed_state_t), ptr(pack.chol), ptr(pack.uniform_embeds)
        d.state_norm_w = g["state_norm.weight"].data_ptr()
        d.rope_cos, d.rope_sin, d.rope_len = pack.rope_cos.data_ptr(), pack.rope_sin.data_ptr(), pack.rope_len
        self.folded = bool(getattr(model, "fold_head", False)) and pack.lm_w is not None
        if self.folded:
            fw, fb = pack.ensure_fold()
            d.lm_fold_w, d.lm_fold_b = fw.data_ptr(), fb.data_ptr()
        self.noise_folded = bool(getattr(model, "fold_noise", False)) and num_steps == 1 and pack.chol is not None
        if self.noise_folded:
            nw, nv, nx = pack.ensure_noise_fold(cfg)
            d.noise_fold_w, d.noise_fold_var, d.noise_fold_x0 = nw.data_ptr(), nv.data_ptr(), nx.data_ptr()
        self.desc = d
        c = _lib.PlanConfig()
        c.batch, c.num_steps, c.jumps = batch, num_steps, jumps
        c.cache = cache.kv.data_ptr()
        c.cache_batch, c.cache_len = cache.kv.shape[2], cache.kv.shape[4]
        c.max_extend_rows = max_extend_rows
        c.launch_mode = launch_mode
        self.cfg = c
        size = ctypes.c_size_t(0)
        _lib.check(lib.fm_plan_workspace_size(ctypes.byref(d), ctypes.byref(c), ctypes.byref(size)), "plan size")
        self.workspace = torch.zeros(size.value, dtype=torch.uint8, device=pack.device)
        handle = ctypes.c_void_p()
        _lib.check(lib.fm_plan_create(ctypes.byref(d), ctypes.byref(c), _ptr(self.workspace), size.value,
                                      ctypes.byref(handle)), "fm_plan_create")
        self.handle = handle
        self.batch, self.num_steps, self.max_extend_rows = batch, num_steps, max_extend_rows
        self.launch_mode = launch_mode
        self.target_key = pack.target_key
        self.pack = pack
        self.cache = cache
        err_ptr = lib.fm_plan_error_word(handle)
        base = self.workspace.data_ptr()
        self.err = self.workspace[err_ptr - base : err_ptr - base + 4].view(torch.int32)

    def __del__(self):
        try:
            if getattr(self, "handle", None) is not None:
                _lib.load().fm_plan_destroy(self.handle)
        except Exception:
            pass

    def draft(self, anchor_ids, seed: int, offset: int, logits=None, ldl=0, scatter=False, tokens=None, z=None,
              noise=None, hidden=None, offset_dev=None):
        io = _lib.DraftIO()
        io.offset_ptr = None if offset_dev is None else offset_dev.data_ptr()
        io.anchor_ids, io.lengths = anchor_ids.data_ptr(), self.cache.lengths.data_ptr()
        io.z = None if z is None else z.data_ptr()
        io.noise = None if noise is None else noise.data_ptr()
        io.seed, io.offset = seed & 0xFFFFFFFFFFFFFFFF, offset & 0xFFFFFFFF
        io.logits = None if logits is None else logits.data_ptr()
        io.ldl, io.scatter = ldl, 1 if scatter else 0
        io.tokens = None if tokens is None else tokens.data_ptr()
        io.hidden = None if hidden is None else hidden.data_ptr()
        _lib.check(_lib.load().fm_draft(self.handle, ctypes.byref(io), _stream_handle()), "fm_draft")

    def forward(self, inputs, positions, ctx_last, mods, hidden):
        io = _lib.ForwardIO()
        io.inputs, io.positions, io.ctx_last = inputs.data_ptr(), positions.data_ptr(), ctx_last.data_ptr()
        io.mods, io.hidden = mods.data_ptr(), hidden.data_ptr()
        _lib.check(_lib.load().fm_forward(self.handle, ctypes.byref(io), _stream_handle()), "fm_forward")

    def extend(self, hidden_rows, cu_rows, batch: int):
        io = _lib.ExtendIO()
        io.target_hidden, io.rows = hidden_rows.data_ptr(), hidden_rows.shape[0]
        io.cu_rows, io.lengths, io.batch = cu_rows.data_ptr(), self.cache.lengths.data_ptr(), batch
        _lib.check(_lib.load().fm_extend_context(self.handle, ctypes.byref(io), _stream_handle()), "fm_extend_context")

    def lm_head(self, logits=None) -> None:
        """Launch the LM-head GEMM of the plan alone (timing the pass's largest kernel)."""
        _lib.check(_lib.load().fm_plan_lm_head(self.handle, _ptr(logits), 0 if logits is None else logits.shape[-1],
                                               _stream_handle()), "fm_plan_lm_head")

    def last_launches(self) -> int:
        return int(_lib.load().fm_plan_last_launches(self.handle))

    def check_device_errors(self):
        code = int(self.err.item())
        if code:
            raise _lib.FlashMapError(f"a FlashMap kernel reported device error {code} (index or wait)")


# ---------------------------------------------------------------- sampled decoding's randomness

# Philox round word of the first target token's draw in spec_generate (the
# token sampled from the prefill logits): a counter of its own, which no
# decoding round (words 0, 1, 2, ...) reaches, so that the anchor and the
# first round's draft are independent draws.
PREFILL_ROUND = 0xFFFFFFFF


def philox_key(generator: Optional[torch.Generator] = None) -> int:
    """The 63-bit Philox key of one ``spec_generate`` call, drawn from
    ``generator`` (or torch's default CPU generator).  The draw advances the
    generator, as the reference's ``torch.rand`` / ``torch.multinomial``
    draws do (modeling_flashmap.py:557, :587, :594): two calls with one
    generator use fresh randomness, and a generator seeded alike reproduces
    a call."""
    device = generator.device if generator is not None else "cpu"
    return int(torch.randint(0, 2 ** 63 - 1, (1,), generator=generator, device=device, dtype=torch.int64).item())


# ---------------------------------------------------------------- the model


class FlashMapDraftModel(PreTrainedModel):
    config_class = FlashMapConfig
    base_model_prefix = "flashmap"
    _no_split_modules = ["FlashMapLayer"]
    _supports_sdpa = True

    def __init__(self, config: FlashMapConfig):
        super().__init__(config)
        dim, target_dim = config.hidden_size, config.target_hidden_size
        self.head_dim = dim // config.num_attention_heads
        self.fc = nn.Linear(len(config.target_layer_ids) * target_dim, dim, bias=False)
        self.hidden_norm = FlashMapRMSNorm(dim, config.rms_norm_eps)
        self.anchor_proj = nn.Linear(target_dim, dim)
        self.anchor_norm = FlashMapRMSNorm(dim, config.rms_norm_eps)
        self.state_norm = FlashMapRMSNorm(target_dim, config.rms_norm_eps)
        self.noise_norm = FlashMapRMSNorm(target_dim, config.rms_norm_eps)
        self.noise_gate = nn.Parameter(torch.ones(1))
        self.x_embed = nn.Linear(target_dim, dim)
        self.time_embed = FlashMapTimeEmbedding(config)
        self.jump_embed = FlashMapTimeEmbedding(config)
        self.layers = nn.ModuleList(FlashMapLayer(config) for _ in range(config.num_hidden_layers))
        self.final_adaln = FlashMapAdaLayerNorm(config)
        self.head = nn.Linear(dim, target_dim)
        if getattr(config, "state_vocab_size", None) is not None:
            self.register_buffer("draft_ids", torch.arange(config.state_vocab_size))
        self._clear_caches()
        self.post_init()

    # values derived from the weights are rebuilt after a move or a reload (:271-285)
    # launch_mode: "kernels" runs a draft as the kernel sequence (one launch per
    # operation); "stream" runs a batch-1, one-jump draft as the streamed
    # single-launch pass (plan creation raises for other shapes); "auto" picks
    # the streamed pass where it applies.
    # fold_head: the serving plugins' fast mode (vllm/fold.py:76-100): the DiT
    # head folded into the LM-head rows, one [S, D] projection of the final
    # AdaLN output instead of the head and the [S, Ht] LM head (0.64 GB less
    # per config-2 draft).  It changes rounding, so it is off by default and
    # outside parity with the HF path.
    fold_head = False
    # fold_noise: the serving plugins' eigen-folded noise (vllm/fold.py:44-73,
    # sglang/model.py:576-595), one-jump drafts only: the first layer's input
    # from one [D, Ht] projection of the noise and a per-token scale, instead
    # of the [Ht, Ht] Cholesky factor, the noise and state norms and x_embed.
    # Same distribution from other draws: off by default, outside parity.
    fold_noise = False
    launch_mode = "auto"

    def _clear_caches(self) -> None:
        self._packs, self._plans, self._counter = {}, {}, 0
        if not hasattr(self, "_caches"):
            self._caches = weakref.WeakSet()

    def _apply(self, fn, *args, **kwargs):
        self._clear_caches()
        return super()._apply(fn, *args, **kwargs)

    def load_state_dict(self, *args, **kwargs):
        self._clear_caches()
        return super().load_state_dict(*args, **kwargs)

    # -------------------------------------------------------------- internals
    def _pack(self, device, embed_tokens=None, lm_head=None) -> _Pack:
        device = torch.device(device)
        pack = self._packs.get(device)
        if pack is None:
            pack = self._packs[device] = _Pack(self, device)
        if embed_tokens is not None:
            if pack.attach_target(embed_tokens.weight, lm_head.weight, getattr(lm_head, "bias", None)):
                self._plans = {k: v for k, v in self._plans.items() if k[-1] != device}
        return pack

    def _plan(self, pack: _Pack, cache: FlashMapCache, batch: int, num_steps: int, extend_rows: int = 0) -> _Plan:
        max_pos = cache.max_length + self.config.block_size + 2
        if pack.ensure_rope(self.config, max_pos):
            self._plans = {}
        mode = {"auto": _lib.LAUNCH_AUTO, "kernels": _lib.LAUNCH_KERNELS, "stream": _lib.LAUNCH_STREAM}[self.launch_mode]
        key = (cache.kv.data_ptr(), tuple(cache.kv.shape), batch, num_steps, mode, bool(self.fold_head),
               bool(self.fold_noise), pack.device)
        plan = self._plans.get(key)
        if plan is None or plan.max_extend_rows < extend_rows or plan.target_key != pack.target_key:
            rows = max(extend_rows, 2 * (plan.max_extend_rows if plan else 0), 64)
            plan = _Plan(self, pack, cache, batch, num_steps, rows, mode)
            self._plans[key] = plan
        return plan

    def _any_plan(self, pack, cache, extend_rows):
        for key, plan in self._plans.items():
            if (key[0] == cache.kv.data_ptr() and key[1] == tuple(cache.kv.shape) and key[-1] == pack.device
                    and plan.max_extend_rows >= extend_rows and plan.target_key == pack.target_key):
                return plan
        return self._plan(pack, cache, cache.kv.shape[2], self.config.num_steps, extend_rows)

    def _seed(self, generator) -> tuple:
        seed = generator.initial_seed() if generator is not None else torch.initial_seed()
        self._counter += 1
        return int(seed), self._counter

    def _check_cache(self, cache: FlashMapCache):
        if cache.kv.dtype != torch.bfloat16 or not cache.kv.is_cuda:
            raise ValueError("the FlashMap CUDA path serves bf16 caches on a CUDA device")

    def _steps(self, num_steps):
        num_steps = num_steps or self.config.num_steps
        if str(num_steps) not in self.config.jump_grids:
            supported = ", ".join(sorted(self.config.jump_grids, key=int))
            raise ValueError(f"num_steps must be one of {supported} (the config's jump_grids), got {num_steps}")
        return int(num_steps)

    # -------------------------------------------------------------- public API
    @torch.no_grad()
    def extend_context(self, cache: FlashMapCache, target_hidden: torch.Tensor, embed_tokens=None,
                       lm_head=None) -> None:
        """Append the target's features ``(B, n, ...)`` at the next ``n`` positions
        (modeling_flashmap.py:342-351): fc, hidden_norm, and every layer's cross
        keys (k_norm + RoPE) and values into the cache, in one launch sequence."""
        self._check_cache(cache)
        B, n = target_hidden.shape[0], target_hidden.shape[1]
        if cache.length + n > cache.max_length:
            raise ValueError(f"FlashMapCache holds {cache.max_length} positions, writing up to {cache.length + n}")
        pack = self._pack(cache.kv.device, embed_tokens, lm_head)
        self._caches.add(cache)
        plan = self._any_plan(pack, cache, B * n)
        rows = target_hidden.to(cache.kv.device, torch.bfloat16).reshape(B * n, -1).contiguous()
        cu = torch.arange(0, B * n + 1, n, device=cache.kv.device, dtype=torch.int32)
        plan.extend(rows, cu, B)
        cache._length += n

    @torch.no_grad()
    def extend_context_varlen(self, cache: FlashMapCache, target_hidden: torch.Tensor, cu_seqlens: torch.Tensor,
                              embed_tokens=None, lm_head=None) -> None:
        """Ragged ``extend_context``: sequence ``b`` appends the rows
        ``target_hidden[cu_seqlens[b]:cu_seqlens[b+1]]`` (packed ``(sum n_b, ...)``)
        at its own next positions; every sequence's length advances by its
        ``n_b`` (the per-sequence form of modeling_flashmap.py:342-351 that the
        serving plugins use with packed ``cu_seqlens``)."""
        self._check_cache(cache)
        cu = cu_seqlens.to(cache.kv.device, torch.int32).contiguous()
        B = cu.shape[0] - 1
        if B != cache.kv.shape[2]:
            raise ValueError(f"cu_seqlens describes {B} sequences, the cache holds {cache.kv.shape[2]}")
        counts = (cu[1:] - cu[:-1]).cpu()
        if (counts < 0).any():
            raise ValueError("cu_seqlens must be non-decreasing")
        after = cache.lengths.cpu() + counts
        if int(after.max()) > cache.max_length:
            raise ValueError(f"FlashMapCache holds {cache.max_length} positions, writing up to {int(after.max())}")
        rows = target_hidden.to(cache.kv.device, torch.bfloat16).reshape(int(cu[-1].item()), -1).contiguous()
        pack = self._pack(cache.kv.device, embed_tokens, lm_head)
        self._caches.add(cache)
        plan = self._any_plan(pack, cache, rows.shape[0])
        plan.extend(rows, cu, B)
        cache._length = int(after.max())

    def attach_target(self, embed_tokens: nn.Module, lm_head: nn.Module) -> None:
        """Prepare the target's embedding-derived constants once (the reference
        computes them lazily on the first draft, :401-420)."""
        self._pack(embed_tokens.weight.device, embed_tokens, lm_head)

    @torch.no_grad()
    def draft(self, anchor_ids: torch.LongTensor, cache: FlashMapCache, embed_tokens: nn.Module, lm_head: nn.Module,
              num_steps: Optional[int] = None, noise: Optional[torch.Tensor] = None,
              generator: Optional[torch.Generator] = None, *, z: Optional[torch.Tensor] = None,
              return_tokens: bool = False):
        """Draft logits ``(B, block_size, V)`` for the block after ``anchor_ids (B,)``
        (modeling_flashmap.py:422-479); ``-inf`` outside the state vocabulary.

        ``noise`` (B, K, S) is the multi-step starting state, as in the
        reference; ``z`` (B, K, target_hidden) optionally fixes the one-step
        noise (otherwise drawn by Philox).  With ``return_tokens`` the fused
        per-slot argmax is returned too."""
        self._check_cache(cache)
        num_steps = self._steps(num_steps)
        pack = self._pack(cache.kv.device, embed_tokens, lm_head)
        self._caches.add(cache)
        B, K = anchor_ids.shape[0], self.config.block_size
        plan = self._plan(pack, cache, B, num_steps)
        dev = cache.kv.device
        V = self.config.vocab_size
        scatter = pack.draft_ids is not None
        logits = torch.empty(B, K, V, device=dev, dtype=torch.bfloat16)
        if scatter:
            logits.fill_(float("-inf"))
        tokens = torch.empty(B, K, device=dev, dtype=torch.int64)
        ids = anchor_ids.to(dev, torch.int64).contiguous()
        zz = None if z is None else z.to(dev, torch.bfloat16).reshape(B * K, -1).contiguous()
        nn_ = None
        if noise is not None and num_steps > 1:
            nn_ = noise.to(dev, torch.float32).reshape(B * K, -1).contiguous()
        seed, offset = self._seed(generator)
        plan.draft(ids, seed, offset, logits=logits, ldl=V, scatter=scatter, tokens=tokens, z=zz, noise=nn_)
        return (logits, tokens) if return_tokens else logits

    @torch.no_grad()
    def forward(self, inputs_embeds, s: float, t: float, position_ids, context) -> torch.Tensor:
        """One jump from ``s`` to ``t`` of the DiT (modeling_flashmap.py:302-313):
        featurised ``inputs_embeds (B, K, target_hidden)`` at ``position_ids (B, K)``
        -> hidden states ``(B, K, target_hidden)``.  ``context`` holds each layer's
        cross-attention (keys, values), e.g. ``cache.context(end)``: a view of a
        FlashMapCache is read in place, other tensors are staged into one."""
        B, K = inputs_embeds.shape[0], inputs_embeds.shape[1]
        keys0 = context[0][0]
        dev = inputs_embeds.device
        end = keys0.shape[2]
        cache = self._cache_of(keys0)
        if cache is None:
            cache = FlashMapCache(self.config, B, end, device=dev, dtype=torch.bfloat16)
            for i, (k, v) in enumerate(context):
                cache.write(i, 0, k.to(torch.bfloat16), v.to(torch.bfloat16))
        pack = self._pack(dev)
        if pack.ensure_rope(self.config, int(position_ids.max()) + 2):
            self._plans = {}
        plan = self._plan(pack, cache, B, self.config.num_steps)
        hidden = torch.empty(B * K, self.config.target_hidden_size, device=dev, dtype=torch.bfloat16)
        ctx_last = torch.full((B,), end - 1, device=dev, dtype=torch.int32)
        plan.forward(inputs_embeds.to(dev, torch.bfloat16).reshape(B * K, -1).contiguous(),
                     position_ids.to(dev, torch.int32).reshape(-1).contiguous(), ctx_last,
                     pack.modulations(self.config, s, t), hidden)
        return hidden.view(B, K, -1)

    def _cache_of(self, keys: torch.Tensor):
        """The registered FlashMapCache whose storage ``keys`` views, if any."""
        ptr = keys.untyped_storage().data_ptr()
        for cache in list(self._caches):
            if cache.kv.untyped_storage().data_ptr() == ptr:
                return cache
        return None

    # -------------------------------------------------------------- speculative decoding
    def check_target(self, target: PreTrainedModel) -> None:
        """Same checks and messages as modeling_flashmap.py:483-512."""
        config = target.config.get_text_config()
        embedding, lm_head = target.get_input_embeddings().weight, target.get_output_embeddings().weight
        expected = (self.config.vocab_size, self.config.target_hidden_size)
        if tuple(embedding.shape) != expected or tuple(lm_head.shape) != expected:
            raise ValueError(
                f"this drafter needs a target with vocabulary {expected[0]} and hidden size {expected[1]} "
                f"({self.config.target_model}), got an embedding of shape {tuple(embedding.shape)}")
        if max(self.config.target_layer_ids) >= config.num_hidden_layers - 1:
            raise ValueError(f"target_layer_ids {self.config.target_layer_ids} need more than "
                             f"{config.num_hidden_layers} target layers")
        name = (getattr(config, "_name_or_path", None) or "").rstrip("/")
        croppable = ("full_attention", "sliding_attention", "chunked_attention")
        recurrent = sorted({k for k in getattr(config, "layer_types", None) or () if k not in croppable})
        if recurrent:
            raise ValueError(
                f"spec_generate cannot decode {name or 'this target'} losslessly: its {', '.join(recurrent)} layers "
                "keep a state that rejected drafts cannot be rolled back from; serve it with vLLM or SGLang")
        if name and name.split("/")[-1] != self.config.target_model.split("/")[-1]:
            warnings.warn(f"this drafter was trained for {self.config.target_model}, not {name}")
        devices = {embedding.device, lm_head.device}
        if len(devices) > 1:
            raise ValueError(f"the drafter and the target's embedding and lm_head must share a device, got {devices}")

    @torch.no_grad()
    def spec_generate(self, target: PreTrainedModel, input_ids: torch.LongTensor, max_new_tokens: int = 256,
                      temperature: float = 0.0, num_steps: Optional[int] = None, stop_token_ids: Optional[list] = None,
                      generator: Optional[torch.Generator] = None, *, _z_source=None) -> FlashMapGenerateOutput:
        """Lossless speculative decoding of ``target`` from ``input_ids (1, P)``
        (modeling_flashmap.py:514-612).  Drafting, draft sampling and the
        acceptance step run on the CUDA path; ``target`` is a transformers
        causal LM on the same CUDA device."""
        if input_ids.shape[0] != 1:
            raise ValueError("spec_generate decodes one sequence at a time")
        self.check_target(target)
        embed_tokens, lm_head = target.get_input_embeddings(), target.get_output_embeddings()
        device = embed_tokens.weight.device
        if stop_token_ids is None:
            eos = target.generation_config.eos_token_id
            stop_token_ids = [] if eos is None else [eos] if isinstance(eos, int) else list(eos)
        stop = set(int(s) for s in stop_token_ids)
        input_ids = input_ids.to(device)
        K, P = self.config.block_size, input_ids.shape[1]
        num_steps = self._steps(num_steps)
        seed = philox_key(generator)

        def native(logits):  # bf16 and fp32 logits are read as they are; other floats widen exactly
            return (logits if logits.dtype in (torch.bfloat16, torch.float32) else logits.float()).contiguous()

        def sample(logits, r):  # (1, n, V) -> tokens (1, n) and their distributions (:553-557)
            lg = native(logits)
            if temperature <= 0:
                return ops.sample_rows(lg, None, 0.0, seed, r), None
            probs = ops.softmax_rows(lg, temperature)
            return ops.sample_rows(lg, probs, temperature, seed, r), probs

        layers, feats = target.get_decoder().layers, {}
        hooks = [layers[i].register_forward_hook(
            (lambda i: lambda m, a, o: feats.__setitem__(i, o[0] if isinstance(o, tuple) else o))(i))
            for i in self.config.target_layer_ids]
        features = lambda: torch.cat([feats[i] for i in self.config.target_layer_ids], dim=-1)  # noqa: E731
        try:
            target_cache = DynamicCache()
            out = target(input_ids, past_key_values=target_cache, use_cache=True, logits_to_keep=1)
            tokens = sample(out.logits[:, -1:], PREFILL_ROUND)[0]
            cache = FlashMapCache(self.config, 1, P + max_new_tokens + K + 1, device=device, dtype=torch.bfloat16)
            self.extend_context(cache, features(), embed_tokens, lm_head)
            lengths, rounds = [], 0
            while tokens.shape[1] < max_new_tokens and int(tokens[0, -1]) not in stop:
                anchor = tokens[:, -1]
                z = None if _z_source is None else _z_source(rounds)
                logits, greedy = self.draft(anchor, cache, embed_tokens, lm_head, num_steps, z=z,
                                            generator=generator, return_tokens=True)
                if temperature <= 0:
                    draft, draft_probs = greedy, None
                else:
                    draft, draft_probs = sample(logits, rounds)
                position = P + tokens.shape[1] - 1
                out = target(torch.cat([anchor[:, None], draft], dim=1),
                             position_ids=torch.arange(position, position + K + 1, device=device)[None],
                             past_key_values=target_cache, use_cache=True)
                tl = native(out.logits)
                if temperature <= 0:
                    acc, bonus = ops.accept_greedy(tl, draft.contiguous())
                else:
                    acc, bonus = ops.accept_rejection(tl, draft.contiguous(), draft_probs.contiguous(), temperature,
                                                      seed, rounds)
                rounds += 1
                accepted, bonus_tok = int(acc[0]), int(bonus[0])
                new = torch.cat([draft[:, :accepted], torch.tensor([[bonus_tok]], device=device)], dim=1)
                hit = [i for i, tkn in enumerate(new[0].tolist()) if tkn in stop]
                if hit:
                    new = new[:, : hit[0] + 1]
                tokens = torch.cat([tokens, new], dim=1)
                lengths.append(new.shape[1])
                excess = target_cache.get_seq_length() - (position + accepted + 1)
                if excess > 0:
                    target_cache.crop(-excess)
                self.extend_context(cache, features()[:, : accepted + 1])
        finally:
            for h in hooks:
                h.remove()
        tokens = tokens[:, :max_new_tokens]
        return FlashMapGenerateOutput(sequences=torch.cat([input_ids, tokens], dim=1), num_new_tokens=tokens.shape[1],
                                      acceptance_lengths=lengths)


class DraftSession:
    """A serving-loop draft: one ``fm_draft`` captured in a CUDA graph over a
    fixed cache, batch and number of jumps, replayed per call.

    ``draft(anchor_ids)`` copies the anchors from pinned host memory, replays
    the graph (all ~100 kernels, chained by programmatic dependent launch) and
    returns the drafted tokens in pinned host memory.  Every replay draws fresh
    Philox noise (a device counter advances per draft).  The cache's per-
    sequence lengths are read on the device, so ``extend_context`` between
    replays is honoured without re-capturing."""

    def __init__(self, model: "FlashMapDraftModel", cache: FlashMapCache, embed_tokens: nn.Module, lm_head: nn.Module,
                 num_steps: Optional[int] = None, with_logits: bool = False, seed: Optional[int] = None,
                 use_graph: bool = True):
        model._check_cache(cache)
        num_steps = model._steps(num_steps)
        self.model, self.cache = model, cache
        pack = model._pack(cache.kv.device, embed_tokens, lm_head)
        model._caches.add(cache)
        B, K = cache.kv.shape[2], model.config.block_size
        self.plan = model._plan(pack, cache, B, num_steps)
        dev = cache.kv.device
        self.B, self.K = B, K
        self.anchor = torch.zeros(B, dtype=torch.int64, device=dev)
        self.tokens = torch.zeros(B * K, dtype=torch.int64, device=dev)
        self.offset = torch.zeros(1, dtype=torch.int32, device=dev)
        self.logits = None
        self.scatter = pack.draft_ids is not None
        if with_logits:
            self.logits = torch.full((B * K, model.config.vocab_size), float("-inf"), device=dev,
                                     dtype=torch.bfloat16)
        self.seed = int(torch.initial_seed() if seed is None else seed)
        self.anchor_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.tokens_host = torch.zeros(B * K, dtype=torch.int64).pin_memory()
        self.graph = None
        self._launch()  # eager warm-up: builds every lazy constant before capture
        torch.cuda.synchronize(dev)
        if use_graph:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._launch()
            torch.cuda.synchronize(dev)

    def _launch(self):
        self.plan.draft(self.anchor, self.seed, 0, logits=self.logits,
                        ldl=0 if self.logits is None else self.logits.shape[1], scatter=self.scatter,
                        tokens=self.tokens, offset_dev=self.offset)

    def replay(self) -> None:
        """One draft on the device with the current contents of the static buffers."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch()

    @property
    def launches(self) -> int:
        """Kernels one draft launches."""
        return self.plan.last_launches()

    def draft(self, anchor_ids) -> torch.Tensor:
        """Anchor ids (B,) (host or device) -> drafted tokens (B, K) in pinned host memory."""
        if isinstance(anchor_ids, torch.Tensor) and anchor_ids.is_cuda:
            self.anchor.copy_(anchor_ids, non_blocking=True)
        else:
            self.anchor_host.copy_(torch.as_tensor(anchor_ids, dtype=torch.int64).reshape(-1))
            self.anchor.copy_(self.anchor_host, non_blocking=True)
        self.replay()
        self.tokens_host.copy_(self.tokens, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return self.tokens_host.view(self.B, self.K)


__all__ = ["DraftSession", "FlashMapCache", "FlashMapDraftModel", "FlashMapGenerateOutput"]
