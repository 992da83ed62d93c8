"""The serving plugins' operators on this library's CUDA kernels, under the
reference's names.

The reference registers its Triton kernels as ``torch.library`` custom ops so
``torch.compile`` keeps them whole inside the draft step it compiles:

* ``flashmap_vllm::rms_norm``, ``::rms_norm_rope``, ``::block_self_attention``
  (flashmap/vllm/kernels.py:48, 100, 193) and ``::paged_cross_attention``
  (flashmap/vllm/model.py:93), plus the plain functions ``rope_table`` and
  ``write_context_kv`` (vllm/kernels.py:27, 311);
* ``flashmap_sglang::block_self_attention``, ``::rms_norm_rope``
  (flashmap/sglang/kernels.py:84, 170), ``::paged_cross_attention`` and
  ``::paged_cross_attention_fp8`` (flashmap/sglang/model.py:127, 154), plus
  ``rms_norm``, ``rope_freqs`` and the context writers ``kv_norm_rope_write_fp8``
  (sglang/kernels.py:132, 319; sglang/model.py:97) and ``kv_norm_rope_write``
  for a bf16 pool (the fused writer sglang/model.py:746-766 calls).

Importing this module registers the same op names with the same schemas, so
plugin code that calls ``torch.ops.flashmap_vllm.*`` / ``torch.ops.flashmap_sglang.*``
runs on the B200 kernels (one process must not import both this module and the
reference's kernel modules: the names would be registered twice).  Each op
checks its arguments where the reference asserts and raises
``OpArgumentError`` (an ``AssertionError`` and a ``ValueError``), runs on the
current CUDA stream, and returns new tensors; the writers mutate the caches
through raw pointers like the reference's.  There is no fallback: without the
library or an sm_100 GPU every call raises.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from . import _lib

__all__ = [
    "OpArgumentError", "rope_table", "rope_freqs", "vllm_rms_norm", "vllm_rms_norm_rope",
    "vllm_block_self_attention", "vllm_paged_cross_attention", "write_context_kv", "sglang_rms_norm",
    "sglang_rms_norm_rope", "sglang_block_self_attention", "sglang_paged_cross_attention",
    "sglang_paged_cross_attention_fp8", "kv_norm_rope_write", "kv_norm_rope_write_fp8", "tree_commit",
]

_FP8 = getattr(torch, "float8_e4m3fn", None)


class OpArgumentError(AssertionError, ValueError):
    """An argument the reference op would reject with ``assert``."""


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise OpArgumentError(msg)


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda(t: torch.Tensor, name: str) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor")


def _weight(w: torch.Tensor, name: str):
    """(tensor, FM_DT_*) of a norm weight: bf16 or fp32, contiguous."""
    _cuda(w, name)
    _need(w.dtype in (torch.bfloat16, torch.float32), f"{name} must be bf16 or fp32, got {w.dtype}")
    w = w.contiguous()
    return w, (_lib.FM_DT_BF16 if w.dtype == torch.bfloat16 else _lib.FM_DT_F32)


def _positions(pos: torch.Tensor):
    _cuda(pos, "positions")
    _need(pos.dtype in (torch.int32, torch.int64), f"positions must be int32 or int64, got {pos.dtype}")
    pos = pos.contiguous()
    return pos, (_lib.FM_DT_I32 if pos.dtype == torch.int32 else _lib.FM_DT_I64)


def _pair_table(table: torch.Tensor, head_dim: int, name: str) -> _lib.RopeView:
    """A fp32 ``(rows..., head_dim / 2, [cos, sin])`` table (vLLM's rope_table, sglang's freqs)."""
    _cuda(table, name)
    _need(table.dtype == torch.float32 and table.is_contiguous(), f"{name} must be contiguous float32")
    _need(table.shape[-2:] == (head_dim // 2, 2), f"{name} must end in ({head_dim // 2}, 2), got {tuple(table.shape)}")
    rows = table.numel() // head_dim
    return _lib.RopeView(table.data_ptr(), table.data_ptr() + 4, head_dim, 2, rows)


def _half_table(cos_sin: torch.Tensor, head_dim: int) -> _lib.RopeView:
    """A fp32 ``(positions, [cos | sin])`` table of rows of head_dim (sglang's writer table)."""
    _cuda(cos_sin, "cos_sin")
    _need(cos_sin.dtype == torch.float32 and cos_sin.is_contiguous() and cos_sin.dim() == 2
          and cos_sin.shape[1] == head_dim, f"cos_sin must be contiguous float32 (positions, {head_dim})")
    return _lib.RopeView(cos_sin.data_ptr(), cos_sin.data_ptr() + 4 * (head_dim // 2), head_dim, 1,
                         cos_sin.shape[0])


_ERR_WORDS: dict = {}


def _err(device) -> torch.Tensor:
    """The device's error word (int32, zero until a kernel records an index or
    timeout code; the first code sticks), allocated once per device so that a
    call launches no fill kernel for it."""
    key = torch.device(device)
    if key.index is None:
        key = torch.device(key.type, torch.cuda.current_device())
    w = _ERR_WORDS.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=key)
        _ERR_WORDS[key] = w
    return w


def _bf16_weight(w: torch.Tensor, name: str) -> torch.Tensor:
    """fm_rmsnorm reads bf16 weights: an fp32 weight must hold bf16 values
    (sglang passes ``weight.float()`` of bf16 parameters)."""
    w, dt = _weight(w, name)
    if dt == _lib.FM_DT_BF16:
        return w
    wb = w.to(torch.bfloat16)
    _need(torch.equal(wb.float(), w), f"{name}: fp32 weights must be bf16-representable")
    return wb


def _rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    _cuda(x, "x")
    _need(x.dtype == torch.bfloat16, f"x must be bf16, got {x.dtype}")
    x = x.contiguous()
    w = _bf16_weight(weight, "weight")
    out = torch.empty_like(x)
    if x.numel():
        cols = x.shape[-1]
        _need(w.numel() == cols, f"weight has {w.numel()} values for rows of {cols}")
        _lib.call("fm_rmsnorm", _p(x), _p(w), _p(out), x.numel() // cols, cols, float(eps), _stream())
    return out


def _norm_rope_rows(x: torch.Tensor, weight: torch.Tensor, rope: _lib.RopeView, positions, eps: float,
                    tokens: int, heads: int, head_dim: int, out: torch.Tensor, x_ts: int, o_ts: int,
                    x_ptr: int, o_ptr: int, mode: int = _lib.FM_NORM_DIT) -> None:
    w, wdt = _weight(weight, "weight")
    _need(w.numel() == head_dim, f"weight has {w.numel()} values for heads of {head_dim}")
    pos_ptr, pdt = None, _lib.FM_DT_I32
    if positions is not None:
        positions, pdt = _positions(positions)
        pos_ptr = _p(positions)
    err = _err(x.device)
    _lib.call("fm_qk_norm_rope", ctypes.c_void_p(x_ptr), x_ts, ctypes.c_void_p(o_ptr), o_ts, tokens, heads,
              head_dim, _p(w), wdt, rope, pos_ptr, pdt, float(eps), mode, _p(err), _stream())
    return err


# ---------------------------------------------------------------------------------------- vLLM


def rope_table(max_positions: int, head_dim: int, base: float, device) -> torch.Tensor:
    """``(max_positions, head_dim / 2, 2)`` fp32 ``(cos, sin)`` of ``position *
    base^(-2i / head_dim)`` (vllm/kernels.py:27-35), from the library's table kernel."""
    from . import ops
    cos, sin = ops.rope_table(max_positions, head_dim, base, device=device)
    return torch.stack([cos, sin], dim=-1).contiguous()


def rope_freqs(positions: torch.Tensor, head_dim: int, theta: float) -> torch.Tensor:
    """sglang's ``(..., head_dim / 2, 2)`` rotary table at ``positions`` (sglang/model.py:97-105)."""
    from . import ops
    inv_freq = ops.rope_inv_freq(head_dim, theta).to(positions.device)
    angles = positions.float()[..., None] * inv_freq
    return torch.stack([angles.cos(), angles.sin()], dim=-1)


@torch.library.custom_op("flashmap_vllm::rms_norm", mutates_args=())
def vllm_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """FlashMap RMSNorm ``x * bf16(weight * rsqrt(mean(x^2) + eps))`` of a bf16
    ``x (..., C)`` (vllm/kernels.py:48-59), one launch of ``fm_rmsnorm``."""
    return _rms_norm(x, weight, eps)


@vllm_rms_norm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op("flashmap_vllm::rms_norm_rope", mutates_args=())
def vllm_rms_norm_rope(x: torch.Tensor, weight: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor,
                       eps: float) -> torch.Tensor:
    """RMSNorm then interleaved RoPE at ``positions (tokens,)`` of ``x (tokens,
    heads, head_dim)`` with the ``rope_table`` ``cos_sin`` (vllm/kernels.py:100-119)."""
    _cuda(x, "x")
    _need(x.dtype == torch.bfloat16 and x.dim() == 3, "x must be bf16 (tokens, heads, head_dim)")
    tokens, heads, head_dim = x.shape
    rope = _pair_table(cos_sin, head_dim, "cos_sin")
    x = x.contiguous()
    out = torch.empty_like(x)
    if tokens:
        _need(positions.numel() == tokens, "one position per token")
        _norm_rope_rows(x, weight, rope, positions, eps, tokens, heads, head_dim, out, heads * head_dim,
                        heads * head_dim, x.data_ptr(), out.data_ptr())
    return out


@vllm_rms_norm_rope.register_fake
def _(x, weight, cos_sin, positions, eps):
    return torch.empty_like(x)


def _block_self_attention(qkv, q_norm, k_norm, rope: _lib.RopeView, positions, eps: float) -> torch.Tensor:
    """(blocks * T, heads * head_dim): the fused kernel for blocks of 16 and
    head_dim 64/128, else q/k norm-rope rows then the block attention kernel."""
    _cuda(qkv, "qkv")
    _need(qkv.dtype == torch.bfloat16 and qkv.dim() == 5 and qkv.shape[2] == 3,
          "qkv must be bf16 (blocks, T, 3, heads, head_dim)")
    blocks, block, _, heads, head_dim = qkv.shape
    qkv = qkv.contiguous()
    out = torch.empty(blocks * block, heads * head_dim, dtype=qkv.dtype, device=qkv.device)
    if blocks == 0:
        return out
    pos_ptr, pdt = None, _lib.FM_DT_I32
    if positions is not None:
        positions, pdt = _positions(positions)
        _need(positions.numel() == blocks * block, "one position per block slot")
        pos_ptr = _p(positions)
    qn, wdt = _weight(q_norm, "q_norm")
    kn, kdt = _weight(k_norm, "k_norm")
    _need(wdt == kdt, "q_norm and k_norm must share a dtype")
    _need(qn.numel() == head_dim and kn.numel() == head_dim, "norm weights of head_dim values")
    err = _err(qkv.device)
    scale = head_dim ** -0.5
    if block == 16 and head_dim in (64, 128):
        _lib.call("fm_block_self_attn_qknorm", _p(qkv), _p(out), blocks, block, heads, head_dim, _p(qn), _p(kn),
                  wdt, rope, pos_ptr, pdt, float(eps), float(scale), _p(err), _stream())
    else:
        staged = torch.empty_like(qkv)
        row = 3 * heads * head_dim
        for part, w in ((0, qn), (1, kn)):
            off = part * heads * head_dim * 2
            _lib.call("fm_qk_norm_rope", ctypes.c_void_p(qkv.data_ptr() + off), row,
                      ctypes.c_void_p(staged.data_ptr() + off), row, blocks * block, heads, head_dim, _p(w), wdt,
                      rope, pos_ptr, pdt, float(eps), _lib.FM_NORM_DIT, _p(err), _stream())
        staged[:, :, 2].copy_(qkv[:, :, 2])
        _lib.call("fm_block_self_attn", _p(staged), _p(out), blocks, block, heads, head_dim, _stream())
    return out


@torch.library.custom_op("flashmap_vllm::block_self_attention", mutates_args=())
def vllm_block_self_attention(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, cos_sin: torch.Tensor,
                              positions: torch.Tensor, eps: float) -> torch.Tensor:
    """Unmasked self-attention within each draft block from its projected ``qkv
    (blocks, T, 3, heads, head_dim)``: q/k RMSNorms, RoPE at ``positions
    (blocks * T,)``, softmax attention; ``(blocks * T, heads * head_dim)``
    (vllm/kernels.py:193-221)."""
    rope = _pair_table(cos_sin, qkv.shape[-1], "cos_sin")
    return _block_self_attention(qkv, q_norm, k_norm, rope, positions, eps)


@vllm_block_self_attention.register_fake
def _(qkv, q_norm, k_norm, cos_sin, positions, eps):
    blocks, block_size, _, heads, head_dim = qkv.shape
    return qkv.new_empty((blocks * block_size, heads * head_dim))


def _paged_attention(query: torch.Tensor, k_base: int, v_base: int, kv_dtype, strides: Sequence[int],
                     page_size: int, num_pages: int, page_table: torch.Tensor, seqused: torch.Tensor,
                     max_seqlen_k: int, cu_seqlens_q: Optional[torch.Tensor], q_per_request: int, max_q: int,
                     softmax_scale: float, descales: Optional[torch.Tensor], quantize_q: bool,
                     out: torch.Tensor) -> None:
    heads, head_dim = query.shape[-2], query.shape[-1]
    _need(page_table.dtype == torch.int32 and page_table.dim() == 2, "the page table must be int32 (requests, cols)")
    _need(seqused.dtype == torch.int32, "sequence lengths must be int32")
    requests = seqused.numel()
    args = _lib.PagedAttn()
    q2 = query.reshape(-1, heads, head_dim)
    args.q = q2.data_ptr()
    args.q_dtype = _lib.FM_DT_E4M3 if query.dtype == _FP8 else _lib.FM_DT_BF16
    args.q_token_stride, args.q_head_stride = q2.stride(0), q2.stride(1)
    if cu_seqlens_q is not None:
        _need(cu_seqlens_q.dtype == torch.int32 and cu_seqlens_q.numel() == requests + 1,
              "cu_seqlens_q must be int32 (requests + 1,)")
        args.cu_seqlens_q = cu_seqlens_q.data_ptr()
    args.q_per_request = q_per_request
    args.max_q = max_q
    args.k, args.v = k_base, v_base
    args.kv_dtype = kv_dtype
    args.kv_page_stride, args.kv_head_stride, args.kv_token_stride = strides
    args.page_size, args.num_pages = page_size, num_pages
    args.page_table = page_table.data_ptr()
    args.page_table_stride, args.page_table_cols = page_table.stride(0), page_table.shape[1]
    args.seqused_k = seqused.data_ptr()
    args.max_seqlen_k = max_seqlen_k
    args.requests, args.heads, args.head_dim = requests, heads, head_dim
    args.softmax_scale = softmax_scale
    if descales is not None:
        _need(descales.dtype == torch.float32 and descales.shape == (3, requests, heads),
              "descales must be float32 (3, requests, heads)")
        descales = descales.contiguous()
        args.descales = descales.data_ptr()
    args.quantize_q = int(quantize_q)
    o2 = out.reshape(-1, heads, head_dim)
    args.out = o2.data_ptr()
    args.out_token_stride, args.out_head_stride = o2.stride(0), o2.stride(1)
    lib = _lib.load()
    nsplit = lib.fm_paged_attn_nsplit(requests, heads, max_q, max_seqlen_k, 0)
    ws_bytes = lib.fm_paged_attn_workspace_size(requests, heads, head_dim, max_q, nsplit)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=query.device)
    err = _err(query.device)
    args.workspace, args.workspace_bytes, args.nsplit, args.err = ws.data_ptr(), ws_bytes, nsplit, err.data_ptr()
    _lib.call("fm_paged_cross_attn", ctypes.byref(args), _stream())


@torch.library.custom_op("flashmap_vllm::paged_cross_attention", mutates_args=())
def vllm_paged_cross_attention(query: torch.Tensor, kv_cache: torch.Tensor, cu_seqlens_q: torch.Tensor,
                               seqused_k: torch.Tensor, block_table: torch.Tensor,
                               scheduler_metadata: Optional[torch.Tensor], descales: Optional[torch.Tensor],
                               max_seqlen_q: int, max_seqlen_k: int, softmax_scale: float,
                               fa_version: int) -> torch.Tensor:
    """Non-causal attention of ``query (tokens, heads, head_dim)`` onto the first
    ``seqused_k`` cached positions of each request in the FlashAttention paged
    cache ``kv_cache (blocks, heads, block_size, 2 * head_dim)`` (keys then
    values in the last axis); an e4m3 cache takes an e4m3 ``query`` and
    ``descales (3, requests, heads)`` (vllm/model.py:93-132).  The FlashAttention
    schedule and version arguments are accepted and not needed."""
    del scheduler_metadata, fa_version
    _cuda(query, "query")
    _cuda(kv_cache, "kv_cache")
    _need(query.dim() == 3 and kv_cache.dim() == 4, "query (tokens, heads, hd), kv_cache (blocks, heads, page, 2hd)")
    heads, head_dim = query.shape[1], query.shape[2]
    _need(kv_cache.shape[1] == heads and kv_cache.shape[3] == 2 * head_dim, "kv_cache does not match the query")
    fp8 = query.dtype == _FP8
    _need(query.dtype == torch.bfloat16 or fp8, f"query must be bf16 or e4m3, got {query.dtype}")
    if fp8:
        _need(kv_cache.dtype in (_FP8, torch.uint8), "an e4m3 query needs an e4m3 cache")
        _need(descales is not None, "an e4m3 cache needs descales")
    else:
        _need(kv_cache.dtype == torch.bfloat16, "a bf16 query needs a bf16 cache")
    _need(kv_cache.stride(3) == 1, "cache rows must be contiguous")
    esz = kv_cache.element_size()
    out = torch.empty(query.shape, dtype=torch.bfloat16, device=query.device)
    if query.shape[0] == 0 or seqused_k.numel() == 0:
        return out
    _paged_attention(query.contiguous(), kv_cache.data_ptr(), kv_cache.data_ptr() + head_dim * esz,
                     _lib.FM_DT_E4M3 if fp8 else _lib.FM_DT_BF16,
                     (kv_cache.stride(0), kv_cache.stride(1), kv_cache.stride(2)), kv_cache.shape[2],
                     kv_cache.shape[0], block_table, seqused_k.to(torch.int32), int(max_seqlen_k), cu_seqlens_q, 0,
                     int(max_seqlen_q), float(softmax_scale), descales, False, out)
    return out


@vllm_paged_cross_attention.register_fake
def _(query, kv_cache, cu_seqlens_q, seqused_k, block_table, *args):
    return torch.empty(query.shape, dtype=torch.bfloat16, device=query.device)


def write_context_kv(kv: torch.Tensor, positions: torch.Tensor, slots: torch.Tensor, k_norm: torch.Tensor,
                     cos_sin: torch.Tensor, cache_ptrs: torch.Tensor, cache_strides: tuple, block_size: int,
                     eps: float, scales: Optional[torch.Tensor] = None, heads_per_cache: Optional[int] = None) -> None:
    """Every layer's context keys (k-normed, rotated) and values of ``kv (tokens,
    layers, 2, heads, head_dim)`` into the paged caches at ``slots`` (negative:
    skipped), heads in layer-major order, ``heads_per_cache`` to a cache;
    ``cache_strides`` = (block, head, token, value offset) in elements; with
    ``scales (layers, 2)`` the caches are e4m3 (vllm/kernels.py:311-364)."""
    tokens, layers, _, heads, head_dim = kv.shape
    if not tokens:
        return
    _cuda(kv, "kv")
    _need(kv.dtype == torch.bfloat16, "kv must be bf16")
    heads_per_cache = heads_per_cache or heads
    num_caches = cache_ptrs.numel()
    if num_caches * heads_per_cache < layers * heads:
        raise ValueError(f"{num_caches} caches of {heads_per_cache} heads cannot hold {layers} x {heads} heads")
    kv = kv.contiguous()
    pos = positions.to(torch.int64).contiguous()
    sl = slots.to(torch.int64).contiguous()
    _need(pos.numel() == tokens and sl.numel() == tokens, "one position and one slot per token")
    kn, kdt = _weight(k_norm, "k_norm")
    _need(kn.numel() == layers * head_dim, "k_norm must be (layers, head_dim)")
    _need(cache_ptrs.dtype == torch.int64 and cache_ptrs.is_cuda, "cache_ptrs must be a CUDA int64 tensor")
    if scales is not None:
        _need(scales.dtype == torch.float32 and scales.numel() == 2 * layers, "scales must be float32 (layers, 2)")
        scales = scales.contiguous()
    rope = _pair_table(cos_sin, head_dim, "cos_sin")
    sb, sh, st, voff = (int(s) for s in cache_strides)
    err = _err(kv.device)
    cache_ptrs = cache_ptrs.contiguous()  # referenced until the launch below
    _lib.call("fm_write_context_kv_paged", _p(kv), tokens, layers, heads, head_dim, _p(pos), _p(sl), _p(kn), kdt,
              rope, _p(cache_ptrs), num_caches, heads_per_cache, sb, sh, st, voff, int(block_size),
              float(eps), _p(scales), _p(err), _stream())


# ---------------------------------------------------------------------------------------- sglang


def sglang_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of a contiguous bf16 ``x (..., C)`` with a float32 ``weight``
    (sglang/kernels.py:132-145)."""
    _need(x.dtype == torch.bfloat16 and x.is_contiguous(), "x must be contiguous bf16")
    _need(weight.dtype == torch.float32, "weight must be float32")
    return _rms_norm(x, weight, eps)


@torch.library.custom_op("flashmap_sglang::rms_norm_rope", mutates_args=())
def sglang_rms_norm_rope(x: torch.Tensor, weight: torch.Tensor, freqs: torch.Tensor, eps: float) -> torch.Tensor:
    """RoPE of RMSNorm(x) for ``x (..., T, heads, head_dim)`` and ``freqs (...,
    T, head_dim / 2, [cos, sin])`` (sglang/kernels.py:170-183)."""
    _cuda(x, "x")
    _need(x.is_contiguous() and freqs.is_contiguous(), "x and freqs must be contiguous")
    _need(x.dtype == torch.bfloat16, "x must be bf16")
    heads, head_dim = x.shape[-2], x.shape[-1]
    rope = _pair_table(freqs, head_dim, "freqs")
    out = torch.empty_like(x)
    tokens = x.numel() // (heads * head_dim)
    if tokens:
        _need(rope.rows == tokens, "one freqs row per token")
        _norm_rope_rows(x, weight, rope, None, eps, tokens, heads, head_dim, out, heads * head_dim,
                        heads * head_dim, x.data_ptr(), out.data_ptr())
    return out


@sglang_rms_norm_rope.register_fake
def _(x, weight, freqs, eps):
    return torch.empty_like(x)


@torch.library.custom_op("flashmap_sglang::block_self_attention", mutates_args=())
def sglang_block_self_attention(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, freqs: torch.Tensor,
                                eps: float) -> torch.Tensor:
    """Self-attention within each draft block from ``qkv (blocks, T, 3, heads,
    head_dim)``: q/k RMSNorms (float32 weights), RoPE by ``freqs (blocks, T,
    head_dim / 2, [cos, sin])``, unmasked softmax attention;
    ``(blocks, T, heads, head_dim)`` (sglang/kernels.py:84-115)."""
    _need(qkv.is_contiguous() and freqs.is_contiguous(), "qkv and freqs must be contiguous")
    _need(freqs.dtype == torch.float32, "freqs must be float32")
    blocks, block, _, heads, head_dim = qkv.shape
    rope = _pair_table(freqs, head_dim, "freqs")
    _need(rope.rows == blocks * block, "freqs must be (blocks, T, head_dim / 2, 2)")
    out = _block_self_attention(qkv, q_norm, k_norm, rope, None, eps)
    return out.view(blocks, block, heads, head_dim)


@sglang_block_self_attention.register_fake
def _(qkv, q_norm, k_norm, freqs, eps):
    blocks, block_size, _, heads, head_dim = qkv.shape
    return qkv.new_empty((blocks, block_size, heads, head_dim))


def _sglang_attention(query, key_buffer, value_buffer, cache_seqlens, page_table, fp8: bool) -> torch.Tensor:
    _cuda(query, "query")
    _need(query.dim() == 4, "query must be (bs, K, heads, head_dim)")
    bs, block, heads, head_dim = query.shape
    _need(key_buffer.shape[1:] == (heads, head_dim) and value_buffer.shape == key_buffer.shape,
          "key/value pools must be (rows, heads, head_dim)")
    _need(key_buffer.stride() == value_buffer.stride() and key_buffer.stride(2) == 1,
          "key and value pools must share their row layout")
    _need(query.dtype == torch.bfloat16, "query must be bf16")
    if fp8:
        _need(key_buffer.dtype == _FP8 and value_buffer.dtype == _FP8, "the fp8 op takes e4m3 pools")
    else:
        _need(key_buffer.dtype == torch.bfloat16 and value_buffer.dtype == torch.bfloat16, "bf16 pools")
    out = torch.empty_like(query)
    if bs == 0:
        return out
    _paged_attention(query.contiguous(), key_buffer.data_ptr(), value_buffer.data_ptr(),
                     _lib.FM_DT_E4M3 if fp8 else _lib.FM_DT_BF16, (key_buffer.stride(0), key_buffer.stride(1), 0),
                     1, key_buffer.shape[0], page_table, cache_seqlens.to(torch.int32), page_table.shape[1], None,
                     block, block, head_dim ** -0.5, None, fp8, out)
    return out


@torch.library.custom_op("flashmap_sglang::paged_cross_attention", mutates_args=())
def sglang_paged_cross_attention(query: torch.Tensor, key_buffer: torch.Tensor, value_buffer: torch.Tensor,
                                 cache_seqlens: torch.Tensor, page_table: torch.Tensor,
                                 scheduler_metadata: torch.Tensor) -> torch.Tensor:
    """``query (bs, K, heads, head_dim)`` onto each request's first
    ``cache_seqlens`` pool rows, listed by ``page_table`` (page size 1)
    (sglang/model.py:127-145).  The schedule argument is not needed."""
    del scheduler_metadata
    return _sglang_attention(query, key_buffer, value_buffer, cache_seqlens, page_table, False)


@sglang_paged_cross_attention.register_fake
def _(query, key_buffer, value_buffer, cache_seqlens, page_table, scheduler_metadata):
    return torch.empty_like(query)


@torch.library.custom_op("flashmap_sglang::paged_cross_attention_fp8", mutates_args=())
def sglang_paged_cross_attention_fp8(query: torch.Tensor, key_buffer: torch.Tensor, value_buffer: torch.Tensor,
                                     cache_seqlens: torch.Tensor, page_table: torch.Tensor,
                                     scheduler_metadata: torch.Tensor) -> torch.Tensor:
    """The same onto an e4m3 pool written with scale 1: the bf16 query is
    quantised per (request, head) with scale amax / 448 inside the kernel
    (sglang/model.py:154-175)."""
    del scheduler_metadata
    return _sglang_attention(query, key_buffer, value_buffer, cache_seqlens, page_table, True)


@sglang_paged_cross_attention_fp8.register_fake
def _(query, key_buffer, value_buffer, cache_seqlens, page_table, scheduler_metadata):
    return torch.empty_like(query)


def _pool_write(kv, meta, k_norm_weights, cos_sin, positions, locs, num_layers, kv_size, head_dim, eps, fp8,
                k_scale, v_scale, commit_lens, locs_row_width) -> None:
    if kv.shape[0] == 0:
        return
    _cuda(kv, "kv")
    _need(kv.dtype == torch.bfloat16, "kv must be bf16")
    tokens = kv.shape[0]
    _need(kv.numel() == tokens * num_layers * 2 * kv_size, "kv must be (tokens, layers * 2 * kv_size)")
    kv = kv.contiguous()
    _need(meta.dtype == torch.int64 and meta.is_cuda and meta.numel() == 4 * num_layers,
          "meta must be CUDA int64 (layers, 4)")
    kn, kdt = _weight(k_norm_weights, "k_norm_weights")
    rope = _half_table(cos_sin, head_dim)
    pos = positions.to(torch.int64).contiguous()
    lc = locs.to(torch.int64).contiguous()
    cl = None
    if commit_lens is not None:
        cl = commit_lens.to(torch.int32).contiguous()
    err = _err(kv.device)
    meta = meta.contiguous()  # referenced until the launch below
    _lib.call("fm_kv_norm_rope_write_pool", _p(kv), tokens, num_layers, kv_size, head_dim, _p(meta),
              _p(kn), kdt, rope, _p(pos), _p(lc), _p(cl), int(locs_row_width or 1),
              _lib.FM_DT_E4M3 if fp8 else _lib.FM_DT_BF16, _lib.FM_NORM_FUSED if fp8 else _lib.FM_NORM_DIT,
              float(k_scale), float(v_scale), float(eps), _p(err), _stream())


def kv_norm_rope_write_fp8(kv, meta, k_norm_weights, cos_sin, positions, locs, num_layers, kv_size, head_dim, eps, *,
                           k_scale=1.0, v_scale=1.0, commit_lens=None, locs_row_width=None) -> None:
    """Context keys (k-normed, rotated) and values into an e4m3 pool, both
    divided by their static scale (sglang/kernels.py:319-331)."""
    _pool_write(kv, meta, k_norm_weights, cos_sin, positions, locs, num_layers, kv_size, head_dim, eps, True,
                k_scale, v_scale, commit_lens, locs_row_width)


def kv_norm_rope_write(kv, meta, k_norm_weights, cos_sin, positions, locs, num_layers, kv_size, head_dim, eps, *,
                       is_neox_style=False, commit_lens=None, locs_row_width=None) -> None:
    """The bf16-pool writer with the arguments of the fused writer that
    sglang/model.py:746-766 calls (FlashMap rotates interleaved pairs, so
    ``is_neox_style`` must be False).  That writer is sglang's own kernel and
    is not in the reference; the keys here take the HF path's k_norm rounding
    (modeling_flashmap.py:76-80), so pool keys equal the HF cache's."""
    if is_neox_style:
        raise OpArgumentError("FlashMap rotates interleaved pairs: is_neox_style must be False")
    _pool_write(kv, meta, k_norm_weights, cos_sin, positions, locs, num_layers, kv_size, head_dim, eps, False,
                1.0, 1.0, commit_lens, locs_row_width)


def attention_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


def tree_commit(accept_index, num_correct, window, predict, req_pool_indices, prefix_lens, req_to_token):
    """The tree path's commit after greedy tree verification, one launch for
    the batch (sglang/kernels.py:363-454): reorders each request's verify
    window in ``req_to_token`` (in place) so the accepted path comes first (no
    KV moves) and returns ``(out_tokens (bs, D1) int64, bonus, commit_lens
    int32, new_seq_lens, inject_locs (bs * W) int64)``."""
    for t, name in ((accept_index, "accept_index"), (num_correct, "num_correct"), (window, "window"),
                    (predict, "predict"), (req_pool_indices, "req_pool_indices"), (prefix_lens, "prefix_lens"),
                    (req_to_token, "req_to_token")):
        _cuda(t, name)
    _need(req_to_token.dtype == torch.int32 and req_to_token.stride(1) == 1, "req_to_token must be int32 rows")
    bs, d1 = accept_index.shape
    width = window.shape[1]
    dev = accept_index.device
    accept = accept_index.to(torch.int32).contiguous()
    correct = num_correct.to(torch.int32).contiguous()
    win = window.to(torch.int64).contiguous()
    pred = predict.to(torch.int32).contiguous()
    pool = req_pool_indices.to(torch.int64).contiguous()
    prefix = prefix_lens.to(torch.int64).contiguous()
    out_tokens = torch.empty(bs, d1, dtype=torch.int64, device=dev)
    bonus = torch.empty(bs, dtype=torch.int64, device=dev)
    commit = torch.empty(bs, dtype=torch.int32, device=dev)
    new_seq_lens = torch.empty(bs, dtype=torch.int64, device=dev)
    inject = torch.empty(bs * width, dtype=torch.int64, device=dev)
    err = _err(dev)
    _lib.call("fm_tree_commit", _p(accept), _p(correct), _p(win), _p(pred), _p(pool), _p(prefix), _p(req_to_token),
              req_to_token.stride(0), req_to_token.shape[0], bs, width, d1, _p(out_tokens), _p(bonus), _p(commit),
              _p(new_seq_lens), _p(inject), _p(err), _stream())
    return out_tokens, bonus, commit, new_seq_lens.to(prefix_lens.dtype), inject
