"""Torch-tensor wrappers of the C-ABI operators (CUDA tensors in, CUDA tensors out).

Each wrapper checks dtypes/contiguity like the reference's torch.library ops
(``assert``s in flashmap/vllm/kernels.py:51, 112) but raises ``ValueError``
instead, runs on the current CUDA stream, and returns new tensors.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

STORE, GELU, SWIGLU, RESID, F32 = (_lib.FM_EPI_STORE, _lib.FM_EPI_GELU, _lib.FM_EPI_SWIGLU, _lib.FM_EPI_RESID,
                                   _lib.FM_EPI_F32)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _logits_dtype(t) -> int:
    if not t.is_cuda or not t.is_contiguous() or t.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"logits must be a contiguous CUDA bf16 or fp32 tensor, got {t.dtype} on {t.device}")
    return 0 if t.dtype == torch.bfloat16 else 1


def _need(t, dtype, name):
    if t is None:
        return
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor, got {t.dtype} on {t.device}")


def gemm(W: torch.Tensor, X: torch.Tensor, epilogue: int = STORE, bias=None, gate=None, out=None,
         err: torch.Tensor | None = None) -> torch.Tensor:
    """``out = epilogue(X @ W.T)`` on the tcgen05 GEMM (``fm_gemm_bf16``)."""
    _need(W, torch.bfloat16, "W")
    _need(X, torch.bfloat16, "X")
    _need(bias, torch.bfloat16, "bias")
    _need(gate, torch.bfloat16, "gate")
    M, K = W.shape
    N = X.shape[0]
    if X.shape[1] != K:
        raise ValueError(f"X has {X.shape[1]} columns, W has {K}")
    width = M // 2 if epilogue == SWIGLU else M
    if out is None:
        if epilogue == RESID:
            raise ValueError("the residual epilogue updates `out` in place")
        out = torch.empty(N, width, device=W.device, dtype=torch.float32 if epilogue == F32 else torch.bfloat16)
    ws_bytes = _lib.load().fm_gemm_workspace_size(M, N, K)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=W.device)
    _lib.call("fm_gemm_bf16", _p(W), _p(X), _p(out), M, N, K, out.shape[1], _p(bias), _p(gate), epilogue, _p(ws),
              ws_bytes, _p(err), _stream())
    return out


def rmsnorm(x, w, eps):
    _need(x, torch.bfloat16, "x")
    _need(w, torch.bfloat16, "w")
    y = torch.empty_like(x)
    cols = x.shape[-1]
    _lib.call("fm_rmsnorm", _p(x), _p(w), _p(y), x.numel() // cols, cols, float(eps), _stream())
    return y


def adaln(x, mod, eps):
    """``mod`` is the (scale | shift | gate) row of 3*D values."""
    _need(x, torch.bfloat16, "x")
    _need(mod, torch.bfloat16, "mod")
    y = torch.empty_like(x)
    cols = x.shape[-1]
    _lib.call("fm_adaln", _p(x), _p(mod), _p(y), x.numel() // cols, cols, float(eps), _stream())
    return y


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    """``1 / theta^(2i/hd)`` in fp32, the reference's expression (modeling_flashmap.py:56)
    evaluated on the host, so that every angle is bit-identical to the reference's."""
    return 1.0 / theta ** (torch.arange(0, head_dim, 2).float() / head_dim)


def rope_table(max_pos: int, head_dim: int, theta: float, device="cuda"):
    cs = torch.empty(max_pos, head_dim // 2, device=device, dtype=torch.float32)
    sn = torch.empty_like(cs)
    inv = rope_inv_freq(head_dim, theta).to(device)
    _lib.call("fm_rope_table", _p(cs), _p(sn), max_pos, head_dim, _p(inv), _stream())
    return cs, sn


def philox_normal(shape, seed: int, offset: int, device="cuda"):
    out = torch.empty(shape, device=device, dtype=torch.bfloat16)
    _lib.call("fm_philox_normal", _p(out), out.numel(), int(seed), int(offset), _stream())
    return out


def block_self_attn(qkv, batch: int, block: int, heads: int, head_dim: int):
    _need(qkv, torch.bfloat16, "qkv")
    out = torch.empty(batch * block, heads * head_dim, device=qkv.device, dtype=torch.bfloat16)
    _lib.call("fm_block_self_attn", _p(qkv), _p(out), batch, block, heads, head_dim, _stream())
    return out


def cross_attn(q, cache_kv, lengths, layer: int, nsplit: int = 0, err=None):
    """``cache_kv`` (L, 2, Bc, H, T, hd); ``lengths`` int32 (B,): keys 0..lengths[b]."""
    _need(q, torch.bfloat16, "q")
    _need(cache_kv, torch.bfloat16, "cache")
    _need(lengths, torch.int32, "lengths")
    L, _, Bc, H, Tc, hd = cache_kv.shape
    B = lengths.shape[0]
    if nsplit <= 0:
        nsplit = max(1, min((148 + B * H - 1) // (B * H), (Tc + 63) // 64))
    out = torch.empty(B * 16, H * hd, device=q.device, dtype=torch.bfloat16)
    wsb = _lib.load().fm_cross_attn_workspace_size(B, H, hd, nsplit)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=q.device)
    _lib.call("fm_cross_attn", _p(q), _p(cache_kv), _p(out), _p(lengths), B, H, hd, L, layer, Bc, Tc, nsplit, _p(ws),
              wsb, _p(err), _stream())
    return out


def row_stats(logits, temperature: float):
    dt = _logits_dtype(logits)
    V = logits.shape[-1]
    rows = logits.numel() // V
    stats = torch.empty(rows, 2, device=logits.device, dtype=torch.float32)
    am = torch.empty(rows, device=logits.device, dtype=torch.int64)
    _lib.call("fm_row_stats", _p(logits), dt, rows, V, float(temperature), _p(stats), _p(am), _stream())
    return stats, am


def softmax_rows(logits, temperature: float):
    dt = _logits_dtype(logits)
    V = logits.shape[-1]
    probs = torch.empty(logits.shape, device=logits.device, dtype=torch.float32)
    _lib.call("fm_softmax_rows", _p(logits), dt, logits.numel() // V, V, float(temperature), _p(probs), _stream())
    return probs


def sample_rows(logits, probs, temperature: float, seed: int, offset: int):
    """Draft tokens (B, K) from logits (B, K, V): argmax at T <= 0, else drawn from probs."""
    B, K, V = logits.shape
    dt = _logits_dtype(logits)
    tokens = torch.empty(B, K, device=logits.device, dtype=torch.int64)
    _lib.call("fm_sample_rows", _p(logits), dt, _p(probs), B, K, V, float(temperature), int(seed), int(offset),
              _p(tokens), _stream())
    return tokens


def accept_greedy(target_logits, draft):
    dt = _logits_dtype(target_logits)
    _need(draft, torch.int64, "draft")
    B, K1, V = target_logits.shape
    acc = torch.empty(B, device=draft.device, dtype=torch.int64)
    bonus = torch.empty_like(acc)
    wsb = _lib.load().fm_accept_workspace_size(B, K1 - 1)
    ws = torch.empty(wsb, dtype=torch.uint8, device=draft.device)
    _lib.call("fm_accept_greedy", _p(target_logits), dt, _p(draft), B, K1 - 1, V, _p(acc), _p(bonus), _p(ws), wsb,
              _stream())
    return acc, bonus


def accept_rejection(target_logits, draft, q, temperature: float, seed: int, offset: int):
    dt = _logits_dtype(target_logits)
    _need(draft, torch.int64, "draft")
    _need(q, torch.float32, "q")
    B, K1, V = target_logits.shape
    acc = torch.empty(B, device=draft.device, dtype=torch.int64)
    bonus = torch.empty_like(acc)
    wsb = _lib.load().fm_accept_workspace_size(B, K1 - 1)
    ws = torch.empty(wsb, dtype=torch.uint8, device=draft.device)
    _lib.call("fm_accept_rejection", _p(target_logits), dt, _p(draft), _p(q), B, K1 - 1, V, float(temperature),
              int(seed), int(offset), _p(acc), _p(bonus), _p(ws), wsb, _stream())
    return acc, bonus


def transpose(x):
    _need(x, torch.bfloat16, "x")
    R, C = x.shape
    out = torch.empty(C, R, device=x.device, dtype=x.dtype)
    _lib.call("fm_transpose_bf16", _p(x), _p(out), R, C, _stream())
    return out


def time_freqs(dim: int) -> torch.Tensor:
    """``exp(-ln(10000) i / half)`` in fp32, the reference's expression (modeling_flashmap.py:94)."""
    half = dim // 2
    return torch.exp(-math.log(10000.0) * torch.arange(half).float() / half)


def time_sinusoid(dim: int, s: float, t: float, scale: float, device="cuda"):
    """Rows 0 and 1: sinusoidal features of ``s`` and ``t`` (bf16)."""
    out = torch.empty(2, dim, device=device, dtype=torch.bfloat16)
    freqs = time_freqs(dim).to(device)
    _lib.call("fm_time_sinusoid", _p(out), dim, float(s), float(t), float(scale), _p(freqs), _stream())
    return out


def silu(x):
    _need(x, torch.bfloat16, "x")
    y = torch.empty_like(x)
    _lib.call("fm_silu", _p(x), _p(y), x.numel(), _stream())
    return y


def add(a, b):
    _need(a, torch.bfloat16, "a")
    _need(b, torch.bfloat16, "b")
    y = torch.empty_like(a)
    _lib.call("fm_add", _p(a), _p(b), _p(y), a.numel(), _stream())
    return y


def attention_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
