"""ctypes wrapper of the C acceptance oracle (``accept_oracle.c``; test infrastructure).

Restates modeling_flashmap.py:553-557 (draft sampling), :579-582 (greedy
acceptance) and :583-594 (rejection sampling) with Philox-injected uniforms;
see the C file's header for the exact arithmetic.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libfm_oracle.so")
_lib = None

_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    """Compile the C oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        try:
            build()  # make rebuilds the library when accept_oracle.c is newer
        except (OSError, subprocess.CalledProcessError):
            if not os.path.exists(_LIB_PATH):
                raise
        L = ctypes.CDLL(_LIB_PATH)
        L.fmo_exp.restype = ctypes.c_float
        L.fmo_exp.argtypes = [ctypes.c_float]
        L.fmo_exp_shifter.restype = ctypes.c_float
        L.fmo_exp_shifter.argtypes = [ctypes.c_float, ctypes.POINTER(ctypes.c_int)]
        L.fmo_exp_shifter_sweep.restype = ctypes.c_int64
        L.fmo_exp_shifter_sweep.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int64,
                                            ctypes.POINTER(ctypes.c_int64)]
        L.fmo_uniform.restype = ctypes.c_float
        L.fmo_uniform.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32]
        L.fmo_philox.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint32)]
        L.fmo_row_stats.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float, _f32p, _f32p]
        L.fmo_rejection_row_stats.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float, _f32p, _f32p]
        L.fmo_argmax.restype = ctypes.c_int64
        L.fmo_argmax.argtypes = [_f32p, ctypes.c_int64]
        L.fmo_categorical.restype = ctypes.c_int64
        L.fmo_categorical.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float]
        L.fmo_categorical_sliced.restype = ctypes.c_int64
        L.fmo_categorical_sliced.argtypes = [_f32p, ctypes.c_int64, ctypes.c_float]
        L.fmo_softmax_rows.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _f32p]
        L.fmo_sample_rows.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                      ctypes.c_uint64, ctypes.c_uint32, _i64p, _f32p]
        L.fmo_accept_greedy.argtypes = [_f32p, _i64p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _i64p, _i64p]
        L.fmo_accept_rejection.argtypes = [_f32p, _i64p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_float, ctypes.c_uint64, ctypes.c_uint32, _i64p, _i64p, _f32p]
        _lib = L
    return _lib


def _rows(t: torch.Tensor) -> np.ndarray:
    """Logit rows as fp32 (bf16 widens exactly)."""
    assert t.dtype in (torch.bfloat16, torch.float32)
    return np.ascontiguousarray(t.detach().cpu().float().contiguous().numpy())


def _ptr(a: np.ndarray, typ):
    return a.ctypes.data_as(typ)


def fm_exp(x: float) -> float:
    return lib().fmo_exp(float(x))


def fm_exp_shifter(x: float):
    """The kernels' paired formulation of fm_exp for one lane: (value, fast)."""
    fast = ctypes.c_int()
    v = lib().fmo_exp_shifter(float(x), ctypes.byref(fast))
    return v, bool(fast.value)


def fm_exp_shifter_sweep(start: int, stride: int, count: int):
    """Over the float bit patterns start + i * stride (i < count, modulo 2^32):
    (inputs on the fast path, those whose value differs from fm_exp)."""
    fast = ctypes.c_int64()
    bad = lib().fmo_exp_shifter_sweep(start & 0xFFFFFFFF, stride & 0xFFFFFFFF, int(count), ctypes.byref(fast))
    return fast.value, bad


def philox(ctr, seed: int) -> list:
    c = (ctypes.c_uint32 * 4)(*[int(v) & 0xFFFFFFFF for v in ctr])
    out = (ctypes.c_uint32 * 4)()
    lib().fmo_philox(c, int(seed), out)
    return list(out)


def uniform(seed: int, a: int, b: int, c: int, purpose: int) -> float:
    return lib().fmo_uniform(int(seed), a, b, c, purpose)


def row_stats(row: torch.Tensor, temperature: float = 1.0):
    bits = _rows(row.reshape(-1))
    m, s = ctypes.c_float(), ctypes.c_float()
    lib().fmo_row_stats(_ptr(bits, _f32p), bits.size, float(temperature), ctypes.byref(m), ctypes.byref(s))
    return m.value, s.value


def rejection_row_stats(row: torch.Tensor, temperature: float = 1.0):
    """(m, S) of a target row as the rejection step forms them: the max of
    x / T and the slice-major fixed-order sum of fm_exp(x / T - m)."""
    bits = _rows(row.reshape(-1))
    m, s = ctypes.c_float(), ctypes.c_float()
    lib().fmo_rejection_row_stats(_ptr(bits, _f32p), bits.size, float(temperature), ctypes.byref(m),
                                  ctypes.byref(s))
    return m.value, s.value


def categorical(weights: np.ndarray, u: float) -> int:
    w = np.ascontiguousarray(weights, dtype=np.float32)
    return int(lib().fmo_categorical(_ptr(w, _f32p), w.size, float(u)))


def categorical_sliced(weights: np.ndarray, u: float) -> int:
    """The rejection bonus draw: the sliced form of ``categorical`` (slices of
    256 ranges of 32 weights, slice totals summed in order)."""
    w = np.ascontiguousarray(weights, dtype=np.float32)
    return int(lib().fmo_categorical_sliced(_ptr(w, _f32p), w.size, float(u)))


def softmax_rows(logits: torch.Tensor, temperature: float = 1.0) -> torch.Tensor:
    """fp32 probabilities of each row (bf16 or fp32 logits), by the fixed-order softmax."""
    bits = _rows(logits)
    V = logits.shape[-1]
    rows = bits.size // V
    out = np.empty(bits.size, dtype=np.float32)
    lib().fmo_softmax_rows(_ptr(bits, _f32p), rows, V, float(temperature), _ptr(out, _f32p))
    return torch.from_numpy(out).view(*logits.shape)


def sample_rows(logits: torch.Tensor, temperature: float, seed: int = 1234, offset: int = 0):
    """Draft tokens (B, K) and, for T > 0, their probabilities (B, K, V)."""
    B, K, V = logits.shape
    bits = _rows(logits)
    tokens = np.empty(B * K, dtype=np.int64)
    probs = np.zeros(B * K * V if temperature > 0 else 1, dtype=np.float32)
    lib().fmo_sample_rows(_ptr(bits, _f32p), B, K, V, float(temperature), int(seed), int(offset),
                          _ptr(tokens, _i64p), _ptr(probs, _f32p))
    toks = torch.from_numpy(tokens).view(B, K)
    return toks, (torch.from_numpy(probs).view(B, K, V) if temperature > 0 else None)


def accept_greedy(target_logits: torch.Tensor, draft: torch.Tensor):
    """(B, K+1, V) bf16/fp32, (B, K) int -> accepted (B,), bonus (B,) int64."""
    B, K1, V = target_logits.shape
    bits = _rows(target_logits)
    d = np.ascontiguousarray(draft.cpu().numpy().astype(np.int64))
    acc = np.empty(B, dtype=np.int64)
    bonus = np.empty(B, dtype=np.int64)
    lib().fmo_accept_greedy(_ptr(bits, _f32p), _ptr(d, _i64p), B, K1 - 1, V, _ptr(acc, _i64p), _ptr(bonus, _i64p))
    return torch.from_numpy(acc), torch.from_numpy(bonus)


def accept_rejection(target_logits: torch.Tensor, draft: torch.Tensor, q: torch.Tensor, temperature: float,
                     seed: int = 1234, offset: int = 0):
    """Rejection sampling of :583-594 with Philox uniforms -> accepted (B,), bonus (B,)."""
    B, K1, V = target_logits.shape
    bits = _rows(target_logits)
    d = np.ascontiguousarray(draft.cpu().numpy().astype(np.int64))
    qq = np.ascontiguousarray(q.detach().cpu().float().numpy())
    acc = np.empty(B, dtype=np.int64)
    bonus = np.empty(B, dtype=np.int64)
    scratch = np.empty(V, dtype=np.float32)
    lib().fmo_accept_rejection(_ptr(bits, _f32p), _ptr(d, _i64p), _ptr(qq, _f32p), B, K1 - 1, V, float(temperature),
                               int(seed), int(offset), _ptr(acc, _i64p), _ptr(bonus, _i64p), _ptr(scratch, _f32p))
    return torch.from_numpy(acc), torch.from_numpy(bonus)


__all__ = [
    "accept_greedy",
    "accept_rejection",
    "build",
    "categorical",
    "categorical_sliced",
    "fm_exp",
    "fm_exp_shifter",
    "fm_exp_shifter_sweep",
    "philox",
    "rejection_row_stats",
    "row_stats",
    "sample_rows",
    "softmax_rows",
    "uniform",
]
