"""The allocation-free greedy acceptance (fm_accept_greedy_noalloc) against the
workspace version (fm_accept_greedy), through the C ABI.

Callers that cannot allocate device memory while they accept a block -- an
engine that plans its buffers before capturing a CUDA graph, or host code in
another language that only holds the tensors it was given -- use the
allocation-free entry point; its scratch is a fixed array in the library.
Acceptance counts and bonus tokens are integers, so the two entry points must
agree exactly, on two calls in a row (the second call must not see the first
call's scratch).  This file is collected last on purpose.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import _lib  # noqa: E402
from tests.golden.inputs import acceptance_inputs  # noqa: E402

DEV = "cuda"


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _with_workspace(lib, target, draft):
    B, K1, V = target.shape
    acc = torch.empty(B, dtype=torch.int64, device=DEV)
    bonus = torch.empty_like(acc)
    wsb = lib.fm_accept_workspace_size(B, K1 - 1)
    ws = torch.empty(wsb, dtype=torch.uint8, device=DEV)
    dt = 0 if target.dtype == torch.bfloat16 else 1
    _lib.check(lib.fm_accept_greedy(_p(target), dt, _p(draft), B, K1 - 1, V, _p(acc), _p(bonus), _p(ws), wsb,
                                    _stream()), "fm_accept_greedy")
    return acc, bonus


def _no_alloc(lib, target, draft):
    B, K1, V = target.shape
    acc = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    bonus = torch.full((B,), -1, dtype=torch.int64, device=DEV)
    dt = 0 if target.dtype == torch.bfloat16 else 1
    _lib.check(lib.fm_accept_greedy_noalloc(_p(target), dt, _p(draft), B, K1 - 1, V, _p(acc), _p(bonus), _stream()),
               "fm_accept_greedy_noalloc")
    return acc, bonus


def test_no_alloc_greedy_acceptance_matches_workspace_version():
    _lib.require_device()
    lib = _lib.load()
    cases = [(34, 16, 3001, 5, torch.bfloat16), (8, 16, 151936, 11, torch.float32)]
    for B, K, V, seed, dtype in cases:  # two calls in a row, different shapes and inputs
        target, draft, _ = acceptance_inputs(B, K, V, seed, 0.0)
        target = target.to(DEV, dtype).contiguous()
        draft = draft.to(DEV).contiguous()
        ref_acc, ref_bonus = _with_workspace(lib, target, draft)
        acc, bonus = _no_alloc(lib, target, draft)
        torch.cuda.synchronize()
        assert acc.tolist() == ref_acc.tolist()
        assert bonus.tolist() == ref_bonus.tolist()


def test_no_alloc_rejects_calls_beyond_its_scratch():
    lib = _lib.load()
    target = torch.zeros(1, 2, 8, dtype=torch.bfloat16, device=DEV)
    draft = torch.zeros(1, 1, dtype=torch.int64, device=DEV)
    acc = torch.empty(1, dtype=torch.int64, device=DEV)
    rows = 16384  # FM_ACCEPT_NOALLOC_MAX_ROWS
    st = lib.fm_accept_greedy_noalloc(_p(target), 0, _p(draft), rows, 1, 8, _p(acc), _p(acc), _stream())
    assert st == 8  # FM_ERR_WORKSPACE, before any launch
    assert b"scratch" in lib.fm_last_error()
