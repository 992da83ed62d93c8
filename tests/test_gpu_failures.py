"""Failure detection on the GPU without a GPU fault.

Every spin wait in the kernels is bounded (2 s of the global timer); a wait
that runs out records a code in the caller's device error word and the
kernel returns, so the context stays usable.  Index checks on values read
from device memory (anchor ids, positions, cache lengths) record
DEV_BAD_INDEX and skip the access.  These tests make both happen on
purpose -- a split-K count that can never be reached, an anchor id beyond
the vocabulary -- and then check that the error word holds the code and
that the same context still computes correct results.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import FlashMapCache, _lib, ops  # noqa: E402
from tests.helpers import CONFIG1, Emb, Head, build  # noqa: E402

DEV = "cuda"
DEV_BAD_INDEX = 4
DEV_TIMEOUT_OTHER = 5


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_bounded_split_k_wait_times_out_and_context_survives():
    """fm_gemm_bf16's workspace is [256 reserved bytes][one int32 counter per
    output tile, zero between calls][split-K partials].  With the counter of
    the only tile preset far below zero, the tile's head CTA never sees its
    contributors' count: its bounded wait gives up, the error word reads
    DEV_TIMEOUT_OTHER, the kernel returns and the output is left unwritten.
    A call with a clean workspace then computes the right product."""
    _lib.require_device()
    lib = _lib.load()
    M, N, K = 128, 16, 8192  # one output tile, 128 k-blocks split over many CTAs
    assert lib.fm_gemm_grid(M, N, K) > 1
    g = torch.Generator(device=DEV).manual_seed(0)
    W = torch.randn(M, K, generator=g, device=DEV).to(torch.bfloat16)
    X = torch.randn(N, K, generator=g, device=DEV).to(torch.bfloat16)
    out = torch.full((N, M), 7.0, device=DEV, dtype=torch.bfloat16)
    wsb = lib.fm_gemm_workspace_size(M, N, K)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=DEV)
    ws[256:260].view(torch.int32).fill_(-(1 << 30))
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.check(lib.fm_gemm_bf16(_p(W), _p(X), _p(out), M, N, K, M, None, None, ops.STORE, _p(ws), wsb, _p(err),
                                _stream()), "fm_gemm_bf16")
    torch.cuda.synchronize()
    assert int(err.item()) == DEV_TIMEOUT_OTHER
    assert bool((out.float() == 7.0).all()), "a tile whose wait gave up must not be written"
    # the context is intact: the same product with a clean workspace
    err.zero_()
    good = ops.gemm(W, X, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = X.float() @ W.float().T
    assert float((good.float() - ref).abs().max() / ref.abs().max()) < 1e-2


def test_out_of_range_anchor_records_bad_index():
    """A draft whose anchor id lies beyond the vocabulary: draft_prep records
    DEV_BAD_INDEX in the plan's error word and reads row 0 instead, the draft
    completes, the host check raises, and a draft with a valid anchor on the
    same plan afterwards reports no error."""
    config, model, _, emb, head = build(CONFIG1, seed=3, with_oracle=False)
    E, W = Emb(emb.to(DEV)), Head(head.to(DEV))
    K = config.block_size
    cache = FlashMapCache(config, 1, 64, device=DEV, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    hidden = torch.randn(1, 20, config.target_hidden_size, generator=g).to(torch.bfloat16)
    model.extend_context(cache, hidden.to(DEV), E, W)
    z = torch.randn(1, K, config.target_hidden_size, generator=g).to(torch.bfloat16).to(DEV)
    bad = torch.tensor([config.vocab_size + 5], device=DEV)
    model.draft(bad, cache, E, W, num_steps=1, z=z)
    torch.cuda.synchronize()
    plan = model._plan(model._pack(cache.kv.device, E, W), cache, 1, 1)  # the draft's own plan
    assert int(plan.err.item()) == DEV_BAD_INDEX
    with pytest.raises(_lib.FlashMapError):
        plan.check_device_errors()
    plan.err.zero_()
    logits = model.draft(torch.tensor([5], device=DEV), cache, E, W, num_steps=1, z=z)
    torch.cuda.synchronize()
    assert int(plan.err.item()) == 0
    assert bool(torch.isfinite(logits).all())
