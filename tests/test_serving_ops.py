"""CPU checks of the serving-plugin operators: the op names and argument lists
of the reference's torch.library ops, shape propagation under fake tensors
(what torch.compile traces), argument errors raised before any CUDA call, and
self-consistency of the CPU restatement the GPU tests compare with."""

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from flashmap_b200 import serving_ops as S
from oracle import flashmap_oracle as O
from oracle import serving_ops as R

# argument names of the reference's ops (flashmap/vllm/kernels.py:48, 100, 193;
# flashmap/vllm/model.py:93; flashmap/sglang/kernels.py:84, 170; flashmap/sglang/model.py:127, 154)
SCHEMAS = {
    ("flashmap_vllm", "rms_norm"): ["x", "weight", "eps"],
    ("flashmap_vllm", "rms_norm_rope"): ["x", "weight", "cos_sin", "positions", "eps"],
    ("flashmap_vllm", "block_self_attention"): ["qkv", "q_norm", "k_norm", "cos_sin", "positions", "eps"],
    ("flashmap_vllm", "paged_cross_attention"): ["query", "kv_cache", "cu_seqlens_q", "seqused_k", "block_table",
                                                 "scheduler_metadata", "descales", "max_seqlen_q", "max_seqlen_k",
                                                 "softmax_scale", "fa_version"],
    ("flashmap_sglang", "block_self_attention"): ["qkv", "q_norm", "k_norm", "freqs", "eps"],
    ("flashmap_sglang", "rms_norm_rope"): ["x", "weight", "freqs", "eps"],
    ("flashmap_sglang", "paged_cross_attention"): ["query", "key_buffer", "value_buffer", "cache_seqlens",
                                                   "page_table", "scheduler_metadata"],
    ("flashmap_sglang", "paged_cross_attention_fp8"): ["query", "key_buffer", "value_buffer", "cache_seqlens",
                                                       "page_table", "scheduler_metadata"],
}


@pytest.mark.parametrize("ns,name", sorted(SCHEMAS))
def test_ops_registered_with_reference_arguments(ns, name):
    op = getattr(getattr(torch.ops, ns), name).default
    assert [a.name for a in op._schema.arguments] == SCHEMAS[(ns, name)]
    assert len(op._schema.returns) == 1
    assert not op._schema.is_mutable


def test_fake_shapes():
    with FakeTensorMode():
        qkv = torch.empty(3, 16, 3, 4, 64, dtype=torch.bfloat16)
        w = torch.empty(64, dtype=torch.bfloat16)
        table = torch.empty(100, 32, 2)
        pos = torch.empty(48, dtype=torch.int64)
        out = torch.ops.flashmap_vllm.block_self_attention(qkv, w, w, table, pos, 1e-5)
        assert out.shape == (48, 256) and out.dtype == torch.bfloat16
        freqs = torch.empty(3, 16, 32, 2)
        out = torch.ops.flashmap_sglang.block_self_attention(qkv, w.float(), w.float(), freqs, 1e-5)
        assert out.shape == (3, 16, 4, 64)
        x = torch.empty(10, 4, 64, dtype=torch.bfloat16)
        assert torch.ops.flashmap_vllm.rms_norm_rope(x, w, table, pos[:10], 1e-5).shape == x.shape
        q = torch.empty(20, 4, 64, dtype=torch.bfloat16)
        cache = torch.empty(8, 4, 16, 128, dtype=torch.bfloat16)
        i32 = torch.empty(3, dtype=torch.int32)
        o = torch.ops.flashmap_vllm.paged_cross_attention(q, cache, torch.empty(4, dtype=torch.int32), i32,
                                                          torch.empty(3, 8, dtype=torch.int32), None, None, 16, 64,
                                                          0.125, 3)
        assert o.shape == q.shape and o.dtype == torch.bfloat16
        q4 = torch.empty(2, 16, 4, 64, dtype=torch.bfloat16)
        pool = torch.empty(300, 4, 64, dtype=torch.bfloat16)
        o = torch.ops.flashmap_sglang.paged_cross_attention(q4, pool, pool, i32[:2],
                                                            torch.empty(2, 150, dtype=torch.int32), i32)
        assert o.shape == q4.shape


def test_argument_errors_before_cuda():
    x = torch.zeros(4, 2, 64, dtype=torch.bfloat16)
    w = torch.ones(64, dtype=torch.bfloat16)
    table = R.rope_pairs(16, 64, 1e4)
    with pytest.raises(AssertionError):
        S.vllm_rms_norm_rope(x, w, table, torch.zeros(4, dtype=torch.int64), 1e-5)
    with pytest.raises(ValueError):
        S.sglang_rms_norm(x.float(), w.float(), 1e-6)
    with pytest.raises(S.OpArgumentError):
        S.kv_norm_rope_write(x.view(4, 128), None, None, None, None, None, 1, 64, 64, 1e-5, is_neox_style=True)


def test_restated_norm_rope_is_the_hf_path():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(9, 3, 64, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(64, generator=g)).to(torch.bfloat16)
    table = R.rope_pairs(40, 64, 1e4)
    pos = torch.randint(0, 40, (9,), generator=g)
    assert R.check_apply_rope_agrees(x, w, table, pos, 1e-5)


def test_restated_paged_attention_is_dense_attention():
    """Gathering pages through a shuffled table equals attention over the
    contiguous context (the page table only relocates rows)."""
    g = torch.Generator().manual_seed(1)
    H, hd, page, n = 2, 64, 16, 45
    ctx_k = torch.randn(n, H, hd, generator=g).to(torch.bfloat16)
    ctx_v = torch.randn(n, H, hd, generator=g).to(torch.bfloat16)
    blocks = torch.randperm(8, generator=g)[:3]
    cache = torch.zeros(8, H, page, 2 * hd, dtype=torch.bfloat16)
    for p in range(n):
        cache[blocks[p // page], :, p % page, :hd] = ctx_k[p]
        cache[blocks[p // page], :, p % page, hd:] = ctx_v[p]
    q = torch.randn(5, H, hd, generator=g).to(torch.bfloat16).float()
    got = R.paged_attention(q, R.gather_vllm(cache, blocks[None].int(), hd), [n], [(0, 5)], hd ** -0.5)
    for h in range(H):
        ref = R.attend(q[:, h], ctx_k[:, h].float(), ctx_v[:, h].float(), hd ** -0.5)
        assert torch.equal(got[:, h], ref)


def test_restated_writer_matches_hf_keys():
    """The paged writer's keys are the HF path's k_norm + RoPE keys (modeling_flashmap.py:139-141)."""
    g = torch.Generator().manual_seed(2)
    T, L, H, hd, bs = 3, 2, 2, 64, 4
    kv = torch.randn(T, L, 2, H, hd, generator=g).to(torch.bfloat16)
    k_norm = (1 + 0.1 * torch.randn(L, hd, generator=g)).to(torch.bfloat16)
    table = R.rope_pairs(32, hd, 1e4)
    pos = torch.tensor([3, 17, 30])
    slots = torch.tensor([5, -1, 9])
    sb, sh, st = H * bs * 2 * hd, bs * 2 * hd, 2 * hd
    caches = [torch.zeros(4 * sb, dtype=torch.bfloat16) for _ in range(L)]
    R.write_context_kv(kv, pos, slots, k_norm, table, caches, (sb, sh, st, hd), bs, 1e-5)
    for t in (0, 2):
        for layer in range(L):
            cos, sin = table[pos[t], :, 0], table[pos[t], :, 1]
            want = O.apply_rope(O.rms_norm(kv[t, layer, 0], k_norm[layer], 1e-5), (cos, sin))
            for h in range(H):
                off = (int(slots[t]) // bs) * sb + h * sh + (int(slots[t]) % bs) * st
                assert torch.equal(caches[layer][off:off + hd], want[h])
                assert torch.equal(caches[layer][off + hd:off + 2 * hd], kv[t, layer, 1, h])
