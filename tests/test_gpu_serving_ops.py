"""GPU parity of the serving-plugin operators (flashmap_b200.serving_ops, on the
kernels of serving.cu) against the CPU restatement in oracle/serving_ops.py.

Tolerances, written per check:
* norms and RoPE: bf16 outputs within 2 bf16 ulps plus 8e-3 of the row's
  largest value, and at least 97% of the elements bit-equal (the fp32 sums run
  in a different order, so the bf16-rounded scale of a row may land one bf16
  step, 2^-8 relative, away; the rotation mixes two such values);
* attention: |got - ref| <= 2e-2 * max|ref| (bf16 inputs and outputs, fp32
  softmax, bf16 numerators as in FlashAttention) and a mean error below 2e-3;
* cache writers: values copied bit-exactly; keys like the norms; e4m3 bytes
  equal on at least 97% of the elements and within one e4m3 step elsewhere.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import _lib  # noqa: E402
from flashmap_b200 import serving_ops as S  # noqa: E402
from oracle import serving_ops as R  # noqa: E402

DEV = "cuda"
FP8 = torch.float8_e4m3fn


@pytest.fixture(scope="module", autouse=True)
def device_ok():
    _lib.require_device()


def _gen(seed):
    return torch.Generator().manual_seed(seed)


def _ulp(x):
    e = torch.floor(torch.log2(x.abs().clamp_min(1e-30)))
    return torch.pow(2.0, e - 7)


def assert_rows_close(got, ref, what, min_exact=0.97):
    g, r = got.float().cpu(), ref.float().cpu()
    assert g.shape == r.shape, what
    assert torch.isfinite(g).all(), what
    tol = 2 * _ulp(r) + 8e-3 * r.abs().amax(dim=-1, keepdim=True)
    bad = (g - r).abs() > tol
    assert not bad.any(), f"{what}: {int(bad.sum())} elements off, max diff {float((g - r).abs().max()):.4g}"
    exact = (g == r).float().mean().item()
    assert exact >= min_exact, f"{what}: only {exact:.4f} bit-equal"


def assert_attn_close(got, ref, what):
    g, r = got.float().cpu(), ref.float().cpu()
    assert g.shape == r.shape, what
    assert torch.isfinite(g).all(), what
    scale = r.abs().max().clamp_min(1e-6)
    err = (g - r).abs()
    assert err.max() <= 2e-2 * scale, f"{what}: max err {float(err.max()):.4g} vs scale {float(scale):.4g}"
    assert err.mean() <= 2e-3 * scale, f"{what}: mean err {float(err.mean()):.4g}"


def assert_fp8_close(got, ref, what):
    gb, rb = got.view(torch.uint8).cpu(), ref.view(torch.uint8).cpu()
    exact = (gb == rb).float().mean().item()
    assert exact >= 0.97, f"{what}: only {exact:.4f} of the e4m3 bytes equal"
    g, r = got.float().cpu(), ref.float().cpu()
    assert ((g - r).abs() <= 0.13 * r.abs() + 2e-3).all(), f"{what}: e4m3 values more than one step apart"


# --------------------------------------------------------------------------- norms and RoPE


@pytest.mark.parametrize("wdtype", [torch.bfloat16, torch.float32])
def test_vllm_rms_norm(wdtype):
    g = _gen(0)
    x = torch.randn(37, 2048, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(2048, generator=g)).to(torch.bfloat16).to(wdtype)
    got = torch.ops.flashmap_vllm.rms_norm(x.to(DEV), w.to(DEV), 1e-6)
    assert_rows_close(got, R.rms_norm(x, w, 1e-6), "rms_norm")


@pytest.mark.parametrize("hd,pdtype", [(128, torch.int64), (64, torch.int32)])
def test_vllm_rms_norm_rope(hd, pdtype):
    g = _gen(1)
    x = torch.randn(50, 4, hd, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    table = R.rope_pairs(5000, hd, 1e4)
    pos = torch.randint(0, 5000, (50,), generator=g).to(pdtype)
    got = torch.ops.flashmap_vllm.rms_norm_rope(x.to(DEV), w.to(DEV), table.to(DEV), pos.to(DEV), 1e-5)
    assert_rows_close(got, R.rms_norm_rope_vllm(x, w, table, pos, 1e-5), "rms_norm_rope")


def test_vllm_rope_table_matches_restatement():
    got = S.rope_table(3000, 128, 1e4, DEV).cpu()
    ref = R.rope_pairs(3000, 128, 1e4)
    assert got.shape == ref.shape
    assert (got - ref).abs().max() <= 1e-5


def test_sglang_rms_norm_rope():
    g = _gen(2)
    x = torch.randn(2, 16, 4, 128, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).float()
    pos = torch.randint(0, 8000, (2, 16), generator=g)
    freqs = R.rope_pairs(8000, 128, 1e6)[pos]
    got = torch.ops.flashmap_sglang.rms_norm_rope(x.to(DEV), w.to(DEV), freqs.to(DEV), 1e-5)
    assert_rows_close(got, R.rms_norm_rope_sglang(x, w, freqs, 1e-5), "sglang rms_norm_rope")
    got2 = S.sglang_rms_norm(x.view(-1, 128).to(DEV), w.to(DEV), 1e-6)
    assert_rows_close(got2, R.rms_norm(x.view(-1, 128), w, 1e-6), "sglang rms_norm")


# --------------------------------------------------------------------------- block self-attention


@pytest.mark.parametrize("blocks,T,H,hd", [(5, 16, 4, 128), (3, 16, 8, 64), (2, 8, 2, 64)])
def test_vllm_block_self_attention(blocks, T, H, hd):
    g = _gen(3)
    qkv = torch.randn(blocks, T, 3, H, hd, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16)
    table = R.rope_pairs(4096, hd, 1e4)
    anchor = torch.randint(0, 4000, (blocks, 1), generator=g)
    pos = (anchor + 1 + torch.arange(T)).reshape(-1)
    got = torch.ops.flashmap_vllm.block_self_attention(qkv.to(DEV), qn.to(DEV), kn.to(DEV), table.to(DEV),
                                                       pos.to(DEV), 1e-5)
    cos, sin = table[pos, :, 0].view(blocks, T, -1), table[pos, :, 1].view(blocks, T, -1)
    ref = R.block_self_attention(qkv, qn, kn, cos, sin, 1e-5)
    assert_attn_close(got.view(blocks, T, H, hd), ref, "vllm block_self_attention")


def test_sglang_block_self_attention():
    g = _gen(4)
    blocks, T, H, hd = 6, 16, 4, 128
    qkv = torch.randn(blocks, T, 3, H, hd, generator=g).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16).float()
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(torch.bfloat16).float()
    pos = torch.randint(0, 9000, (blocks, 1), generator=g) + torch.arange(T)
    freqs = R.rope_pairs(9100, hd, 1e6)[pos].contiguous()
    got = torch.ops.flashmap_sglang.block_self_attention(qkv.to(DEV), qn.to(DEV), kn.to(DEV), freqs.to(DEV), 1e-5)
    ref = R.block_self_attention(qkv, qn, kn, freqs[..., 0], freqs[..., 1], 1e-5)
    assert got.shape == (blocks, T, H, hd)
    assert_attn_close(got, ref, "sglang block_self_attention")


# --------------------------------------------------------------------------- paged cross-attention


def _vllm_case(g, hd, H, page, seqused, qrows, num_blocks, dtype=torch.bfloat16):
    R_ = len(seqused)
    cols = max(1, max((s + page - 1) // page for s in seqused))
    perm = torch.randperm(num_blocks, generator=g)
    table = perm[: R_ * cols].view(R_, cols).int()
    cache = torch.randn(num_blocks, H, page, 2 * hd, generator=g)
    cu = torch.tensor([0] + list(torch.tensor(qrows).cumsum(0)), dtype=torch.int32)
    q = torch.randn(int(cu[-1]), H, hd, generator=g)
    return table, cache, cu, q


@pytest.mark.parametrize("hd,page", [(128, 16), (64, 32)])
def test_vllm_paged_cross_attention(hd, page):
    g = _gen(5)
    H = 4
    seqused = [700, 1, 0, 260, 33]
    qrows = [16, 5, 16, 1, 40]
    table, cache, cu, q = _vllm_case(g, hd, H, page, seqused, qrows, 240)
    cache = cache.to(torch.bfloat16)
    q = q.to(torch.bfloat16)
    su = torch.tensor(seqused, dtype=torch.int32)
    got = torch.ops.flashmap_vllm.paged_cross_attention(q.to(DEV), cache.to(DEV), cu.to(DEV), su.to(DEV),
                                                        table.to(DEV), None, None, max(qrows), max(seqused),
                                                        hd ** -0.5, 3)
    ranges = [(int(cu[i]), int(cu[i + 1])) for i in range(len(seqused))]
    ref = R.paged_attention(q.float(), R.gather_vllm(cache, table, hd), seqused, ranges, hd ** -0.5)
    assert_attn_close(got, ref, "vllm paged attention")
    a, b = ranges[2]
    assert torch.equal(got[a:b].float().cpu(), torch.zeros(b - a, H, hd))  # no context: zero rows


def test_vllm_paged_cross_attention_fp8():
    g = _gen(6)
    hd, H, page = 128, 4, 16
    seqused = [513, 64, 1000]
    qrows = [16, 16, 7]
    table, cache, cu, q = _vllm_case(g, hd, H, page, seqused, qrows, 200)
    cache8 = (2 * cache).to(FP8)
    q8 = (2 * q).to(FP8)
    R_ = len(seqused)
    descales = 0.5 + torch.rand(3, R_, H, generator=g)
    su = torch.tensor(seqused, dtype=torch.int32)
    got = torch.ops.flashmap_vllm.paged_cross_attention(q8.to(DEV), cache8.to(DEV), cu.to(DEV), su.to(DEV),
                                                        table.to(DEV), None, descales.to(DEV), 16, max(seqused),
                                                        hd ** -0.5, 3)
    ranges = [(int(cu[i]), int(cu[i + 1])) for i in range(R_)]
    qf = q8.float().clone()
    for r, (a, b) in enumerate(ranges):
        qf[a:b] *= descales[0, r][None, :, None]
    ref = R.paged_attention(qf, R.gather_vllm(cache8, table, hd, descales), seqused, ranges, hd ** -0.5)
    assert_attn_close(got, ref, "vllm paged attention (e4m3)")


@pytest.mark.parametrize("fp8", [False, True])
def test_sglang_paged_cross_attention(fp8):
    g = _gen(7)
    bs, K, H, hd, rows = 3, 16, 4, 128, 900
    lens = [300, 17, 1]
    page_table = torch.stack([torch.randperm(rows, generator=g)[:300] for _ in range(bs)]).int()
    kb = torch.randn(rows, H, hd, generator=g)
    vb = torch.randn(rows, H, hd, generator=g)
    kb, vb = (kb.to(FP8), vb.to(FP8)) if fp8 else (kb.to(torch.bfloat16), vb.to(torch.bfloat16))
    query = torch.randn(bs, K, H, hd, generator=g).to(torch.bfloat16)
    seqlens = torch.tensor(lens, dtype=torch.int32)
    op = torch.ops.flashmap_sglang.paged_cross_attention_fp8 if fp8 else torch.ops.flashmap_sglang.paged_cross_attention
    got = op(query.to(DEV), kb.to(DEV), vb.to(DEV), seqlens.to(DEV), page_table.to(DEV),
             torch.zeros(1, dtype=torch.int32, device=DEV))
    qf = R.quantize_query_fp8(query) if fp8 else query.float()
    ref = R.paged_attention(qf.view(bs * K, H, hd), R.gather_pool(kb, vb, page_table), lens,
                            [(r * K, (r + 1) * K) for r in range(bs)], hd ** -0.5)
    assert got.shape == query.shape
    assert_attn_close(got.view(bs * K, H, hd), ref, f"sglang paged attention (fp8={fp8})")


# --------------------------------------------------------------------------- cache writers


@pytest.mark.parametrize("hpc,fp8", [(None, False), (3, False), (None, True)])
def test_vllm_write_context_kv(hpc, fp8):
    g = _gen(8)
    T, L, H, hd, bs, nblk = 40, 2, 4, 128, 16, 12
    per = hpc or H
    n_caches = (L * H + per - 1) // per
    kv = torch.randn(T, L, 2, H, hd, generator=g).to(torch.bfloat16)
    k_norm = (1 + 0.1 * torch.randn(L, hd, generator=g)).to(torch.bfloat16)
    table = R.rope_pairs(6000, hd, 1e4)
    pos = torch.randint(0, 6000, (T,), generator=g)
    slots = torch.randperm(nblk * bs, generator=g)[:T]
    slots[3] = -1
    dt = FP8 if fp8 else torch.bfloat16
    caches = [torch.zeros(nblk, per, bs, 2 * hd, dtype=dt, device=DEV) for _ in range(n_caches)]
    ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64, device=DEV)
    c0 = caches[0]
    strides = (c0.stride(0), c0.stride(1), c0.stride(2), hd)
    scales = (0.5 + torch.rand(L, 2, generator=g)) if fp8 else None
    S.write_context_kv(kv.to(DEV), pos.to(DEV), slots.to(DEV), k_norm.to(DEV), table.to(DEV), ptrs, strides, bs,
                       1e-5, scales=None if scales is None else scales.to(DEV), heads_per_cache=hpc)
    torch.cuda.synchronize()
    ref = [torch.zeros(c.numel(), dtype=dt) for c in caches]
    R.write_context_kv(kv, pos, slots, k_norm, table, ref, strides, bs, 1e-5, scales=scales, heads_per_cache=hpc)
    for c, r in zip(caches, ref):
        got = c.view(-1).cpu().view(-1, 2 * hd)
        want = r.view(-1, 2 * hd)
        if fp8:
            assert_fp8_close(got[:, :hd], want[:, :hd], "e4m3 keys")
            assert_fp8_close(got[:, hd:], want[:, hd:], "e4m3 values")
        else:
            assert_rows_close(got[:, :hd], want[:, :hd], "keys")
            assert torch.equal(got[:, hd:], want[:, hd:]), "values"


@pytest.mark.parametrize("fp8,commit", [(False, False), (True, True)])
def test_sglang_kv_norm_rope_write(fp8, commit):
    g = _gen(9)
    T, L, H, hd, rows = 48, 3, 4, 128, 200
    kv_size = H * hd
    kv = torch.randn(T, L * 2 * kv_size, generator=g).to(torch.bfloat16)
    k_norm = (1 + 0.1 * torch.randn(L, hd, generator=g)).to(torch.bfloat16).float()
    pairs = R.rope_pairs(7000, hd, 1e6)
    cos_sin = torch.cat([pairs[..., 0], pairs[..., 1]], dim=-1).contiguous()
    pos = torch.randint(0, 7000, (T,), generator=g)
    locs = torch.randperm(rows, generator=g)[:T]
    locs[5] = -1
    dt = FP8 if fp8 else torch.bfloat16
    kp = [torch.zeros(rows, kv_size, dtype=dt, device=DEV) for _ in range(L)]
    vp = [torch.zeros(rows, kv_size, dtype=dt, device=DEV) for _ in range(L)]
    meta = torch.tensor([[k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0)] for k, v in zip(kp, vp)],
                        dtype=torch.int64, device=DEV)
    commit_lens = torch.tensor([16, 3, 0], dtype=torch.int32) if commit else None
    kw = dict(commit_lens=None if commit_lens is None else commit_lens.to(DEV), locs_row_width=16 if commit else None)
    if fp8:
        S.kv_norm_rope_write_fp8(kv.to(DEV), meta, k_norm.to(DEV), cos_sin.to(DEV), pos.to(DEV), locs.to(DEV), L,
                                 kv_size, hd, 1e-5, k_scale=0.75, v_scale=1.25, **kw)
    else:
        S.kv_norm_rope_write(kv.to(DEV), meta, k_norm.to(DEV), cos_sin.to(DEV), pos.to(DEV), locs.to(DEV), L,
                             kv_size, hd, 1e-5, **kw)
    torch.cuda.synchronize()
    rk = [torch.zeros(rows, kv_size, dtype=dt) for _ in range(L)]
    rv = [torch.zeros(rows, kv_size, dtype=dt) for _ in range(L)]
    R.kv_norm_rope_write_pool(kv, rk, rv, k_norm, cos_sin, pos, locs, L, kv_size, hd, 1e-5, fp8,
                              k_scale=0.75 if fp8 else 1.0, v_scale=1.25 if fp8 else 1.0, commit_lens=commit_lens,
                              row_width=16)
    for layer in range(L):
        if fp8:
            assert_fp8_close(kp[layer].cpu(), rk[layer], "e4m3 pool keys")
            assert_fp8_close(vp[layer].cpu(), rv[layer], "e4m3 pool values")
        else:
            assert_rows_close(kp[layer].cpu().view(rows, H, hd), rk[layer].view(rows, H, hd), "pool keys")
            assert torch.equal(vp[layer].cpu(), rv[layer]), "pool values"
