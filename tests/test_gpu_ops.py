"""GPU parity of the primitive kernels against fp32 torch math and the CPU oracle.

Tolerances: bf16 outputs may differ from an fp32-accumulated reference only
by the order of fp32 summation, so at most one bf16 unit in the last place
and on a small fraction of elements; fp32 GEMM outputs within 1e-4 relative.
Sampling and acceptance are bit-exact against the C oracle.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU, skipped there
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import _lib, ops  # noqa: E402
from oracle import accept as oracle_accept  # noqa: E402
from oracle import flashmap_oracle as O  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def device_ok():
    _lib.require_device()


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    """Size of one bf16 unit in the last place at |x| (fp32 tensor)."""
    e = torch.floor(torch.log2(x.abs().clamp_min(1e-30)))
    return torch.pow(2.0, e - 7)


def assert_bf16_close(got: torch.Tensor, ref: torch.Tensor, max_ulps=1, min_exact=0.98, what=""):
    g, r = got.float(), ref.float()
    assert g.shape == r.shape
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    diff = (g - r).abs()
    tol = max_ulps * bf16_ulp(torch.maximum(g.abs(), r.abs())) + 1e-30
    bad = diff > tol
    if bad.any():
        idx = bad.nonzero()[:8].tolist()
        detail = "; ".join(f"{tuple(i)}: got {g[tuple(i)].item():.8g} ref {r[tuple(i)].item():.8g}" for i in idx)
        raise AssertionError(f"{what}: {int(bad.sum())} elements beyond {max_ulps} ulp: {detail}")
    exact = (g == r).float().mean().item()
    assert exact >= min_exact, f"{what}: only {exact:.4f} of elements bit-equal"


def assert_close_scaled(got, ref, ulps=1, atol_frac=1e-5, what="", extra_tol=None):
    """|got - ref| <= ulps * ulp(ref) + atol_frac * max|ref| (+ extra_tol): rounding
    differences only, with an absolute floor for values that cancel to ~0."""
    g, r = got.float(), ref.float()
    assert g.shape == r.shape
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    tol = ulps * bf16_ulp(r) + atol_frac * r.abs().max().clamp_min(1e-30)
    if extra_tol is not None:
        tol = tol + extra_tol
    bad = (g - r).abs() > tol
    if bad.any():
        idx = bad.nonzero()[:8].tolist()
        detail = "; ".join(f"{tuple(i)}: got {g[tuple(i)].item():.8g} ref {r[tuple(i)].item():.8g}" for i in idx)
        raise AssertionError(f"{what}: {int(bad.sum())} elements out of tolerance: {detail}")


def rand(shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


GEMM_SHAPES = [
    (128, 1, 64), (256, 16, 256), (2048, 16, 2048), (3000, 17, 320), (6144, 16, 2048), (2048, 16, 8192),
    (16384, 16, 4096), (512, 64, 1024), (512, 128, 1024), (1024, 200, 512), (2048, 1024, 2048), (384, 2048, 256),
    (4096, 5, 4096),
    # wide blocks split over up to 8 CTAs per tile (head-CTA fix-up from staged partials)
    (2048, 256, 2048), (256, 96, 4096), (640, 64, 8192), (2048, 1024, 8192),
    # at least two tiles per CTA over several column blocks: tiles relabelled column-major
    (40000, 512, 256), (20000, 300, 512),
    # 256-token blocks on CTA pairs (256 x 256 tiles): config-5 shapes, a pair
    # tile whose second half lies past M, ragged token tails in either half
    (7680, 1024, 2560), (2560, 1024, 2560), (13824, 1024, 2560), (130, 1000, 640), (5120, 257, 2560),
    # long reductions (>= 512 k-blocks) on whole tiles, all groups advancing through K together
    (4096, 1024, 32768), (14336, 100, 32768),
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_store_bias(M, N, K):
    W = rand((M, K), 1 / math.sqrt(K), 1)
    X = rand((N, K), 1.0, 2)
    b = rand((M,), 0.1, 3)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = ops.gemm(W, X, ops.STORE, bias=b, err=err)
    acc = X.float() @ W.float().T + b.float()
    ref = acc.to(torch.bfloat16)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # near a rounding boundary the fp32 sums of two summation orders may round apart
    near = ((acc - ref.float()).abs() > 0.45 * bf16_ulp(acc)).float().mean().item()
    # the two orders' fp32 sums drift apart further as K grows (one accumulator
    # over K / 16 tensor-core steps here): the absolute floor scales with K past 8192
    long_k = max(1.0, K / 8192)
    assert_close_scaled(out, ref, ulps=1, atol_frac=1e-5 * long_k, what=f"gemm {M}x{N}x{K} (near-boundary {near:.4f})")
    assert (out == ref).float().mean().item() > (0.98 if long_k == 1.0 else 0.95)


@pytest.mark.parametrize("M,N,K", [(2048, 16, 2048), (3000, 17, 320), (1024, 200, 512), (256, 96, 4096),
                                   (20000, 300, 512)])
def test_gemm_fp32_and_determinism(M, N, K):
    W = rand((M, K), 1 / math.sqrt(K), 4)
    X = rand((N, K), 1.0, 5)
    a = ops.gemm(W, X, ops.F32)
    b = ops.gemm(W, X, ops.F32)
    ref = X.float() @ W.float().T
    assert torch.equal(a, b), "split-K reduction must not depend on arrival order"
    torch.testing.assert_close(a, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("N", [16, 64, 300])
def test_gemm_gelu(N):
    M, K = 8192, 2048
    W = rand((M, K), 1 / math.sqrt(K), 6)
    X = rand((N, K), 1.0, 7)
    b = rand((M,), 0.1, 8)
    out = ops.gemm(W, X, ops.GELU, bias=b)
    y = (X.float() @ W.float().T + b.float()).to(torch.bfloat16).float()
    ref = (0.5 * y * (1.0 + torch.erf(y * 0.7071067811865476))).to(torch.bfloat16)
    # a one-ulp flip of the rounded pre-activation y moves gelu by about gelu'(y) * ulp(y)
    assert_close_scaled(out, ref, ulps=2, atol_frac=1e-5, what="gelu", extra_tol=1.2 * bf16_ulp(y))
    assert (out == ref).float().mean().item() > 0.97


@pytest.mark.parametrize("N,I,K", [(16, 384, 256), (48, 384, 256), (300, 384, 256), (1024, 6912, 2560)])
def test_gemm_swiglu(N, I, K):
    Wg = rand((I, K), 1 / math.sqrt(K), 9)
    Wu = rand((I, K), 1 / math.sqrt(K), 10)
    W = torch.stack([Wg.view(I // 64, 64, K), Wu.view(I // 64, 64, K)], dim=1).reshape(2 * I, K).contiguous()
    X = rand((N, K), 1.0, 11)
    out = ops.gemm(W, X, ops.SWIGLU)
    g = (X.float() @ Wg.float().T).to(torch.bfloat16)
    u = (X.float() @ Wu.float().T).to(torch.bfloat16)
    sg = torch.nn.functional.silu(g.float()).to(torch.bfloat16).float()
    ref = (sg * u.float()).to(torch.bfloat16)
    # another fp32 summation order may round g or u one bf16 step apart: the
    # product then moves by |silu'(g) u| ulp(g) (silu' <= 1.1) or |silu(g)| ulp(u)
    extra = 1.1 * u.float().abs() * bf16_ulp(g.float()) + sg.abs() * bf16_ulp(u.float())
    assert_close_scaled(out, ref, ulps=2, atol_frac=1e-5, what="swiglu", extra_tol=extra)
    assert (out == ref).float().mean().item() > 0.97


@pytest.mark.parametrize("M,N,K", [(2048, 16, 2048), (2048, 16, 8192), (256, 1024, 512), (2048, 256, 2048),
                                   (2048, 1024, 8192), (16384, 640, 512), (2560, 1024, 6912), (384, 520, 1024)])
def test_gemm_gated_residual(M, N, K):
    W = rand((M, K), 1 / math.sqrt(K), 12)
    X = rand((N, K), 1.0, 13)
    b = rand((M,), 0.1, 14)
    gate = rand((M,), 0.5, 15)
    x0 = rand((N, M), 1.0, 16)
    out = x0.clone()
    ops.gemm(W, X, ops.RESID, bias=b, gate=gate, out=out)
    y = (X.float() @ W.float().T + b.float()).to(torch.bfloat16)
    gy = (gate.float() * y.float()).to(torch.bfloat16)
    ref = (x0.float() + gy.float()).to(torch.bfloat16)
    # a one-ulp flip of the rounded y moves gate*y by |gate| ulp(y), plus its own rounding
    extra = gate.float().abs() * bf16_ulp(y.float()) + bf16_ulp(gy.float())
    assert_close_scaled(out, ref, ulps=1, atol_frac=1e-5, what="residual", extra_tol=extra)
    assert (out == ref).float().mean().item() > 0.97


@pytest.mark.parametrize("cols", [2048, 4096, 5120, 6144])
def test_rmsnorm_matches_oracle(cols):
    x = rand((37, cols), 2.0, 20)
    w = (1 + 0.1 * rand((cols,), 1.0, 21).float()).to(torch.bfloat16)
    got = ops.rmsnorm(x, w, 1e-6)
    ref = O.rms_norm(x.cpu(), w.cpu(), 1e-6)
    assert_bf16_close(got.cpu(), ref, max_ulps=1, min_exact=0.995, what="rmsnorm")
    # the vector paths (rows <= 2048, wide rows) sum in the canonical order of the
    # generic path, which an unaligned view of the same rows takes: bit for bit
    xs = torch.empty(37 * cols + 8, dtype=torch.bfloat16, device=x.device)
    xu = xs[1:1 + 37 * cols].view(37, cols)
    xu.copy_(x)
    assert torch.equal(ops.rmsnorm(xu, w, 1e-6), got)


@pytest.mark.parametrize("D", [2048, 2560, 5120])
def test_adaln_matches_oracle(D):
    x = rand((16, D), 3.0, 22)
    mod = rand((3 * D,), 0.5, 23)
    got = ops.adaln(x, mod, 1e-6)
    scale, shift, gate = mod.cpu().view(1, 3 * D).chunk(3, dim=-1)
    ref, _ = O.ada_layer_norm(x.cpu(), (scale, shift, gate), 1e-6)
    # the statistics sum in another order than the CPU's: a one-ulp flip of the
    # rounded normalised value moves the bf16 (1 + scale) product by up to one ulp
    # of the product, which the shift's addition can leave on a smaller result
    sc, sh = scale.float().view(-1), shift.float().view(-1)
    prod = (ref.float() - sh).abs()
    extra = bf16_ulp(prod * (1 + sc.abs())) + bf16_ulp(prod)
    assert_close_scaled(got.cpu(), ref, ulps=1, atol_frac=0.0, what="adaln", extra_tol=extra)
    assert (got.cpu() == ref).float().mean().item() > 0.995
    xs = torch.empty(16 * D + 8, dtype=torch.bfloat16, device=x.device)
    xu = xs[1:1 + 16 * D].view(16, D)
    xu.copy_(x)
    assert torch.equal(ops.adaln(xu, mod, 1e-6), got)


@pytest.mark.parametrize("hd,theta", [(128, 10000.0), (64, 1e6)])
def test_rope_table_matches_oracle(hd, theta):
    cs, sn = ops.rope_table(9000, hd, theta)
    pos = torch.arange(9000)[None]
    rc, rs = O.rope_tables(pos, hd, theta)
    torch.testing.assert_close(cs.cpu(), rc[0, :, 0], rtol=0, atol=2e-6)
    torch.testing.assert_close(sn.cpu(), rs[0, :, 0], rtol=0, atol=2e-6)


def test_philox_normal_statistics_and_determinism():
    a = ops.philox_normal((64, 4096), seed=1234, offset=3)
    b = ops.philox_normal((64, 4096), seed=1234, offset=3)
    c = ops.philox_normal((64, 4096), seed=1234, offset=4)
    assert torch.equal(a, b) and not torch.equal(a, c)
    f = a.float()
    assert abs(f.mean().item()) < 0.01 and abs(f.std().item() - 1.0) < 0.01


def sdpa_ref(q, k, v):
    """fp32 softmax attention with bf16-rounded numerators (the CPU flash order)."""
    s = (q.float() @ k.float().transpose(-1, -2)) * (1.0 / math.sqrt(q.shape[-1]))
    m = s.max(-1, keepdim=True).values
    e = torch.exp(s - m)
    return ((e.to(torch.bfloat16).float() @ v.float()) / e.sum(-1, keepdim=True)).to(torch.bfloat16)


@pytest.mark.parametrize("B,H,hd", [(1, 16, 128), (3, 4, 64)])
def test_block_self_attention(B, H, hd):
    D = H * hd
    qkv = rand((B * 16, 3 * D), 1.0, 30)
    got = ops.block_self_attn(qkv, B, 16, H, hd)
    q, k, v = qkv.view(B, 16, 3, H, hd).permute(2, 0, 3, 1, 4)
    ref = sdpa_ref(q, k, v).permute(0, 2, 1, 3).reshape(B * 16, D)
    assert_bf16_close(got, ref, max_ulps=2, min_exact=0.95, what="self-attn")
    # and against the reference's own op (torch SDPA on the CPU)
    cpu = torch.nn.functional.scaled_dot_product_attention(q.cpu(), k.cpu(), v.cpu())
    cpu = cpu.permute(0, 2, 1, 3).reshape(B * 16, D)
    assert_close_scaled(got.cpu(), cpu, ulps=2, atol_frac=2 ** -8, what="self-attn vs CPU SDPA")


@pytest.mark.parametrize("B,H,hd,lens,nsplit", [
    (1, 16, 128, [2048], 0), (1, 16, 128, [2048], 1), (3, 4, 64, [0, 17, 129], 0), (2, 20, 128, [4096, 1023], 3),
    (4, 16, 128, [63, 64, 65, 4000], 0),
])
def test_cross_attention(B, H, hd, lens, nsplit):
    L, Tc = 2, max(lens) + 20
    cache = rand((L, 2, B + 1, H, Tc, hd), 1.0, 40)
    q = rand((B * 16, H * hd), 1.0, 41)
    lengths = torch.tensor(lens, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    for layer in range(L):
        got = ops.cross_attn(q, cache, lengths, layer, nsplit, err=err)
        for b, n in enumerate(lens):
            k = cache[layer, 0, b, :, : n + 1]
            v = cache[layer, 1, b, :, : n + 1]
            qb = q[b * 16 : (b + 1) * 16].view(16, H, hd).transpose(0, 1)
            ref = sdpa_ref(qb, k, v).transpose(0, 1).reshape(16, H * hd)
            # numerators are rounded to bf16 relative to a running (per split) maximum
            assert_close_scaled(got[b * 16 : (b + 1) * 16], ref, ulps=2, atol_frac=2 ** -9,
                                what=f"cross-attn b={b} len={n}")
    torch.cuda.synchronize()
    assert int(err.item()) == 0


# ------------------------------------------------------------------ sampling / acceptance (bit-exact)

@pytest.mark.parametrize("V", [2048, 3001, 151936])
def test_row_stats_and_softmax_bit_exact(V):
    logits = (2.0 * torch.randn(5, V, generator=torch.Generator().manual_seed(V))).to(torch.bfloat16)
    stats, am = ops.row_stats(logits.to(DEV), 0.7)
    for r in range(5):
        m, s = oracle_accept.row_stats(logits[r], 0.7)
        assert stats[r, 0].item() == m and stats[r, 1].item() == s
        assert am[r].item() == int(logits[r].argmax())
    probs = ops.softmax_rows(logits.to(DEV), 0.7).cpu()
    assert torch.equal(probs, oracle_accept.softmax_rows(logits, 0.7))


def test_fm_exp_full_range_bit_exact():
    """fm_exp over its whole finite range through fp32 softmax rows at T = 1:
    x - m spans [-110, 0] (normal, subnormal and zero results), each row's max
    is 0, and every probability must equal the C oracle's bit for bit."""
    g = torch.Generator().manual_seed(17)
    logits = -110.0 * torch.rand(4, 65536, generator=g)
    logits[:, 0] = 0.0
    logits[1] = -torch.logspace(-8, 2.04, 65536)  # dense near 0 and out to -110
    logits[1, 0] = 0.0
    probs = ops.softmax_rows(logits.to(DEV), 1.0).cpu()
    assert torch.equal(probs, oracle_accept.softmax_rows(logits, 1.0))
    assert int((probs == 0).sum()) > 0 and int(((probs > 0) & (probs < 1.1754944e-38)).sum()) > 0


@pytest.mark.parametrize("V,T", [(2048, 1.0), (3001, 0.7), (151936, 1.0)])
def test_sample_rows_bit_exact(V, T):
    B, K = 2, 16
    logits = (2.0 * torch.randn(B, K, V, generator=torch.Generator().manual_seed(7))).to(torch.bfloat16)
    ld = logits.to(DEV)
    probs = ops.softmax_rows(ld, T)
    toks = ops.sample_rows(ld, probs, T, seed=1234, offset=5).cpu()
    ref, _ = oracle_accept.sample_rows(logits, T, seed=1234, offset=5)
    assert torch.equal(toks, ref)
    greedy = ops.sample_rows(ld, None, 0.0, 1234, 5).cpu()
    assert torch.equal(greedy, logits.argmax(-1))


@pytest.mark.parametrize("B,K,V,seed", [(34, 16, 3001, 5), (8, 16, 151936, 11), (64, 16, 151936, 12)])
def test_accept_greedy_bit_exact(B, K, V, seed):
    from tests.golden.inputs import acceptance_inputs

    target, draft, _ = acceptance_inputs(B, K, V, seed, 0.0)
    acc, bonus = ops.accept_greedy(target.to(DEV), draft.to(DEV))
    racc, rbonus = oracle_accept.accept_greedy(target, draft)
    assert acc.cpu().tolist() == racc.tolist() and bonus.cpu().tolist() == rbonus.tolist()


@pytest.mark.parametrize("logits_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("B,K,V,seed,T", [(24, 16, 3001, 6, 1.0), (24, 16, 2048, 7, 0.7), (6, 16, 151936, 9, 1.0),
                                         (64, 16, 151936, 13, 1.0)])
def test_accept_rejection_bit_exact(B, K, V, seed, T, logits_dtype):
    """bf16 and fp32 target logits (the fp32 rows hold the same values: bf16 widens exactly)."""
    from tests.golden.inputs import acceptance_inputs

    target, draft, q = acceptance_inputs(B, K, V, seed, T)
    target = target.to(logits_dtype)
    acc, bonus = ops.accept_rejection(target.to(DEV), draft.to(DEV), q.to(DEV), T, seed=1234, offset=0)
    racc, rbonus = oracle_accept.accept_rejection(target, draft, q, T, seed=1234, offset=0)
    assert acc.cpu().tolist() == racc.tolist()
    assert bonus.cpu().tolist() == rbonus.tolist()


@pytest.mark.parametrize("T", [1.0, 0.7])
def test_accept_rejection_near_ties_bit_exact(T):
    """Tests the approximate row sums cannot settle: u q is placed 1-8 parts
    per million below p (accepted) on slots before j_b and above p (rejected)
    at slot j_b = b mod (K + 1), far inside the 2^-10 settling margin, so every
    such test is decided with the exact slice-major sums.  Accepted lengths and
    bonus tokens equal the C oracle's, and the lengths are the planted ones."""
    import numpy as np

    from tests.golden.inputs import acceptance_inputs

    B, K, V = 17, 16, 151936
    target, draft, q = acceptance_inputs(B, K, V, 21, T)
    q = q.clone()
    g = torch.Generator().manual_seed(3)
    f32 = np.float32
    for b in range(B):
        jb = b % (K + 1)
        for k in range(min(jb + 1, K)):
            row = target[b, k]
            m, s = oracle_accept.rejection_row_stats(row, T)
            x = f32(row[draft[b, k]].float().item())
            e = f32(oracle_accept.fm_exp(float(f32(f32(x / f32(T)) - f32(m)))))
            p = float(f32(e / f32(s)))
            u = oracle_accept.uniform(1234, k, b, 0, 1)
            ppm = float(torch.randint(1, 9, (1,), generator=g)) * 1e-6
            q[b, k, draft[b, k]] = p / u * (1.0 + ppm if k == jb else 1.0 - ppm)
    acc, bonus = ops.accept_rejection(target.to(DEV), draft.to(DEV), q.to(DEV), T, seed=1234, offset=0)
    racc, rbonus = oracle_accept.accept_rejection(target, draft, q, T, seed=1234, offset=0)
    assert racc.tolist() == [b % (K + 1) for b in range(B)]
    assert acc.cpu().tolist() == racc.tolist()
    assert bonus.cpu().tolist() == rbonus.tolist()


def test_acceptance_golden_cases_through_cuda():
    """The reference's own acceptance decisions (golden file) reproduced on the GPU."""
    import os

    from tests.golden.inputs import acceptance_inputs

    cases = torch.load(os.path.join(os.path.dirname(__file__), "golden", "acceptance_cases.pt"))
    for name, c in cases.items():
        target, draft, q = acceptance_inputs(c["B"], c["K"], c["V"], c["seed"], c["temperature"])
        if c["temperature"] <= 0:
            acc, bonus = ops.accept_greedy(target.to(DEV), draft.to(DEV))
        else:
            acc, bonus = ops.accept_rejection(target.to(DEV), draft.to(DEV), q.to(DEV), c["temperature"],
                                              seed=c["rng_seed"], offset=0)
        assert acc.cpu().tolist() == c["accepted"], name
        assert bonus.cpu().tolist() == c["bonus"], name


@pytest.mark.parametrize("logits_dtype", [torch.bfloat16, torch.float32])
def test_signed_zero_maximum_takes_first_index(logits_dtype):
    """A row whose maximum is zero held as both -0.0 and +0.0: torch.argmax
    compares them equal and returns the first index, whichever sign it has.
    Greedy acceptance (bonus token), the row statistics' argmax and draft
    sampling at T = 0 must do the same, wherever the two zeros sit in the row
    (one vocabulary slice or two)."""
    V = 151936
    for first, second in ((5, 9), (5, 100000), (70000, 140000)):
        for sign_first in (-0.0, 0.0):
            row = torch.full((V,), -1.0)
            row[first] = sign_first
            row[second] = -0.0 if sign_first == 0.0 else 0.0
            target = row.repeat(1, 17, 1).to(logits_dtype)  # (1, K + 1, V): every row the same
            draft = torch.full((1, 16), first, dtype=torch.int64)
            acc, bonus = ops.accept_greedy(target.to(DEV), draft.to(DEV))
            assert int(acc[0]) == 16 and int(bonus[0]) == first, (first, second, sign_first)
            _, am = ops.row_stats(target[0].to(DEV).contiguous(), 1.0)
            assert am.cpu().tolist() == [first] * 17
            tok = ops.sample_rows(target[:, :16].to(DEV).contiguous(), None, 0.0, 1234, 0)
            assert tok.cpu().tolist() == [[first] * 16]
