"""The CUDA serving operators and folds against the reference's own code: the
golden vectors of tests/golden/serving_cases.pt (the Triton kernels of
flashmap/vllm/kernels.py and flashmap/sglang/kernels.py run by Triton's CPU
interpreter, and flashmap/vllm/fold.py), made by
tests/golden/make_serving_golden.py.

Tolerances, written per check (the tolerances of tests/test_gpu_serving_ops.py,
which holds the same kernels to the CPU restatement): norms and RoPE within
2 bf16 ulps plus 8e-3 of the row's largest value with >= 97% bit-equal;
attention within 2e-2 of the largest output (mean 2e-3); cache values
bit-exact; greedy sampling exact; the folded head within one bf16 step
(the GEMM accumulates in another order); the folded noise, once each
eigenvector's sign is matched (the device eigen-solver may return -q for q),
within one bf16 step on >= 99.9% of the elements and within 1% of its
column's largest magnitude everywhere (the device accumulates the fp32 Gram
matrix in another order, which perturbs the eigenvectors).
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import FlashMapConfig, FlashMapDraftModel, _lib, ops  # noqa: E402
from flashmap_b200 import serving_ops as S  # noqa: E402
from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head  # noqa: E402
from tests.helpers import CONFIG1, CONFIG5S, Emb, Head  # noqa: E402
from tests.test_gpu_serving_ops import assert_attn_close, assert_rows_close  # noqa: E402
from tests.test_serving_golden import CASES, close_bf16  # noqa: E402

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def device_ok():
    _lib.require_device()


def test_vllm_rms_norm_rope_vs_reference_kernel():
    for c in CASES["vllm_rms_norm_rope"]:
        got = torch.ops.flashmap_vllm.rms_norm_rope(c["x"].to(DEV), c["weight"].to(DEV), c["cos_sin"].to(DEV),
                                                    c["positions"].to(DEV), c["eps"])
        assert_rows_close(got.cpu(), c["out"], "vllm rms_norm_rope")


def test_vllm_block_self_attention_vs_reference_kernel():
    for c in CASES["vllm_block_self_attention"]:
        got = torch.ops.flashmap_vllm.block_self_attention(c["qkv"].to(DEV), c["q_norm"].to(DEV),
                                                           c["k_norm"].to(DEV), c["cos_sin"].to(DEV),
                                                           c["positions"].to(DEV), c["eps"])
        assert_attn_close(got.cpu(), c["out"], "vllm block_self_attention")


def test_sglang_rms_norm_rope_vs_reference_kernel():
    for c in CASES["sglang_rms_norm_rope"]:
        got = torch.ops.flashmap_sglang.rms_norm_rope(c["x"].to(DEV), c["weight"].to(DEV), c["freqs"].to(DEV),
                                                      c["eps"])
        assert_rows_close(got.cpu(), c["out"], "sglang rms_norm_rope")


def test_sglang_block_self_attention_vs_reference_kernel():
    for c in CASES["sglang_block_self_attention"]:
        got = torch.ops.flashmap_sglang.block_self_attention(c["qkv"].to(DEV), c["q_norm"].to(DEV),
                                                             c["k_norm"].to(DEV), c["freqs"].to(DEV), c["eps"])
        assert_attn_close(got.cpu(), c["out"], "sglang block_self_attention")


def test_vllm_write_context_kv_vs_reference_kernel():
    for c in CASES["vllm_write_context_kv"]:
        caches = [torch.zeros(c["cache_shape"], dtype=torch.bfloat16, device=DEV) for _ in c["caches"]]
        ptrs = torch.tensor([x.data_ptr() for x in caches], dtype=torch.int64, device=DEV)
        S.write_context_kv(c["kv"].to(DEV), c["positions"].to(DEV), c["slots"].to(DEV), c["k_norm"].to(DEV),
                           c["cos_sin"].to(DEV), ptrs, c["strides"], c["block_size"], c["eps"],
                           heads_per_cache=c["heads_per_cache"])
        torch.cuda.synchronize()
        hd = c["kv"].shape[-1]
        for got, ref in zip(caches, c["caches"]):
            g, r = got.cpu().view(-1, 2 * hd), ref.view(-1, 2 * hd)
            assert_rows_close(g[:, :hd], r[:, :hd], "keys")
            assert torch.equal(g[:, hd:], r[:, hd:]), "values"


def test_greedy_rows_vs_reference_sample_rows():
    """sglang/kernels.py:196-254 on greedy rows: the first index of the row maximum."""
    for c in CASES["sglang_sample_rows_greedy"]:
        got = ops.row_stats(c["logits"].to(DEV), 1.0)[1]
        assert torch.equal(got.cpu(), c["out"])


@pytest.mark.parametrize("idx,cfg", [(0, CONFIG1), (1, CONFIG5S)])
def test_cuda_folds_vs_reference_fold_py(idx, cfg):
    config = FlashMapConfig(**cfg)
    sd = synthetic_state_dict(config, seed=0, dtype=torch.bfloat16)
    emb, head = synthetic_target_head(config, seed=0, dtype=torch.bfloat16)
    model = FlashMapDraftModel(config)
    model.load_state_dict(sd, strict=True)
    model = model.to(DEV, torch.bfloat16).eval()
    pack = model._pack(torch.device(DEV), Emb(emb.to(DEV)), Head(head.to(DEV)))
    w, b = pack.ensure_fold()
    fh = CASES["fold_head"][idx]
    bad, err = close_bf16(w.cpu(), fh["weight"], floor=1e-3)
    assert bad == 0, f"folded head weight: {bad} elements off, max {err}"
    bad, err = close_bf16(b.cpu(), fh["bias"], floor=1e-3)
    assert bad == 0, f"folded head bias: {bad} elements off, max {err}"
    weight, var, _ = pack.ensure_noise_fold(config)
    fn = CASES["fold_noise"][idx]
    got, ref = weight.cpu().float(), fn["M"].float()
    sign = torch.sign((got * ref).sum(0))
    sign[sign == 0] = 1
    bad, err = close_bf16(got * sign[None, :], ref, floor=1e-3)
    assert bad <= 1e-3 * ref.numel(), f"folded noise: {bad} elements more than one bf16 step off, max {err}"
    col = ref.abs().amax(dim=0, keepdim=True)
    worst = float(((got * sign[None, :] - ref).abs() / col).max())
    assert worst <= 1e-2, f"folded noise: an element {worst:.4f} of its column's scale off"
    assert torch.allclose(var.cpu(), fn["var"], rtol=1e-5, atol=1e-7)
