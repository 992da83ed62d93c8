"""The persistent single-launch draft (batch 1, one jump) against the kernel
sequence of the same plan: identical bits for the logits, argmax tokens,
hidden states and the anchor's cache rows, with caller-given noise and with
Philox noise drawn in place; the device noise counter advances alike; the
graph-captured session replays the same draws.  The kernel sequence itself
is held to the CPU oracle by test_gpu_draft.py."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import DraftSession, FlashMapCache  # noqa: E402
from tests.helpers import CONFIG1, CONFIG2, CONFIG5S, Emb, Head, build  # noqa: E402

DEV = "cuda"


def _setup(cfg, ctx_len, seed=3):
    config, model, _, emb, head = build(cfg, seed=seed, with_oracle=False)
    E, W = Emb(emb.to(DEV)), Head(head.to(DEV))
    K = config.block_size
    g = torch.Generator().manual_seed(1000 + seed)
    hidden = torch.randn(1, ctx_len, len(config.target_layer_ids) * config.target_hidden_size, generator=g)
    cache = FlashMapCache(config, 1, ctx_len + K + 2, device=DEV, dtype=torch.bfloat16)
    model.extend_context(cache, hidden.to(DEV, torch.bfloat16), E, W)
    pack = model._pack(DEV, E, W)
    model.launch_mode = "kernels"
    seq = model._plan(pack, cache, 1, 1)
    model.launch_mode = "persistent"
    one = model._plan(pack, cache, 1, 1)
    return config, model, pack, cache, seq, one, E, W


def _bits(t):
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


def _run(plan, config, pack, cache, anchor, seed, offset, z=None, offset_dev=None):
    K, V, Ht = config.block_size, config.vocab_size, config.target_hidden_size
    scatter = pack.draft_ids is not None
    logits = torch.full((K, V), float("-inf"), device=DEV, dtype=torch.bfloat16)
    tokens = torch.full((K,), -1, device=DEV, dtype=torch.int64)
    hidden = torch.empty(K, Ht, device=DEV, dtype=torch.bfloat16)
    plan.draft(anchor, seed, offset, logits=logits, ldl=V, scatter=scatter, tokens=tokens, z=z, hidden=hidden,
               offset_dev=offset_dev)
    torch.cuda.synchronize()
    plan.check_device_errors()
    return logits, tokens, hidden, cache.kv.clone()


@pytest.mark.parametrize("cfg,ctx_len", [(CONFIG1, 40), (CONFIG5S, 29), (CONFIG1, 300), (CONFIG2, 2048)])
def test_persistent_pass_equals_kernel_sequence(cfg, ctx_len):
    config, model, pack, cache, seq, one, _, _ = _setup(cfg, ctx_len)
    on, why = one.persistent()
    assert on, why
    assert not seq.persistent()[0]
    K, Ht = config.block_size, config.target_hidden_size
    g = torch.Generator().manual_seed(7)
    for trial in range(3):
        anchor = torch.randint(0, config.vocab_size, (1,), generator=g).to(DEV)
        z = None
        if trial == 0:
            z = torch.randn(K, Ht, generator=g).to(DEV, torch.bfloat16)
        a = _run(seq, config, pack, cache, anchor, 1234, trial, z=z)
        b = _run(one, config, pack, cache, anchor, 1234, trial, z=z)
        for name, x, y in zip(("logits", "tokens", "hidden", "cache"), a, b):
            assert torch.equal(_bits(x), _bits(y)), f"{name} differs (trial {trial})"
        assert torch.equal(b[1], b[0].float().argmax(-1))
    assert one.last_launches() == 1


def test_persistent_pass_device_noise_counter():
    config, model, pack, cache, seq, one, _, _ = _setup(CONFIG1, 57)
    anchor = torch.tensor([5], device=DEV)
    cnt_a = torch.zeros(1, dtype=torch.int32, device=DEV)
    cnt_b = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(3):
        a = _run(seq, config, pack, cache, anchor, 99, 0, offset_dev=cnt_a)
        b = _run(one, config, pack, cache, anchor, 99, 0, offset_dev=cnt_b)
        assert torch.equal(_bits(a[0]), _bits(b[0]))
    assert int(cnt_a.item()) == int(cnt_b.item()) == 3


def test_persistent_pass_in_a_cuda_graph():
    config, model, pack, cache, seq, one, E, W = _setup(CONFIG5S, 33)
    assert model.launch_mode == "persistent"
    eager = DraftSession(model, cache, E, W, seed=11, use_graph=False)
    graph = DraftSession(model, cache, E, W, seed=11, use_graph=True)
    assert graph.launches == 1
    for anchor in (3, 17, 256):
        assert torch.equal(eager.draft([anchor]).clone(), graph.draft([anchor]).clone())
