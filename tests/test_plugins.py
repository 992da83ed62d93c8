"""CPU checks of the vLLM and sglang plugin entry points: the reference's method
signatures and attributes, construction checks, weight loading, and the
context-cache layout planner (engines absent: their objects are stand-ins)."""

import inspect
from types import SimpleNamespace

import pytest
import torch

from flashmap_b200 import FlashMapConfig
from flashmap_b200 import sglang_model as SG
from flashmap_b200 import vllm_model as VL
from flashmap_b200.synthetic import synthetic_state_dict

CFG = dict(target_hidden_size=256, vocab_size=2048, target_layer_ids=[0], block_size=16, hidden_size=256,
           num_hidden_layers=2, num_attention_heads=4, intermediate_size=1024, mlp_type="gelu")

# parameter lists of the reference's plugin models (flashmap/vllm/model.py, flashmap/sglang/model.py)
VLLM_METHODS = {
    "load_weights": ["weights"],
    "prepare": [],
    "set_noise_keys": ["seeds", "rows"],
    "combine_hidden_states": ["hidden_states"],
    "precompute_and_store_context_kv": ["context_states", "context_positions", "context_slot_mapping"],
    "defer_context_kv": ["context_states", "context_positions", "context_slot_mapping"],
    "forward": ["input_ids", "positions", "inputs_embeds"],
    "compute_draft_logits": ["hidden_states"],
}
SGLANG_METHODS = {
    "load_weights": ["weights"],
    "attach_shared_modules": ["embed_tokens", "lm_head"],
    "prepare": ["lm_head_weight"],
    "head_logits": ["hidden"],
    "forward_embed": ["input_ids"],
    "compute_base_logits": ["hidden"],
    "write_target_hidden_kv": ["target_hidden", "pool", "positions", "cache_loc", "cache_loc_2d", "commit_lens",
                               "target_hidden_is_projected"],
    "forward": ["input_ids", "positions", "forward_batch", "input_embeds", "get_embedding", "pp_proxy_tensors"],
}


def _params(fn):
    return [p for p in inspect.signature(fn).parameters if p != "self"]


def vllm_config(config, **over):
    cfg = dict(parallel_config=SimpleNamespace(tensor_parallel_size=1), use_v2_model_runner=True,
               speculative_config=SimpleNamespace(draft_model_config=SimpleNamespace(hf_config=config)),
               model_config=SimpleNamespace(dtype=torch.bfloat16, max_model_len=512, is_hybrid=False),
               cache_config=SimpleNamespace(cache_dtype="auto"))
    cfg.update(over)
    return SimpleNamespace(**cfg)


@pytest.mark.parametrize("name", sorted(VLLM_METHODS))
def test_vllm_signatures(name):
    assert _params(getattr(VL.FlashMapDraftModel, name)) == VLLM_METHODS[name]


@pytest.mark.parametrize("name", sorted(SGLANG_METHODS))
def test_sglang_signatures(name):
    assert _params(getattr(SG.FlashMapDraftModel, name)) == SGLANG_METHODS[name]


def test_vllm_construction_checks():
    config = FlashMapConfig(**CFG)
    m = VL.FlashMapDraftModel(vllm_config=vllm_config(config))
    assert m.noise_scale == 1.0 and m.compile is True and m.hot_ids is None
    assert m.block_size == 16 and not m.cache_plan.packed
    with pytest.raises(ValueError, match="tensor parallel"):
        VL.FlashMapDraftModel(vllm_config=vllm_config(config, parallel_config=SimpleNamespace(tensor_parallel_size=2)))
    with pytest.raises(ValueError, match="V2 model runner"):
        VL.FlashMapDraftModel(vllm_config=vllm_config(config, use_v2_model_runner=False))
    with pytest.raises(ValueError, match="bfloat16"):
        VL.FlashMapDraftModel(vllm_config=vllm_config(
            config, model_config=SimpleNamespace(dtype=torch.float16, max_model_len=512)))
    with pytest.raises(RuntimeError):
        m.combine_hidden_states(torch.zeros(1, 256))  # prepare() has not run


def test_vllm_load_weights():
    config = FlashMapConfig(**CFG)
    sd = synthetic_state_dict(config, seed=0, dtype=torch.float32)
    m = VL.FlashMapDraftModel(vllm_config=vllm_config(config))
    names = m.load_weights(list(sd.items()) + [("embed_tokens.weight", torch.zeros(1)), ("counts", torch.zeros(1))])
    assert "model.layers.0.self_attn.q_proj.weight" in names
    assert torch.equal(m.model.fc.weight, sd["fc.weight"])
    with pytest.raises(ValueError, match="unexpected"):
        m.load_weights([("nonsense.weight", torch.zeros(1))])
    with pytest.raises(ValueError, match="missing"):
        m.load_weights(list(sd.items())[:-3])


def test_vllm_state_vocab_d2t():
    config = FlashMapConfig(**dict(CFG, state_vocab_size=512))
    sd = synthetic_state_dict(config, seed=1, dtype=torch.float32)
    m = VL.FlashMapDraftModel(vllm_config=vllm_config(config))
    m.load_weights(sd.items())
    ids = sd["draft_ids"]
    assert torch.equal(m.d2t + torch.arange(512), ids)
    assert torch.equal(m.model.draft_ids, ids)


def test_sglang_construction_and_loading():
    config = FlashMapConfig(**CFG)
    m = SG.FlashMapDraftModel(config)
    assert m.flashmap and m.sample_from_anchor and m.gamma == 16 and m.lm_head is None
    assert m.folded_head is None and m.hot_ids is None and isinstance(m.markov_head, SG.IdentityMarkov)
    sd = synthetic_state_dict(config, seed=0, dtype=torch.float32)
    m.load_weights(list(sd.items()) + [("ids", torch.arange(2048)), ("counts", torch.ones(2048))])
    assert m._vocab_ranking is not None
    with pytest.raises(KeyError):
        m.load_weights([("nonsense", torch.zeros(1))])
    bad = FlashMapConfig(**CFG)
    bad.flow_map = False
    with pytest.raises(ValueError, match="stage-1 flow"):
        SG.FlashMapDraftModel(bad)
    with pytest.raises(ValueError, match="padded or sharded"):
        m.attach_shared_modules(embed_tokens=SimpleNamespace(weight=torch.zeros(10, 256)),
                                lm_head=SimpleNamespace(weight=torch.zeros(10, 256)))


def test_context_layout():
    """The packed layout of the reference plugin's hybrid-target mode: the
    DiT's heads layer-major in target-sized caches, a layer's heads cut at
    cache boundaries into runs."""
    lay = VL.context_layout(6, 20, 128, hybrid=True, target_attention_layers=16, target_kv_heads=8,
                            target_head_size=128, bf16_cache=True)
    assert lay.packed and lay.caches == 16 and lay.per_cache == 8
    # layer 0's 20 heads span caches 0, 1, 2 (8 + 8 + 4); layer 1 starts at slot 4 of cache 2
    assert lay.runs(0) == [(0, 0, 8, 0), (1, 0, 8, 8), (2, 0, 4, 16)]
    assert lay.runs(1)[0] == (2, 4, 4, 0)
    covered = sorted(lay.where(l, h) for l in range(6) for h in range(20))
    assert len(set(covered)) == 120 and max(covered)[0] < 16
    for layer in range(6):  # the runs cover each layer's heads once, in order
        heads = [r.head + i for r in lay.runs(layer) for i in range(r.count)]
        assert heads == list(range(20))
        assert all(lay.where(layer, r.head) == (r.cache, r.slot) for r in lay.runs(layer))
    assert not VL.context_layout(6, 20, 128, hybrid=False, target_attention_layers=16, target_kv_heads=8,
                                 target_head_size=128, bf16_cache=True).packed
    assert not VL.context_layout(6, 20, 128, hybrid=True, target_attention_layers=16, target_kv_heads=8,
                                 target_head_size=128, bf16_cache=False).packed
    small = VL.context_layout(6, 20, 128, hybrid=True, target_attention_layers=4, target_kv_heads=8,
                              target_head_size=128, bf16_cache=True)
    assert not small.packed and small.caches == 6 and small.runs(3) == [(3, 0, 20, 0)]
    with pytest.raises(ValueError):
        VL.context_layout(2, 4, 64, hybrid=False, target_attention_layers=0, target_kv_heads=0,
                          target_head_size=0, bf16_cache=True, mode="bogus")
    q = torch.arange(2 * 20 * 3.0).view(2, 20, 3)
    caches = [torch.zeros(1, 8, 1, 6) for _ in range(16)]
    out = VL.attend_runs(q, caches, lay.runs(0), lambda pq, pc, n: pq * 2)
    assert torch.equal(out, q * 2)
