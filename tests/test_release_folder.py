"""A FlashMap release folder, laid out as the reference's converter writes it
(scripts/convert_checkpoint.py:351-400): ``model.safetensors`` in bf16 with
``{"format": "pt"}`` metadata; ``config.json`` with the model's fields, the
``architectures`` / ``auto_map`` entries, vLLM's speculators header
(``speculators_model_type``, ``speculators_config``,
``transformer_layer_config``, ``draft_vocab_size``) and sglang's fields
(``max_position_embeddings``, ``dspark_config``); and, for a drafter over the
full vocabulary with a restricted draft vocabulary, ``draft_vocab.safetensors``
(``counts``, ``ids``).  The folder loads through
``FlashMapDraftModel.from_pretrained`` and the vLLM and sglang plugins'
``load_weights`` with every tensor and model field as written."""

import json
import os

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

from flashmap_b200 import FlashMapConfig, FlashMapDraftModel
from flashmap_b200.synthetic import synthetic_state_dict
from tests.helpers import CONFIG1, CONFIG5S


def write_release(folder, cfg, seed=5, draft_vocab=0):
    config = FlashMapConfig(**cfg)
    weights = {k: (v.to(torch.bfloat16) if v.is_floating_point() else v)
               for k, v in synthetic_state_dict(config, seed=seed, dtype=torch.float32).items()}
    os.makedirs(folder, exist_ok=True)
    save_file(weights, os.path.join(folder, "model.safetensors"), metadata={"format": "pt"})
    fields = config.to_dict()
    fields.update(
        architectures=["FlashMapDraftModel"],
        auto_map={"AutoConfig": "configuration_flashmap.FlashMapConfig",
                  "AutoModel": "modeling_flashmap.FlashMapDraftModel"},
        dtype="bfloat16",
        speculators_model_type="flashmap",
        speculators_config={
            "algorithm": "flashmap", "default_proposal_method": "greedy",
            "proposal_methods": [{"proposal_type": "greedy", "speculative_tokens": config.block_size,
                                  "accept_tolerance": 0.0, "verifier_accept_k": 1}],
            "verifier": {"name_or_path": config.target_model, "architectures": ["Qwen3ForCausalLM"]}},
        transformer_layer_config={},
        max_position_embeddings=131072,
        dspark_config={"markov_rank": 1, "markov_head_type": "vanilla", "mask_token_id": config.vocab_size - 1},
    )
    ranking = None
    if config.state_vocab_size is not None:
        fields["draft_vocab_size"] = config.state_vocab_size
    elif draft_vocab:
        fields["draft_vocab_size"] = draft_vocab
        g = torch.Generator().manual_seed(seed)
        counts = torch.randint(0, 1000, (config.vocab_size,), generator=g)
        order = torch.argsort(counts, descending=True, stable=True)
        ranking = {"counts": counts[order], "ids": order}
        save_file(ranking, os.path.join(folder, "draft_vocab.safetensors"), metadata={"format": "pt"})
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(fields, f, indent=2)
    return config, weights, ranking


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
def test_from_pretrained_loads_release_folder(tmp_path, cfg):
    config, weights, _ = write_release(str(tmp_path / "release"), cfg)
    model, info = FlashMapDraftModel.from_pretrained(str(tmp_path / "release"), output_loading_info=True,
                                                     dtype=torch.bfloat16)
    assert not info["missing_keys"] and not info["unexpected_keys"], info
    state = model.state_dict()
    for name, tensor in weights.items():
        assert torch.equal(state[name].cpu(), tensor), name
    for field in ("target_hidden_size", "vocab_size", "state_vocab_size", "block_size", "hidden_size",
                  "num_hidden_layers", "num_attention_heads", "intermediate_size", "mlp_type", "rope_theta",
                  "jump_grids"):
        assert getattr(model.config, field) == getattr(config, field), field
    assert model.config.speculators_model_type == "flashmap"
    assert model.config.dspark_config["mask_token_id"] == config.vocab_size - 1


def folder_entries(folder):
    """(name, tensor) of the folder's safetensors files, as an engine's loader iterates them."""
    for name in ("model.safetensors", "draft_vocab.safetensors"):
        path = os.path.join(folder, name)
        if os.path.exists(path):
            with safe_open(path, "pt") as handle:
                for key in handle.keys():
                    yield key, handle.get_tensor(key)


@pytest.mark.parametrize("cfg,draft_vocab", [(CONFIG1, 512), (CONFIG5S, 0)])
def test_sglang_plugin_loads_release_folder(tmp_path, cfg, draft_vocab):
    from flashmap_b200 import sglang_model as SG

    folder = str(tmp_path / "release")
    config, weights, ranking = write_release(folder, cfg, draft_vocab=draft_vocab)
    loaded_config = FlashMapConfig.from_pretrained(folder)
    sm = SG.FlashMapDraftModel(loaded_config)
    sm.load_weights(folder_entries(folder))
    params = {**dict(sm.named_parameters()), **dict(sm.named_buffers())}
    for name, tensor in weights.items():
        assert torch.equal(params[name].to(tensor.dtype), tensor), name
    want = config.state_vocab_size or draft_vocab
    assert sm.draft_vocab_size == want
    if ranking is not None:
        assert torch.equal(sm._vocab_ranking, ranking["ids"])


@pytest.mark.parametrize("cfg,draft_vocab", [(CONFIG1, 512), (CONFIG5S, 0)])
def test_vllm_plugin_loads_release_folder(tmp_path, cfg, draft_vocab):
    """vLLM's loader: ``draft_vocab_size`` from the folder's header sizes d2t,
    ``draft_ids`` (state vocabulary) or the ranking's ``ids`` fill it."""
    from flashmap_b200 import vllm_model as VL
    from tests.test_plugins import vllm_config

    folder = str(tmp_path / "release")
    config, weights, ranking = write_release(folder, cfg, draft_vocab=draft_vocab)
    m = VL.FlashMapDraftModel(vllm_config=vllm_config(FlashMapConfig.from_pretrained(folder)))
    m.load_weights(folder_entries(folder))
    params = {**dict(m.named_parameters()), **dict(m.named_buffers())}
    for name, tensor in weights.items():
        assert torch.equal(params["model." + name].to(tensor.dtype), tensor), name
    size = config.state_vocab_size or draft_vocab
    assert m.d2t is not None and m.d2t.shape[0] == size
    hot = weights["draft_ids"] if config.state_vocab_size else ranking["ids"][:size].sort().values
    assert torch.equal(m.d2t + torch.arange(size), hot)
