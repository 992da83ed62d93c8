"""The vLLM and sglang plugin models on the GPU against stand-in engines: the
context written through each engine's paged layout, one draft step, and the
draft logits compared with the CPU oracle's draft of the same context and
noise.  The plugins fold like their reference counterparts (vLLM: the head
and the noise; sglang: the head, the noise with ``FLASHMAP_FOLDED_NOISE``),
so the oracle drafts folded too, fed the plugin's own noise-fold tensors (the
eigenbasis is defined up to signs).  The noise rows are given: each test
replaces the plugin core's noise draw with fixed normals.

Tolerances are the north star's: logits within 2e-2 of the reference's
scale, and no argmax disagreement (tie-aware) at a decisive position, one
whose reference top-1/top-2 gap exceeds twice the block's largest logit
difference.
"""

from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import sglang_model as SG  # noqa: E402
from flashmap_b200 import vllm_model as VL  # noqa: E402
from oracle.flashmap_oracle import OracleCache  # noqa: E402
from tests.helpers import CONFIG1, CONFIG5S, LOGITS_RTOL, Emb, Head, build, decisive_disagreements  # noqa: E402

DEV = "cuda"
PAGE = 16


def _contexts(config, lengths, seed):
    g = torch.Generator().manual_seed(seed)
    width = len(config.target_layer_ids) * config.target_hidden_size
    return [torch.randn(n, width, generator=g).to(torch.bfloat16) for n in lengths]


def _oracle_logits(config, oracle, emb, head, hidden, anchor, z, noise_fold, steps=1, state=None):
    K = config.block_size
    oc = OracleCache(config, 1, hidden.shape[0] + K + 2, torch.bfloat16)
    oracle.extend_context(oc, hidden[None])
    if steps == 1:
        ref = oracle.draft(torch.tensor([anchor]), oc, emb, head, num_steps=1, z=z[None], folded=True,
                           noise_fold=noise_fold)[0]
    else:
        ref = oracle.draft(torch.tensor([anchor]), oc, emb, head, num_steps=steps, noise=state[None], folded=True)[0]
    if config.state_vocab_size:
        ref = ref[:, oracle.p["draft_ids"].long()] if "draft_ids" in oracle.p else ref
    return ref


def _check(config, got, ref, what):
    g, r = got.float().cpu(), ref.float().cpu()
    fin = torch.isfinite(r)
    r = torch.where(fin, r, torch.zeros_like(r))
    g = torch.where(fin, g, torch.zeros_like(g))
    rel = float((g - r).abs().max() / r.abs().max())
    assert rel <= LOGITS_RTOL, f"{what}: logits relative error {rel:.4g}"
    bad, under, thr = decisive_disagreements(got.float().argmax(-1), got, ref)
    assert bad == 0, f"{what}: {bad} argmax disagreements at decisive positions (margin {thr:.4g})"


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
@pytest.mark.parametrize("steps", [1, 2])
def test_vllm_plugin_draft_matches_oracle(cfg, steps):
    """One jump (folded noise and head) or two (the exact vocabulary-sized state,
    the folded jump head) against the oracle's draft of the same noise."""
    config, model, oracle, emb, head = build(cfg, seed=4)
    config.num_steps = steps
    K, H, hd, L = config.block_size, config.num_attention_heads, config.hidden_size // config.num_attention_heads, \
        config.num_hidden_layers
    vconf = SimpleNamespace(parallel_config=SimpleNamespace(tensor_parallel_size=1), use_v2_model_runner=True,
                            speculative_config=SimpleNamespace(draft_model_config=SimpleNamespace(hf_config=config)),
                            model_config=SimpleNamespace(dtype=torch.bfloat16, max_model_len=1024, is_hybrid=False),
                            cache_config=SimpleNamespace(cache_dtype="auto"))
    vm = VL.FlashMapDraftModel(vllm_config=vconf).to(DEV)
    vm.model.to(torch.bfloat16)
    vm.load_weights(model.state_dict().items())
    vm.model.embed_tokens = Emb(emb.to(DEV))
    vm.lm_head = Head(head.to(DEV))
    num_blocks = 64
    caches = [torch.zeros(num_blocks, H, PAGE, 2 * hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    layers = [SimpleNamespace(kv_cache=c, layer_name=f"ctx.{i}", kv_cache_dtype="auto") for i, c in enumerate(caches)]
    vm.bind_cache_layers(layers)
    vm.prepare()
    lengths = [40, 23, 130]
    gz = torch.Generator().manual_seed(16)
    z = torch.randn(len(lengths) * K, config.target_hidden_size, generator=gz).to(torch.bfloat16)
    vm._core.noise = lambda *args, **kwargs: z.to(DEV)
    state = torch.randn(len(lengths) * K, vm._core.pack.S, generator=gz)
    vm._core.state_noise = lambda *args, **kwargs: state.to(DEV).clone()
    fold = tuple(t.cpu() for t in vm._core.pack.ensure_noise_fold(config))

    hiddens = _contexts(config, lengths, 5)
    g = torch.Generator().manual_seed(6)
    cols = (max(lengths) + K + PAGE) // PAGE
    table = torch.randperm(num_blocks, generator=g)[: len(lengths) * cols].view(len(lengths), cols).int()

    def slot(r, p):
        return int(table[r, p // PAGE]) * PAGE + p % PAGE

    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        states = vm.combine_hidden_states(h.to(DEV))
        pos = torch.arange(n, device=DEV)
        slots = torch.tensor([slot(r, p) for p in range(n)], device=DEV)
        if r == 1:  # the deferred path: written by the next forward with the anchors
            vm.defer_context_kv(states, pos, slots)
        else:
            vm.precompute_and_store_context_kv(states, pos, slots)
    anchors = torch.randint(0, config.vocab_size, (len(lengths),), generator=g)
    input_ids = torch.stack([torch.cat([a[None], torch.zeros(K - 1, dtype=torch.long)]) for a in anchors]).view(-1)
    positions = torch.cat([n + torch.arange(K) for n in lengths])
    slot_mapping = torch.tensor([slot(r, n + k) for r, n in enumerate(lengths) for k in range(K)])
    meta = SimpleNamespace(seq_lens=torch.tensor(lengths, dtype=torch.int32, device=DEV) + K,
                           slot_mapping=slot_mapping.to(DEV),
                           query_start_loc=torch.arange(0, (len(lengths) + 1) * K, K, dtype=torch.int32, device=DEV),
                           block_table=table.to(DEV))
    vm.forward_context = lambda: SimpleNamespace(attn_metadata={"ctx.0": meta})
    hidden = vm.forward(input_ids.to(DEV), positions.to(DEV))
    logits = vm.compute_draft_logits(hidden)
    torch.cuda.synchronize()
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        ref = _oracle_logits(config, oracle, emb, head, h, int(anchors[r]), z[r * K:(r + 1) * K], fold, steps,
                             state[r * K:(r + 1) * K])
        _check(config, logits[r * K:(r + 1) * K], ref, f"vllm request {r} ({steps} jumps)")


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
@pytest.mark.parametrize("folded_noise", [False, True])
def test_sglang_plugin_draft_matches_oracle(cfg, folded_noise):
    config, model, oracle, emb, head = build(cfg, seed=7)
    K, H, hd, L = config.block_size, config.num_attention_heads, config.hidden_size // config.num_attention_heads, \
        config.num_hidden_layers
    sm = SG.FlashMapDraftModel(config).to(DEV, torch.bfloat16)
    sm.load_weights(model.state_dict().items())
    sm.folded_noise = folded_noise  # FLASHMAP_FOLDED_NOISE, read at construction
    sm.attach_shared_modules(embed_tokens=Emb(emb.to(DEV)), lm_head=Head(head.to(DEV)))
    assert sm.folded_head is not None and sm.lm_head.weight.shape[1] == config.hidden_size
    gz = torch.Generator().manual_seed(17)
    z = torch.randn(2 * K, config.target_hidden_size, generator=gz).to(torch.bfloat16)
    sm._core.noise = lambda *args, **kwargs: z.to(DEV)
    fold = tuple(t.cpu() for t in sm._core.pack.ensure_noise_fold(config)) if folded_noise else None
    rows = 1024
    kb = [torch.zeros(rows, H, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    vb = [torch.zeros(rows, H, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    pool = SimpleNamespace(get_key_buffer=lambda i: kb[i], get_value_buffer=lambda i: vb[i])
    lengths = [33, 200]
    g = torch.Generator().manual_seed(8)
    req_to_token = torch.randperm(rows, generator=g)[: 2 * 300].view(2, 300).int().to(DEV)
    sm.token_to_kv_pool = lambda: pool
    sm.req_to_token = lambda: req_to_token
    hiddens = _contexts(config, lengths, 9)
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        sm.write_target_hidden_kv(target_hidden=h.to(DEV), pool=pool, positions=torch.arange(n, device=DEV),
                                  cache_loc=req_to_token[r, :n].long())
    anchors = torch.randint(0, config.vocab_size, (len(lengths),), generator=g)
    input_ids = torch.stack([torch.cat([a[None], torch.zeros(K - 1, dtype=torch.long)]) for a in anchors]).view(-1)
    positions = torch.cat([n + torch.arange(K) for n in lengths]).to(DEV)
    out_cache_loc = torch.cat([req_to_token[r, n:n + K].long() for r, n in enumerate(lengths)])
    batch = SimpleNamespace(batch_size=len(lengths), seq_lens=torch.tensor(lengths, device=DEV),
                            out_cache_loc=out_cache_loc, req_pool_indices=torch.arange(len(lengths), device=DEV))
    out = sm.forward(input_ids.to(DEV), positions, batch)
    logits, _ = sm.compute_base_logits(out.hidden_states)
    torch.cuda.synchronize()
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        ref = _oracle_logits(config, oracle, emb, head, h, int(anchors[r]), z[r * K:(r + 1) * K], fold)
        _check(config, logits[r * K:(r + 1) * K], ref, f"sglang request {r}")
