"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference FlashMap code itself (al-jshen/flashmap v0.2.1, imported
from a checkout given by ``--reference``) on the CPU with seeded synthetic
weights (``flashmap_b200.synthetic``) and injected random draws, and saves
inputs and outputs to ``tests/golden/*.pt``.  ``tests/test_oracle_golden.py``
replays the same inputs through ``oracle/`` and requires identical results.

The reference cannot be imported on the measurement box, so the fixtures are
committed; rerun this script only to regenerate them:

    python tests/golden/make_golden.py --reference /path/to/flashmap
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
from contextlib import contextmanager

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head  # noqa: E402

CONFIG1 = dict(
    target_hidden_size=256, vocab_size=2048, target_layer_ids=[0], block_size=16, hidden_size=256,
    num_hidden_layers=2, num_attention_heads=4, intermediate_size=1024, mlp_type="gelu",
)
# a config-5-shaped drafter at toy size: SwiGLU, a state vocabulary, two target layers
CONFIG5S = dict(
    target_hidden_size=320, vocab_size=3000, state_vocab_size=1024, target_layer_ids=[0, 1], block_size=16,
    hidden_size=256, num_hidden_layers=2, num_attention_heads=4, intermediate_size=384, mlp_type="swiglu",
)
TARGET1 = dict(vocab_size=2048, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, head_dim=64, rope_theta=1e6, intermediate_size=512)


def tensor_sha(t: torch.Tensor) -> str:
    """sha256 of a tensor's bytes (contiguous, as stored): a bit-exact pin."""
    t = t.detach().contiguous()
    raw = t.view(torch.int16) if t.dtype == torch.bfloat16 else t
    return hashlib.sha256(raw.numpy().tobytes()).hexdigest()


@contextmanager
def patched(module, name, fn):
    old = getattr(module, name)
    setattr(module, name, fn)
    try:
        yield
    finally:
        setattr(module, name, old)


def build_drafter(flashmap, cfg_kwargs, dtype, seed=0):
    config = flashmap.FlashMapConfig(**cfg_kwargs)
    model = flashmap.FlashMapDraftModel(config)
    sd = synthetic_state_dict(config, seed=seed, dtype=torch.float32)
    missing, unexpected = model.load_state_dict(sd, strict=True), None
    del missing, unexpected
    return model.to(dtype).eval(), config


class Emb(torch.nn.Module):
    def __init__(self, w):
        super().__init__()
        self.weight = torch.nn.Parameter(w, requires_grad=False)

    def forward(self, ids):
        return torch.nn.functional.embedding(ids, self.weight)


class Head(torch.nn.Module):
    def __init__(self, w):
        super().__init__()
        self.weight = torch.nn.Parameter(w, requires_grad=False)
        self.bias = None


def draft_case(flashmap, cfg_kwargs, dtype, *, ctx_len, num_steps, seed):
    """extend_context over ``ctx_len`` rows, then one draft with injected noise."""
    model, config = build_drafter(flashmap, cfg_kwargs, dtype, seed)
    emb_w, head_w = synthetic_target_head(config, seed=seed, dtype=dtype)
    g = torch.Generator().manual_seed(1000 + seed)
    hidden = torch.randn(1, ctx_len, len(config.target_layer_ids) * config.target_hidden_size, generator=g).to(dtype)
    anchor = torch.randint(0, config.vocab_size, (1,), generator=g)
    cache = flashmap.FlashMapCache(config, 1, ctx_len + config.block_size + 2, dtype=dtype)
    model.extend_context(cache, hidden)
    case = dict(config=cfg_kwargs, dtype=str(dtype), seed=seed, ctx_len=ctx_len, num_steps=num_steps,
                hidden=hidden, anchor=anchor, kv_after_extend_sha=tensor_sha(cache.kv[:, :, :, :, :ctx_len]))
    s_size = config.state_vocab_size or config.vocab_size
    if num_steps == 1:
        z = torch.randn(1, config.block_size, config.target_hidden_size, generator=g).to(dtype)
        case["z"] = z

        def fake_randn(*shape, **kw):
            return z.clone()

        with patched(torch, "randn", fake_randn):
            logits = model.draft(anchor, cache, Emb(emb_w), Head(head_w), num_steps=1)
    else:
        noise = torch.randn(1, config.block_size, s_size, generator=g)
        case["noise"] = noise
        logits = model.draft(anchor, cache, Emb(emb_w), Head(head_w), num_steps=num_steps, noise=noise)
    case["logits"] = logits
    case["anchor_kv_sha"] = tensor_sha(cache.kv[:, :, :, :, ctx_len])
    return case


def spec_case(flashmap, temperature, max_new_tokens=64, seed=0, rng_seed=1234):
    """spec_generate of the config-1 pair.

    Injected draws: round r's one-step noise z is the r-th draw of
    ``torch.randn((1, 16, 256), generator=Generator().manual_seed(77))``; at
    T > 0 the acceptance uniforms are Philox (k, 0, r, 1), the draft rows'
    categorical draws use Philox (k, 0, r, 3), the bonus draw (0, 0, r, 2)
    and the first target token (sampled from the prefill) (0, 0, 2^32 - 1, 3),
    a counter no round reaches, all through the oracle's categorical sampler
    (its sliced form for the bonus)."""
    from transformers import Qwen3Config, Qwen3ForCausalLM

    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import accept

    torch.manual_seed(0)
    target = Qwen3ForCausalLM(Qwen3Config(**TARGET1)).eval()
    model, config = build_drafter(flashmap, CONFIG1, torch.float32, seed)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 2048, (1, 128), generator=g)
    zs, rounds = [], {"n": 0, "draft_calls": 0, "prefill_done": False}
    zg = torch.Generator().manual_seed(77)
    real_randn = torch.randn

    def fake_randn(*shape, **kw):
        shape = shape[0] if len(shape) == 1 and isinstance(shape[0], tuple) else shape
        z = real_randn(*shape, generator=zg, dtype=kw.get("dtype") or torch.float32)
        zs.append(z.clone())
        return z

    def fake_rand(shape, **kw):
        r = rounds["n"]
        return torch.tensor([accept.uniform(rng_seed, k, 0, r, 1) for k in range(shape[0])])

    def fake_multinomial(probs, n, generator=None, **kw):
        r = rounds["n"]
        if probs.dim() == 2:  # the prefill's row (:562), then each round's K draft rows (:557)
            if rounds["prefill_done"]:
                rounds["draft_calls"] += 1
            word = r if rounds["prefill_done"] else 0xFFFFFFFF
            rounds["prefill_done"] = True
            out = [accept.categorical(probs[k].float().numpy(), accept.uniform(rng_seed, k, 0, word, 3))
                   for k in range(probs.shape[0])]
            return torch.tensor(out, dtype=torch.int64)[:, None]
        tok = accept.categorical_sliced(probs.float().numpy(), accept.uniform(rng_seed, 0, 0, r, 2))  # bonus (:594)
        rounds["n"] += 1
        return torch.tensor([tok], dtype=torch.int64)

    with patched(torch, "randn", fake_randn):
        if temperature > 0:
            with patched(torch, "rand", fake_rand), patched(torch, "multinomial", fake_multinomial):
                out = model.spec_generate(target, prompt, max_new_tokens=max_new_tokens, temperature=temperature)
        else:
            out = model.spec_generate(target, prompt, max_new_tokens=max_new_tokens, temperature=temperature)
    return dict(temperature=temperature, prompt=prompt, sequences=out.sequences,
                acceptance_lengths=list(out.acceptance_lengths), num_z=len(zs), rng_seed=rng_seed,
                max_new_tokens=max_new_tokens)


def reference_acceptance_block(flashmap):
    """The acceptance statements of the reference's spec_generate, as source.

    Taken from the loaded module at run time (the ``if temperature <= 0:``
    block whose first statement is the target argmax, up to the line that
    builds ``new_tokens``), so the golden outputs come from the reference's
    own code, not from a restatement."""
    import inspect
    import textwrap

    src = inspect.getsource(flashmap.modeling_flashmap.FlashMapDraftModel.spec_generate).splitlines()
    start = next(i for i, line in enumerate(src)
                 if line.strip() == "if temperature <= 0:" and "target_tokens" in src[i + 1])
    end = next(i for i in range(start, len(src)) if "new_tokens = torch.cat" in src[i])
    return textwrap.dedent("\n".join(src[start:end]))


def acceptance_case(flashmap, B, K, V, seed, temperature, rng_seed=1234):
    """Run the reference's acceptance block row by row on recipe inputs."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import accept
    from tests.golden.inputs import acceptance_inputs

    code = compile(reference_acceptance_block(flashmap), "reference_acceptance", "exec")
    target, draft, q = acceptance_inputs(B, K, V, seed, temperature)
    accepted, bonus = [], []
    for b in range(B):
        def fake_rand(shape, **kw):
            return torch.tensor([accept.uniform(rng_seed, k, b, 0, 1) for k in range(shape[0])])

        def fake_multinomial(probs, n, generator=None, **kw):
            return torch.tensor([accept.categorical_sliced(probs.float().numpy(),
                                                           accept.uniform(rng_seed, 0, b, 0, 2))])

        class Out:
            logits = target[b : b + 1]

        ns = dict(torch=torch, out=Out, draft=draft[b : b + 1], temperature=temperature, generator=None,
                  block_size=K, draft_probs=None if q is None else q[b : b + 1])
        with patched(torch, "rand", fake_rand), patched(torch, "multinomial", fake_multinomial):
            exec(code, ns)
        accepted.append(int(ns["accepted"]))
        bonus.append(int(ns["bonus"].reshape(-1)[0]))
    return dict(B=B, K=K, V=V, seed=seed, temperature=temperature, rng_seed=rng_seed,
                accepted=accepted, bonus=bonus)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of a flashmap checkout (its parent of flashmap/)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import flashmap  # noqa: F401  (the reference itself)

    torch.set_num_threads(8)
    cases = {
        "c1_fp32_1step": draft_case(flashmap, CONFIG1, torch.float32, ctx_len=40, num_steps=1, seed=0),
        "c1_bf16_1step": draft_case(flashmap, CONFIG1, torch.bfloat16, ctx_len=40, num_steps=1, seed=1),
        "c1_fp32_2step": draft_case(flashmap, CONFIG1, torch.float32, ctx_len=33, num_steps=2, seed=2),
        "c5s_bf16_1step": draft_case(flashmap, CONFIG5S, torch.bfloat16, ctx_len=29, num_steps=1, seed=3),
        "c5s_bf16_2step": draft_case(flashmap, CONFIG5S, torch.bfloat16, ctx_len=21, num_steps=2, seed=4),
    }
    torch.save(cases, os.path.join(HERE, "draft_cases.pt"))
    spec = {"greedy": spec_case(flashmap, 0.0), "t1": spec_case(flashmap, 1.0)}
    torch.save(spec, os.path.join(HERE, "spec_cases.pt"))
    acc = {
        "greedy": acceptance_case(flashmap, 34, 16, 3001, seed=5, temperature=0.0),
        "t1": acceptance_case(flashmap, 24, 16, 3001, seed=6, temperature=1.0),
        "t07": acceptance_case(flashmap, 24, 16, 2048, seed=7, temperature=0.7),
    }
    torch.save(acc, os.path.join(HERE, "acceptance_cases.pt"))
    for k, v in acc.items():
        print(k, v["accepted"], v["bonus"][:8])
    for k, v in cases.items():
        print(k, tuple(v["logits"].shape), float(v["logits"].float().abs().max()))
    for k, v in spec.items():
        print(k, v["sequences"].shape, v["acceptance_lengths"])


if __name__ == "__main__":
    main()
