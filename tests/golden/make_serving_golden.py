"""Generate the golden vectors that pin the serving operators and the folds to
the reference's own code (al-jshen/flashmap v0.2.1, imported from a checkout
given by ``--reference``): the Triton kernels of flashmap/vllm/kernels.py
(``rms_norm_rope`` :68-121, ``block_self_attention`` :128-228,
``write_context_kv`` :236-365) and flashmap/sglang/kernels.py
(``block_self_attention`` :19-116, ``rms_norm_rope`` :150-185,
``sample_rows`` :196-254, greedy rows), run by Triton's CPU interpreter, and
the plain-torch folds of flashmap/vllm/fold.py (``noise_factor`` :45-58,
``fold_noise`` :61-74, ``fold_head`` :77-101).  Saves ``tests/golden/serving_cases.pt``.

    python tests/golden/make_serving_golden.py --reference /path/to/flashmap

The interpreter (triton 3.6) is made to follow the compiled kernels' numerics
in two places, both in its emulation of instructions and neither in the
reference's code: a float -> bf16 conversion rounds to nearest even (the
interpreter truncates, where ``.to(tl.bfloat16)`` compiles to a
round-to-nearest conversion), and ``tl.dot`` of bf16 operands multiplies their
values with fp32 accumulation (the interpreter multiplies the bf16 bit
patterns as integers).
"""

from __future__ import annotations

import argparse
import importlib.util
import os

os.environ.setdefault("TRITON_INTERPRET", "1")  # before triton is imported

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def load(reference: str, sub: str, name: str):
    spec = importlib.util.spec_from_file_location(f"ref_{sub}_{name}", os.path.join(reference, "flashmap", sub,
                                                                                     f"{name}.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def fix_interpreter():
    """Round-to-nearest-even float -> bf16 casts and value-level bf16 dots in the interpreter."""
    import triton.language as tl
    from triton.runtime import interpreter as I

    original_convert = I._convert_float

    def to_bf16_rne(bits_f32: np.ndarray) -> np.ndarray:
        u = bits_f32.astype(np.uint32)
        nan = (u & 0x7FFFFFFF) > 0x7F800000
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
        return r

    def convert(input, input_dtype, output_dtype, rounding_mode):
        if input_dtype == tl.float32 and output_dtype == tl.bfloat16:
            bits = np.frombuffer(np.ascontiguousarray(input).tobytes(), dtype=np.uint32).reshape(input.shape)
            return to_bf16_rne(bits)
        return original_convert(input, input_dtype, output_dtype, rounding_mode)

    I._convert_float = convert

    def bf16_values(h):
        bits = h.data.astype(np.uint32) << 16
        return bits.view(np.float32)

    original_dot = I.InterpreterBuilder.create_dot

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            av = bf16_values(a) if a.dtype.scalar == tl.bfloat16 else a.data.astype(np.float32)
            bv = bf16_values(b) if b.dtype.scalar == tl.bfloat16 else b.data.astype(np.float32)
            return I.TensorHandle(np.matmul(av, bv, dtype=np.float32) + d.data, d.dtype.scalar)
        return original_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    I.InterpreterBuilder.create_dot = create_dot


def bf(t):
    return t.to(torch.bfloat16)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a checkout of al-jshen/flashmap (the directory holding flashmap/)")
    args = ap.parse_args()
    fix_interpreter()
    vk = load(args.reference, "vllm", "kernels")
    sk = load(args.reference, "sglang", "kernels")
    fold = load(args.reference, "vllm", "fold")
    g = torch.Generator().manual_seed(11)
    eps = 1e-6
    cases = {"vllm_rms_norm_rope": [], "vllm_block_self_attention": [], "vllm_write_context_kv": [],
             "sglang_rms_norm_rope": [], "sglang_block_self_attention": [], "sglang_sample_rows_greedy": [],
             "fold_noise": [], "fold_head": []}

    for tokens, heads, hd in [(7, 4, 64), (5, 2, 128)]:
        x = bf(2 * torch.randn(tokens, heads, hd, generator=g))
        w = bf(1 + 0.2 * torch.randn(hd, generator=g))
        table = vk.rope_table(96, hd, 1e6, "cpu")
        pos = torch.randint(0, 96, (tokens,), generator=g)
        out = vk.rms_norm_rope(x, w, table, pos, eps)
        cases["vllm_rms_norm_rope"].append(dict(x=x, weight=w, cos_sin=table, positions=pos, eps=eps, out=out))

    for blocks, heads, hd in [(2, 4, 64), (1, 2, 128)]:
        T = 16
        qkv = bf(torch.randn(blocks, T, 3, heads, hd, generator=g))
        qn, kn = bf(1 + 0.2 * torch.randn(hd, generator=g)), bf(1 + 0.2 * torch.randn(hd, generator=g))
        table = vk.rope_table(128, hd, 1e6, "cpu")
        pos = torch.randint(0, 128, (blocks * T,), generator=g)
        out = vk.block_self_attention(qkv, qn, kn, table, pos, eps)
        cases["vllm_block_self_attention"].append(dict(qkv=qkv, q_norm=qn, k_norm=kn, cos_sin=table, positions=pos,
                                                       eps=eps, out=out))

    for tokens, L, heads, hd, hpc, page in [(6, 2, 4, 64, None, 4), (5, 3, 2, 64, 3, 8)]:
        kv = bf(torch.randn(tokens, L, 2, heads, hd, generator=g))
        hpc_ = hpc or heads
        n_caches = -(-L * heads // hpc_)
        blocks = 4
        caches = [torch.zeros(blocks, hpc_, page, 2 * hd, dtype=torch.bfloat16) for _ in range(n_caches)]
        ptrs = torch.tensor([c.data_ptr() for c in caches], dtype=torch.int64)
        slots = torch.randperm(blocks * page, generator=g)[:tokens]
        slots[1] = -1  # a skipped token
        kn = bf(1 + 0.2 * torch.randn(L, hd, generator=g))
        table = vk.rope_table(64, hd, 1e6, "cpu")
        pos = torch.randint(0, 64, (tokens,), generator=g)
        st = caches[0].stride()
        vk.write_context_kv(kv, pos, slots, kn, table, ptrs, (st[0], st[1], st[2], hd), page, eps,
                            heads_per_cache=hpc)
        cases["vllm_write_context_kv"].append(dict(kv=kv, positions=pos, slots=slots, k_norm=kn, cos_sin=table,
                                                   strides=(st[0], st[1], st[2], hd), block_size=page, eps=eps,
                                                   heads_per_cache=hpc, cache_shape=tuple(caches[0].shape),
                                                   caches=[c.clone() for c in caches]))

    for T, heads, hd in [(16, 4, 64), (16, 2, 128)]:
        x = bf(2 * torch.randn(2, T, heads, hd, generator=g))
        w = (1 + 0.2 * torch.randn(hd, generator=g)).float()
        ang = torch.rand(2, T, hd // 2, generator=g) * 6.283
        freqs = torch.stack([ang.cos(), ang.sin()], -1).contiguous()
        out = sk.rms_norm_rope(x, w, freqs, eps)
        cases["sglang_rms_norm_rope"].append(dict(x=x, weight=w, freqs=freqs, eps=eps, out=out))
        qkv = bf(torch.randn(2, T, 3, heads, hd, generator=g))
        qn, kn = (1 + 0.2 * torch.randn(hd, generator=g)).float(), (1 + 0.2 * torch.randn(hd, generator=g)).float()
        out = sk.block_self_attention(qkv, qn, kn, freqs, eps)
        cases["sglang_block_self_attention"].append(dict(qkv=qkv, q_norm=qn, k_norm=kn, freqs=freqs, eps=eps,
                                                         out=out))

    for rows, V in [(6, 5000), (3, 9000)]:
        logits = bf(3 * torch.randn(rows, V, generator=g))
        logits[0, 17] = logits[0, 4000] = logits[0].max() + 1  # a tie: the first index wins
        temps = torch.ones(rows)
        greedy = torch.ones(rows, dtype=torch.int32)
        seed = torch.tensor(7, dtype=torch.int64)
        out = sk.sample_rows(logits, temps, greedy, seed)
        cases["sglang_sample_rows_greedy"].append(dict(logits=logits, out=out))

    # the folds on the synthetic drafters of the tests (tests/helpers.py CONFIG1, CONFIG5S): the
    # inputs regenerate from the seeded synthetic law, the fixture keeps the reference's outputs
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from flashmap_b200 import FlashMapConfig
    from flashmap_b200.synthetic import synthetic_state_dict, synthetic_target_head
    from tests.helpers import CONFIG1, CONFIG5S

    for name, cfg in (("CONFIG1", CONFIG1), ("CONFIG5S", CONFIG5S)):
        config = FlashMapConfig(**cfg)
        sd = synthetic_state_dict(config, seed=0, dtype=torch.bfloat16)
        emb, head = synthetic_target_head(config, seed=0, dtype=torch.bfloat16)
        rows = sd.get("draft_ids")
        emb_s = emb if rows is None else emb[rows]
        m, lam_h = fold.fold_noise(emb_s, sd["noise_norm.weight"], sd["x_embed.weight"])
        cases["fold_noise"].append(dict(config=name, seed=0, M=m, var=lam_h))
        w, bias = fold.fold_head(head, sd["head.weight"], sd["head.bias"], rows=rows, chunk=512)
        cases["fold_head"].append(dict(config=name, seed=0, weight=w, bias=bias))

    path = os.path.join(HERE, "serving_cases.pt")
    torch.save(cases, path)
    print("saved", path, {k: len(v) for k, v in cases.items()})


if __name__ == "__main__":
    main()
