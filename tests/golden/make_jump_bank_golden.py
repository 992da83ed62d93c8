"""Generate the golden vectors that pin the banked multi-jump oracle
(``oracle/jump_bank_oracle.py``) to the reference's ``flashmap/sglang/jump_bank.py``.

Runs the reference module itself (al-jshen/flashmap v0.2.1, imported from a
checkout given by ``--reference``; it needs only torch) on the CPU: the
per-(seed, token) normals, the jump coefficients of several grids, a small
noise bank (its draws recorded by replaying the bank's own generator) and the
embedded jump inputs for given bank rows, seeds and prediction supports.  The
reference's draft object is a stand-in holding the fields the bank reads
(``state_embedding``, ``state_norm``, ``noise_norm``, ``jump_gate``), its
norms the reference's ``FlashMapRMSNorm``.  Saves ``tests/golden/jump_bank_cases.pt``;
``tests/test_jump_bank_oracle.py`` replays the inputs through the oracle.

    python tests/golden/make_jump_bank_golden.py --reference /path/to/flashmap
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))

V, H, M, CHUNK = 96, 32, 12, 5
TEMPERATURE, BANK_SEED, EPS, NOISE_GATE = 0.8, 3, 1e-6, 0.6
GRID = [0.0, 0.4, 0.8, 1.0]
GRIDS = [[0.0, 1.0], [0.0, 0.5, 1.0], [0.0, 0.3, 0.7, 1.0], [0.0, 0.25, 0.5, 0.75, 1.0]]


def load(reference: str):
    sys.path.insert(0, reference)
    from flashmap.modeling_flashmap import FlashMapRMSNorm  # noqa: E402

    spec = importlib.util.spec_from_file_location("ref_jump_bank",
                                                  os.path.join(reference, "flashmap", "sglang", "jump_bank.py"))
    bank = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bank)
    return bank, FlashMapRMSNorm


class StandIn:
    """The fields of the sglang draft model the bank reads, for grid ``GRID``."""

    def __init__(self, rmsnorm_cls, embedding, w_state, w_noise):
        self.state_embedding = embedding
        self.state_norm = rmsnorm_cls(H, EPS).to(torch.bfloat16)
        self.noise_norm = rmsnorm_cls(H, EPS).to(torch.bfloat16)
        with torch.no_grad():
            self.state_norm.weight.copy_(w_state)
            self.noise_norm.weight.copy_(w_noise)
        self.noise_gate = torch.tensor(NOISE_GATE).to(torch.bfloat16)
        self.jumps = [(a, b, b) for a, b in zip(GRID[:-1], GRID[1:])]

    def jump_gate(self, step: int) -> torch.Tensor:
        start, end, _ = self.jumps[step]
        return (self.noise_gate.float() * (end - start)).to(self.noise_gate.dtype)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="a checkout of al-jshen/flashmap (the directory holding flashmap/)")
    args = ap.parse_args()
    bank_mod, rmsnorm_cls = load(args.reference)
    g = torch.Generator().manual_seed(11)

    # per-(seed, token) normals, including ids past 2^31 and repeated ids
    seeds = torch.tensor([0, 1, 12345, 2**31 - 2, 987654321], dtype=torch.int64)
    ids = torch.randint(0, 2**32 - 1, (5, 40), generator=g, dtype=torch.int64)
    ids[:, 5] = ids[:, 2]
    normals = bank_mod.token_normals(seeds, ids)

    coefficients = {str(grid): bank_mod.jump_coefficients(grid) for grid in GRIDS}

    embedding = (torch.randn(V, H, generator=g) * 0.5).to(torch.bfloat16)
    w_state = (1.0 + 0.2 * torch.randn(H, generator=g)).to(torch.bfloat16)
    w_noise = (1.0 + 0.2 * torch.randn(H, generator=g)).to(torch.bfloat16)
    draft = StandIn(rmsnorm_cls, embedding, w_state, w_noise)
    bank = bank_mod.JumpNoiseBank(draft, GRID, size=M, temperature=TEMPERATURE, seed=BANK_SEED, chunk=CHUNK)
    # the bank's draws, replayed from its generator in its chunk order
    gz = torch.Generator(device="cpu").manual_seed(BANK_SEED)
    z = torch.cat([TEMPERATURE * torch.randn(min(CHUNK, M - s), V, generator=gz) for s in range(0, M, CHUNK)])

    posterior = torch.full((1, V), 1.0 / V).to(torch.bfloat16)
    uniform = draft.state_norm(posterior @ embedding)[0]
    rows = torch.tensor([0, 5, 11, 5, 7], dtype=torch.int64)
    slot_seeds = torch.tensor([1, 2**31 - 2, 77, 1234, 5], dtype=torch.int64)
    k = 6
    supports = []
    for m in range(2):
        logits = torch.randn(rows.numel(), V, generator=g) * 3.0
        sid, sp = bank_mod.top_predictions(logits, k)
        if m == 1:
            sid[:, 0] = supports[0][0][:, 1]  # a token both predictions hold
        supports.append((sid, sp))
    first = bank.first_input(draft, rows, uniform)
    jump1 = bank.jump_input(draft, 1, rows, slot_seeds, supports[:1])
    jump2 = bank.jump_input(draft, 2, rows, slot_seeds, supports[:2])
    topk_logits = torch.randn(3, V, generator=g).to(torch.bfloat16)
    topk_rows = torch.randperm(V, generator=g)
    topk_ids, topk_probs = bank_mod.top_predictions(topk_logits, k, topk_rows)

    out = dict(
        V=V, H=H, M=M, temperature=TEMPERATURE, eps=EPS, noise_gate=NOISE_GATE, grid=GRID, k=k,
        seeds=seeds, ids=ids, normals=normals, coefficients=coefficients,
        embedding=embedding, w_state=w_state, w_noise=w_noise, z=z,
        noise_embed=bank.noise_embed, mean_embed=bank.mean_embed, log_mass=bank.log_mass,
        evidence=bank.evidence, slopes=bank.slopes,
        uniform=uniform, rows=rows, slot_seeds=slot_seeds, supports=supports,
        first=first, jump1=jump1, jump2=jump2,
        topk_logits=topk_logits, topk_rows=topk_rows, topk_ids=topk_ids, topk_probs=topk_probs,
    )
    out = {k: (v.detach() if isinstance(v, torch.Tensor) else v) for k, v in out.items()}
    out["supports"] = [(i.detach(), q.detach()) for i, q in out["supports"]]
    path = os.path.join(HERE, "jump_bank_cases.pt")
    torch.save(out, path)
    print("wrote", path)


if __name__ == "__main__":
    main()
