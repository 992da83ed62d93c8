"""The banked multi-jump kernels (csrc/bank.cu) and the sglang plugin's banked
draft on the GPU: each kernel against the golden vectors of the reference's
flashmap/sglang/jump_bank.py (tests/golden/jump_bank_cases.pt), and a two-jump
plugin draft against the oracle's banked draft of the same bank rows, seeds
and supports.

Tolerances: bf16 results within 2 bf16 ulps of the reference (different fp32
summation orders round apart); fp32 log-masses and probabilities within 1e-5
relative; the hashed normals within 2e-5 (CUDA's log, cos and sqrt against
torch's CPU ones); the jump rows within 1e-2 of their scale (the weights
exp(a z - log Z) carry the normals' last-ulp differences); draft logits
within the north star's 2e-2."""

import ctypes
import os
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from flashmap_b200 import _lib, ops  # noqa: E402
from flashmap_b200 import sglang_model as SG  # noqa: E402
from oracle import jump_bank_oracle as JB  # noqa: E402
from oracle.flashmap_oracle import OracleCache  # noqa: E402
from tests.helpers import CONFIG1, CONFIG5S, LOGITS_RTOL, Emb, Head, build  # noqa: E402

DEV = "cuda"
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "jump_bank_cases.pt")
p_ = ops._p


@pytest.fixture(scope="module")
def case():
    return torch.load(GOLDEN)


def _ulps(got, ref, n):
    g, r = got.float().cpu(), ref.float().cpu()
    ulp = torch.pow(2.0, torch.floor(torch.log2(r.abs().clamp_min(1e-30))) - 7)
    bad = (g - r).abs() > n * ulp + 1e-6
    assert not bool(bad.any()), f"{int(bad.sum())} of {bad.numel()} beyond {n} bf16 ulps"


def test_token_normals(case):
    seeds, ids = case["seeds"].to(DEV), case["ids"].to(DEV)
    out = torch.empty(ids.shape, device=DEV)
    _lib.call("fm_token_normals", p_(seeds), p_(ids), ids.shape[0], ids.shape[1], p_(out), ops._stream())
    torch.testing.assert_close(out.cpu(), case["normals"], atol=2e-5, rtol=1e-5)


def test_bank_rows_and_products(case):
    z, E = case["z"].to(DEV), case["embedding"].to(DEV)
    slopes = case["slopes"]
    rows, V = z.shape
    zb = torch.empty(rows, V, device=DEV, dtype=torch.bfloat16)
    probs = torch.empty(len(slopes), rows, V, device=DEV, dtype=torch.bfloat16)
    mass = torch.empty(len(slopes), rows, device=DEV)
    arr = (ctypes.c_float * 8)(*slopes)
    _lib.call("fm_bank_rows", p_(z), p_(zb), p_(probs), p_(mass), rows, V, ctypes.cast(arr, ctypes.c_void_p),
              len(slopes), ops._stream())
    et = E.t().contiguous()
    _ulps(ops.gemm(et, zb), case["noise_embed"], 2)
    for j in range(len(slopes)):
        _ulps(ops.gemm(et, probs[j]), case["mean_embed"][j], 2)
    torch.testing.assert_close(mass.cpu(), case["log_mass"], atol=0.0, rtol=1e-5)


def test_topk_rows(case):
    logits, row_map, k = case["topk_logits"].to(DEV), case["topk_rows"].to(DEV), case["k"]
    R, V = logits.shape
    ids = torch.empty(R, k, device=DEV, dtype=torch.int64)
    probs = torch.empty(R, k, device=DEV)
    err = torch.zeros(1, device=DEV, dtype=torch.int32)
    _lib.call("fm_topk_rows", p_(logits), V, R, V, k, p_(row_map), V, p_(ids), p_(probs), p_(err), ops._stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    torch.testing.assert_close(probs.cpu(), case["topk_probs"], atol=0.0, rtol=1e-5)
    # the same tokens up to exact ties of the bf16 logits (this kernel breaks them by index)
    ref_ids, lg = case["topk_ids"], case["topk_logits"].float()
    inv = torch.argsort(case["topk_rows"])
    for r in range(R):
        got_vals = lg[r, inv[ids[r].cpu()]]
        want_vals = lg[r, inv[ref_ids[r]]]
        assert torch.equal(got_vals, want_vals)


def _gate(case, n):
    grid = case["grid"]
    return (torch.tensor(case["noise_gate"]).to(torch.bfloat16).float() * (grid[n + 1] - grid[n])).to(torch.bfloat16)


def _mix(case, post, stride, state, n):
    R, H = state.shape
    out = torch.empty(R, H, device=DEV, dtype=torch.bfloat16)
    w_state, w_noise = case["w_state"].to(DEV), case["w_noise"].to(DEV)  # held until the kernel has run
    _lib.call("fm_mix_state", p_(post), stride, p_(state), p_(w_state), p_(w_noise), p_(out),
              float(_gate(case, n).float()), float(case["eps"]), R, H, ops._stream())
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("n", [0, 1, 2])
def test_jump_inputs(case, n):
    E = case["embedding"].to(DEV)
    V, H = E.shape
    rows, seeds = case["rows"].to(DEV), case["slot_seeds"].to(DEV)
    R = rows.shape[0]
    noise_embed = case["noise_embed"].to(DEV)
    if n == 0:
        gathered = torch.empty(R, H, device=DEV, dtype=torch.bfloat16)
        _lib.call("fm_bank_gather", p_(noise_embed), noise_embed.shape[0], H, p_(rows), R, p_(gathered), None,
                  ops._stream())
        uniform = ops.gemm(E.t().contiguous(), torch.full((1, V), 1.0 / V, device=DEV).to(torch.bfloat16))
        got = _mix(case, uniform.reshape(-1), 0, gathered, 0)
        _ulps(got, case["first"], 2)
        return
    supports = case["supports"][:n]
    ids = torch.cat([i for i, _ in supports], 1).to(DEV).contiguous()
    probs = torch.cat([q for _, q in supports], 1).float().to(DEV).contiguous()
    coefficients = JB.jump_coefficients(case["grid"])
    alpha, betas = coefficients[n]
    beta_t = torch.tensor(betas, device=DEV, dtype=torch.float32)
    mean_embed, log_mass = case["mean_embed"][n - 1].to(DEV), case["log_mass"][n - 1].to(DEV)
    out = torch.empty(2 * R, H, device=DEV, dtype=torch.bfloat16)
    err = torch.zeros(1, device=DEV, dtype=torch.int32)
    a = _lib.BankJump()
    a.noise_embed, a.mean_embed, a.log_mass, a.embed = (noise_embed.data_ptr(), mean_embed.data_ptr(),
                                                        log_mass.data_ptr(), E.data_ptr())
    a.state_map = None
    a.bank_rows, a.state_rows, a.hidden, a.slots = noise_embed.shape[0], V, H, R
    a.rows, a.seeds, a.ids, a.probs, a.betas = (rows.data_ptr(), seeds.data_ptr(), ids.data_ptr(), probs.data_ptr(),
                                                beta_t.data_ptr())
    a.support, a.topk = ids.shape[1], supports[0][0].shape[1]
    a.alpha, a.evidence, a.slope = alpha, case["evidence"][n - 1], case["slopes"][n - 1]
    a.temperature, a.out, a.err = case["temperature"], out.data_ptr(), err.data_ptr()
    _lib.call("fm_bank_jump_rows", ctypes.byref(a), ops._stream())
    post, noise = JB.jump_rows((case["noise_embed"], case["mean_embed"], case["log_mass"]), case["grid"], n,
                               case["rows"], case["slot_seeds"], supports, case["embedding"], case["temperature"])
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for got, want in ((out[:R], post), (out[R:], noise)):
        g, w = got.float().cpu(), want.float()
        assert float((g - w).abs().max() / w.abs().max()) < 1e-2
    got = _mix(case, out[:R], H, out[R:], n).float().cpu()
    want = case[f"jump{n}"].float()
    assert float((got - want).abs().max() / want.abs().max()) < 1e-2


@pytest.mark.parametrize("cfg", [CONFIG1, CONFIG5S])
def test_sglang_banked_two_jump_draft_matches_oracle(cfg):
    """Two banked jumps through the plugin against the oracle's: the same bank
    (the plugin's), bank rows and slot seeds (fixed), and the supports the
    plugin's top-k chose after jump 0 (they agree with the oracle's own top-k of
    its jump-0 logits up to near-ties)."""
    config, model, oracle, emb, head = build(cfg, seed=21)
    config.num_steps = 2
    K, H, hd, L = config.block_size, config.num_attention_heads, config.hidden_size // config.num_attention_heads, \
        config.num_hidden_layers
    sm = SG.FlashMapDraftModel(config).to(DEV, torch.bfloat16)
    sm.load_weights(model.state_dict().items())
    sm.jump_bank_size, sm.jump_topk = 96, 8
    sm.attach_shared_modules(embed_tokens=Emb(emb.to(DEV)), lm_head=Head(head.to(DEV)))
    core = sm._core
    bank = sm.jump_bank
    assert bank is not None and bank.size == 96
    rows_pool = 1024
    kb = [torch.zeros(rows_pool, H, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    vb = [torch.zeros(rows_pool, H, hd, dtype=torch.bfloat16, device=DEV) for _ in range(L)]
    pool = SimpleNamespace(get_key_buffer=lambda i: kb[i], get_value_buffer=lambda i: vb[i])
    lengths = [37, 90]
    g = torch.Generator().manual_seed(22)
    req_to_token = torch.randperm(rows_pool, generator=g)[: 2 * 200].view(2, 200).int().to(DEV)
    sm.token_to_kv_pool = lambda: pool
    sm.req_to_token = lambda: req_to_token
    width = len(config.target_layer_ids) * config.target_hidden_size
    hiddens = [torch.randn(n, width, generator=g).to(torch.bfloat16) for n in lengths]
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        sm.write_target_hidden_kv(target_hidden=h.to(DEV), pool=pool, positions=torch.arange(n, device=DEV),
                                  cache_loc=req_to_token[r, :n].long())
    T = len(lengths) * K
    bank_rows = torch.randint(0, bank.size, (T,), generator=g)
    slot_seeds = torch.randint(0, 2**31 - 1, (T,), generator=g)
    core.bank_draw = lambda *args, **kwargs: (bank_rows.to(DEV), slot_seeds.to(DEV))
    recorded = []
    top = core.top_predictions

    def record(*args, **kwargs):
        out = top(*args, **kwargs)
        recorded.append(out)
        return out

    core.top_predictions = record
    anchors = torch.randint(0, config.vocab_size, (len(lengths),), generator=g)
    input_ids = torch.stack([torch.cat([a[None], torch.zeros(K - 1, dtype=torch.long)]) for a in anchors]).view(-1)
    positions = torch.cat([n + torch.arange(K) for n in lengths]).to(DEV)
    out_cache_loc = torch.cat([req_to_token[r, n:n + K].long() for r, n in enumerate(lengths)])
    batch = SimpleNamespace(batch_size=len(lengths), seq_lens=torch.tensor(lengths, device=DEV),
                            out_cache_loc=out_cache_loc, req_pool_indices=torch.arange(len(lengths), device=DEV))
    out = sm.forward(input_ids.to(DEV), positions, batch)
    logits, _ = sm.compute_base_logits(out.hidden_states)
    torch.cuda.synchronize()
    assert len(recorded) == 1
    sup_ids, sup_probs = (t.cpu() for t in recorded[0])

    cpu_bank = (bank.noise_embed.cpu(), bank.mean_embed.cpu(), bank.log_mass.cpu())
    state_e = emb if config.state_vocab_size is None else emb[oracle.p["draft_ids"]]
    fold = oracle.fold_head(head)
    (s0, t0, _), (s1, t1, _) = [(a, b, b) for a, b in zip(bank.grid[:-1], bank.grid[1:])]
    uniform_embeds = oracle.target_constants(state_e)[0]
    for r, (n, h) in enumerate(zip(lengths, hiddens)):
        sl = slice(r * K, (r + 1) * K)
        oc = OracleCache(config, 1, n + K + 2, torch.bfloat16)
        oracle.extend_context(oc, h[None])
        anchor = torch.tensor([int(anchors[r])])
        oracle.anchor_context(oc, anchor, emb)
        context = oc.context(n + 1)
        pos = n + 1 + torch.arange(K)[None]
        inputs0 = oracle.mix_state(uniform_embeds, JB.first_rows(cpu_bank[0], bank_rows[sl])[None], s0, t0)
        logits0 = oracle.forward(inputs0, s0, t0, pos, context, head=fold)[0]
        ref_ids, _ = JB.top_predictions(logits0, sm.jump_topk)
        overlap = sum(len(set(a.tolist()) & set(b.tolist())) for a, b in zip(ref_ids, sup_ids[sl])) / ref_ids.numel()
        assert overlap >= 0.9, f"request {r}: jump-0 top-k overlap {overlap}"
        post, noise = JB.jump_rows(cpu_bank, bank.grid, 1, bank_rows[sl], slot_seeds[sl],
                                   [(sup_ids[sl], sup_probs[sl])], state_e, bank.temperature)
        inputs1 = oracle.mix_state(post[None], noise[None], s1, t1)
        ref = oracle.forward(inputs1, s1, t1, pos, context, head=fold)[0]
        got = logits[sl].float().cpu()
        rel = float((got - ref.float()).abs().max() / ref.float().abs().max())
        assert rel <= LOGITS_RTOL, f"request {r}: banked two-jump logits relative error {rel}"
