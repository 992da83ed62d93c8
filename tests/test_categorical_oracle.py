"""CPU properties of the oracle's categorical draws (oracle/accept_oracle.c):
``categorical`` (the draft-sampling draw, :553-557 of modeling_flashmap.py
draws by torch.multinomial) and ``categorical_sliced`` (the rejection step's
bonus draw, :594), both inverse-CDF draws over unnormalised non-negative
weights with a fixed summation order, as the CUDA kernels compute them.

With integer weights every partial sum is exact in fp32, so both draws must
equal the exact inverse CDF ``first v with cumsum(w)[v] > u * total``; with
general weights they must stay monotone in u, never pick a zero weight, and
match the weights' frequencies."""

import numpy as np
import pytest

from oracle import accept as A

SLICE = 256 * 32


def exact_inverse_cdf(w: np.ndarray, u: float) -> int:
    c = np.cumsum(w.astype(np.float64))
    target = np.float32(u) * np.float32(c[-1])  # u * total rounded as the draw rounds it
    idx = int(np.searchsorted(c, float(target), side="right"))
    return min(idx, len(w) - 1)


@pytest.mark.parametrize("V", [1, 31, 4099, SLICE, 2 * SLICE + 77, 19 * SLICE - 5])
def test_integer_weights_equal_exact_inverse_cdf(V):
    rng = np.random.default_rng(V)
    w = rng.integers(0, 4, V).astype(np.float32)
    w[rng.integers(0, V)] = 1.0  # at least one positive weight
    for u in list(rng.random(40)) + [0.0, 0.999999]:
        u = float(np.float32(u))
        want = exact_inverse_cdf(w, u)
        assert A.categorical(w, u) == want, (V, u)
        assert A.categorical_sliced(w, u) == want, (V, u)


@pytest.mark.parametrize("V", [5, 3000, 3 * SLICE + 1])
def test_single_positive_weight_is_always_drawn(V):
    rng = np.random.default_rng(V + 1)
    for k in (0, V // 2, V - 1):
        w = np.zeros(V, dtype=np.float32)
        w[k] = 0.37
        for u in (0.0, 0.5, float(np.float32(0.9999999))):
            assert A.categorical(w, u) == k
            assert A.categorical_sliced(w, u) == k


def test_all_zero_weights_give_index_zero():
    for V in (7, SLICE + 3):
        w = np.zeros(V, dtype=np.float32)
        assert A.categorical_sliced(w, 0.3) == 0


@pytest.mark.parametrize("sliced", [False, True])
def test_monotone_in_u_and_never_a_zero_weight(sliced):
    rng = np.random.default_rng(7)
    V = 2 * SLICE + 513
    w = (rng.random(V) * (rng.random(V) < 0.3)).astype(np.float32)
    draw = A.categorical_sliced if sliced else A.categorical
    us = np.sort(rng.random(300).astype(np.float32))
    picks = [draw(w, float(u)) for u in us]
    assert all(a <= b for a, b in zip(picks, picks[1:]))
    assert all(w[p] > 0 for p in picks)


@pytest.mark.parametrize("sliced", [False, True])
def test_frequencies_follow_the_weights(sliced):
    rng = np.random.default_rng(11)
    V = SLICE + 1000
    w = np.zeros(V, dtype=np.float32)
    hot = rng.choice(V, 8, replace=False)
    w[hot] = rng.random(8).astype(np.float32) + 0.1
    draw = A.categorical_sliced if sliced else A.categorical
    n = 4000
    counts = {int(k): 0 for k in hot}
    for u in rng.random(n).astype(np.float32):
        counts[draw(w, float(u))] += 1
    p = w[hot] / w[hot].sum()
    for k, pk in zip(hot, p):
        # binomial standard deviation at n = 4000 is at most 0.8%; allow 5 sigma
        assert abs(counts[int(k)] / n - pk) < 5 * np.sqrt(pk * (1 - pk) / n) + 1e-3
