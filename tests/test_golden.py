"""The oracle against the committed golden fixtures (tests/golden/, written by
tests/golden/make_golden.py from the cases of golden_cases.py): the seeded
inputs hash to the recorded digests, and the oracle reproduces every stored
array and every digested output bit for bit."""
import numpy as np
import pytest

import golden_cases
from helpers import digest, golden, golden_digests


def same_bits(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.dtype == b.dtype and a.shape == b.shape and a.tobytes() == b.tobytes()


@pytest.mark.parametrize("case", golden_cases.CASES)
def test_oracle_reproduces_golden_fixture(case):
    inputs, arrays, outs = getattr(golden_cases, case)()
    recorded = golden_digests()
    keys = {k for k in recorded if k.startswith(case + "/")}
    assert keys == ({f"{case}/input/{k}" for k in inputs} | {f"{case}/{k}" for k in outs})
    # inputs first: a mismatch here means numpy's seeded streams changed, not the oracle
    for k, a in inputs.items():
        assert digest(a) == recorded[f"{case}/input/{k}"], f"seeded input {k} changed"
    stored = golden(case)
    assert set(stored) == set(arrays)
    for k, a in arrays.items():
        assert same_bits(a, stored[k]), k
    for k, a in outs.items():
        assert digest(a) == recorded[f"{case}/{k}"], k


def test_fixture_invariants():
    """Properties of the stored vectors themselves: the router's top-8 are
    distinct, in range, in descending logit order, with weights summing to the
    renormalised per-expert scales; the schedule is a stable histogram of the
    local routes; the scalar grids sit inside the reference's error bounds."""
    st, fw = golden("moe_stages"), golden("moe_forward")
    for idx, w, lg in ((st["router_idx"], st["router_w"], st["router_logits"]),
                       (fw["idx"], fw["w"], fw["logits"])):
        assert ((idx >= 0) & (idx < golden_cases.E)).all()
        assert all(len(set(r)) == 8 for r in idx.tolist())
        sel = np.take_along_axis(lg, idx, axis=1)
        assert (np.diff(sel, axis=1) <= 0).all()
        assert (w > 0).all()
    off = st["sched_offset"]
    sidx, _ = golden_cases.skewed_routes(golden_cases.SCHED_T, golden_cases.SCHED_BASE)
    local = sidx - golden_cases.SCHED_BASE
    local = local[(local >= 0) & (local < golden_cases.SCHED_EPR)]
    assert np.array_equal(np.diff(off), np.bincount(local, minlength=golden_cases.SCHED_EPR))
    for e in range(golden_cases.SCHED_EPR):
        tok = st["sched_token"][off[e]:off[e + 1]]
        assert (np.diff(tok) > 0).all()      # token-major, one route per token per expert
    sm = golden("scalar_math")
    x = sm["softmax_exp_x"].astype(np.float64)
    rel = sm["softmax_exp"] / np.exp(x) - 1
    ok = x >= -86        # below, the exponent field underflows (results < 1e-37)
    assert rel[ok].max() <= 1e-6 and rel[ok].min() > -7.5e-3
    g = sm["gelu_x"].astype(np.float64)
    exact = 0.5 * g * (1 + np.tanh(np.sqrt(2 / np.pi) * (g + 0.044715 * g ** 3)))
    assert np.abs(sm["gelu"] - exact).max() < 1e-2


@pytest.mark.parametrize("case", ["moe_stages", "moe_forward", "dense_mlp"])
def test_oracle_bits_independent_of_thread_count(case):
    """The fixtures hold on any host: the oracle's OpenMP loops split work
    over tokens, rows or experts, never inside one sum, so 1 and 3 threads
    give the bits of the default thread count."""
    from oracle import oracle as O
    L = O.lib()
    n = L.orc_num_threads()
    stored = golden(case)
    try:
        for threads in (1, 3):
            L.orc_set_num_threads(threads)
            _, arrays, _ = getattr(golden_cases, case)()
            for k, a in arrays.items():
                assert same_bits(a, stored[k]), (threads, k)
    finally:
        L.orc_set_num_threads(n)
