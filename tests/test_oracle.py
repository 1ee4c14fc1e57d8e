"""The CPU oracle, pinned against the reference sampler's own outputs and hand-computed cases.

Golden vectors come from vinfer's ``filtered_probs`` / ``sample`` (``tests/golden/make_golden.py``).
Penalties, min-p and the inverse-CDF draw have no counterpart in the reference and are pinned
by known answers computed by hand below.
"""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.reference_port import reference_filtered_probs, reference_sample
from oracle.sampler_oracle import (
    RowParams,
    canonical_order,
    filtered_probs,
    penalize,
    position_seed,
    process_row,
    splitmix64,
    uniform_from_seed,
)

GOLDEN = np.load(Path(__file__).parent / "golden" / "sampler_golden.npz")
NAMES = list(GOLDEN["names"])
GRID = GOLDEN["grid"]
TOY = np.array([2.0, 1.0, 0.5, 0.0, -1.0, -3.0], dtype=np.float32)


def _params(t, k, p):
    return RowParams(temperature=float(t), top_k=int(k), top_p=float(p))


@pytest.mark.parametrize("i", range(len(NAMES)), ids=NAMES)
def test_oracle_filtered_probs_match_the_reference(i):
    x = GOLDEN[f"logits_{i}"]
    ref = GOLDEN[f"fp_{i}"]
    for g, (t, k, p) in enumerate(GRID):
        res = process_row(x, _params(t, k, p))
        want, got = ref[g], res.probs
        if res.topp_margin < 1e-6:
            continue  # float32 (reference) vs float64 (oracle) cumsum may flip this cut
        if res.tie_at_topp_cut:
            # torch.sort is unstable on CPU: the reference keeps an arbitrary subset of the tie
            # group, of the same size and mass; compare sizes and the sorted values only.
            assert int((want > 0).sum()) == int((got > 0).sum())
            np.testing.assert_allclose(np.sort(want), np.sort(got), rtol=1e-5, atol=1e-7)
            continue
        np.testing.assert_array_equal(want > 0, got > 0, err_msg=f"kept set, params {t, k, p}")
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-8, err_msg=f"params {t, k, p}")


@pytest.mark.parametrize("i", range(len(NAMES)), ids=NAMES)
def test_oracle_greedy_matches_the_reference(i):
    x = GOLDEN[f"logits_{i}"]
    assert process_row(x, RowParams(temperature=0)).token == int(GOLDEN[f"greedy_{i}"][0])


@pytest.mark.parametrize("i", range(len(NAMES)), ids=NAMES)
def test_reference_port_is_bit_exact_with_the_reference(i):
    x = torch.from_numpy(GOLDEN[f"logits_{i}"])
    ref_fp = GOLDEN[f"fp_{i}"]
    for g in (0, 5, 17, 42, 79):
        t, k, p = GRID[g]
        got = reference_filtered_probs(x, float(t), int(k), float(p)).numpy()
        if (ref_fp[g] > 0).sum() == (got > 0).sum():
            np.testing.assert_allclose(np.sort(got), np.sort(ref_fp[g]), rtol=1e-6, atol=0)
    for g, seed, pos, tok in GOLDEN[f"race_{i}"]:
        t, k, p = GRID[g]
        assert reference_sample(x, _params(t, k, p), int(seed), int(pos)) == int(tok)


def test_position_seed_matches_the_reference():
    for s, p, want in GOLDEN["position_seed"]:
        assert position_seed(int(s), int(p)) == int(want)


# ---- known answers for the extensions --------------------------------------------------------


def test_penalties_known_answer():
    x = np.array([2.0, -2.0, 0.0, 1.5, 3.0], dtype=np.float32)
    ids = np.array([0, 1, 2, 4])
    counts = np.array([3, 1, 2, 0])  # a zero count is ignored
    y = penalize(x, ids, counts, repetition=2.0, presence=0.5, frequency=0.25)
    # 2/2 - 0.75 - 0.5 ; -2*2 - 0.25 - 0.5 ; 0*2 - 0.5 - 0.5 ; untouched ; untouched
    np.testing.assert_array_equal(y, np.array([-0.25, -4.75, -1.0, 1.5, 3.0], dtype=np.float32))
    # defaults change nothing, bit for bit
    np.testing.assert_array_equal(penalize(x, ids, counts, 1.0, 0.0, 0.0), x)


def test_penalties_change_the_greedy_token():
    x = np.array([1.0, 3.0, 2.9], dtype=np.float32)
    assert process_row(x, RowParams(temperature=0)).token == 1
    res = process_row(x, RowParams(temperature=0, repetition_penalty=1.1), 0.0,
                      np.array([1]), np.array([1]))
    assert res.token == 2  # 3/1.1 = 2.727 < 2.9


def test_min_p_known_answer():
    x = np.log(np.array([0.5, 0.3, 0.15, 0.05], dtype=np.float64)).astype(np.float32)
    res = process_row(x, RowParams(min_p=0.2), 0.0)
    # p >= 0.2 * 0.5 keeps 0.5, 0.3, 0.15; renormalised over 0.95
    np.testing.assert_allclose(res.probs, [0.5 / 0.95, 0.3 / 0.95, 0.15 / 0.95, 0.0], rtol=1e-6)
    assert res.kept == 3


def test_inverse_cdf_draw_known_answer():
    x = np.log(np.array([0.1, 0.6, 0.3], dtype=np.float64)).astype(np.float32)
    # canonical order: id 1 (0.6), id 2 (0.3), id 0 (0.1); edges 0.6, 0.9
    for u, tok in ((0.0, 1), (0.59, 1), (0.61, 2), (0.89, 2), (0.91, 0), (0.999999, 0)):
        assert process_row(x, RowParams(), u).token == tok, u
    assert process_row(x, RowParams(), 0.6000001).draw_margin < 1e-6


def test_canonical_order_breaks_ties_by_id_and_folds_signed_zero():
    v = np.array([1.0, 3.0, 1.0, -0.0, 0.0, 3.0], dtype=np.float32)
    assert canonical_order(v).tolist() == [1, 5, 0, 2, 3, 4]


def test_topk_keeps_every_tie_at_the_kth_value():
    x = np.array([5.0, 5.0, 5.0, 1.0, 0.0], dtype=np.float32)
    res = process_row(x, RowParams(top_k=1), 0.7)
    assert res.kept == 3 and res.token == 2  # thirds: edges 1/3, 2/3


def test_topp_cut_in_a_tie_group_keeps_lowest_ids():
    x = np.zeros(10, dtype=np.float32)
    res = process_row(x, RowParams(top_p=0.35), 0.5)
    # mass before token j is j/10: kept while j/10 < 0.35 -> ids 0..3
    assert res.kept == 4 and (res.probs > 0).tolist() == [True] * 4 + [False] * 6
    assert res.tie_at_topp_cut and res.token == 2


def test_uniform_from_seed_is_a_24_bit_grid_in_unit_interval():
    assert splitmix64(0) == 0xE220A8397B1DCDAF  # the published first SplitMix64 output
    for s in range(200):
        u = float(uniform_from_seed(position_seed(s, s * 3)))
        assert 0.0 <= u < 1.0 and math.isclose(u * 2**24, round(u * 2**24))


@pytest.mark.parametrize("params", [RowParams(), RowParams(temperature=0.5), RowParams(top_k=3),
                                    RowParams(top_p=0.8), RowParams(min_p=0.1)])
def test_inverse_cdf_frequencies_match_the_filtered_distribution(params):
    # the reference's own distribution test (test_sampler.py:24-38), with a uniform grid of u
    n = 20000
    counts = np.zeros(len(TOY))
    for j in range(n):
        counts[process_row(TOY, params, (j + 0.5) / n).token] += 1
    tv = 0.5 * np.abs(counts / n - filtered_probs(TOY, params)).sum()
    assert tv < 0.015
