"""The partial-attention bound can fail: mistakes planted in a CPU restatement
of the attention (never in a GPU kernel) violate it on the peaked GPU cases,
while the exact result rounded to the output type stays inside it.

Runs on the CPU over the q heads of the first KV head of each case, and on the
20K case over the rows that the mistakes touch: its first 256 selected rows
and every row of a split tile (the bound is element by element, so a
violation there is a violation of the whole case)."""
import numpy as np
import pytest

import attn_check as ac

MISTAKES = ["causal_plus_one", "causal_minus_one", "drop_split_chunk", "merge_without_max"]
PEAKED = ["mistral7k_peaked", "g8_peaked", "long_split_peaked"]


def _rows(case, pos):
    """All rows of the smaller cases; for the 20K case the first 256 selected
    rows (short causal prefixes) and every row of a split tile of KV head 0."""
    n_sel = case[2]
    if n_sel <= 1000:
        return np.arange(n_sel)
    row_tile, tile_pair, cuts = ac.plan(pos.numpy(), n_sel, case[3] // case[4], case[4])
    split = np.array([bool(cuts[(0, tile_pair[t])]) for t in row_tile])
    return np.union1d(np.arange(256), np.nonzero(split)[0])


@pytest.fixture(scope="module", params=PEAKED)
def case_data(request):
    case = ac.CASE[request.param]
    q, k, v, pos = ac.make_inputs(case)
    G = case[3] // case[4]
    heads = list(range(G))
    rows = _rows(case, pos)
    exp, absm = ac.oracle(case, q, k, v, pos, heads=heads, rows=rows)
    cols = np.concatenate([np.arange(h * case[5], (h + 1) * case[5]) for h in heads])
    return case, (q, k, v, pos), heads, cols, exp, absm, rows


def test_rounded_exact_result_is_inside(case_data):
    case, _, _, cols, exp, absm, _ = case_data
    n_bad, worst = ac.violations(ac.round_to(exp, case[6]), exp, absm, case[6], cols)
    assert n_bad == 0 and worst < ac.TOL[case[6]] / 2, worst


@pytest.mark.parametrize("mistake", MISTAKES)
def test_planted_mistake_is_caught(case_data, mistake):
    case, inputs, heads, cols, exp, absm, rows = case_data
    _, _, cuts = ac.plan(inputs[3].numpy(), case[2], case[3] // case[4], case[4])
    if mistake in ("drop_split_chunk", "merge_without_max"):
        assert any(cuts[(0, p)] for (h, p) in cuts if h == 0), "the case must have split tiles"
    bad = ac.round_to(ac.planted(case, *inputs, mistake, heads, rows=rows), case[6])
    n_bad, worst = ac.violations(bad, exp, absm, case[6], cols)
    assert n_bad > 0 and worst > 4 * ac.TOL[case[6]], (mistake, n_bad, worst)


def test_in_place_masking_stays_inside(case_data):
    """The kernel masks diagonal key tiles in place (scores -inf, then the
    full-tile code): masked keys may keep a weight of 2^-126 and a split piece
    in which a row sees no key merges with weight 0.  Restated on the CPU with
    every masked key at 2^-126, the rounded result stays as far inside the
    bound as the exact result does."""
    case, inputs, heads, cols, exp, absm, rows = case_data
    got = ac.round_to(ac.in_place_masked(case, *inputs, heads, rows=rows), case[6])
    n_bad, worst = ac.violations(got, exp, absm, case[6], cols)
    _, worst_exact = ac.violations(ac.round_to(exp, case[6]), exp, absm, case[6], cols)
    assert n_bad == 0 and worst <= worst_exact * (1 + 1e-6) + 1e-12, (worst, worst_exact)
