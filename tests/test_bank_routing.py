"""The built-in bank of per-expert count tables (`harness/routing.py` `BANK`): every scenario is
realised exactly as a top-k table (histogram equal to the counts, distinct experts per token, no
count above the token count), deterministically per (rank, seed), and the placements permute it."""
import numpy as np
import pytest

from deepep_slingshot_b200.harness import routing as R


@pytest.mark.parametrize('name', R.BANK)
@pytest.mark.parametrize('rank', [0, 3])
def test_bank_scenario_is_exact(name, rank):
    N, E, K, ranks = 300, 64, 6, 4
    counts = R.bank_counts(name, rank, ranks, N, E, K, seed=2)
    assert counts.sum() == N * K and counts.max() <= N and counts.min() >= 0
    idx = R.make_routing(f'bank:{name}', rank, ranks, N, E, K, seed=2).numpy()
    assert idx.shape == (N, K)
    assert (np.bincount(idx[idx >= 0], minlength=E) == counts).all()
    assert all(len(set(row.tolist())) == K for row in idx)
    again = R.make_routing(f'bank:{name}', rank, ranks, N, E, K, seed=2).numpy()
    assert (idx == again).all()


def test_bank_shapes():
    N, E, K = 256, 32, 4
    hot = R.bank_counts('hot8', 0, 2, N, E, K, 0)
    assert np.sort(hot)[-8:].sum() >= N * K // 2 - 8
    dead = R.bank_counts('dead', 1, 2, N, E, K, 0)
    assert (dead == 0).sum() == E // 4
    assert (dead == 0).tolist() == (R.bank_counts('dead', 0, 2, N, E, K, 0) == 0).tolist()  # shared dead set
    sat = R.bank_counts('saturated', 0, 2, N, E, K, 0)
    assert (sat == N).sum() == K - 1
    d0, d1 = R.bank_counts('drift', 0, 2, N, E, K, 0), R.bank_counts('drift', 1, 2, N, E, K, 0)
    assert np.argmax(d0) != np.argmax(d1) or not (d0 == d1).all()


def test_bank_greedy_placement_keeps_histogram_up_to_permutation():
    N, E, K, ranks = 200, 32, 4, 4
    plain = R.make_routing('bank:drift', 1, ranks, N, E, K, seed=1).numpy()
    placed = R.make_routing('bank:drift:greedy', 1, ranks, N, E, K, seed=1).numpy()
    assert sorted(np.bincount(plain.ravel(), minlength=E)) == sorted(np.bincount(placed.ravel(), minlength=E))


def test_unknown_bank_scenario():
    with pytest.raises(ValueError):
        R.bank_counts('nope', 0, 2, 8, 8, 2, 0)
