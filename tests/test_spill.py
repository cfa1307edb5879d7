"""Host logic of the expert spill: splitting a long call into token runs
whose distinct experts fit in the HBM slots (kandiga_b200.spill.token_runs)."""
import numpy as np
import pytest

from kandiga_b200.spill import token_runs


def check_runs(idx, E, S, runs):
    assert runs[0][0] == 0 and runs[-1][1] == idx.shape[0]
    for (a, b), (c, _) in zip(runs, runs[1:]):
        assert b == c and a < b
    for i, (a, b) in enumerate(runs):
        used = {int(e) for e in idx[a:b].ravel() if 0 <= e < E}
        assert len(used) <= S
        if i + 1 < len(runs):  # greedy: the next token would not have fitted
            more = used | {int(e) for e in idx[b] if 0 <= e < E}
            assert len(more) > S


@pytest.mark.parametrize("E,S,K,T", [(32, 8, 8, 20), (64, 20, 8, 200), (256, 64, 8, 512), (16, 16, 4, 50)])
def test_token_runs_cover_and_fit(E, S, K, T):
    rng = np.random.RandomState(E + S)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    runs = token_runs(idx, E, S)
    check_runs(idx, E, S, runs)
    if S >= E:
        assert runs == [(0, T)]


def test_token_runs_edges():
    assert token_runs(np.zeros((0, 8), np.int32), 16, 8) == [(0, 0)]
    idx = np.array([[1, 2, -1, 99], [1, 2, 3, 3]], np.int32)  # invalid ids take no slot
    assert token_runs(idx, 16, 3) == [(0, 2)]
    with pytest.raises(ValueError):
        token_runs(np.array([[0, 1, 2, 3]], np.int32), 16, 3)
