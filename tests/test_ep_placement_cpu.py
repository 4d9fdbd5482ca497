"""Expert placement: skew model figures, equal-size placements that cut the busiest rank's expected
load on a skewed routing profile, JSON round trip and validation."""
import numpy as np
import pytest

from r9700_stack_b200.parallel import ep_placement as P


def _zipf(E, s=1.2, seed=0):
    rng = np.random.default_rng(seed)
    p = 1.0 / np.arange(1, E + 1) ** s
    rng.shuffle(p)
    return p / p.sum()


def test_profile_and_skew():
    ids = np.array([[0, 1], [0, 2], [0, 1], [3, -1]])
    p = P.profile(ids, 4)
    assert np.allclose(p, [3 / 7, 2 / 7, 1 / 7, 1 / 7])
    s = P.skew(p, [[0, 1], [2, 3]], tokens=1, k=2)
    assert s["imbalance"] > 1.0 and len(s["touched_per_rank"]) == 2
    uni = P.skew(np.full(8, 1 / 8), P.contiguous(8, 4), tokens=4, k=2)
    assert abs(uni["imbalance"] - 1.0) < 1e-9


@pytest.mark.parametrize("E,R", [(64, 4), (288, 8), (256, 2)])
def test_place_beats_contiguous_on_skew(E, R):
    p = np.sort(_zipf(E))[::-1].copy()  # hottest experts first: the worst case for contiguous ranges
    base = P.skew(p, P.contiguous(E, R), tokens=16, k=8)
    pl = P.place(p, R, tokens=16, k=8)
    P.validate(pl, E)
    got = P.skew(p, pl, tokens=16, k=8)
    assert got["imbalance"] < base["imbalance"]
    assert got["imbalance"] < 1.05, got["imbalance"]


def test_json_roundtrip(tmp_path):
    pl = P.place(_zipf(32), 4)
    f = tmp_path / "placement.json"
    P.save(str(f), pl)
    assert P.load(str(f)) == pl
    with pytest.raises(ValueError):
        P.validate([[0, 1], [1, 2]], 4)
    with pytest.raises(ValueError):
        P.validate([[0, 1, 2], [3]], 4)
