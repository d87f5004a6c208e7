"""Replica choice for expert parallelism (gyro_moe.balance): loads add up, replication evens out
a Zipf-skewed expert popularity, and nothing is replicated when the load is already even."""
import numpy as np

from gyro_moe import balance


def test_rank_loads_add_up_and_spread_replicas():
    counts = np.array([10, 0, 0, 0, 5, 5, 0, 0], np.float64)
    assert balance.rank_loads(counts, 2).tolist() == [10, 10]
    assert balance.rank_loads(counts, 2, [0]).tolist() == [5, 15]
    assert balance.rank_loads(counts, 4, [0]).sum() == counts.sum()


def test_zipf_popularity_is_evened_out():
    rng = np.random.default_rng(3)
    p = (rng.permutation(256) + 1.0) ** -1.1
    counts = np.round(p / p.sum() * 32768)
    for world in (2, 4, 8):
        before = balance.rank_loads(counts, world).max() / (counts.sum() / world)
        rep = balance.choose_replicas(counts, world)
        after = balance.rank_loads(counts, world, rep).max() / (counts.sum() / world)
        assert after <= max(1.1, before) and len(rep) <= 32 and len(set(rep)) == len(rep)
        if before > 1.3:
            assert after < before


def test_even_load_needs_no_replicas():
    assert balance.choose_replicas(np.ones(64), 8) == []
    assert balance.choose_replicas(np.ones(64), 1) == []
