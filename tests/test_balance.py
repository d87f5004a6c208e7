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


def test_bench_sequence_placement_covers_the_batch_evenly():
    # bench.rank_sequences: every sequence on exactly one rank, in batch order within a rank, and
    # the busiest rank within one sequence of an even share (longest-first greedy placement)
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    import bench
    lengths, offsets, _ = bench.ep_batch()
    for world in (1, 2, 4, 8):
        seqs = bench.rank_sequences(lengths, world)
        flat = sorted(i for q in seqs for i in q)
        assert flat == list(range(len(lengths)))
        assert all(q == sorted(q) for q in seqs)
        loads = [int(sum(lengths[i] for i in q)) for q in seqs]
        assert max(loads) <= lengths.sum() / world + lengths.max()
        assert sum(bench.rank_tokens(offsets, np.zeros((offsets[-1], 1), np.uint16), r, world).shape[0]
                   for r in range(world)) == offsets[-1]
