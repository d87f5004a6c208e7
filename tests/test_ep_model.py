"""Expert parallelism on the CPU: two gloo ranks run the exchange of the expert-parallel layer
(dispatch plan, count exchange, row dispatch, expert phase on the local shard, partial-row
return, source sum) with the oracle in place of the kernels, and must reproduce the
single-device layer (src/engine.zig:520-642). Also: ranks without tokens, all traffic to one
rank, and a rank that leaves before the exchange (the other must fail, not hang)."""
import os
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

import ep_model  # noqa: E402


def run(tmp_path, case, world=2):
    store = tmp_path / "store"
    mp.spawn(ep_model.worker, args=(world, str(store), case, str(tmp_path)), nprocs=world, join=True)
    return [dict(np.load(tmp_path / f"rank{r}.npz")) if (tmp_path / f"rank{r}.npz").exists() else None
            for r in range(world)]


BASE = {"seed": 5, "NE": 16, "E": 256, "F": 128, "U": 4}


def check(res):
    for r in res:
        assert r is not None and "error" not in r, r
        np.testing.assert_allclose(r["out"], r["want"], rtol=2e-5, atol=2e-6)


def test_plan_layout_matches_the_kernel_contract():
    ids = np.array([[0, 9], [8, 15], [1, 2], [9, 3]])
    w = np.array([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5], [0.9, 0.1]], np.float32)
    pos_of, sends = ep_model.plan(ids, w, 16, 2)
    assert pos_of.tolist() == [[0, 0], [-1, 1], [1, -1], [2, 2]]
    toks, loc, wt = sends[1]
    assert toks.tolist() == [0, 1, 3]
    assert loc.tolist() == [[ep_model.NO_SLOT, 1], [0, 7], [1, ep_model.NO_SLOT]]
    np.testing.assert_allclose(wt, [[0.0, 0.4], [0.7, 0.3], [0.9, 0.0]], rtol=1e-6)


def test_two_ranks_match_the_single_device_layer(tmp_path):
    check(run(tmp_path, dict(BASE, n_tok=[7, 5])))


def test_zipf_routing_and_a_rank_without_tokens(tmp_path):
    check(run(tmp_path, dict(BASE, seed=8, zipf=1.1, n_tok=[9, 0])))


def test_all_traffic_to_one_rank(tmp_path):
    check(run(tmp_path, dict(BASE, seed=9, n_tok=[4, 6], only_rank=1)))


def test_replicated_hot_experts_are_served_where_the_token_is(tmp_path):
    # experts 1 and 9 (one from each shard) served locally on every rank: same layer output
    check(run(tmp_path, dict(BASE, seed=12, zipf=1.1, n_tok=[8, 6], replicas=(9, 1))))


def test_route_table_of_replicas():
    r = ep_model.route_table(16, 2, 1, replicas=(9, 1))
    assert r[9].tolist() == [-1, 1] and r[1].tolist() == [-1, 8 + 1] and r[0].tolist() == [0, 0]
    ids = np.array([[1, 2], [9, 12]])
    pos_of, sends = ep_model.plan(ids, np.ones((2, 2), np.float32), 16, 2, rank=1, replicas=(9, 1))
    assert sends[0][0].tolist() == [0] and sends[1][0].tolist() == [0, 1]
    assert sends[1][1].tolist() == [[9, ep_model.NO_SLOT], [1, 4]]


def test_rank_that_never_joins_ends_the_exchange_with_an_error(tmp_path):
    t0 = time.time()
    res = run(tmp_path, dict(BASE, seed=10, n_tok=[3, 3], leave_rank=1, timeout=5.0))
    assert res[1] is None
    assert res[0] is not None and "error" in res[0]
    assert time.time() - t0 < 120
