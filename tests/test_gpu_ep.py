"""Expert parallelism on 2 GPUs through the C ABI: two processes, one context each (world 2),
experts sharded 50/50, rows exchanged over NVLink peer memory (and, for the layer cases, over
NCCL as well). Every rank's output must match the CPU oracle
of the whole layer (src/engine.zig:520-642) on its own tokens, within the tolerance of the
tensor-core path (its f16 operands). Cases:

- a small layer;
- Zipf routing with a rank that has no tokens;
- the config-0 layer shape with ragged per-expert segments;
- a two-layer pre-norm stack on bf16 tokens;
- device-pointer calls twice in a row;
- the no-alloc decode entry, which the expert-parallel context must refuse;
- replicated experts;
- the exchange in use (peer memory on distinct GPUs, NCCL when asked for)."""
import numpy as np
import pytest

from oracle import oracle
from gyro_moe import metrics

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
REL_RMS, COSINE = 1e-2, 0.9999          # north-star layer tolerance
PREFILL_TIGHT = 5e-3                    # f16 operands of the tensor-core path


def check(ref, got, tight=PREFILL_TIGHT):
    if ref.size == 0:
        assert got.size == 0
        return
    m = metrics.compare(ref, got)
    assert m["rel_rms"] <= REL_RMS and m["cosine"] >= COSINE and m["rel_rms"] <= tight, m


@pytest.fixture(scope="module")
def ranks(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import ep_gpu_worker
    out = tmp_path_factory.mktemp("ep2")
    mp.spawn(ep_gpu_worker.worker, args=(2, str(out)), nprocs=2, join=True)
    return [dict(np.load(out / f"rank{r}.npz")) for r in range(2)]


def test_group_caps(ranks):
    for r, res in enumerate(ranks):
        assert res["caps_world"].tolist() == [r, 2]


def test_exchange_kind(ranks):
    from gyro_moe import abi
    import ep_gpu_worker
    for res in ranks:
        assert int(res["exchange"]) == abi.GX_EP_PEER
        assert int(res["nccl_exchange0"]) == abi.GX_EP_NONE
        assert int(res["nccl_exchange"]) == abi.GX_EP_NCCL
        # every layer case took the peer exchange, the config-0 shape included although a
        # narrower layer set the exchange up first
        assert [int(res[f"{c[0]}_peer_layers"]) for c in ep_gpu_worker.CASES] == \
            list(range(1, len(ep_gpu_worker.CASES) + 1))


@pytest.fixture(scope="module")
def fault(tmp_path_factory):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import ep_gpu_worker
    out = tmp_path_factory.mktemp("ep2fault")
    mp.spawn(ep_gpu_worker.fault_worker, args=(2, str(out)), nprocs=2, join=True)
    return [dict(np.load(out / f"fault{r}.npz")) for r in range(2)]


def test_missing_rows_end_in_an_error_on_every_rank(fault):
    """One rank skips its push: the peer's bounded device-side wait expires, the failure is passed
    on through the return flags, both ranks report GX_E_KERNEL within seconds (not a result with
    rows missing), later calls are refused, and both contexts close."""
    from gyro_moe import abi
    for res in fault:
        assert int(res["exchange"]) == abi.GX_EP_PEER
        assert int(res["first_rc"]) == -9
        assert float(res["first_s"]) < 10.0
        assert int(res["second_rc"]) == -4
        assert int(res["destroy_rc"]) == 0


@pytest.mark.parametrize("exchange", ["", "nccl_"])
@pytest.mark.parametrize("case", [c[0] for c in __import__("ep_gpu_worker").CASES])
def test_layer_matches_oracle_on_every_rank(ranks, case, exchange):
    import ep_gpu_worker
    kw = dict(next(c for c in ep_gpu_worker.CASES if c[0] == case)[1])
    layer = ep_gpu_worker.make(kw)
    for res in ranks:
        x, y, ids = res[f"{case}_x"], res[f"{exchange}{case}_y"], res[f"{exchange}{case}_ids"]
        if x.shape[0] == 0:
            assert y.shape[0] == 0
            continue
        want, wids, _ = oracle.moe_ffn(layer, x)
        assert metrics.topk_sets(wids, ids)["flips"] == 0
        check(want, y)


def test_stack_matches_oracle_on_every_rank(ranks):
    import ep_gpu_worker
    layers = [ep_gpu_worker.make(dict(seed=41 + l, n_expert=16, E=256, F=128, U=4)) for l in range(2)]
    for res in ranks:
        x = (res["stack_x"].astype(np.uint32) << 16).view(np.float32)
        check(oracle.stack(layers, x), res["stack_y"])


def test_device_calls_twice_and_noalloc_refused(ranks):
    import ep_gpu_worker
    layer = ep_gpu_worker.make(dict(seed=42, n_expert=16, E=256, F=128, U=4))
    for res in ranks:
        for rep in range(2):
            x, y = res[f"dev{rep}_x"], res[f"dev{rep}_y"]
            if x.shape[0]:
                check(oracle.moe_ffn(layer, x)[0], y)
        assert int(res["noalloc_rc"]) == -5


def test_replicated_experts_keep_outputs_and_counts(ranks):
    import ep_gpu_worker
    layer = ep_gpu_worker.make(ep_gpu_worker.REPLICATION_LAYER)
    for res in ranks:
        x = res["rep_x"]
        want, wids, _ = oracle.moe_ffn(layer, x)
        check(want, res["rep_y0"])
        check(want, res["rep_y1"])
        assert metrics.topk_sets(wids, res["rep_ids1"])["flips"] == 0
        # counts are this rank's routed slots per global expert, before and after replication
        assert res["rep_counts0"].sum() == x.shape[0] * layer["n_used"]
        np.testing.assert_array_equal(res["rep_counts1"], np.bincount(wids.ravel(), minlength=32))
        assert int(res["rep_dup_rc"]) == -1
