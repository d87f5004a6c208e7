"""One rank of the 2-GPU expert-parallel parity test (tests/test_gpu_ep.py).

Every rank makes the same C-ABI calls, in the same order, for every case. All collective work
is done before any comparison, so that a failed check on one rank cannot leave the other
waiting in an exchange. Results go to <out>/rank<r>.npz for the parent to check against the
oracle.
"""
from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "gyro-dx_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

CASES = [
    # name, layer kwargs, tokens per rank
    ("small", dict(seed=31, n_expert=16, E=256, F=128, U=4), [37, 21]),
    ("zipf_empty_rank", dict(seed=32, n_expert=32, E=256, F=256, U=4, zipf=1.1), [70, 0]),
    ("config0_shape", dict(seed=33, zipf=1.1), [300, 180]),
    # a Q8_0 shared expert: every rank computes it for its own tokens, beside the exchanged rows
    ("shared_expert", dict(seed=35, n_expert=32, E=256, F=256, U=4, shared=256), [45, 20]),
]


REPLICATION_LAYER = dict(seed=34, n_expert=32, E=256, F=256, U=4, zipf=1.1)
REPLICAS = [3, 20, 9]


def make(kw):
    from gyro_moe import synth
    kw = dict(kw)
    seed = kw.pop("seed")
    sf = kw.pop("shared", None)
    layer = synth.make_layer(seed, **kw)
    if sf:
        layer["shared"] = synth.make_shared(seed + 500, E=layer["n_embd"], SF=sf, type_id=8)
    return layer


def tokens(case_i, rank, n, E):
    from gyro_moe import synth
    return synth.tokens(9000 + 10 * case_i + rank, max(n, 1), E=E)[:n]


def worker(rank: int, world: int, out_dir: str) -> None:
    os.environ.setdefault("GX_COMM_TIMEOUT_MS", "30000")
    import torch
    torch.cuda.set_device(rank)
    from gyro_moe import abi

    def shared_id(name: str) -> bytes:
        """A fresh NCCL id from rank 0 (one per communicator), passed through a file."""
        idf = Path(out_dir) / name
        if rank == 0:
            tmp = idf.with_suffix(".tmp")
            tmp.write_bytes(abi.unique_id())
            tmp.rename(idf)
        t0 = time.time()
        while not idf.exists():
            if time.time() - t0 > 60:
                raise RuntimeError("no NCCL id from rank 0")
            time.sleep(0.05)
        return idf.read_bytes()

    nccl_id = shared_id("nccl_id")
    res = {}
    max_tok = max(max(n) for _, _, n in CASES)
    with abi.Context(device=rank, max_tokens=max_tok, max_layers=2, rank=rank, world=world, nccl_id=nccl_id) as ctx:
        caps = ctx.caps()
        res["caps_world"] = np.array([caps.rank, caps.world])
        for i, (name, kw, n_tok) in enumerate(CASES):
            layer = make(kw)
            ctx.upload_layer(0, layer)
            x = tokens(i, rank, n_tok[rank], layer["n_embd"])
            y, ids, w = ctx.forward_host(0, x, want_routing=True)
            res[f"{name}_x"], res[f"{name}_y"], res[f"{name}_ids"] = x, y, ids
            # which exchange this call took: the count of peer-memory layer calls so far
            res[f"{name}_peer_layers"] = np.array(ctx.caps().ep_peer_layers)
        # a two-layer pre-norm stack, bf16 tokens in
        layers = [make(dict(seed=41 + l, n_expert=16, E=256, F=128, U=4)) for l in range(2)]
        for l, layer in enumerate(layers):
            ctx.upload_layer(l, layer)
        xs = tokens(7, rank, [50, 30][rank], 256)
        xb = (xs.view(np.uint32) >> 16).astype(np.uint16)
        res["stack_x"] = xb
        res["stack_y"] = ctx.stack_forward_host(0, 2, xb)
        # device pointers, one rank without tokens, twice in a row (buffers reused)
        dev = torch.device("cuda", rank)
        for rep in range(2):
            n = [12, 0][rank]
            xt = torch.from_numpy(tokens(8 + rep, rank, n, 256)).to(dev)
            yt = torch.empty_like(xt)
            ctx.wait(ctx.forward(1, xt, yt))
            res[f"dev{rep}_x"], res[f"dev{rep}_y"] = xt.cpu().numpy(), yt.cpu().numpy()
        try:
            ctx.forward_noalloc(1, xt, yt)
            res["noalloc_rc"] = np.array(0)
        except abi.GxError as e:
            res["noalloc_rc"] = np.array(e.code)
        # hot experts served where the token is: one from each shard, and a list naming one twice
        layer = make(REPLICATION_LAYER)
        ctx.upload_layer(0, layer)
        x = tokens(20, rank, [40, 24][rank], layer["n_embd"])
        res["rep_x"] = x
        res["rep_y0"] = ctx.forward_host(0, x)
        res["rep_counts0"] = ctx.expert_counts(0, reset=True)
        ctx.replicate_experts(0, REPLICAS)
        res["rep_y1"], res["rep_ids1"], _ = ctx.forward_host(0, x, want_routing=True)
        res["rep_counts1"] = ctx.expert_counts(0)
        try:
            ctx.replicate_experts(0, [3, 3])
            res["rep_dup_rc"] = np.array(0)
        except abi.GxError as e:
            res["rep_dup_rc"] = np.array(e.code)
        res["exchange"] = np.array(ctx.caps().ep_exchange)
    # the same layer cases with the rows exchanged over NCCL (read when the first layer runs)
    os.environ["GX_EP_NCCL"] = "1"
    try:
        with abi.Context(device=rank, max_tokens=max_tok, max_layers=1, rank=rank, world=world,
                         nccl_id=shared_id("nccl_id2")) as ctx:
            res["nccl_exchange0"] = np.array(ctx.caps().ep_exchange)
            for i, (name, kw, n_tok) in enumerate(CASES):
                layer = make(kw)
                ctx.upload_layer(0, layer)
                x = tokens(i, rank, n_tok[rank], layer["n_embd"])
                y, ids, w = ctx.forward_host(0, x, want_routing=True)
                res[f"nccl_{name}_y"], res[f"nccl_{name}_ids"] = y, ids
            res["nccl_exchange"] = np.array(ctx.caps().ep_exchange)
    finally:
        del os.environ["GX_EP_NCCL"]
    np.savez(Path(out_dir) / f"rank{rank}.npz", **res)


def fault_worker(rank: int, world: int, out_dir: str) -> None:
    """Failure detection without a GPU fault: rank 0 does not send its rows for its first
    peer-exchange layer call (the GX_EP_FAULT_SKIP_PUSH host hook), while staying alive with its
    exchange block mapped. Rank 1's bounded wait for those rows runs out (GX_EP_WAIT_MS), rank 1
    fails its return so rank 0 fails too, and both report GX_E_KERNEL instead of a result. The
    contexts then refuse further calls and close cleanly."""
    os.environ.setdefault("GX_COMM_TIMEOUT_MS", "30000")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["GX_EP_WAIT_MS"] = "300"
    if rank == 0:
        os.environ["GX_EP_FAULT_SKIP_PUSH"] = "1"
    import torch
    torch.cuda.set_device(rank)
    from gyro_moe import abi

    idf = Path(out_dir) / "nccl_id_fault"
    if rank == 0:
        tmp = idf.with_suffix(".tmp")
        tmp.write_bytes(abi.unique_id())
        tmp.rename(idf)
    t0 = time.time()
    while not idf.exists():
        if time.time() - t0 > 60:
            raise RuntimeError("no NCCL id from rank 0")
        time.sleep(0.05)
    res = {}
    ctx = abi.Context(device=rank, max_tokens=64, max_layers=1, rank=rank, world=world, nccl_id=idf.read_bytes())
    layer = make(dict(seed=51, n_expert=16, E=256, F=128, U=4))
    ctx.upload_layer(0, layer)
    x = tokens(50, rank, 20, 256)
    t0 = time.time()
    try:
        ctx.forward_host(0, x, timeout_ms=20000)
        res["first_rc"] = np.array(0)
    except abi.GxError as e:
        res["first_rc"] = np.array(e.code)
    res["first_s"] = np.array(time.time() - t0)
    try:
        ctx.forward_host(0, x, timeout_ms=20000)
        res["second_rc"] = np.array(0)
    except abi.GxError as e:
        res["second_rc"] = np.array(e.code)
    res["exchange"] = np.array(ctx.caps().ep_exchange)
    try:
        ctx.close()
        res["destroy_rc"] = np.array(0)
    except abi.GxError as e:
        res["destroy_rc"] = np.array(e.code)
    np.savez(Path(out_dir) / f"fault{rank}.npz", **res)
