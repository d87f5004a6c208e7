"""CPU model of the expert-parallel routed layer, run as torch.distributed (gloo) ranks.

Test infrastructure: it restates the exchange the library performs over NCCL
(gyro-dx_b200/csrc/gx_ep.cu and enqueue_layer_ep in gx_abi.cu) with the CPU oracle standing in for
the kernels. It checks the decomposition itself on the CPU:

- Each rank routes its own tokens with the replicated router.
- Replicated experts are served by the token's own rank (route table of gx_replicate_experts).
- A token goes once to every rank that serves one of its U experts. It carries its U slots
  there: destination-local expert id, or NO_SLOT for experts served elsewhere.
- The serving rank returns sum_k w_k * Expert_k(x) over its own slots.
- The source adds the returned partial rows.

The result must equal the single-device layer (src/engine.zig:520-642).
"""
from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "gyro-dx_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

NO_SLOT = 0xFFFFFFFF


def route_table(n_expert: int, world: int, rank: int, replicas=()) -> np.ndarray:
    """[n_expert][2]: (serving rank or -1 = the token's own rank, local expert index there), as
    gx_replicate_experts sets it on `rank`: shard experts at their shard index, replica i of a
    listed expert at slot per + i (or the shard index on the expert's own rank)."""
    per = n_expert // world
    route = np.stack([np.arange(n_expert) // per, np.arange(n_expert) % per], axis=1)
    for i, e in enumerate(replicas):
        route[e] = (-1, e % per if e // per == rank else per + i)
    return route


def plan(ids: np.ndarray, weights: np.ndarray, n_expert: int, world: int, rank: int = 0, replicas=()):
    """Dispatch plan, as ep_plan_kernel lays it out.

    For destination d, the send rows are the tokens with a slot served by d, in token order.
    Returns pos_of [n][world] (-1 if the token is not sent there) and, per destination, (tokens,
    local ids [rows][U], weights [rows][U])."""
    n, U = ids.shape
    route = route_table(n_expert, world, rank, replicas)
    dest = np.where(route[ids, 0] < 0, rank, route[ids, 0]) if n else np.zeros((0, U), np.int64)
    pos_of = -np.ones((n, world), np.int64)
    sends = []
    for d in range(world):
        here = dest == d
        toks = np.nonzero(here.any(axis=1))[0]
        loc = np.where(here[toks], route[ids[toks], 1], NO_SLOT).astype(np.uint32)
        w = np.where(here[toks], weights[toks], 0.0).astype(np.float32)
        pos_of[toks, d] = np.arange(len(toks))
        sends.append((toks, loc.reshape(-1, U), w.reshape(-1, U)))
    return pos_of, sends


def local_slice(layer: dict, rank: int, world: int, replicas=()) -> dict:
    """The experts rank `rank` holds: its shard (rows [r*NE/W*F, ...) of gate/up, [r*NE/W*E, ...)
    of down), then a copy of every replicated expert in list order."""
    per = layer["n_expert"] // world
    F, E = layer["n_ff"], layer["n_embd"]
    experts = list(range(rank * per, (rank + 1) * per)) + list(replicas)
    out = dict(layer)
    out["n_expert"] = len(experts)
    out["gate"] = np.concatenate([layer["gate"][e * F:(e + 1) * F] for e in experts])
    out["up"] = np.concatenate([layer["up"][e * F:(e + 1) * F] for e in experts])
    out["down"] = np.concatenate([layer["down"][e * E:(e + 1) * E] for e in experts])
    return out


def _exchange(parts: list, rank: int, world: int, dtype, width):
    """Sends parts[d] (an array [rows][width]) to rank d and returns what every source sent here."""
    import torch
    import torch.distributed as dist
    counts = torch.tensor([len(p) for p in parts], dtype=torch.int64)
    table = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(table, counts)
    got = [None] * world
    reqs = []
    for d in range(world):
        if d == rank:
            got[d] = np.asarray(parts[d]).reshape(-1, width).astype(dtype, copy=True)
            continue
        if len(parts[d]):
            reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(parts[d]).reshape(-1, width)), d))
    for s in range(world):
        if s == rank:
            continue
        n = int(table[s][rank])
        buf = torch.from_numpy(np.zeros((n, width), dtype=dtype))
        if n:
            dist.irecv(buf, s).wait()
        got[s] = buf.numpy()
    for r in reqs:
        r.wait()
    return got


def ep_layer(layer: dict, x: np.ndarray, rank: int, world: int, replicas=()) -> np.ndarray:
    """One expert-parallel layer on this rank's tokens x [n][E]; returns out [n][E]."""
    from oracle import oracle
    E, U, NE = layer["n_embd"], layer["n_used"], layer["n_expert"]
    n = x.shape[0]
    if n:
        _, ids, w = oracle.moe_ffn(layer, x)          # selection with the replicated router
    else:
        ids, w = np.zeros((0, U), np.uint32), np.zeros((0, U), np.float32)
    pos_of, sends = plan(ids.astype(np.int64), w, NE, world, rank, replicas)
    rows = _exchange([x[t] for t, _, _ in sends], rank, world, np.float32, E)
    rids = _exchange([loc.astype(np.int64) for _, loc, _ in sends], rank, world, np.int64, U)
    rw = _exchange([wt for _, _, wt in sends], rank, world, np.float32, U)
    mine = local_slice(layer, rank, world, replicas)
    R = [len(r) for r in rows]
    allrows = np.concatenate(rows) if sum(R) else np.zeros((0, E), np.float32)
    if sum(R):
        part = oracle.moe_experts(mine, allrows, np.concatenate(rids).astype(np.uint32), np.concatenate(rw))
    else:
        part = np.zeros((0, E), np.float32)
    offs = np.cumsum([0] + R)
    back = _exchange([part[offs[s]:offs[s + 1]] for s in range(world)], rank, world, np.float32, E)
    out = np.zeros((n, E), np.float32)
    for d in range(world):
        sel = pos_of[:, d] >= 0
        out[sel] += back[d][pos_of[sel, d]]
    return out


def init(rank: int, world: int, store: str, timeout_s: float = 20.0) -> None:
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"file://{store}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=timeout_s))


def worker(rank: int, world: int, store: str, case: dict, result_dir: str) -> None:
    """One rank of a test case; writes its outcome to result_dir/rank<r>.npz."""
    import torch.distributed as dist
    from gyro_moe import synth
    layer = synth.make_layer(case["seed"], n_expert=case["NE"], E=case["E"], F=case["F"], U=case["U"],
                             zipf=case.get("zipf"))
    if case.get("only_rank") is not None:       # every expert but those of one rank made unreachable
        per = case["NE"] // world
        bias = np.full(case["NE"], -np.inf, np.float32)
        r = case["only_rank"]
        bias[r * per:(r + 1) * per] = 0.0
        layer["router_bias"] = bias
    n_tok = case["n_tok"][rank]
    x = synth.tokens(case["seed"] + 100 + rank, max(n_tok, 1), E=case["E"])[:n_tok]
    init(rank, world, store, case.get("timeout", 20.0))
    try:
        if case.get("leave_rank") == rank:
            return                               # never joins the exchange
        try:
            out = ep_layer(layer, x, rank, world, case.get("replicas", ()))
        except RuntimeError as e:                # a peer that left: the collective ends with an error
            np.savez(os.path.join(result_dir, f"rank{rank}.npz"), error=str(e))
            return
        from oracle import oracle
        want = oracle.moe_ffn(layer, x)[0] if n_tok else np.zeros((0, case["E"]), np.float32)
        np.savez(os.path.join(result_dir, f"rank{rank}.npz"), out=out, want=want)
    finally:
        if case.get("leave_rank") is None:
            dist.destroy_process_group()
