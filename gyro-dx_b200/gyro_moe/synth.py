"""Seeded synthetic routed-MoE layers with the shapes and value distributions of the
benchmark configurations (there is no model file on these machines).

- Codes: stream bytes uniform random from the seed. Block scales are fixed, not random:
  d = fp16(1/sqrt(cols)) (a random fp16 is Inf/NaN with probability 1/32). With the unit-variance
  codebook the weights come out ~N(0, 1/cols).
- Signs: one +-1 vector of width E shared by gate and up, one of width F for down (the
  reference looks signs up by width, src/model.zig:316-330).
- Router: f32 [n_expert, E] ~ N(0, 0.02).
- Optional Zipf(s) expert popularity: a fixed logit bias beta_e = ln p_e, p_e ~ rank_e^-s over
  a seeded permutation (a harness hook with no reference counterpart).

All arrays use the reference layout (stacked expert rows of packed 128-weight blocks,
src/model.zig:115-123), i.e. exactly what the Zig host passes as Matrix.data slices.
"""
from __future__ import annotations

import hashlib

import numpy as np

BLOCK_BYTES = {144: 34, 145: 26, 146: 30, 147: 42, 148: 50, 149: 58, 150: 22, 151: 18}
TYPE_NAMES = {144: "TQ2_T", 145: "TQK6", 146: "TQK7", 147: "TQP5", 148: "TQP6", 149: "TQP7",
              150: "TQK5", 151: "TQK4"}


def fp16_bits(value: float) -> int:
    return int(np.array([value], dtype=np.float16).view(np.uint16)[0])


def packed_matrix(rng: np.random.Generator, type_id: int, rows: int, cols: int,
                  scale: float | None = None) -> np.ndarray:
    """rows x (cols/128) blocks of random stream bytes with scale d = fp16(scale) (default
    1/sqrt(cols)); returns uint8 [rows, row_bytes]."""
    bb = BLOCK_BYTES[type_id]
    nb = cols // 128
    data = rng.integers(0, 256, rows * nb * bb, dtype=np.uint8)
    d = fp16_bits(1.0 / np.sqrt(cols) if scale is None else scale)
    # every block size is even, so each block's little-endian fp16 scale is one uint16 word
    data.view("<u2").reshape(rows * nb, bb // 2)[:, 0] = d
    return data.reshape(rows, nb * bb)


def zipf_bias(rng: np.random.Generator, n_expert: int, s: float = 1.1) -> np.ndarray:
    ranks = rng.permutation(n_expert) + 1
    p = ranks.astype(np.float64) ** (-s)
    p /= p.sum()
    return np.log(p).astype(np.float32)


def make_layer(seed: int, n_expert: int = 256, E: int = 2048, F: int = 512, U: int = 8,
               type_id: int = 144, zipf: float | None = None, signs: bool = True,
               expert_weights_scale: float = 0.0) -> dict:
    rng = np.random.default_rng(seed)
    layer = {
        "type_id": type_id, "n_expert": n_expert, "n_embd": E, "n_ff": F, "n_used": U,
        "expert_weights_scale": expert_weights_scale,
        "gate": packed_matrix(rng, type_id, n_expert * F, E),
        "up": packed_matrix(rng, type_id, n_expert * F, E),
        "down": packed_matrix(rng, type_id, n_expert * E, F),
        "router": rng.normal(0.0, 0.02, size=(n_expert, E)).astype(np.float32),
        "gate_signs": (rng.integers(0, 2, E) * 2 - 1).astype(np.float32) if signs else None,
        "down_signs": (rng.integers(0, 2, F) * 2 - 1).astype(np.float32) if signs else None,
        "router_bias": zipf_bias(rng, n_expert, zipf) if zipf else None,
    }
    h = hashlib.sha256()
    for key in ("gate", "up", "down", "router", "gate_signs", "down_signs", "router_bias"):
        if layer[key] is not None:
            h.update(np.ascontiguousarray(layer[key]).tobytes())
    layer["sha256"] = h.hexdigest()
    return layer


SHARED_TYPES = {"f32": 0, "q8_0": 8, "bf16": 30}


def make_shared(seed: int, E: int = 2048, SF: int = 512, type_id: int = 8) -> dict:
    """A shared expert (src/model.zig:418-421) in one of the non-expert encodings the reference GPU
    engine multiplies (src/gpu_engine.zig:846-850): Q8_0 (blocks of an fp16 scale and 32 int8, with
    d = fp16(1 / (73 sqrt(cols))) so the weights come out with a standard deviation near
    1 / sqrt(cols)), bf16 or f32 (~N(0, 1/cols)). Its sigmoid gate is f32 ~N(0, 0.02)."""
    rng = np.random.default_rng(seed)

    def mat(rows: int, cols: int) -> np.ndarray:
        return dense_matrix(rng, type_id, rows, cols, 1.0 / np.sqrt(cols))

    return {"type_id": type_id, "n_ff": SF, "gate": mat(SF, E), "up": mat(SF, E), "down": mat(E, SF),
            "gate_inp": rng.normal(0.0, 0.02, size=E).astype(np.float32)}


def dense_matrix(rng: np.random.Generator, type_id: int, rows: int, cols: int, std: float) -> np.ndarray:
    """Row-major bytes of a plain matrix with weights of about the given deviation: Q8_0 (blocks of
    an fp16 scale d = fp16(std / 73) and 32 int8 ~U[-127, 127]), bf16 or f32 (~N(0, std^2))."""
    if type_id == 8:
        q = rng.integers(-127, 128, (rows, cols // 32, 32), dtype=np.int8)
        d = np.full((rows, cols // 32, 1), fp16_bits(std / 73.0), np.uint16)
        return np.concatenate([d.view(np.uint8), q.view(np.uint8)], axis=2).reshape(rows, cols // 32 * 34)
    w = rng.normal(0.0, std, size=(rows, cols)).astype(np.float32)
    if type_id == 30:
        return bf16_bits(w).view(np.uint8).reshape(rows, cols * 2)
    if type_id == 0:
        return w.view(np.uint8).reshape(rows, cols * 4)
    raise ValueError(f"unsupported non-expert type {type_id}")


def make_hc(seed: int, E: int = 2048, n_streams: int = 4, rank: int = 256, eps: float = 1e-6,
            type_id: int = 8) -> dict:
    """Hyper-connection mixer weights of the FFN block (src/model.zig:361-366: hc_ffn_norm, down,
    up, inject) in one non-expert encoding (Q8_0 by default); norm weights ~1 + N(0, 0.1).
    HD = n_streams * E. The reference model has 4 streams of rank 320."""
    rng = np.random.default_rng(seed)
    HD = n_streams * E
    return {"n_streams": n_streams, "rank": rank, "n_embd": E, "type_id": type_id, "eps": eps,
            "norm": (1.0 + 0.1 * rng.standard_normal(HD)).astype(np.float32),
            "down": dense_matrix(rng, type_id, rank, HD, 1.0 / np.sqrt(HD)),
            "up": dense_matrix(rng, type_id, HD, rank, 1.0 / np.sqrt(rank)),
            "inject": dense_matrix(rng, type_id, n_streams, HD, 1.0 / np.sqrt(HD))}


def tokens(seed: int, n: int, E: int = 2048, dtype=np.float32) -> np.ndarray:
    """x ~ N(0, 1); bf16 inputs are produced by rounding (returned as float32 values that are
    exactly representable in bf16 when dtype is 'bf16')."""
    x = np.random.default_rng(seed).standard_normal((n, E)).astype(np.float32)
    if dtype == "bf16":
        x = bf16_round(x)
    return x


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def loguniform_lengths(seed: int, count: int = 32, lo: int = 1, hi: int = 512) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.floor(np.exp(rng.uniform(np.log(lo), np.log(hi + 1), count))).astype(np.int64).clip(lo, hi)
