"""ctypes front end of the CPU oracle (oracle/gxo.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm, always as the checker or the timed CPU baseline, never as the
product. It restates the reference CPU engine of mattneel/gyro-dx (src/gyro.zig,
src/kernels.zig, src/engine.zig:520-686); see gxo.h for the line-by-line mapping.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CODEBOOK = ROOT / "gyro-dx_b200" / "gyro_moe" / "data" / "gyro_codebook.f16"

_F32P = ctypes.POINTER(ctypes.c_float)
_U32P = ctypes.POINTER(ctypes.c_uint32)


class _Layer(ctypes.Structure):
    _fields_ = [
        ("type_id", ctypes.c_uint32),
        ("n_expert", ctypes.c_uint32),
        ("n_embd", ctypes.c_uint32),
        ("n_ff", ctypes.c_uint32),
        ("n_used", ctypes.c_uint32),
        ("expert_weights_scale", ctypes.c_float),
        ("gate", ctypes.c_void_p),
        ("up", ctypes.c_void_p),
        ("down", ctypes.c_void_p),
        ("router", ctypes.c_void_p),
        ("gate_signs", ctypes.c_void_p),
        ("down_signs", ctypes.c_void_p),
        ("router_bias", ctypes.c_void_p),
    ]


def build(force: bool = False) -> None:
    """Compiles liboracle.so / liboracle_fast.so (and oracle/_ref when the reference exists)."""
    targets = ["all"]
    if Path("/root/reference/third_party/agention-gyro/src/tq_ref.c").exists():
        targets.append("ref")
    cmd = ["make", "-s", "-C", str(HERE)] + (["-B"] if force else []) + targets
    subprocess.run(cmd, check=True)


_LIBS: dict[str, ctypes.CDLL] = {}


def lib(fast: bool = False) -> ctypes.CDLL:
    name = "liboracle_fast.so" if fast else "liboracle.so"
    if name in _LIBS:
        return _LIBS[name]
    path = HERE / name
    if not path.exists():
        build()
    L = ctypes.CDLL(str(path))
    L.gxo_set_codebook.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    L.gxo_type_info.argtypes = [ctypes.c_uint32] + [ctypes.POINTER(ctypes.c_int)] * 3
    L.gxo_fp16_to_fp32.argtypes = [ctypes.c_uint16]
    L.gxo_fp16_to_fp32.restype = ctypes.c_float
    L.gxo_state.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    L.gxo_state.restype = ctypes.c_uint32
    L.gxo_decode_row.argtypes = [ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                 _F32P, ctypes.c_size_t]
    L.gxo_rotate.argtypes = [_F32P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]
    L.gxo_unrotate.argtypes = L.gxo_rotate.argtypes
    L.gxo_rotate_f32.argtypes = [_F32P, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p]
    L.gxo_rotate_f32.restype = None
    L.gxo_dot_row.argtypes = [ctypes.c_uint32, ctypes.c_void_p, _F32P, ctypes.c_size_t]
    L.gxo_dot_row.restype = ctypes.c_float
    L.gxo_softmax.argtypes = [_F32P, ctypes.c_size_t]
    L.gxo_softmax.restype = None
    L.gxo_topk.argtypes = [_F32P, ctypes.c_size_t, _U32P, _F32P, ctypes.c_size_t]
    L.gxo_topk.restype = None
    L.gxo_moe_ffn.argtypes = [ctypes.POINTER(_Layer), _F32P, ctypes.c_size_t, _F32P, _U32P, _F32P,
                              ctypes.c_int]
    L.gxo_moe_experts.argtypes = [ctypes.POINTER(_Layer), _F32P, ctypes.c_size_t, _U32P, _F32P, _F32P,
                                  ctypes.c_int]
    L.gxo_shared_expert.argtypes = [ctypes.POINTER(_Shared), _F32P, ctypes.c_size_t, ctypes.c_size_t, _F32P,
                                    ctypes.c_int]
    L.gxo_hc_mix.argtypes = [ctypes.POINTER(_Hc), _F32P, ctypes.c_size_t, _F32P, ctypes.c_void_p, ctypes.c_int]
    L.gxo_hc_combine.argtypes = [ctypes.POINTER(_Hc), _F32P, ctypes.c_size_t, _F32P, _F32P]
    L.gxo_max_threads.restype = ctypes.c_int
    L.gxo_rms_norm.argtypes = [_F32P, _F32P, ctypes.c_size_t, ctypes.c_float]
    L.gxo_rms_norm.restype = None
    table = CODEBOOK.read_bytes()
    if L.gxo_set_codebook(table, len(table)) != 0:
        raise RuntimeError("oracle rejected the codebook")
    _LIBS[name] = L
    return L


class _Shared(ctypes.Structure):
    _fields_ = [
        ("type_id", ctypes.c_uint32),
        ("n_ff", ctypes.c_uint32),
        ("gate", ctypes.c_void_p),
        ("up", ctypes.c_void_p),
        ("down", ctypes.c_void_p),
        ("gate_inp", ctypes.c_void_p),
    ]


class _Hc(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("n_embd", ctypes.c_uint32),
                ("type_id", ctypes.c_uint32), ("eps", ctypes.c_float), ("norm", ctypes.c_void_p),
                ("down", ctypes.c_void_p), ("up", ctypes.c_void_p), ("inject", ctypes.c_void_p)]


def _f32p(a: np.ndarray):
    return a.ctypes.data_as(_F32P)


def type_info(type_id: int):
    k, s, b = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    if lib().gxo_type_info(type_id, ctypes.byref(k), ctypes.byref(s), ctypes.byref(b)) != 0:
        raise ValueError(f"unknown Gyro type {type_id}")
    return k.value, s.value, b.value


def decode_row(type_id: int, packed: bytes | np.ndarray, n: int, state_bits: int = 15) -> np.ndarray:
    """Strict decode (src/gyro.zig:81-105). Raises ValueError with the gyro.Error code."""
    src = np.frombuffer(bytes(packed), dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    rc = lib().gxo_decode_row(type_id, state_bits, src.ctypes.data, src.size, _f32p(out), n)
    if rc != 0:
        raise ValueError(rc)
    return out


def rotate(values: np.ndarray, block: int, signs: np.ndarray | None, inverse: bool = False) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32).copy()
    s = None if signs is None else np.ascontiguousarray(signs, dtype=np.int8)
    fn = lib().gxo_unrotate if inverse else lib().gxo_rotate
    rc = fn(_f32p(v), v.size, block, None if s is None else s.ctypes.data)
    if rc != 0:
        raise ValueError(rc)
    return v


def moe_ffn(layer: dict, x: np.ndarray, threads: int = 1, fast: bool = False):
    """src/engine.zig:520-642 on f32 tokens x [n, E]; returns (out [n,E], ids [n,U], w [n,U])."""
    L = lib(fast)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, E = x.shape
    U = layer["n_used"]
    keep = []

    def ptr(a, dtype):
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dtype)
        keep.append(a)
        return a.ctypes.data

    desc = _Layer(layer["type_id"], layer["n_expert"], E, layer["n_ff"], U,
                  layer.get("expert_weights_scale", 0.0),
                  ptr(layer["gate"], np.uint8), ptr(layer["up"], np.uint8), ptr(layer["down"], np.uint8),
                  ptr(layer["router"], np.float32), ptr(layer.get("gate_signs"), np.float32),
                  ptr(layer.get("down_signs"), np.float32), ptr(layer.get("router_bias"), np.float32))
    out = np.empty((n, E), dtype=np.float32)
    ids = np.empty((n, U), dtype=np.uint32)
    w = np.empty((n, U), dtype=np.float32)
    rc = L.gxo_moe_ffn(ctypes.byref(desc), _f32p(x), n, _f32p(out), ids.ctypes.data_as(_U32P), _f32p(w), threads)
    if rc != 0:
        raise RuntimeError(f"gxo_moe_ffn failed ({rc})")
    if layer.get("shared") is not None:
        shared_expert(layer["shared"], x, out, threads=threads, fast=fast)
    return out, ids, w


def shared_expert(shared: dict, x: np.ndarray, out: np.ndarray, threads: int = 1, fast: bool = False) -> None:
    """src/engine.zig:644-653: adds sigmoid(gate_inp . x) * Down(silu(Gate x) * Up x) into out [n, E]."""
    L = lib(fast)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, E = x.shape
    keep = [np.ascontiguousarray(shared[k], dtype=np.uint8) for k in ("gate", "up", "down")]
    gi = np.ascontiguousarray(shared["gate_inp"], dtype=np.float32)
    desc = _Shared(shared["type_id"], shared["n_ff"], keep[0].ctypes.data, keep[1].ctypes.data, keep[2].ctypes.data,
                   gi.ctypes.data)
    if not (out.flags["C_CONTIGUOUS"] and out.dtype == np.float32 and out.shape == (n, E)):
        raise ValueError("out must be a contiguous float32 [n, E] array")
    rc = L.gxo_shared_expert(ctypes.byref(desc), _f32p(x), n, E, _f32p(out), threads)
    if rc != 0:
        raise RuntimeError(f"gxo_shared_expert failed ({rc})")


def moe_experts(layer: dict, x: np.ndarray, ids: np.ndarray, weights: np.ndarray, threads: int = 1,
                fast: bool = False) -> np.ndarray:
    """Expert half of src/engine.zig:547-641 for a given routing (ids local to the layer's experts;
    ids >= n_expert contribute nothing). Returns out [n, E]."""
    L = lib(fast)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, E = x.shape
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    keep = []

    def ptr(a, dtype):
        if a is None:
            return None
        a = np.ascontiguousarray(a, dtype=dtype)
        keep.append(a)
        return a.ctypes.data

    desc = _Layer(layer["type_id"], layer["n_expert"], E, layer["n_ff"], layer["n_used"],
                  layer.get("expert_weights_scale", 0.0),
                  ptr(layer["gate"], np.uint8), ptr(layer["up"], np.uint8), ptr(layer["down"], np.uint8),
                  ptr(layer.get("router"), np.float32), ptr(layer.get("gate_signs"), np.float32),
                  ptr(layer.get("down_signs"), np.float32), None)
    out = np.zeros((n, E), dtype=np.float32)
    rc = L.gxo_moe_experts(ctypes.byref(desc), _f32p(x), n, ids.ctypes.data_as(_U32P), _f32p(weights), _f32p(out),
                           threads)
    if rc != 0:
        raise RuntimeError(f"gxo_moe_experts failed ({rc})")
    return out


STACK_NORM_EPS = 1e-6


def rms_norm(x: np.ndarray, eps: float = STACK_NORM_EPS) -> np.ndarray:
    """Row-wise RMSNorm with unit weight (src/kernels.zig:281-291)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    for r in range(x.shape[0]):
        lib().gxo_rms_norm(_f32p(out[r]), _f32p(x[r]), x.shape[1], eps)
    return out


def stack(layers: list, x: np.ndarray, threads: int = 1, fast: bool = False) -> np.ndarray:
    """The benchmark stack: x_{l+1} = x_l + MoE_l(RMSNorm(x_l)), a pre-norm residual stand-in
    for the mixer between the reference model's layers."""
    cur = np.ascontiguousarray(x, dtype=np.float32)
    for layer in layers:
        out, _, _ = moe_ffn(layer, rms_norm(cur), threads=threads, fast=fast)
        cur = cur + out
    return cur


def max_threads() -> int:
    return int(lib(True).gxo_max_threads())


def ref_lib() -> ctypes.CDLL | None:
    """The reference's own C decoder compiled from its sources (oracle/_ref), if built."""
    path = HERE / "_ref" / "libtq_ref.so"
    if not path.exists():
        return None
    R = ctypes.CDLL(str(path))
    R.tq_dequantize_row.argtypes = [ctypes.c_int, ctypes.c_void_p, _F32P, ctypes.c_int64]
    R.tq_hadamard_rotate.argtypes = [_F32P, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    R.tq_hadamard_unrotate.argtypes = R.tq_hadamard_rotate.argtypes
    return R


if __name__ == "__main__":
    build(force=bool(os.environ.get("FORCE")))
    print("oracle built; threads:", max_threads())


def _hc_desc(hc: dict, keep: list):
    arrs = [np.ascontiguousarray(hc[k], dtype=np.uint8) for k in ("down", "up", "inject")]
    norm = np.ascontiguousarray(hc["norm"], dtype=np.float32)
    keep += arrs + [norm]
    return _Hc(hc["n_streams"], hc["rank"], hc["n_embd"], hc["type_id"], hc["eps"], norm.ctypes.data,
               arrs[0].ctypes.data, arrs[1].ctypes.data, arrs[2].ctypes.data)


def hc_mix(hc: dict, res: np.ndarray, threads: int = 1, fast: bool = False):
    """src/engine.zig:184-215: res [n, hc*E] -> (cur [n, E], inject [n, hc])."""
    L = lib(fast)
    res = np.ascontiguousarray(res, dtype=np.float32)
    n = res.shape[0]
    keep = []
    desc = _hc_desc(hc, keep)
    out = np.empty((n, hc["n_embd"]), np.float32)
    inj = np.empty((n, hc["n_streams"]), np.float32)
    if L.gxo_hc_mix(ctypes.byref(desc), _f32p(res), n, _f32p(out), inj.ctypes.data, threads) != 0:
        raise RuntimeError("gxo_hc_mix failed")
    return out, inj


def hc_combine(hc: dict, res: np.ndarray, block_out: np.ndarray, inject: np.ndarray) -> np.ndarray:
    """src/engine.zig:217-228: a new res with the block output added to every stream."""
    L = lib()
    res = np.ascontiguousarray(res, dtype=np.float32).copy()
    block_out = np.ascontiguousarray(block_out, dtype=np.float32)
    inject = np.ascontiguousarray(inject, dtype=np.float32)
    keep = []
    desc = _hc_desc(hc, keep)
    if L.gxo_hc_combine(ctypes.byref(desc), _f32p(res), res.shape[0], _f32p(block_out), _f32p(inject)) != 0:
        raise RuntimeError("gxo_hc_combine failed")
    return res


def ffn_block(layer: dict, hc: dict, res: np.ndarray, threads: int = 1, fast: bool = False) -> np.ndarray:
    """The reference's FFN block (src/engine.zig:162-165): hc mixer, routed + shared experts,
    hc combine. res [n, hc*E] -> res'."""
    cur, inj = hc_mix(hc, res, threads=threads, fast=fast)
    out, _, _ = moe_ffn(layer, cur, threads=threads, fast=fast)
    return hc_combine(hc, res, out, inj)
