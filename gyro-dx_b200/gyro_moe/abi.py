"""ctypes mirror of include/gyro_moe.h — the host-side binding a Python caller (tests, bench)
uses; the Zig host binds the same symbols through gyro-dx_b200/zig/gx_abi.zig.

It loads the in-tree libgyromoe.so and fails loudly when it is missing: there is no CPU
fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libgyromoe.so"
CODEBOOK_PATH = PKG / "data" / "gyro_codebook.f16"

GX_OK = 0
ERRORS = {-1: "GX_E_INVALIDARG", -2: "GX_E_OUTOFMEMORY", -3: "GX_E_TIMEOUT", -4: "GX_E_DEVICE",
          -5: "GX_E_UNSUPPORTED", -6: "GX_E_STATE", -7: "GX_E_MISMATCH", -8: "GX_E_COMM", -9: "GX_E_KERNEL",
          -10: "GX_E_RANGE"}
GX_F32, GX_Q8_0, GX_BF16 = 0, 8, 30
GX_FLAG_PROFILE = 1
GX_EP_NONE, GX_EP_NCCL, GX_EP_PEER = 0, 1, 2     # gx_caps.ep_exchange


class GxError(RuntimeError):
    def __init__(self, code: int, call: str):
        super().__init__(f"{call} failed: {ERRORS.get(code, code)}")
        self.code = code


class Options(ctypes.Structure):
    _fields_ = [("device", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("world", ctypes.c_uint32),
                ("max_tokens", ctypes.c_uint32), ("max_layers", ctypes.c_uint32), ("flags", ctypes.c_uint32),
                ("codebook", ctypes.c_void_p), ("codebook_bytes", ctypes.c_uint64),
                ("nccl_id", ctypes.c_uint8 * 128)]


class Caps(ctypes.Structure):
    _fields_ = [("abi_version", ctypes.c_uint32), ("sm_count", ctypes.c_uint32), ("cc_major", ctypes.c_uint32),
                ("cc_minor", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("world", ctypes.c_uint32),
                ("max_tokens", ctypes.c_uint32), ("max_layers", ctypes.c_uint32), ("hbm_bytes", ctypes.c_uint64),
                ("free_bytes", ctypes.c_uint64), ("l2_bytes", ctypes.c_uint64), ("arena_bytes", ctypes.c_uint64),
                ("device_name", ctypes.c_char * 120), ("ep_exchange", ctypes.c_uint32), ("ep_peer_layers", ctypes.c_uint32)]


class LayerDesc(ctypes.Structure):
    _fields_ = [("type_id", ctypes.c_uint32), ("n_expert", ctypes.c_uint32), ("n_embd", ctypes.c_uint32),
                ("n_ff", ctypes.c_uint32), ("n_used", ctypes.c_uint32), ("expert_weights_scale", ctypes.c_float),
                ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("gate_bytes", ctypes.c_uint64), ("up_bytes", ctypes.c_uint64), ("down_bytes", ctypes.c_uint64),
                ("router", ctypes.c_void_p), ("gate_signs", ctypes.c_void_p), ("up_signs", ctypes.c_void_p),
                ("down_signs", ctypes.c_void_p), ("router_bias", ctypes.c_void_p)]


class SharedDesc(ctypes.Structure):
    _fields_ = [("type_id", ctypes.c_uint32), ("n_ff", ctypes.c_uint32), ("gate", ctypes.c_void_p),
                ("up", ctypes.c_void_p), ("down", ctypes.c_void_p), ("gate_bytes", ctypes.c_uint64),
                ("up_bytes", ctypes.c_uint64), ("down_bytes", ctypes.c_uint64), ("gate_inp", ctypes.c_void_p)]


class HcDesc(ctypes.Structure):
    _fields_ = [("n_streams", ctypes.c_uint32), ("rank", ctypes.c_uint32), ("type_id", ctypes.c_uint32),
                ("eps", ctypes.c_float), ("norm", ctypes.c_void_p), ("down", ctypes.c_void_p),
                ("up", ctypes.c_void_p), ("inject", ctypes.c_void_p), ("down_bytes", ctypes.c_uint64),
                ("up_bytes", ctypes.c_uint64), ("inject_bytes", ctypes.c_uint64)]


class GgufLayerInfo(ctypes.Structure):
    _fields_ = [("type_id", ctypes.c_uint32), ("n_expert", ctypes.c_uint32), ("n_embd", ctypes.c_uint32),
                ("n_ff", ctypes.c_uint32), ("n_used", ctypes.c_uint32), ("expert_weights_scale", ctypes.c_float),
                ("shared_type", ctypes.c_uint32), ("shared_ff", ctypes.c_uint32), ("rotated", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


GX_SHARED_NONE = 0xFFFFFFFF


class Timings(ctypes.Structure):
    _fields_ = [("router_ns", ctypes.c_uint64), ("gate_up_ns", ctypes.c_uint64), ("down_ns", ctypes.c_uint64),
                ("experts_ns", ctypes.c_uint64), ("total_ns", ctypes.c_uint64), ("layers", ctypes.c_uint64)]


assert ctypes.sizeof(Options) == 168 and ctypes.sizeof(Caps) == 192 and ctypes.sizeof(LayerDesc) == 112
assert ctypes.sizeof(SharedDesc) == 64 and ctypes.sizeof(GgufLayerInfo) == 40 and ctypes.sizeof(HcDesc) == 72

# (name, argtypes) of every exported entry point; include/gyro_moe.h declares exactly these.
_P, _U32, _U64, _F = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_float
SIGNATURES = {
    "gx_create": [ctypes.POINTER(Options), ctypes.POINTER(_P)],
    "gx_comm_unique_id": [ctypes.c_char_p, _U64],
    "gx_get_caps": [_P, ctypes.POINTER(Caps)],
    "gx_upload_layer": [_P, _U32, ctypes.POINTER(LayerDesc), _U32],
    "gx_upload_shared": [_P, _U32, ctypes.POINTER(SharedDesc), _U32],
    "gx_upload_hc": [_P, _U32, ctypes.POINTER(HcDesc), _U32],
    "gx_ffn_block": [_P, _U32, _P, _U32, _P, ctypes.POINTER(_U64)],
    "gx_gguf_inspect_layer": [ctypes.c_char_p, _U32, ctypes.POINTER(GgufLayerInfo)],
    "gx_upload_layer_gguf": [_P, _U32, ctypes.c_char_p, _U32, _U32],
    "gx_moe_forward": [_P, _U32, _P, _U32, _U32, _P, _U32, _P, _P, ctypes.POINTER(_U64)],
    "gx_moe_forward_host": [_P, _U32, _P, _U32, _U32, _P, _U32, _P, _P, _U32],
    "gx_stack_forward": [_P, _U32, _U32, _P, _U32, _U32, _P, _U32, ctypes.POINTER(_U64)],
    "gx_stack_forward_host": [_P, _U32, _U32, _P, _U32, _U32, _P, _U32, _U32],
    "gx_wait": [_P, _U64, _U32],
    "gx_poll": [_P, ctypes.POINTER(_U64)],
    "gx_get_stream": [_P, ctypes.POINTER(_P)],
    "gx_decode_blocks": [_P, _U32, _P, _U64, _P, _U32, _P, ctypes.POINTER(_F), _U32],
    "gx_upload_matrix": [_P, _U32, _U32, _U32, _P, _U64, ctypes.POINTER(_U32), _U32],
    "gx_matvec": [_P, _U32, _P, _U32, _P, ctypes.POINTER(_U64)],
    "gx_read_timings": [_P, ctypes.POINTER(Timings)],
    "gx_read_expert_counts": [_P, _U32, _P, _U32, _U32],
    "gx_replicate_experts": [_P, _U32, _P, _U32, _U32],
    "gx_moe_forward_noalloc": [_P, _U32, _P, _U32, _U32, _P, _U32, _P, _P, ctypes.POINTER(_U64)],
    "gx_set_flags": [_P, _U32],
    "gx_destroy": [_P, _U32],
}

NOALLOC_MAX_TOKENS = 16          # GX_NOALLOC_MAX_TOKENS

_LIB = None


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Loads libgyromoe.so (raises if it was not built). GYRO_MOE_LIB in the environment names
    another build of the same library (for side-by-side timing)."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path else Path(os.environ.get("GYRO_MOE_LIB", "") or LIB_PATH)
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with gyro-dx_b200/gyro_moe/build.py (no CPU fallback exists)")
    lib = ctypes.CDLL(str(p))
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int32
    if path is None:
        _LIB = lib
    return lib


def _check(rc: int, call: str) -> None:
    if rc != GX_OK:
        raise GxError(rc, call)


def _ptr(a) -> int | None:
    """Device pointer of a torch tensor, host pointer of a numpy array, or None."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def _dtype_code(a) -> int:
    name = str(a.dtype)
    if "bfloat16" in name:
        return GX_BF16
    if "float32" in name:
        return GX_F32
    if name == "uint16":  # numpy bf16 bit patterns
        return GX_BF16
    raise ValueError(f"unsupported activation dtype {name}")


def gguf_layer_info(path, gguf_layer: int) -> GgufLayerInfo:
    """gx_gguf_inspect_layer: shapes and types of one layer of a GGUF file (no device needed)."""
    info = GgufLayerInfo()
    _check(load().gx_gguf_inspect_layer(str(path).encode(), gguf_layer, ctypes.byref(info)), "gx_gguf_inspect_layer")
    return info


def unique_id() -> bytes:
    """A fresh NCCL unique id for gx_options.nccl_id (rank 0 makes it, the others receive it)."""
    buf = ctypes.create_string_buffer(128)
    _check(load().gx_comm_unique_id(buf, 128), "gx_comm_unique_id")
    return buf.raw


class Context:
    """One device context (gx_create ... gx_destroy)."""

    def __init__(self, device: int = 0, max_tokens: int = 64, max_layers: int = 1, flags: int = 0,
                 rank: int = 0, world: int = 1, nccl_id: bytes | None = None):
        self.lib = load()
        table = CODEBOOK_PATH.read_bytes()
        self._codebook = ctypes.create_string_buffer(table, len(table))
        opts = Options(device, rank, world, max_tokens, max_layers, flags,
                       ctypes.cast(self._codebook, ctypes.c_void_p), len(table))
        if nccl_id:
            ctypes.memmove(opts.nccl_id, nccl_id, min(128, len(nccl_id)))
        h = ctypes.c_void_p()
        _check(self.lib.gx_create(ctypes.byref(opts), ctypes.byref(h)), "gx_create")
        self.handle = h
        self.max_tokens = max_tokens
        self.layers: dict[int, dict] = {}

    # --- lifecycle -----------------------------------------------------------------------
    def close(self, timeout_ms: int = 60000) -> None:
        if self.handle:
            _check(self.lib.gx_destroy(self.handle, timeout_ms), "gx_destroy")
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def caps(self) -> Caps:
        c = Caps()
        _check(self.lib.gx_get_caps(self.handle, ctypes.byref(c)), "gx_get_caps")
        return c

    def stream(self) -> int:
        s = ctypes.c_void_p()
        _check(self.lib.gx_get_stream(self.handle, ctypes.byref(s)), "gx_get_stream")
        return s.value or 0

    # --- upload ----------------------------------------------------------------------------
    def upload_layer(self, index: int, layer: dict, timeout_ms: int = 600000) -> None:
        keep = []

        def arr(a, dtype):
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=dtype)
            keep.append(a)
            return a.ctypes.data

        gate, up, down = (np.ascontiguousarray(layer[k], dtype=np.uint8) for k in ("gate", "up", "down"))
        keep += [gate, up, down]
        gs = layer.get("gate_signs")
        desc = LayerDesc(layer["type_id"], layer["n_expert"], layer["n_embd"], layer["n_ff"], layer["n_used"],
                         layer.get("expert_weights_scale", 0.0), gate.ctypes.data, up.ctypes.data, down.ctypes.data,
                         gate.nbytes, up.nbytes, down.nbytes, arr(layer["router"], np.float32),
                         arr(gs, np.float32), arr(layer.get("up_signs", gs), np.float32),
                         arr(layer.get("down_signs"), np.float32), arr(layer.get("router_bias"), np.float32))
        _check(self.lib.gx_upload_layer(self.handle, index, ctypes.byref(desc), timeout_ms), "gx_upload_layer")
        self.layers[index] = {k: layer[k] for k in ("n_embd", "n_used", "n_expert")}
        if layer.get("shared") is not None:
            self.upload_shared(index, layer["shared"], timeout_ms)

    def upload_shared(self, index: int, shared: dict | None, timeout_ms: int = 600000) -> None:
        """gx_upload_shared: the layer's shared expert (synth.make_shared layout), or None to drop it."""
        if shared is None:
            _check(self.lib.gx_upload_shared(self.handle, index, None, timeout_ms), "gx_upload_shared")
            return
        mats = [np.ascontiguousarray(shared[k], dtype=np.uint8) for k in ("gate", "up", "down")]
        gi = np.ascontiguousarray(shared["gate_inp"], dtype=np.float32)
        desc = SharedDesc(shared["type_id"], shared["n_ff"], mats[0].ctypes.data, mats[1].ctypes.data,
                          mats[2].ctypes.data, mats[0].nbytes, mats[1].nbytes, mats[2].nbytes, gi.ctypes.data)
        _check(self.lib.gx_upload_shared(self.handle, index, ctypes.byref(desc), timeout_ms), "gx_upload_shared")

    def upload_hc(self, index: int, hc: dict | None, timeout_ms: int = 600000) -> None:
        """gx_upload_hc: the FFN block's hyper-connection mixer (synth.make_hc layout), or None."""
        if hc is None:
            _check(self.lib.gx_upload_hc(self.handle, index, None, timeout_ms), "gx_upload_hc")
            return
        mats = [np.ascontiguousarray(hc[k], dtype=np.uint8) for k in ("down", "up", "inject")]
        norm = np.ascontiguousarray(hc["norm"], dtype=np.float32)
        desc = HcDesc(hc["n_streams"], hc["rank"], hc["type_id"], hc["eps"], norm.ctypes.data, mats[0].ctypes.data,
                      mats[1].ctypes.data, mats[2].ctypes.data, mats[0].nbytes, mats[1].nbytes, mats[2].nbytes)
        _check(self.lib.gx_upload_hc(self.handle, index, ctypes.byref(desc), timeout_ms), "gx_upload_hc")

    def upload_layer_gguf(self, index: int, path, gguf_layer: int, timeout_ms: int = 600000) -> None:
        """gx_upload_layer_gguf: layer gguf_layer of a GGUF file into slot index."""
        _check(self.lib.gx_upload_layer_gguf(self.handle, index, str(path).encode(), gguf_layer, timeout_ms),
               "gx_upload_layer_gguf")
        info = gguf_layer_info(path, gguf_layer)
        self.layers[index] = {"n_embd": info.n_embd, "n_used": info.n_used, "n_expert": info.n_expert}

    # --- forward ---------------------------------------------------------------------------
    def forward(self, layer: int, x, y, ids=None, weights=None) -> int:
        """Device tensors (torch, on this context's device). Returns the ticket."""
        t = ctypes.c_uint64()
        n_tok = x.shape[0]
        _check(self.lib.gx_moe_forward(self.handle, layer, _ptr(x), _dtype_code(x), n_tok, _ptr(y), _dtype_code(y),
                                       _ptr(ids), _ptr(weights), ctypes.byref(t)), "gx_moe_forward")
        return t.value

    def ffn_block(self, layer: int, res, n_tok: int | None = None, mixed=None) -> int:
        """gx_ffn_block on a device f32 tensor res [n_tok, hc * n_embd], updated in place; mixed
        (optional device f32 [n_tok, n_embd]) receives the mixer's output. Returns the ticket."""
        t = ctypes.c_uint64()
        n = res.shape[0] if n_tok is None else n_tok
        _check(self.lib.gx_ffn_block(self.handle, layer, _ptr(res), n, _ptr(mixed), ctypes.byref(t)), "gx_ffn_block")
        return t.value

    def expert_counts(self, layer: int, reset: bool = False, timeout_ms: int = 60000) -> np.ndarray:
        """This rank's routed slots per global expert of a layer (expert-parallel contexts)."""
        n = self.layers[layer]["n_expert"]
        out = np.zeros(n, np.uint32)
        _check(self.lib.gx_read_expert_counts(self.handle, layer, out.ctypes.data, int(reset), timeout_ms),
               "gx_read_expert_counts")
        return out

    def replicate_experts(self, layer: int, experts, timeout_ms: int = 120000) -> None:
        """Collective: every rank serves the listed global experts of the layer for its own tokens."""
        ids = np.ascontiguousarray(np.asarray(experts, dtype=np.uint32))
        _check(self.lib.gx_replicate_experts(self.handle, layer, ids.ctypes.data if ids.size else None, ids.size,
                                             timeout_ms), "gx_replicate_experts")

    def forward_noalloc(self, layer: int, x, y, ids=None, weights=None) -> int:
        """gx_moe_forward_noalloc on device tensors: the decode layer on the library's static
        scratch, for at most NOALLOC_MAX_TOKENS tokens. Returns the ticket."""
        t = ctypes.c_uint64()
        _check(self.lib.gx_moe_forward_noalloc(self.handle, layer, _ptr(x), _dtype_code(x), x.shape[0], _ptr(y),
                                               _dtype_code(y), _ptr(ids), _ptr(weights), ctypes.byref(t)),
               "gx_moe_forward_noalloc")
        return t.value

    def forward_host(self, layer: int, x: np.ndarray, out_dtype=np.float32, timeout_ms: int = 60000,
                     want_routing: bool = False):
        """Host numpy in/out (bf16 passed as uint16 bit patterns)."""
        x = np.ascontiguousarray(x)
        n_tok, E = x.shape
        y = np.empty((n_tok, E), dtype=out_dtype)
        U = self.layers[layer]["n_used"]
        ids = np.empty((n_tok, U), np.uint32) if want_routing else None
        w = np.empty((n_tok, U), np.float32) if want_routing else None
        _check(self.lib.gx_moe_forward_host(self.handle, layer, x.ctypes.data, _dtype_code(x), n_tok, y.ctypes.data,
                                            _dtype_code(y), _ptr(ids), _ptr(w), timeout_ms), "gx_moe_forward_host")
        return (y, ids, w) if want_routing else y

    def stack_forward(self, first: int, n_layers: int, x, y) -> int:
        t = ctypes.c_uint64()
        _check(self.lib.gx_stack_forward(self.handle, first, n_layers, _ptr(x), _dtype_code(x), x.shape[0], _ptr(y),
                                         _dtype_code(y), ctypes.byref(t)), "gx_stack_forward")
        return t.value

    def stack_forward_host(self, first: int, n_layers: int, x: np.ndarray, out_dtype=np.float32,
                           timeout_ms: int = 60000) -> np.ndarray:
        x = np.ascontiguousarray(x)
        y = np.empty(x.shape, dtype=out_dtype)
        _check(self.lib.gx_stack_forward_host(self.handle, first, n_layers, x.ctypes.data, _dtype_code(x), x.shape[0],
                                              y.ctypes.data, _dtype_code(y), timeout_ms), "gx_stack_forward_host")
        return y

    def wait(self, ticket: int, timeout_ms: int = 60000) -> None:
        _check(self.lib.gx_wait(self.handle, ticket, timeout_ms), "gx_wait")

    def poll(self) -> int:
        t = ctypes.c_uint64()
        _check(self.lib.gx_poll(self.handle, ctypes.byref(t)), "gx_poll")
        return t.value

    def set_flags(self, flags: int) -> None:
        _check(self.lib.gx_set_flags(self.handle, flags), "gx_set_flags")

    def timings(self) -> Timings:
        t = Timings()
        _check(self.lib.gx_read_timings(self.handle, ctypes.byref(t)), "gx_read_timings")
        return t

    # --- conformance / standalone GEMV -----------------------------------------------------
    def decode_blocks(self, type_id: int, packed: bytes | np.ndarray, value_count: int,
                      expected: np.ndarray | None = None, timeout_ms: int = 60000):
        src = np.frombuffer(bytes(packed), dtype=np.uint8)
        out = np.empty(value_count, np.float32)
        err = ctypes.c_float(0.0)
        exp = None if expected is None else np.ascontiguousarray(expected, dtype=np.float32)
        rc = self.lib.gx_decode_blocks(self.handle, type_id, src.ctypes.data, src.size, out.ctypes.data, value_count,
                                       _ptr(exp), ctypes.byref(err), timeout_ms)
        return rc, out, err.value

    def upload_matrix(self, type_id: int, rows: int, cols: int, packed: np.ndarray, timeout_ms: int = 60000) -> int:
        p = np.ascontiguousarray(packed, dtype=np.uint8)
        h = ctypes.c_uint32()
        _check(self.lib.gx_upload_matrix(self.handle, type_id, rows, cols, p.ctypes.data, p.nbytes, ctypes.byref(h),
                                         timeout_ms), "gx_upload_matrix")
        return h.value

    def matvec(self, handle: int, x, y) -> int:
        t = ctypes.c_uint64()
        _check(self.lib.gx_matvec(self.handle, handle, _ptr(x), x.shape[0], _ptr(y), ctypes.byref(t)), "gx_matvec")
        return t.value
