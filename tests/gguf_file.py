"""A minimal GGUF version-3 writer for tests: synthetic routed-MoE layers stored the way the
reference model file stores them (stacked expert tensors blk.L.ffn_{gate,up,down}_exps.weight with
the innermost dimension first, the router blk.L.ffn_gate_inp.weight, the shared expert and its
gate, <arch>.expert_* hyper-parameters and the prism.hadamard.* rotation metadata; the layout of
src/gguf.zig:263-334 and the bindings of src/model.zig:395-421). Test infrastructure only."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
ALIGN = 32


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(kind: int, v) -> bytes:
    if kind == U32:
        return struct.pack("<I", v)
    if kind == F32:
        return struct.pack("<f", v)
    if kind == STR:
        return _str(v)
    if kind == BOOL:
        return struct.pack("<B", v)
    if kind == ARR:
        elem, items = v
        body = b"".join(_value(elem, x) for x in items)
        return struct.pack("<IQ", elem, len(items)) + body
    if kind == I32:
        return struct.pack("<i", v)
    raise ValueError(kind)


def write(path, metadata: list, tensors: list, version: int = 3, misalign: str | None = None,
          overlap: tuple | None = None) -> None:
    """metadata: [(key, kind, value)]; tensors: [(name, dims (innermost first), type id, bytes)].
    misalign / overlap break the header on purpose for the negative tests."""
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata))
    for key, kind, v in metadata:
        head += _str(key) + struct.pack("<I", kind) + _value(kind, v)
    offsets, off = [], 0
    for name, dims, typ, data in tensors:
        offsets.append(off)
        off = (off + len(data) + ALIGN - 1) // ALIGN * ALIGN
    if overlap:
        offsets[overlap[1]] = offsets[overlap[0]]
    for i, (name, dims, typ, data) in enumerate(tensors):
        rel = offsets[i] + (1 if misalign == name else 0)
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", typ, rel)
    pad = (-len(head)) % ALIGN
    blob = bytearray(head + b"\0" * pad)
    base = len(blob)
    blob += b"\0" * off
    for i, (name, dims, typ, data) in enumerate(tensors):
        blob[base + offsets[i]:base + offsets[i] + len(data)] = bytes(data)
    with open(path, "wb") as f:
        f.write(bytes(blob))


def layer_records(index: int, layer: dict) -> tuple[list, list]:
    """GGUF tensors and rotation entries of one synthetic layer (synth.make_layer layout)."""
    E, F, NE = layer["n_embd"], layer["n_ff"], layer["n_expert"]
    t = layer["type_id"]
    pre = f"blk.{index}."
    tensors = [
        (pre + "ffn_gate_exps.weight", [E, F, NE], t, np.ascontiguousarray(layer["gate"]).tobytes()),
        (pre + "ffn_up_exps.weight", [E, F, NE], t, np.ascontiguousarray(layer["up"]).tobytes()),
        (pre + "ffn_down_exps.weight", [F, E, NE], t, np.ascontiguousarray(layer["down"]).tobytes()),
        (pre + "ffn_gate_inp.weight", [E, NE], 0, np.ascontiguousarray(layer["router"], np.float32).tobytes()),
    ]
    sh = layer.get("shared")
    if sh is not None:
        SF, st = sh["n_ff"], sh["type_id"]
        tensors += [
            (pre + "ffn_gate_shexp.weight", [E, SF], st, np.ascontiguousarray(sh["gate"]).tobytes()),
            (pre + "ffn_up_shexp.weight", [E, SF], st, np.ascontiguousarray(sh["up"]).tobytes()),
            (pre + "ffn_down_shexp.weight", [SF, E], st, np.ascontiguousarray(sh["down"]).tobytes()),
            (pre + "ffn_gate_inp_shexp.weight", [E], 0, np.ascontiguousarray(sh["gate_inp"], np.float32).tobytes()),
        ]
    rotated = []
    if layer.get("gate_signs") is not None:
        rotated += [pre + "ffn_gate_exps.weight", pre + "ffn_up_exps.weight"]
    if layer.get("down_signs") is not None:
        rotated.append(pre + "ffn_down_exps.weight")
    return tensors, rotated


def model_file(path, layers: list, arch: str = "qwen4exp", **kw) -> None:
    """Layers that share one E / F and one sign vector per width (the reference model's layout:
    prism.hadamard.sign_widths lists each width once)."""
    tensors, rotated = [], []
    for i, l in enumerate(layers):
        t, r = layer_records(i, l)
        tensors += t
        rotated += r
    l0 = layers[0]
    meta = [("general.architecture", STR, arch),
            (f"{arch}.expert_used_count", U32, l0["n_used"]),
            (f"{arch}.expert_count", U32, l0["n_expert"]),
            ("agention.trellis.state_bits", U32, 15)]
    if l0.get("expert_weights_scale", 0.0):
        meta.append((f"{arch}.expert_weights_scale", F32, l0["expert_weights_scale"]))
    if rotated:
        widths, values = [], []
        for key, width in (("gate_signs", l0["n_embd"]), ("down_signs", l0["n_ff"])):
            if l0.get(key) is not None:
                widths.append(width)
                values += [int(v) for v in l0[key]]
        meta += [("prism.hadamard.version", U32, 1), ("prism.hadamard.block_size", U32, 128),
                 ("prism.hadamard.transform", STR, "normalized-sylvester-walsh-hadamard"),
                 ("prism.hadamard.axis", STR, "input-last-dimension"),
                 ("prism.hadamard.sign_mode", STR, kw.pop("sign_mode", "explicit")),
                 ("prism.hadamard.weight_names", ARR, (STR, rotated)),
                 ("prism.hadamard.sign_widths", ARR, (I32, widths)),
                 ("prism.hadamard.sign_values", ARR, (I32, values))]
    write(path, meta, tensors, **kw)
