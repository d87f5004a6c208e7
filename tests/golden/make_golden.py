#!/usr/bin/env python3
"""Regenerates the committed golden fixtures under tests/golden/.

Needs the reference tree (mattneel/gyro-dx) at /root/reference (or $GYRO_REFERENCE); the GPU
machines do not have it, which is why the outputs are committed.

1. gyro_vectors.bin / .json — decoder and rotation fixture. The reference's C decoder
   (third_party/agention-gyro/src/tq_ref.c, built from the reference tree into oracle/_ref by
   oracle/Makefile) is driven through the fixture recipe of the reference's
   tests/gyro_vectors_generate.py:21-68 (same seed 0x4759524F, Python `random` draws, the 12
   edge scales, widths 640 and 2560, the GYROV1 record layout). The result must be
   byte-identical to the reference's own tests/gyro_vectors.bin: its SHA-256 must equal the
   value recorded in tests/gyro_vectors.json:13 (8f739c3e...818c). The script aborts otherwise.
2. spec_kats.json — the worked examples of third_party/agention-gyro/SPEC.md section 10
   (TQK4 d=1.0, TQ2_T d=0.5, TQP5 d=-2.0, rotation (1,2,3,4)), parsed from the SPEC text.
3. layer_small.json — one small routed layer (seeded inputs from tests/layer_case.py) through
   the strict CPU oracle, so GPU tests can check against frozen numbers as well as the live
   oracle.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import random
import re
import struct
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

REFERENCE = Path(os.environ.get("GYRO_REFERENCE", "/root/reference"))
TYPES = [(144, 34), (145, 26), (146, 30), (147, 42), (148, 50), (149, 58), (150, 22), (151, 18)]
SEED = 0x4759524F
EDGE_SCALES = [0x0000, 0x8000, 0x0001, 0x8001, 0x03FF, 0x83FF, 0x0400, 0x8400, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF]
REFERENCE_SHA = "8f739c3eb9cd3099ec7ccd1f46f60fb115cf2ec87d2ac6c373f2a49ed032818c"


def make_vectors(ref) -> bytes:
    """Fixture recipe of tests/gyro_vectors_generate.py:21-68, driven through the reference C
    decoder. Record layout: b'GYROV1\\0\\0', u32 cases, then per case (u32 type, u32 size,
    size packed bytes, 128 f32), then u32 rotations, per rotation (u32 width, u32 block,
    width f32 input, width i8 signs, width f32 rotated, width f32 unrotated)."""
    rng = random.Random(SEED)
    out = bytearray(b"GYROV1\0\0" + struct.pack("<I", len(TYPES) * 64))
    for type_id, size in TYPES:
        for case in range(64):
            scale = EDGE_SCALES[case] if case < len(EDGE_SCALES) else rng.randrange(65536)
            while scale & 0x7C00 == 0x7C00:
                scale = rng.randrange(65536)
            raw = struct.pack("<H", scale) + bytes(rng.randrange(256) for _ in range(size - 2))
            packed = ctypes.create_string_buffer(raw)
            decoded = (ctypes.c_float * 128)()
            if ref.tq_dequantize_row(type_id, packed, decoded, 128) != 0:
                raise RuntimeError("reference decoder rejected a valid block")
            out += struct.pack("<II", type_id, size) + raw + struct.pack("<128f", *decoded)
    out += struct.pack("<I", 2)
    for width in (640, 2560):
        source = [rng.uniform(-2.0, 2.0) for _ in range(width)]
        values = (ctypes.c_float * width)(*source)
        signs = (ctypes.c_int8 * width)(*(rng.choice([-1, 1]) for _ in range(width)))
        out += struct.pack("<II", width, 128) + struct.pack(f"<{width}f", *values)
        out += bytes(s & 255 for s in signs)
        if ref.tq_hadamard_rotate(values, width, 128, signs) != 0:
            raise RuntimeError("reference rotate failed")
        out += struct.pack(f"<{width}f", *values)
        if ref.tq_hadamard_unrotate(values, width, 128, signs) != 0:
            raise RuntimeError("reference unrotate failed")
        out += struct.pack(f"<{width}f", *values)
    return bytes(out)


def parse_spec_kats(spec: str) -> dict:
    """SPEC.md section 10: block bytes and the per-step tables (state, idx0, idx1, values)."""
    kats = {}
    sections = re.split(r"^### ", spec, flags=re.M)
    for sec in sections:
        m = re.match(r"10\.(\d) (\S+) block, d = (-?[0-9.]+)", sec)
        if not m:
            continue
        name = m.group(2)
        type_id = {"TQK4": 151, "TQ2_T": 144, "TQP5": 147}[name]
        blocks = re.findall(r"```\n(.*?)```", sec, flags=re.S)
        byte_text = blocks[0]
        hexes = re.findall(r"\b[0-9a-f]{2}\b", byte_text.split("\\")[0] if name == "TQK4" else byte_text)
        raw = bytes(int(h, 16) for h in hexes)
        rows = []
        for line in blocks[1].splitlines():
            parts = line.split()
            if not parts or not parts[0].isdigit():
                continue
            step = int(parts[0])
            state = int(parts[1], 16)
            masked = int(parts[2], 16)
            if type_id == 147:
                idx = [int(parts[3])]
                vals = [float(v) for v in parts[4:6]]
            else:
                idx = [int(parts[3]), int(parts[4])]
                vals = [float(v) for v in parts[5:9]]
            rows.append({"step": step, "state": state, "masked": masked, "idx": idx, "values": vals})
        kats[name] = {"type_id": type_id, "d": float(m.group(3)), "bytes": raw.hex(), "rows": rows}
    rot = {"block": 4, "signs": [1, -1, 1, 1], "input": [1.0, 2.0, 3.0, 4.0], "rotated": [3.0, 1.0, -4.0, 2.0]}
    if "H_4 (s ⊙ v) = (1-2+3+4, 1+2+3-4, 1-2-3-4, 1+2-3+4) / 2 = (3, 1, -4, 2)" not in spec:
        raise RuntimeError("SPEC rotation example not found")
    kats["rotation"] = rot
    return kats


def main() -> None:
    from oracle import oracle

    oracle.build()
    ref = oracle.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libtq_ref.so missing: the reference tree is needed")
    data = make_vectors(ref)
    sha = hashlib.sha256(data).hexdigest()
    ref_fixture = REFERENCE / "tests" / "gyro_vectors.bin"
    if sha != REFERENCE_SHA or (ref_fixture.exists() and ref_fixture.read_bytes() != data):
        raise SystemExit(f"fixture mismatch: {sha}")
    (HERE / "gyro_vectors.bin").write_bytes(data)
    (HERE / "gyro_vectors.json").write_text(json.dumps({
        "source": "reference C decoder tq_ref.c (oracle/_ref) through the recipe of "
                  "tests/gyro_vectors_generate.py:21-68",
        "seed": SEED, "decode_cases": 512, "decoded_values": 65536, "rotation_widths": [640, 2560],
        "sha256": sha, "identical_to_reference_fixture": True}, indent=2) + "\n")

    spec = (REFERENCE / "third_party" / "agention-gyro" / "SPEC.md").read_text()
    kats = parse_spec_kats(spec)
    (HERE / "spec_kats.json").write_text(json.dumps(kats, indent=1) + "\n")

    import numpy as np
    from layer_case import small_layer

    layer, x = small_layer()
    out, ids, w = oracle.moe_ffn(layer, x)
    (HERE / "layer_small.json").write_text(json.dumps({
        "case": "tests/layer_case.py small_layer()", "inputs_sha256": layer["sha256"],
        "ids": ids.tolist(), "weights": [[float(v) for v in r] for r in w],
        "out": [[float(v) for v in r] for r in out]}) + "\n")
    print("fixtures written:", sha, {k: len(v.get("rows", [])) for k, v in kats.items()})


if __name__ == "__main__":
    main()
