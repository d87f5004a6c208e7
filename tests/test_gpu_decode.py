"""GPU conformance of the Gyro decoder through the C ABI (gx_decode_blocks, the replacement of
gd_validate_gyro, native/gyro_native.cpp:597-730): every fixture block of the reference bit for
bit, random blocks of all eight types against the CPU oracle, and the argument rules."""
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, synth
from test_oracle import read_vectors

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def ctx():
    with abi.Context(device=0, max_tokens=16, max_layers=1) as c:
        yield c


def test_fixture_blocks_bit_exact(ctx):
    blocks, _ = read_vectors()
    for type_id in sorted(synth.BLOCK_BYTES):
        mine = [(raw, exp) for t, raw, exp in blocks if t == type_id]
        packed = b"".join(raw for raw, _ in mine)
        expected = np.concatenate([exp for _, exp in mine]).view(np.float32)
        rc, out, err = ctx.decode_blocks(type_id, packed, 128 * len(mine), expected)
        assert rc == 0, (type_id, err)
        assert np.array_equal(out.view(np.uint32), expected.view(np.uint32))


@pytest.mark.parametrize("type_id", sorted(synth.BLOCK_BYTES))
def test_random_blocks_match_oracle(ctx, type_id):
    rng = np.random.default_rng(100 + type_id)
    bb = synth.BLOCK_BYTES[type_id]
    n_blocks = 4096
    raw = bytearray(rng.bytes(bb * n_blocks))
    for b in range(n_blocks):
        d = int(rng.integers(0, 65536))
        while d & 0x7C00 == 0x7C00:
            d = int(rng.integers(0, 65536))
        raw[b * bb:b * bb + 2] = struct.pack("<H", d)
    want = oracle.decode_row(type_id, bytes(raw), 128 * n_blocks)
    rc, out, _ = ctx.decode_blocks(type_id, bytes(raw), 128 * n_blocks, want)
    assert rc == 0
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def test_spec_worked_examples_on_gpu(ctx):
    kats = json.loads((GOLDEN / "spec_kats.json").read_text())
    for name in ("TQK4", "TQ2_T", "TQP5"):
        kat = kats[name]
        raw = bytes.fromhex(kat["bytes"])
        rc, out, _ = ctx.decode_blocks(kat["type_id"], raw, 128)
        assert rc == 0
        per = 2 if kat["type_id"] == 147 else 4
        for row in kat["rows"]:
            t = row["step"]
            np.testing.assert_allclose(out[t * per:(t + 1) * per], row["values"], atol=5.1e-7, rtol=0)


def test_mismatch_is_reported(ctx):
    blocks, _ = read_vectors()
    type_id, raw, exp = blocks[20]
    wrong = exp.view(np.float32).copy()
    wrong[5] = np.nextafter(wrong[5], np.float32(np.inf))
    rc, _, err = ctx.decode_blocks(type_id, raw, 128, wrong)
    assert rc == -7 and err > 0


def test_argument_rules(ctx):
    # native/gyro_native.cpp:601-607: multiple of 128, positive, <= 2^24, exact byte count, known type
    lib, h = ctx.lib, ctx.handle
    buf = np.zeros(34 * 2, np.uint8)
    out = np.zeros(256, np.float32)
    import ctypes
    err = ctypes.c_float()
    assert lib.gx_decode_blocks(h, 144, buf.ctypes.data, 68, out.ctypes.data, 0, None, ctypes.byref(err), 1000) == -1
    assert lib.gx_decode_blocks(h, 144, buf.ctypes.data, 68, out.ctypes.data, 200, None, ctypes.byref(err), 1000) == -1
    assert lib.gx_decode_blocks(h, 144, buf.ctypes.data, 67, out.ctypes.data, 256, None, ctypes.byref(err), 1000) == -1
    assert lib.gx_decode_blocks(h, 35, buf.ctypes.data, 68, out.ctypes.data, 256, None, ctypes.byref(err), 1000) == -1
    assert lib.gx_decode_blocks(h, 144, buf.ctypes.data, 68, out.ctypes.data, 256, None, ctypes.byref(err), 1000) == 0
