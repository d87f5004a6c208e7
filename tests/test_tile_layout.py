"""CPU check of the HBM tile layout and the mma fragment K-permutation (no GPU needed).

tests/tile_emu.cpp compiles the kernels' own header (gyro-dx_b200/csrc/gx_tile.h) with g++ and
emulates one warp: repack -> per-lane run load -> trellis state/hash -> B fragments, times A
fragments of up to 8 tokens split into fp16 hi/lo. The result must equal the dense product of
the strictly decoded weights (CPU oracle) with the tokens.
"""
import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from gyro_moe import synth

HERE = Path(__file__).resolve().parent


@pytest.fixture(scope="module")
def emu(tmp_path_factory):
    so = tmp_path_factory.mktemp("emu") / "libtile_emu.so"
    subprocess.run(["g++", "-std=c++17", "-O1", "-fPIC", "-shared", str(HERE / "tile_emu.cpp"), "-o", str(so)],
                   check=True)
    lib = ctypes.CDLL(str(so))
    lib.emu_tile_gemv.argtypes = [ctypes.c_uint32, ctypes.c_int] + [ctypes.c_void_p] * 3 + [ctypes.c_int] + \
        [ctypes.c_void_p] * 3
    return lib


@pytest.mark.parametrize("type_id", sorted(synth.BLOCK_BYTES))
@pytest.mark.parametrize("ntok", [1, 3, 8])
def test_warp_emulation_matches_dense(emu, type_id, ntok):
    rng = np.random.default_rng(type_id * 10 + ntok)
    NB = 3
    raw = synth.packed_matrix(rng, type_id, 8, NB * 128, scale=None)
    # random finite scales per block to exercise the scale placement
    for r in range(8):
        for b in range(NB):
            d = synth.fp16_bits(float(rng.uniform(-0.2, 0.2)))
            off = b * synth.BLOCK_BYTES[type_id]
            raw[r, off], raw[r, off + 1] = d & 0xFF, d >> 8
    x = rng.standard_normal((ntok, NB * 128)).astype(np.float32)
    xhi = x.astype(np.float16)
    xlo = (x - xhi.astype(np.float32)).astype(np.float16)
    cb = np.frombuffer(oracle.CODEBOOK.read_bytes(), dtype=np.uint16)
    out = np.zeros((ntok, 8), np.float64)
    tiles = np.zeros(NB * 8 * synth.BLOCK_BYTES[type_id], np.uint8)
    raw = np.ascontiguousarray(raw)
    rc = emu.emu_tile_gemv(type_id, NB, raw.ctypes.data, xhi.view(np.uint16).ctypes.data,
                           xlo.view(np.uint16).ctypes.data, ntok, cb.ctypes.data, out.ctypes.data, tiles.ctypes.data)
    assert rc == 0
    W = np.stack([oracle.decode_row(type_id, raw[r].tobytes(), NB * 128) for r in range(8)]).astype(np.float64)
    want = x.astype(np.float64) @ W.T
    np.testing.assert_allclose(out, want, rtol=2e-6, atol=2e-6 * np.abs(want).max())
    # the tile layout is a permutation of the block bytes: nothing lost, nothing padded
    assert sorted(tiles.tolist()) == sorted(raw.reshape(-1).tolist())
