"""Pins the CPU oracle (the parity checker) before anything is checked against it.

Sources of truth, in order: the reference fixture tests/gyro_vectors.bin (regenerated here
byte-identically from the reference C decoder, SHA 8f739c3e...818c), the worked examples of
SPEC.md section 10, the unit tests of src/gyro.zig:197-238 and src/kernels.zig:384-419, and
(when the reference tree exists) the reference decoder itself compiled into oracle/_ref.
"""
import hashlib
import json
import struct
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from gyro_moe import synth

GOLDEN = Path(__file__).resolve().parent / "golden"


def read_vectors():
    data = (GOLDEN / "gyro_vectors.bin").read_bytes()
    assert hashlib.sha256(data).hexdigest() == json.loads((GOLDEN / "gyro_vectors.json").read_text())["sha256"]
    pos = 8
    assert data[:8] == b"GYROV1\0\0"
    (cases,) = struct.unpack_from("<I", data, pos)
    pos += 4
    blocks = []
    for _ in range(cases):
        type_id, size = struct.unpack_from("<II", data, pos)
        pos += 8
        raw = data[pos:pos + size]
        pos += size
        expected = np.frombuffer(data, dtype=np.uint32, count=128, offset=pos).copy()
        pos += 512
        blocks.append((type_id, raw, expected))
    (rotations,) = struct.unpack_from("<I", data, pos)
    pos += 4
    rots = []
    for _ in range(rotations):
        width, block = struct.unpack_from("<II", data, pos)
        pos += 8
        values = np.frombuffer(data, dtype=np.float32, count=width, offset=pos).copy()
        pos += 4 * width
        signs = np.frombuffer(data, dtype=np.int8, count=width, offset=pos).copy()
        pos += width
        rotated = np.frombuffer(data, dtype=np.uint32, count=width, offset=pos).copy()
        pos += 4 * width
        back = np.frombuffer(data, dtype=np.uint32, count=width, offset=pos).copy()
        pos += 4 * width
        rots.append((width, block, values, signs, rotated, back))
    assert pos == len(data)
    return blocks, rots


def test_fixture_is_the_reference_fixture():
    # tests/gyro_vectors.json:13 of the reference records this digest.
    digest = hashlib.sha256((GOLDEN / "gyro_vectors.bin").read_bytes()).hexdigest()
    assert digest == "8f739c3eb9cd3099ec7ccd1f46f60fb115cf2ec87d2ac6c373f2a49ed032818c"


def test_codebook_hash():
    # src/gyro.zig:197-202, SPEC.md section 4.
    digest = hashlib.sha256(oracle.CODEBOOK.read_bytes()).hexdigest()
    assert digest == "ee481f151d8947ce8b08817fdf89d0a56d647b6435ceb3df0f079ea748e0e588"


def test_oracle_decodes_fixture_bit_exact():
    blocks, _ = read_vectors()
    assert len(blocks) == 512
    for type_id, raw, expected in blocks:
        got = oracle.decode_row(type_id, raw, 128).view(np.uint32)
        assert np.array_equal(got, expected), type_id


def test_oracle_rotation_fixture_bit_exact():
    _, rots = read_vectors()
    assert [r[0] for r in rots] == [640, 2560]
    for width, block, values, signs, rotated, back in rots:
        r = oracle.rotate(values, block, signs)
        assert np.array_equal(r.view(np.uint32), rotated)
        u = oracle.rotate(r, block, signs, inverse=True)
        assert np.array_equal(u.view(np.uint32), back)


def test_spec_worked_examples():
    kats = json.loads((GOLDEN / "spec_kats.json").read_text())
    L = oracle.lib()
    for name in ("TQK4", "TQ2_T", "TQP5"):
        kat = kats[name]
        raw = bytes.fromhex(kat["bytes"])
        _, steps, bb = oracle.type_info(kat["type_id"])
        assert len(raw) == bb
        assert L.gxo_fp16_to_fp32(raw[0] | raw[1] << 8) == kat["d"]
        stream = raw[2:]
        decoded = oracle.decode_row(kat["type_id"], raw, 128)
        per = 2 if steps == 64 else 4
        for row in kat["rows"]:
            t = row["step"]
            s = L.gxo_state(kat["type_id"], stream, len(stream), t)
            assert s == row["state"], (name, t)
            assert s & 0x7FFF == row["masked"]
            h = (row["masked"] * 0x9E3779B1) & 0xFFFFFFFF
            idx = [h >> 21, (h >> 10) & 2047][:len(row["idx"])]
            assert idx == row["idx"], (name, t)
            np.testing.assert_allclose(decoded[t * per:(t + 1) * per], row["values"], atol=5.1e-7, rtol=0)
    rot = kats["rotation"]
    v = oracle.rotate(np.array(rot["input"], np.float32), rot["block"], np.array(rot["signs"], np.int8))
    assert v.tolist() == rot["rotated"]
    back = oracle.rotate(v, rot["block"], np.array(rot["signs"], np.int8), inverse=True)
    assert back.tolist() == rot["input"]


def test_fail_closed_lengths_and_types():
    # src/gyro.zig:204-214
    with pytest.raises(ValueError):
        oracle.type_info(35)
    src = bytes(34)
    with pytest.raises(ValueError, match="-2"):
        oracle.decode_row(144, src, 128, state_bits=-1)
    with pytest.raises(ValueError, match="-3"):
        oracle.decode_row(144, src, 128, state_bits=16)
    with pytest.raises(ValueError, match="-5"):
        oracle.decode_row(144, src[:33], 128)
    with pytest.raises(ValueError, match="-4"):
        oracle.decode_row(144, src, 127)
    assert oracle.lib().gxo_decode_row(35, 15, src, 34, None, 128) == -1


def test_binary16_edges():
    # src/gyro.zig:216-224
    f = oracle.lib().gxo_fp16_to_fp32
    bits = lambda v: struct.unpack("<I", struct.pack("<f", v))[0]
    assert bits(f(0)) == 0x00000000
    assert bits(f(0x8000)) == 0x80000000
    assert bits(f(1)) == 0x33800000
    assert bits(f(0x0400)) == 0x38800000
    assert f(0x7BFF) == 65504.0
    assert np.isinf(f(0x7C00))
    assert np.isnan(f(0x7E00))
    # every pattern against numpy's exact conversion
    allh = np.arange(65536, dtype=np.uint32)
    ref = allh.astype(np.uint16).view(np.float16).astype(np.float32)
    got = np.array([f(int(h)) for h in allh[::37]], np.float32)
    finite = np.isfinite(ref[::37])
    assert np.array_equal(got[finite].view(np.uint32), ref[::37][finite].view(np.uint32))


def test_rotation_invalid_signs_leave_values():
    # src/gyro.zig:226-238
    with pytest.raises(ValueError, match="-1"):
        oracle.rotate(np.array([1, 2, 3, 4], np.float32), 3, None)
    with pytest.raises(ValueError, match="-7"):
        oracle.rotate(np.array([1, 2, 3, 4], np.float32), 4, np.array([1, -1, 0, 1], np.int8))


@pytest.mark.parametrize("type_id", sorted(synth.BLOCK_BYTES))
def test_oracle_matches_reference_decoder(type_id):
    """Random blocks and random finite scales through both decoders (needs oracle/_ref)."""
    ref = oracle.ref_lib()
    if ref is None:
        pytest.skip("reference decoder not built (needs the reference tree)")
    import ctypes
    rng = np.random.default_rng(type_id)
    bb = synth.BLOCK_BYTES[type_id]
    raw = bytearray(rng.bytes(bb * 256))
    for b in range(256):
        d = int(rng.integers(0, 65536))
        while d & 0x7C00 == 0x7C00:
            d = int(rng.integers(0, 65536))
        raw[b * bb:b * bb + 2] = struct.pack("<H", d)
    n = 256 * 128
    want = np.empty(n, np.float32)
    assert ref.tq_dequantize_row(type_id, bytes(raw), want.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n) == 0
    got = oracle.decode_row(type_id, bytes(raw), n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("type_id", sorted(synth.BLOCK_BYTES))
def test_fused_dot_matches_strict_decode(type_id):
    # src/kernels.zig:384-403: scale 0.03125, two blocks, tolerance 1e-4.
    rng = np.random.default_rng(7)
    bb = synth.BLOCK_BYTES[type_id]
    raw = bytearray(rng.bytes(2 * bb))
    for b in range(2):
        raw[b * bb:b * bb + 2] = struct.pack("<H", synth.fp16_bits(0.03125))
    ref = oracle.decode_row(type_id, bytes(raw), 256)
    x = (rng.random(256, dtype=np.float32) - 0.5).astype(np.float32)
    want = float(np.dot(ref.astype(np.float64), x.astype(np.float64)))
    got = oracle.lib().gxo_dot_row(type_id, bytes(raw), x.ctypes.data_as(oracle._F32P), 256)
    assert abs(got - want) <= 1e-4


def test_topk_ties_prefer_lower_index():
    import ctypes
    v = np.array([0.1, 0.5, 0.5, 0.2, 0.5, 0.0], np.float32)
    ids = np.empty(3, np.uint32)
    w = np.empty(3, np.float32)
    oracle.lib().gxo_topk(v.ctypes.data_as(oracle._F32P), 6, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
                          w.ctypes.data_as(oracle._F32P), 3)
    assert ids.tolist() == [1, 2, 4]


def test_layer_matches_frozen_fixture():
    from layer_case import small_layer
    gold = json.loads((GOLDEN / "layer_small.json").read_text())
    layer, x = small_layer()
    assert layer["sha256"] == gold["inputs_sha256"]
    out, ids, w = oracle.moe_ffn(layer, x)
    assert ids.tolist() == gold["ids"]
    np.testing.assert_allclose(w, gold["weights"], rtol=1e-6, atol=0)
    np.testing.assert_allclose(out, gold["out"], rtol=1e-5, atol=1e-6)


def test_layer_properties_and_threaded_build():
    from layer_case import small_layer
    layer, x = small_layer(seed=3, n_tok=7)
    out, ids, w = oracle.moe_ffn(layer, x)
    assert all(len(set(r)) == len(r) for r in ids.tolist())
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-5)
    assert np.all(np.diff(w, axis=1) <= 0)
    fast, fids, fw = oracle.moe_ffn(layer, x, threads=4, fast=True)
    assert np.array_equal(fids, ids)
    rel = np.sqrt(((fast - out) ** 2).sum() / (out ** 2).sum())
    assert rel < 1e-5


def test_layer_dense_definition():
    """The layer equals its dense definition: decode every weight strictly, unrotate nothing,
    rotate x and the SwiGLU output, accumulate in float64."""
    from layer_case import small_layer
    layer, x = small_layer(seed=5, n_tok=3)
    out, ids, w = oracle.moe_ffn(layer, x)
    E, F, NE = layer["n_embd"], layer["n_ff"], layer["n_expert"]
    dec = lambda m, cols: np.stack([oracle.decode_row(layer["type_id"], r.tobytes(), cols) for r in m])
    G = dec(layer["gate"], E).reshape(NE, F, E).astype(np.float64)
    Up = dec(layer["up"], E).reshape(NE, F, E).astype(np.float64)
    D = dec(layer["down"], F).reshape(NE, E, F).astype(np.float64)

    def fwht(v):
        v = v.reshape(-1, 128).astype(np.float64).copy()
        h = 1
        while h < 128:
            v = v.reshape(-1, 128 // (2 * h), 2, h)
            a, b = v[:, :, 0, :].copy(), v[:, :, 1, :].copy()
            v[:, :, 0, :], v[:, :, 1, :] = a + b, a - b
            h *= 2
        return (v.reshape(-1) / np.sqrt(128))

    for t in range(x.shape[0]):
        xh = fwht(x[t] * layer["gate_signs"])
        acc = np.zeros(E)
        for k in range(layer["n_used"]):
            e = ids[t, k]
            g, u = G[e] @ xh, Up[e] @ xh
            a = fwht(g / (1 + np.exp(-g)) * u * layer["down_signs"])
            acc += w[t, k] * (D[e] @ a)
        rel = np.sqrt(((acc - out[t]) ** 2).sum() / (acc ** 2).sum())
        assert rel < 1e-5


@pytest.mark.parametrize("type_id", [0, 8, 30])
def test_shared_expert_matches_dense_definition(type_id):
    """src/engine.zig:644-653 with the Q8_0 / bf16 / f32 dots of src/kernels.zig:72-120, against a
    float64 numpy restatement of the same definition."""
    layer = synth.make_layer(5, n_expert=16, E=256, F=128, U=4)
    x = synth.tokens(6, 3, E=256)
    sh = synth.make_shared(9, E=256, SF=128, type_id=type_id)
    base, _, _ = oracle.moe_ffn(layer, x)
    out, _, _ = oracle.moe_ffn(dict(layer, shared=sh), x)

    def dense(m, rows, cols):
        if type_id == 8:
            b = m.reshape(rows, cols // 32, 34)
            d = b[:, :, :2].copy().view(np.float16).astype(np.float64)
            q = b[:, :, 2:].view(np.int8).astype(np.float64)
            return (d * q).reshape(rows, cols)
        if type_id == 30:
            return (m.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(rows, cols).astype(np.float64)
        return m.view(np.float32).reshape(rows, cols).astype(np.float64)

    xd = x.astype(np.float64)
    g, u = xd @ dense(sh["gate"], 128, 256).T, xd @ dense(sh["up"], 128, 256).T
    y = (g / (1 + np.exp(-g)) * u) @ dense(sh["down"], 256, 128).T
    gate = 1 / (1 + np.exp(-(xd @ sh["gate_inp"].astype(np.float64))))
    np.testing.assert_allclose(out, base + y * gate[:, None], rtol=1e-5, atol=1e-5)


def dense_f64(m: np.ndarray, type_id: int, rows: int, cols: int) -> np.ndarray:
    """Plain matrix bytes (Q8_0 / bf16 / f32 rows) as float64 values."""
    if type_id == 8:
        b = m.reshape(rows, cols // 32, 34)
        d = b[:, :, :2].copy().view(np.float16).astype(np.float64)
        q = b[:, :, 2:].view(np.int8).astype(np.float64)
        return (d * q).reshape(rows, cols)
    if type_id == 30:
        return (m.view(np.uint16).astype(np.uint32) << 16).view(np.float32).reshape(rows, cols).astype(np.float64)
    return m.view(np.float32).reshape(rows, cols).astype(np.float64)


@pytest.mark.parametrize("type_id", [0, 8, 30])
def test_hc_mixer_matches_dense_definition(type_id):
    """hcMix and hcCombine (src/engine.zig:184-228) against a float64 numpy restatement: per-stream
    RMSNorm with the stream's weight, lo = silu(Down xn / hc), cur = mean_c xn_c sigmoid((Up lo)_c),
    inject = Inject xn, res_c += y 2 sigmoid(inject_c / hc). Rank 320 as in the reference model."""
    E, H, R = 256, 4, 320
    hc = synth.make_hc(11, E=E, n_streams=H, rank=R, type_id=type_id)
    res = np.random.default_rng(12).standard_normal((5, H * E)).astype(np.float32) * 3.0
    cur, inj = oracle.hc_mix(hc, res)
    r = res.astype(np.float64).reshape(5, H, E)
    xn = r / np.sqrt((r ** 2).mean(axis=2, keepdims=True) + hc["eps"]) * hc["norm"].reshape(H, E)
    xn = xn.reshape(5, H * E)
    lo = xn @ dense_f64(hc["down"], type_id, R, H * E).T / H
    lo = lo / (1 + np.exp(-lo))
    gate = lo @ dense_f64(hc["up"], type_id, H * E, R).T
    want = (xn * (1 / (1 + np.exp(-gate)))).reshape(5, H, E).mean(axis=1)
    np.testing.assert_allclose(cur, want, rtol=2e-5, atol=2e-5)
    want_inj = xn @ dense_f64(hc["inject"], type_id, H, H * E).T
    np.testing.assert_allclose(inj, want_inj, rtol=2e-5, atol=2e-5)
    y = np.random.default_rng(13).standard_normal((5, E)).astype(np.float32)
    got = oracle.hc_combine(hc, res, y, inj)
    w = 2 / (1 + np.exp(-inj.astype(np.float64) / H))
    want_res = r + y.astype(np.float64)[:, None, :] * w[:, :, None]
    np.testing.assert_allclose(got, want_res.reshape(5, H * E), rtol=1e-6, atol=1e-6)


def test_ffn_block_is_mix_layer_combine():
    layer = synth.make_layer(14, n_expert=16, E=256, F=128, U=4)
    layer["shared"] = synth.make_shared(15, E=256, SF=128)
    hc = synth.make_hc(16, E=256, n_streams=4, rank=128)
    res = np.random.default_rng(17).standard_normal((3, 1024)).astype(np.float32)
    cur, inj = oracle.hc_mix(hc, res)
    y, _, _ = oracle.moe_ffn(layer, cur)
    np.testing.assert_array_equal(oracle.ffn_block(layer, hc, res), oracle.hc_combine(hc, res, y, inj))
    with pytest.raises(RuntimeError):
        oracle.hc_mix(dict(hc, rank=0), res)
