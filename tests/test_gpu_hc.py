"""GPU parity of the FFN block with its hyper-connection mixer (gx_upload_hc, gx_ffn_block), through
the C ABI, against the CPU oracle of src/engine.zig:162-165 (hcMix, the routed + shared experts,
hcCombine; src/engine.zig:184-228, :520-653). res [n, hc*E] is updated in place.

Two comparisons per case. (1) The mixer's output (the hc_mixed observation, returned through
gx_ffn_block's `mixed`) against oracle.hc_mix. (2) The block's increment res' - res against the
oracle's block run on the GPU's own mixer output: routing is recomputed from that output, and a
token whose U-th and (U+1)-th router logits lie closer than the mixer's rounding may select
another expert set from an input that differs in the 4th digit, so the increment is checked on
the same input the GPU routed (with the oracle's injection logits). Tolerances: the north-star
bound (relative RMS <= 1e-2, cosine >= 0.9999) and the tighter bound each path holds."""
import os

import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, metrics, synth

pytestmark = pytest.mark.gpu
REL_RMS, COSINE = 1e-2, 0.9999
DECODE_TIGHT = 5e-5        # CUDA-core mixer and experts, f32 accumulation
PREFILL_TIGHT = 5e-3       # tensor-core mixer and experts: f16 operands
MIX_TIGHT = {DECODE_TIGHT: 2e-5, PREFILL_TIGHT: 2e-3}

THREADS = min(16, os.cpu_count() or 1)

torch = pytest.importorskip("torch")


def run_block(layer, hc, res, max_tokens=256):
    with abi.Context(device=0, max_tokens=max_tokens, max_layers=1) as ctx:
        ctx.upload_layer(0, layer)
        ctx.upload_hc(0, hc)
        rt = torch.from_numpy(res).cuda()
        mixed = torch.empty(res.shape[0], hc["n_embd"], device="cuda")
        ctx.wait(ctx.ffn_block(0, rt, mixed=mixed))
        return rt.cpu().numpy(), mixed.cpu().numpy()


def check(ref, got, tight):
    m = metrics.compare(ref, got)
    assert np.isfinite(got).all()
    assert m["rel_rms"] <= REL_RMS and m["cosine"] >= COSINE, m
    assert m["rel_rms"] <= tight, m
    return m


def check_block(layer, hc, res, tight):
    got, mixed = run_block(layer, hc, res)
    cur, inj = oracle.hc_mix(hc, res, threads=THREADS)
    check(cur, mixed, MIX_TIGHT[tight])
    y, _, _ = oracle.moe_ffn(layer, mixed, threads=THREADS)
    want = oracle.hc_combine(hc, res, y, inj)
    return check(want - res, got - res, tight)


@pytest.fixture(scope="module")
def config0_block():
    """Config-0 routed layer (hidden 2048, 256 experts, F 512, top-8) with a Q8_0 shared expert and a
    Q8_0 mixer of 4 streams at the reference model's rank 320."""
    layer = synth.make_layer(0)
    layer["shared"] = synth.make_shared(1, E=2048, SF=512, type_id=abi.GX_Q8_0)
    return layer, synth.make_hc(2, E=2048, n_streams=4, rank=320)


@pytest.mark.parametrize("n_tok", [1, 4, 13, 64, 150])
def test_config0_ffn_block(config0_block, n_tok):
    layer, hc = config0_block
    res = np.random.default_rng(700 + n_tok).standard_normal((n_tok, 4 * 2048)).astype(np.float32) * 2.0
    check_block(layer, hc, res, PREFILL_TIGHT if n_tok >= 64 else DECODE_TIGHT)


@pytest.mark.parametrize("hc_type", [abi.GX_BF16, abi.GX_F32])
@pytest.mark.parametrize("n_tok", [3, 96])
def test_bf16_and_f32_mixers(hc_type, n_tok):
    """bf16 mixer weights are stored as fp16 exactly; f32 ones are rounded to fp16 once on upload."""
    layer = synth.make_layer(710, n_expert=32, E=256, F=256, U=4)
    hc = synth.make_hc(711, E=256, n_streams=2, rank=128, type_id=hc_type)
    res = np.random.default_rng(712).standard_normal((n_tok, 512)).astype(np.float32)
    tight = PREFILL_TIGHT if n_tok >= 64 or hc_type == abi.GX_F32 else DECODE_TIGHT
    check_block(layer, hc, res, tight)


@pytest.mark.parametrize("n_tok", [2, 80])
def test_reference_model_shape(n_tok):
    """The reference model's FFN block widths (hidden 2560, 256 experts of 640, top-10, shared
    expert 640, 4 streams of rank 320)."""
    layer = synth.make_layer(720, n_expert=256, E=2560, F=640, U=10)
    layer["shared"] = synth.make_shared(721, E=2560, SF=640, type_id=abi.GX_Q8_0)
    hc = synth.make_hc(722, E=2560, n_streams=4, rank=320)
    res = np.random.default_rng(723).standard_normal((n_tok, 4 * 2560)).astype(np.float32)
    check_block(layer, hc, res, PREFILL_TIGHT if n_tok >= 64 else DECODE_TIGHT)


def test_repeated_blocks_and_errors():
    """Three blocks in a row on the same streams (the residual grows), against the oracle applied
    three times; a block without a mixer, a misaligned res and an odd rank are refused."""
    layer = synth.make_layer(730, n_expert=16, E=256, F=128, U=4)
    hc = synth.make_hc(731, E=256, n_streams=4, rank=128)
    res = np.random.default_rng(732).standard_normal((6, 1024)).astype(np.float32)
    want = res
    for _ in range(3):
        want = oracle.ffn_block(layer, hc, want)
    with abi.Context(device=0, max_tokens=16, max_layers=1) as ctx:
        ctx.upload_layer(0, layer)
        rt = torch.from_numpy(res).cuda()
        with pytest.raises(abi.GxError) as e:
            ctx.ffn_block(0, rt)
        assert e.value.code == -6
        with pytest.raises(abi.GxError):
            ctx.upload_hc(0, dict(hc, rank=96))
        ctx.upload_hc(0, hc)
        for _ in range(3):
            ctx.ffn_block(0, rt)
        ctx.wait(ctx.ffn_block(0, rt, n_tok=0))
        got = rt.cpu().numpy()
        big = torch.zeros(6 * 1024 + 1, device="cuda")
        with pytest.raises(abi.GxError):
            ctx.ffn_block(0, big[1:].view(6, 1024))
        ctx.upload_hc(0, None)
        with pytest.raises(abi.GxError):
            ctx.ffn_block(0, rt)
    m = metrics.compare(want - res, got - res)
    assert m["rel_rms"] <= DECODE_TIGHT, m
