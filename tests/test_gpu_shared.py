"""GPU parity of a layer with its shared expert and sigmoid gate (gx_upload_shared), through the C
ABI, against the CPU oracle of src/engine.zig:520-653 (routed experts, then
out += sigmoid(gate_inp . x) * Down(silu(Gate x) * Up x)). The shared matrices are Q8_0, bf16 or
f32, the encodings the reference GPU engine multiplies them in (src/gpu_engine.zig:846-850).
Few-token calls take the CUDA-core shared-expert kernels, many-token calls the tensor-core grouped
GEMM with the Q8_0 / fp16 decoders. Tolerances: the north-star bound (relative RMS <= 1e-2, cosine
>= 0.9999) and the tighter bound each path holds."""
import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, metrics, synth

pytestmark = pytest.mark.gpu
REL_RMS, COSINE = 1e-2, 0.9999
DECODE_TIGHT = 2e-5        # decode path: exact Q8_0 / bf16 shared weights, f32 accumulation
PREFILL_TIGHT = 5e-3       # tensor-core path: f16 operands

torch = pytest.importorskip("torch")


def check(ref, got, tight):
    m = metrics.compare(ref, got)
    assert np.isfinite(got).all()
    assert m["rel_rms"] <= REL_RMS and m["cosine"] >= COSINE, m
    assert m["rel_rms"] <= tight, m
    return m


@pytest.fixture(scope="module")
def config0():
    """Config-0 routed layer (hidden 2048, 256 experts, F 512, top-8) with a Q8_0 shared expert of
    width 512 (the reference model's shared width equals its expert width, docs/MODEL.md:61-66)."""
    layer = synth.make_layer(0)
    layer["shared"] = synth.make_shared(1, E=2048, SF=512, type_id=abi.GX_Q8_0)
    return layer


@pytest.mark.parametrize("n_tok", [1, 3, 12, 100])
def test_config0_layer_with_q8_shared_expert(config0, n_tok):
    x = synth.tokens(600 + n_tok, n_tok)
    want, wids, ww = oracle.moe_ffn(config0, x)
    routed, _, _ = oracle.moe_ffn({k: v for k, v in config0.items() if k != "shared"}, x)
    assert metrics.compare(want, routed)["rel_rms"] > 0.05     # the shared term is not negligible
    with abi.Context(device=0, max_tokens=128, max_layers=1) as ctx:
        ctx.upload_layer(0, config0)
        got, ids, w = ctx.forward_host(0, x, want_routing=True)
        gb = ctx.forward_host(0, synth.bf16_bits(synth.bf16_round(x)), out_dtype=np.float32)
    assert metrics.topk_sets(wids, ids)["flips"] == 0
    tight = PREFILL_TIGHT if n_tok >= 64 else DECODE_TIGHT
    check(want, got, tight)
    want_b, _, _ = oracle.moe_ffn(config0, synth.bf16_round(x))
    check(want_b, gb, tight)


@pytest.mark.parametrize("sh_type,tight", [(abi.GX_BF16, DECODE_TIGHT), (abi.GX_F32, 5e-4)])
@pytest.mark.parametrize("n_tok", [5, 80])
def test_bf16_and_f32_shared_experts(sh_type, tight, n_tok):
    """bf16 matrices are stored as fp16 exactly; f32 ones are rounded to fp16 once on upload."""
    layer = synth.make_layer(610, n_expert=32, E=256, F=256, U=4)
    layer["shared"] = synth.make_shared(611, E=256, SF=256, type_id=sh_type)
    x = synth.tokens(612, n_tok, E=256)
    want, _, _ = oracle.moe_ffn(layer, x)
    with abi.Context(device=0, max_tokens=128, max_layers=1) as ctx:
        ctx.upload_layer(0, layer)
        got = ctx.forward_host(0, x)
    check(want, got, PREFILL_TIGHT if n_tok >= 64 else tight)


@pytest.mark.parametrize("n_tok", [2, 80])
def test_stack_with_shared_experts(n_tok):
    """Pre-norm stack (the shared expert sees RMSNorm(x) like the routed ones), graph replay."""
    layers = []
    for i in range(3):
        l = synth.make_layer(620 + i, n_expert=16, E=256, F=128, U=4)
        l["shared"] = synth.make_shared(630 + i, E=256, SF=256, type_id=abi.GX_Q8_0)
        layers.append(l)
    x = synth.tokens(640, n_tok, E=256) * 2.0
    ref = oracle.stack(layers, x)
    with abi.Context(device=0, max_tokens=128, max_layers=3) as ctx:
        for i, l in enumerate(layers):
            ctx.upload_layer(i, l)
        for _ in range(3):
            got = ctx.stack_forward_host(0, 3, x)
            check(ref, got, PREFILL_TIGHT if n_tok >= 64 else 5e-5)


def test_removing_the_shared_expert_and_noalloc_refusal():
    layer = synth.make_layer(650, n_expert=16, E=256, F=128, U=4)
    shared = synth.make_shared(651, E=256, SF=128, type_id=abi.GX_Q8_0)
    x = synth.tokens(652, 4, E=256)
    routed, _, _ = oracle.moe_ffn(layer, x)
    with abi.Context(device=0, max_tokens=16, max_layers=1) as ctx:
        ctx.upload_layer(0, layer)
        ctx.upload_shared(0, shared)
        xt = torch.from_numpy(x).cuda()
        yt = torch.empty_like(xt)
        with pytest.raises(abi.GxError) as e:
            ctx.forward_noalloc(0, xt, yt)
        assert e.value.code == -5
        ctx.upload_shared(0, None)
        check(routed, ctx.forward_host(0, x), DECODE_TIGHT)
        with pytest.raises(abi.GxError):
            ctx.upload_shared(0, dict(shared, n_ff=100))     # not a multiple of 128
