"""Range of the f16 operands on the GPU paths, through the C ABI.

The tensor-core path (64 tokens and more) feeds the MMAs f16 rotated tokens and f16 down operands,
and the decode path splits activations into f16 hi/lo halves; the CPU engine keeps everything in
f32 (src/engine.zig:547-641). Relative f16 precision does not depend on scale while values stay
normal (2^-14 .. 65504), so large but representable activations (x 16) must match the oracle at the
tight tolerances the paths hold at unit scale. Small ones (x 0.01) reach f16 subnormals in the
SwiGLU products (which scale as x^2) and hold the north-star tolerance only. Activations whose f16
image would overflow must not come back as Inf: every layer-output writer checks its values, and
the call returns GX_E_RANGE; the context stays usable afterwards."""
import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, metrics, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
REL_RMS, COSINE = 1e-2, 0.9999          # north-star layer tolerance
TIGHT = {"prefill": 5e-3, "decode": 2e-5}


@pytest.fixture(scope="module")
def setup():
    layer = synth.make_layer(77, n_expert=32, E=256, F=128, U=4)
    with abi.Context(device=0, max_tokens=256, max_layers=1) as c:
        c.upload_layer(0, layer)
        yield c, layer


@pytest.mark.parametrize("path,n_tok", [("decode", 5), ("prefill", 160)])
@pytest.mark.parametrize("scale", [16.0, 0.01])
def test_scaled_activations_match_oracle(setup, path, n_tok, scale):
    ctx, layer = setup
    x = synth.tokens(91, n_tok, E=256) * np.float32(scale)
    want, wids, _ = oracle.moe_ffn(layer, x)
    got, ids, _ = ctx.forward_host(0, x, want_routing=True)
    assert metrics.topk_sets(wids, ids)["flips"] == 0
    m = metrics.compare(want, got)
    assert m["rel_rms"] <= REL_RMS and m["cosine"] >= COSINE, m
    if scale >= 1.0:
        assert m["rel_rms"] <= TIGHT[path], m


@pytest.mark.parametrize("path,n_tok", [("decode", 5), ("prefill", 160)])
def test_overflow_is_reported_not_returned(setup, path, n_tok):
    ctx, layer = setup
    # x ~ N(0, 4096^2): the SwiGLU products reach ~1e7, beyond f16 (65504)
    x = synth.tokens(92, n_tok, E=256) * np.float32(4096.0)
    with pytest.raises(abi.GxError) as e:
        ctx.forward_host(0, x)
    assert e.value.code == -10                               # GX_E_RANGE
    # an input holding Inf is reported the same way
    x = synth.tokens(93, n_tok, E=256)
    x[n_tok // 2, 7] = np.inf
    with pytest.raises(abi.GxError) as e:
        ctx.forward_host(0, x)
    assert e.value.code == -10
    # the context stays usable: a normal call afterwards matches the oracle
    x = synth.tokens(94, n_tok, E=256)
    want, _, _ = oracle.moe_ffn(layer, x)
    got, _, _ = ctx.forward_host(0, x, want_routing=True)
    m = metrics.compare(want, got)
    assert m["rel_rms"] <= TIGHT[path], m
