"""Layers loaded from a GGUF file (gx_upload_layer_gguf) give the same results as the same layers
uploaded from host arrays (gx_upload_layer + gx_upload_shared), and match the CPU oracle; the file is
written like the reference model file (tests/gguf_file.py)."""
import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, metrics, synth
import gguf_file

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def check(ref, got, tight):
    m = metrics.compare(ref, got)
    assert m["rel_rms"] <= 1e-2 and m["cosine"] >= 0.9999 and m["rel_rms"] <= tight, m


@pytest.mark.parametrize("n_tok,tight", [(3, 2e-5), (100, 5e-3)])
def test_gguf_layers_match_host_upload_and_oracle(tmp_path, n_tok, tight):
    layers = [synth.make_layer(0, U=8), synth.make_layer(1, U=8)]
    layers[1]["gate_signs"], layers[1]["down_signs"] = layers[0]["gate_signs"], layers[0]["down_signs"]
    layers[1]["shared"] = synth.make_shared(2, E=2048, SF=512, type_id=abi.GX_Q8_0)
    path = tmp_path / "model.gguf"
    gguf_file.model_file(path, layers)
    x = synth.tokens(3, n_tok)
    with abi.Context(device=0, max_tokens=128, max_layers=4) as ctx:
        for i, l in enumerate(layers):
            ctx.upload_layer(i, l)
            ctx.upload_layer_gguf(2 + i, path, i)
        for i, l in enumerate(layers):
            a = ctx.forward_host(i, x)
            b = ctx.forward_host(2 + i, x)
            assert np.array_equal(a, b)
            check(oracle.moe_ffn(l, x)[0], b, tight)
        ref = oracle.stack(layers, x)
        check(ref, ctx.stack_forward_host(2, 2, x), 5e-3 if n_tok >= 64 else 5e-5)
