"""The decode stack as one persistent cooperative kernel (gx_decode_stack.cu, opt-in with
GX_STACK_KERNEL=1) through gx_stack_forward: every Gyro type, token counts at the kernel's limits,
bf16 in/out, in-place calls, and agreement with the per-phase kernels and with the CPU oracle of
the pre-norm chain x_{l+1} = x_l + MoE_l(RMSNorm(x_l)) (src/engine.zig:520-642 per layer)."""
import os

import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, metrics, synth

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(autouse=True)
def stack_kernel_on(monkeypatch):
    monkeypatch.setenv("GX_STACK_KERNEL", "1")
REL_RMS, COSINE = 1e-2, 0.9999


def check(ref, got, tight=5e-5):
    m = metrics.compare(ref, got)
    assert m["rel_rms"] <= REL_RMS and m["cosine"] >= COSINE and m["rel_rms"] <= tight, m


def run(ctx, n_layers, x, out_dtype=torch.float32, inplace=False):
    xt = torch.from_numpy(x).cuda()
    if inplace:
        ctx.wait(ctx.stack_forward(0, n_layers, xt, xt))
        return xt.float().cpu().numpy()
    yt = torch.empty(xt.shape, dtype=out_dtype, device="cuda")
    ctx.wait(ctx.stack_forward(0, n_layers, xt, yt))
    return yt.float().cpu().numpy()


@pytest.mark.parametrize("type_id", sorted(synth.BLOCK_BYTES))
def test_stack_kernel_all_types(type_id):
    layers = [synth.make_layer(300 + 10 * type_id + i, n_expert=32, E=512, F=256, U=4, type_id=type_id)
              for i in range(3)]
    with abi.Context(device=0, max_tokens=16, max_layers=3) as ctx:
        for i, l in enumerate(layers):
            ctx.upload_layer(i, l)
        for n in (1, 5):
            x = synth.tokens(type_id + n, n, E=512)
            check(oracle.stack(layers, x), run(ctx, 3, x))


def test_stack_kernel_config_shape_token_limits_and_per_phase_agreement():
    layers = [synth.make_layer(700 + i, n_expert=256, zipf=1.1) for i in range(3)]
    with abi.Context(device=0, max_tokens=32, max_layers=3) as ctx:
        for i, l in enumerate(layers):
            ctx.upload_layer(i, l)
        for n in (1, 16, 17):                      # 17 tokens: per-phase kernels
            x = synth.tokens(800 + n, n)
            got = run(ctx, 3, x)
            check(oracle.stack(layers, x), got, tight=1e-4)
            os.environ["GX_STACK_KERNEL"] = "0"
            try:
                ref = run(ctx, 3, x)
            finally:
                os.environ["GX_STACK_KERNEL"] = "1"
            np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def test_stack_kernel_bf16_inplace_and_repeats():
    layers = [synth.make_layer(710 + i, n_expert=64, E=1024, F=512, U=8) for i in range(2)]
    with abi.Context(device=0, max_tokens=8, max_layers=2) as ctx:
        for i, l in enumerate(layers):
            ctx.upload_layer(i, l)
        x = synth.tokens(811, 3, E=1024, dtype="bf16")
        ref = oracle.stack(layers, x)
        xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
        for _ in range(3):                                  # the barrier counter restarts per call
            yb = torch.empty_like(xb)
            ctx.wait(ctx.stack_forward(0, 2, xb, yb))
            check(ref, yb.float().cpu().numpy(), tight=5e-3)   # bf16 output rounding
        got = run(ctx, 2, x, inplace=True)
        check(ref, got)
        one = run(ctx, 1, x)                                # a single layer is a stack of one
        check(oracle.stack(layers[:1], x), one)
