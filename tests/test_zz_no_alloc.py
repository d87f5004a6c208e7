"""gx_moe_forward_noalloc (the decode layer on the library's static scratch, no allocation on
any call) against gx_moe_forward on the same layer and tokens, through the C ABI, and against the
CPU oracle directly. The file sorts last so the check also runs after every other GPU test in one
process; it passes alone too."""
import numpy as np
import pytest

from oracle import oracle
from gyro_moe import abi, metrics, synth
from layer_case import small_layer

pytestmark = pytest.mark.gpu
REL_RMS, COSINE = 1e-2, 0.9999          # north-star layer tolerance
TIGHT = 2e-5                            # what the decode kernels hold against the oracle

torch = pytest.importorskip("torch")


def close(ref, got):
    m = metrics.compare(ref, got)
    assert m["rel_rms"] <= REL_RMS and m["cosine"] >= COSINE and m["rel_rms"] <= TIGHT, m


def run(ctx, fn, layer, x, U, y_dtype=torch.float32):
    n = x.shape[0]
    y = torch.empty((n, x.shape[1]), dtype=y_dtype, device="cuda")
    ids = torch.empty((n, U), dtype=torch.int32, device="cuda")
    w = torch.empty((n, U), dtype=torch.float32, device="cuda")
    ctx.wait(fn(layer, x, y, ids, w))
    return y.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy()


@pytest.mark.parametrize("type_id", [144, 147])
def test_noalloc_matches_forward_on_two_calls_in_a_row(type_id):
    layer, _ = small_layer(seed=31, type_id=type_id)
    big = synth.make_layer(7, n_expert=64, E=1024, F=512, U=8, zipf=1.1)
    with abi.Context(device=0, max_tokens=64, max_layers=2) as ctx:
        ctx.upload_layer(0, layer)
        ctx.upload_layer(1, big)
        cases = [(0, synth.tokens(5, abi.NOALLOC_MAX_TOKENS, E=256), 4),
                 (1, synth.tokens(6, 3, E=1024), 8),
                 (0, synth.tokens(8, 1, E=256), 4)]
        for idx, x, U in cases:
            xt = torch.from_numpy(x).cuda()
            want = run(ctx, ctx.forward, idx, xt, U)
            ref, ref_ids, _ = oracle.moe_ffn(layer if idx == 0 else big, x)
            for _ in range(2):                         # two calls in a row on the same scratch
                got = run(ctx, ctx.forward_noalloc, idx, xt, U)
                close(want[0], got[0])
                close(ref, got[0])                     # and on its own against the oracle
                assert metrics.topk_sets(want[1], got[1])["flips"] == 0
                assert metrics.topk_sets(ref_ids, got[1])["flips"] == 0
                np.testing.assert_allclose(got[2], want[2], rtol=1e-6, atol=0)


def test_noalloc_bf16_tokens_and_output():
    layer, x = small_layer(seed=41, n_tok=7)
    with abi.Context(device=0, max_tokens=16, max_layers=1) as ctx:
        ctx.upload_layer(0, layer)
        xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
        want = run(ctx, ctx.forward, 0, xt, 4, torch.bfloat16)
        got = run(ctx, ctx.forward_noalloc, 0, xt, 4, torch.bfloat16)
        close(want[0], got[0])


def test_noalloc_rejects_more_tokens_than_its_scratch_holds():
    layer, _ = small_layer(seed=51)
    with abi.Context(device=0, max_tokens=64, max_layers=1) as ctx:
        ctx.upload_layer(0, layer)
        x = torch.zeros((abi.NOALLOC_MAX_TOKENS + 1, 256), dtype=torch.float32, device="cuda")
        y = torch.empty_like(x)
        with pytest.raises(abi.GxError) as e:
            ctx.forward_noalloc(0, x, y)
        assert e.value.code == -1
        ctx.wait(ctx.forward_noalloc(0, x[:0], y[:0]))   # zero tokens: nothing to do
