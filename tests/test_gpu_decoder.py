"""The decode-step matmul stack (b200_decoder) against the oracle's CPU step (oracle/stack.py).

The chain re-quantizes each product's input, so float differences of earlier products can move later q8 roundings:
end-to-end logits are judged by cosine similarity >= 0.9999, the bar stated for decoder stacks.
"""

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu

SMALL = {
    # rows too short for the persistent step: chain mode only
    "q8": dict(n_layer=3, hidden=256, n_head=4, n_kv_head=2, head_dim=64, ffn=512, n_vocab=300,
               type_attn=8, type_ffn_up=8, type_ffn_down=8, type_head=8),
    "kquant": dict(n_layer=2, hidden=512, n_head=8, n_kv_head=2, head_dim=64, ffn=1024, n_vocab=1000,
                   type_attn=12, type_ffn_up=12, type_ffn_down=14, type_head=14),
    # shapes the persistent step takes (K % 1024, K % 2048 for K-quants)
    "q8_mk": dict(n_layer=2, hidden=1024, n_head=8, n_kv_head=2, head_dim=128, ffn=3072, n_vocab=500,
                  type_attn=8, type_ffn_up=8, type_ffn_down=8, type_head=8),
    "kquant_mk": dict(n_layer=2, hidden=2048, n_head=16, n_kv_head=4, head_dim=128, ffn=2048, n_vocab=700,
                      type_attn=12, type_ffn_up=12, type_ffn_down=14, type_head=14),
}


@pytest.fixture(scope="module")
def b200():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return load_package()


@pytest.fixture(scope="module")
def ctx(b200):
    c = b200.Context(0)
    yield c
    c.close()


def load(b200, ctx, c, model):
    d = b200.Decoder(ctx, **c)
    names = ["attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down"]
    for l, L in enumerate(model["layers"]):
        for i, n in enumerate(names):
            d.set_tensor(l, i, L[n])
        d.set_tensor(l, b200.DEC_ATTN_NORM, L["attn_norm"])
        d.set_tensor(l, b200.DEC_FFN_NORM, L["ffn_norm"])
    d.set_tensor(0, b200.DEC_OUTPUT, model["output"])
    d.set_tensor(0, b200.DEC_OUTPUT_NORM, model["output_norm"])
    return d


def cosine(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.mark.parametrize("name", sorted(SMALL))
def test_decoder_step_matches_cpu(b200, ctx, name):
    import torch

    from oracle import stack

    c = SMALL[name]
    model = stack.random_model(c, seed=7)
    rng = np.random.default_rng(8)
    x = rng.normal(0, 1, size=c["hidden"]).astype(np.float32)
    want = stack.step(c, model, x)
    d = load(b200, ctx, c, model)
    xd = torch.from_numpy(x).cuda()
    d.set_launch(mode=b200.DEC_MODE_CHAIN)
    got = d.step(xd).cpu().numpy()
    assert d.launches == 4 * c["n_layer"] + 1
    assert cosine(got, want) >= 0.9999
    host = d.step_host(x)
    assert np.array_equal(host, got)
    # chain launch options change scheduling only, never results
    d.set_launch(mode=b200.DEC_MODE_CHAIN, pdl=False, ctas_per_sm=0)
    again = d.step(xd).cpu().numpy()
    assert np.array_equal(again, got)
    if name.endswith("_mk"):
        d.set_launch(mode=-1)
        pers = d.step(xd).cpu().numpy()
        assert d.launches == 1  # the automatic choice is the persistent step
        ctx.synchronize()
        assert cosine(pers, want) >= 0.9999
        assert cosine(pers, got) >= 0.99999
        for _ in range(3):  # replays of the captured step are deterministic
            assert np.array_equal(d.step(xd).cpu().numpy(), pers)
        assert np.array_equal(d.step_host(x), pers)
    else:
        d.set_launch(mode=-1)
        d.step(xd)
        assert d.launches == 4 * c["n_layer"] + 1  # not eligible: the automatic choice is the chain
        with pytest.raises(b200.B200Error):
            d.set_launch(mode=b200.DEC_MODE_PERSISTENT)
            d.step(xd)
    d.close()


def test_decoder_rejects_bad_tensor(b200, ctx):
    d = b200.Decoder(ctx, **SMALL["q8"])
    with pytest.raises(b200.B200Error):
        d.set_tensor(5, 0, np.zeros(10, dtype=np.uint8))  # no such layer
    with pytest.raises(b200.B200Error):
        d.set_tensor(0, b200.DEC_ATTN_NORM, np.zeros(1000, dtype=np.float32))  # too long
    d.close()
