"""Q8_0 products with M >= 32 activation rows take the int8 tensor-core path (tcgen05.mma kind::i8, TMEM accumulators,
TMA operands, optional split-K). Same bar as every product: |err| <= 1e-4 * sum |w x| per element against the oracle."""

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu

CASES = [
    (256, 128, 32),     # one tile, one stage
    (1024, 3072, 64),   # config 4-like rows, split-K
    (2048, 1000, 100),  # ragged rows and tokens
    (6144, 2048, 64),   # config 4's down projection
    (2048, 384, 257),   # several token tiles
    (2048, 6144, 64),   # the 32-token tile kernel (96 items), config 4's gate|up shape
    (1024, 6000, 100),  # tile kernel: ragged rows and a 4-token last tile
]


@pytest.mark.parametrize("K,N,M", CASES)
def test_q8_0_tensor_core_products(oracle, K, N, M):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    b200 = load_package()
    ctx = b200.Context(0)
    try:
        rng = np.random.default_rng(K + N + M)
        wb = oracle.quantize(8, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
        x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
        w = ctx.weight(8, K, N, data=wb)
        got = ctx.mul_mat(w, torch.from_numpy(x).cuda()).cpu().numpy()
        ctx.synchronize()
        want = oracle.mul_mat(8, wb, K, N, x)
        wd = oracle.dequantize(8, wb, K).astype(np.float64)
        xd = oracle.dequantize(8, oracle.quantize(8, x), K).astype(np.float64)
        bound = 1e-4 * (np.abs(xd) @ np.abs(wd).T) + 1e-30
        err = np.abs(got.astype(np.float64) - want)
        assert np.all(err <= bound), f"max err/bound {np.max(err / bound):.3g}"
        # run again: split-K tickets were left at zero, results are identical
        again = ctx.mul_mat(w, torch.from_numpy(x).cuda()).cpu().numpy()
        assert np.array_equal(again, got)
        ctx.free_weight(w)
    finally:
        ctx.close()


Q4_K, Q6_K, Q8_K = 12, 14, 15

KQ_CASES = [
    (Q4_K, 256, 128, 32),    # one super-block, one token tile
    (Q4_K, 2048, 1000, 100), # ragged rows, four token tiles (the last of 4 tokens)
    (Q6_K, 2048, 640, 64),
    (Q6_K, 6144, 384, 33),   # config 3's down projection K, a 1-token last tile
    (Q4_K, 4096, 256, 257),
]


def _kq_bound(oracle, qtype, wb, K, x):
    wd = oracle.dequantize(qtype, wb, K).astype(np.float64)
    xd = oracle.dequantize(Q8_K, oracle.quantize(Q8_K, x), K).astype(np.float64)
    return 1e-4 * (np.abs(xd) @ np.abs(wd).T) + 1e-30


@pytest.mark.parametrize("qtype,K,N,M", KQ_CASES)
def test_kquant_tensor_core_products(oracle, qtype, K, N, M):
    """Q4_K / Q6_K products with M >= 32 run on the int8 tensor cores over an expanded copy of the weights, with
    ggml's integer super-block sums (q8_K activations)."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    b200 = load_package()
    ctx = b200.Context(0)
    try:
        rng = np.random.default_rng(K * 3 + N + M + qtype)
        wb = oracle.quantize(qtype, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
        x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
        w = ctx.weight(qtype, K, N, data=wb)
        got = ctx.mul_mat(w, torch.from_numpy(x).cuda()).cpu().numpy()
        ctx.synchronize()
        want = oracle.mul_mat(qtype, wb, K, N, x)
        err = np.abs(got.astype(np.float64) - want)
        b = _kq_bound(oracle, qtype, wb, K, x)
        assert np.all(err <= b), f"max err/bound {np.max(err / b):.3g}"
        # new bytes for the same weight: the expanded copy is rebuilt, not reused
        wb2 = oracle.quantize(qtype, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
        ctx.set_weight(w, wb2)
        got2 = ctx.mul_mat(w, torch.from_numpy(x).cuda()).cpu().numpy()
        want2 = oracle.mul_mat(qtype, wb2, K, N, x)
        assert np.all(np.abs(got2.astype(np.float64) - want2) <= _kq_bound(oracle, qtype, wb2, K, x))
        ctx.free_weight(w)
    finally:
        ctx.close()
