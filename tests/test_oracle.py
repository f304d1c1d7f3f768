"""The CPU oracle against gguf-py's golden vectors (tests/golden/make_golden.py) and against its own float restatement.

CPU only. Pins: Q8_0 quantization and Q8_0 / Q4_K / Q6_K / BF16 (de)quantization bit for bit against gguf-py, which
the reference's checks/compare/quantize_compare.py:1-11 pins against ggml.
"""

import numpy as np
import pytest

Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 8, 12, 13, 14, 15, 30


@pytest.mark.parametrize("case", ["normal", "kat", "edge"])
def test_q8_0_quantize_matches_gguf_py(oracle, golden, case):
    x = golden[f"q8_0_{case}_x"]
    want = golden[f"q8_0_{case}_q"]
    got = oracle.quantize(Q8_0, x)
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("qtype,name,k", [(Q8_0, "q8_0", 32), (Q4_K, "q4_K", 256), (Q5_K, "q5_K", 256), (Q6_K, "q6_K", 256)])
def test_dequantize_matches_gguf_py(oracle, golden, qtype, name, k):
    blocks = golden[f"deq_{name}_blocks"]
    want = golden[f"deq_{name}_y"].reshape(-1, k)
    got = oracle.dequantize(qtype, blocks, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_bf16_matches_gguf_py(oracle, golden):
    x = golden["bf16_x"]
    got = oracle.quantize(BF16, x.reshape(1, -1)).reshape(-1)
    assert np.array_equal(got, golden["bf16_q"])
    y = oracle.dequantize(BF16, got, x.size).reshape(-1)
    assert np.array_equal(y.view(np.uint32), golden["bf16_y"].view(np.uint32))


def test_fp16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(7)
    x = np.concatenate([
        rng.normal(0, 1, 2000), 2.0 ** rng.uniform(-30, 17, 4000) * rng.choice([-1, 1], 4000),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, 2.0**-24, 2.0**-25, 2.0**-25 * 1.0001, 3 * 2.0**-26, np.inf, -np.inf]),
    ]).astype(np.float32)
    L = oracle.lib()
    got = np.array([L.oracle_fp32_to_fp16(float(v)) for v in x], dtype=np.uint16)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    h = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    fin = (h & 0x7C00) != 0x7C00
    back = np.array([L.oracle_fp16_to_fp32(int(v)) for v in h[fin]], dtype=np.float32)
    assert np.array_equal(back.view(np.uint32), h[fin].view(np.float16).astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("qtype", [Q4_K, Q5_K, Q6_K])
def test_k_quantizers_make_valid_blocks(oracle, qtype):
    """Our own Q4_K / Q5_K / Q6_K weight quantizers round-trip through gguf-py's dequantizer."""
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    rng = np.random.default_rng(3)
    x = rng.normal(0, 0.02, size=(4, 512)).astype(np.float32)
    b = oracle.quantize(qtype, x)
    ours = oracle.dequantize(qtype, b, 512)
    theirs = quants.dequantize(b, {Q4_K: T.Q4_K, Q5_K: T.Q5_K, Q6_K: T.Q6_K}[qtype]).reshape(4, 512)
    assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32))
    rel = np.abs(ours - x).max() / np.abs(x).max()
    assert rel < {Q4_K: 0.08, Q5_K: 0.04, Q6_K: 0.03}[qtype]


def test_q8_K_quantizer_properties(oracle):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, size=(3, 512)).astype(np.float32)
    x[1, :256] = 0.0
    x[2, 7] = 5.0
    x[2, 9] = -5.0  # equal magnitudes: the first one sets the sign of d
    b = oracle.quantize(Q8_K, x)
    assert b.shape == (3, 2 * 292)
    for r in range(3):
        for s in range(2):
            blk = b[r, s * 292:(s + 1) * 292]
            d = blk[:4].view(np.float32)[0]
            qs = blk[4:260].view(np.int8).astype(np.int32)
            bs = blk[260:292].view(np.int16).astype(np.int32)
            assert np.array_equal(bs, qs.reshape(16, 16).sum(1))
            xs = x[r, s * 256:(s + 1) * 256]
            if not xs.any():
                assert d == 0 and not qs.any()
                continue
            assert qs.max() <= 127 and qs.min() >= -128
            assert np.abs(d * qs - xs).max() <= abs(d) * 0.5 + 1e-6
    blk = b[2, 0:292]
    assert blk[:4].view(np.float32)[0] < 0  # max is +5 at index 7: iscale = -127/5 < 0
    assert blk[4 + 7].view(np.int8) == -127


@pytest.mark.parametrize("qtype,K", [(Q8_0, 1024), (Q4_K, 1024), (Q6_K, 1024), (BF16, 256)])
def test_mul_mat_matches_dequantized_float(oracle, qtype, K):
    """The integer dot products equal the float dot of the dequantized weight and quantized activation rows."""
    rng = np.random.default_rng(11)
    N, M = 24, 3
    w = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    wb = oracle.quantize(qtype, w)
    y = oracle.mul_mat(qtype, wb, K, N, x)
    wd = oracle.dequantize(qtype, wb, K).astype(np.float64)
    vt = {Q8_0: Q8_0, Q4_K: Q8_K, Q6_K: Q8_K, BF16: BF16}[qtype]
    xd = oracle.dequantize(vt, oracle.quantize(vt, x), K).astype(np.float64)
    ref = xd @ wd.T
    bound = 1e-4 * (np.abs(xd) @ np.abs(wd).T) + 1e-6
    assert np.all(np.abs(y - ref) <= bound)


def test_block_sums_are_exact(oracle):
    rng = np.random.default_rng(13)
    K = 512
    for qtype in (Q8_0, Q4_K, Q5_K, Q6_K):
        w = oracle.quantize(qtype, rng.normal(0, 0.02, size=(1, K)).astype(np.float32))
        vt = Q8_0 if qtype == Q8_0 else Q8_K
        x = oracle.quantize(vt, rng.normal(0, 1, size=(1, K)).astype(np.float32))
        s = oracle.block_sums(qtype, w[0], x[0], K)
        if qtype == Q8_0:
            qw = w[0].reshape(-1, 34)[:, 2:].view(np.int8).astype(np.int64)
            qx = x[0].reshape(-1, 34)[:, 2:].view(np.int8).astype(np.int64)
            assert np.array_equal(s, (qw * qx).sum(1))


def test_mul_mat_id_matches_per_expert_mul_mat(oracle):
    rng = np.random.default_rng(17)
    E, K, N, T, top_k = 6, 256, 40, 5, 3
    w = rng.normal(0, 0.02, size=(E * N, K)).astype(np.float32)
    wb = oracle.quantize(Q8_0, w)
    ids = np.stack([rng.permutation(E)[:top_k] for _ in range(T)]).astype(np.int32)
    b = rng.normal(0, 1, size=(T, 1, K)).astype(np.float32)
    y = oracle.mul_mat_id(Q8_0, wb, K, N, E, b, ids)
    for t in range(T):
        for s in range(top_k):
            e = ids[t, s]
            ref = oracle.mul_mat(Q8_0, wb[e * N:(e + 1) * N], K, N, b[t, 0][None])
            assert np.array_equal(y[t, s], ref[0])
    with pytest.raises(ValueError):
        oracle.mul_mat_id(Q8_0, wb, K, N, E, b, np.full_like(ids, E))


def test_get_rows_dequantizes(oracle):
    rng = np.random.default_rng(19)
    K, rows = 512, 9
    t = oracle.quantize(Q4_K, rng.normal(0, 0.02, size=(rows, K)).astype(np.float32))
    ids = np.array([3, 0, 8, 3], dtype=np.int32)
    got = oracle.get_rows(Q4_K, t, K, rows, ids)
    assert np.array_equal(got, oracle.dequantize(Q4_K, t[ids], K))
