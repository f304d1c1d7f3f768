"""Parity of the B200 kernels with the CPU oracle, through the C ABI (include/b200.h).

Bars (stated by the task): bit-exact for integer / byte work (activation quantization, (sub-)block int32 sums, weight
bytes, GET_ROWS dequantization); float outputs within |err| <= 1e-4 * sum_i |w_i * x_i| per element, where w_i are
the dequantized weights and x_i the quantized activations the CPU's vec_dot multiplies.
"""

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 8, 12, 13, 14, 15, 30
VEC = {Q8_0: Q8_0, Q4_K: Q8_K, Q5_K: Q8_K, Q6_K: Q8_K, BF16: BF16}
TOL = 1e-4


@pytest.fixture(scope="module")
def b200():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    m = load_package()
    return m


@pytest.fixture(scope="module")
def ctx(b200):
    c = b200.Context(0)
    yield c
    c.close()


def cuda(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bound(oracle, qtype, wb, K, x):
    wd = oracle.dequantize(qtype, wb, K).astype(np.float64)
    vt = VEC[qtype]
    xd = oracle.dequantize(vt, oracle.quantize(vt, x), K).astype(np.float64)
    return TOL * (np.abs(xd) @ np.abs(wd).T) + 1e-30


def rand_w(rng, qtype, N, K, oracle, sigma=0.02):
    w = rng.normal(0, sigma, size=(N, K)).astype(np.float32)
    return oracle.quantize(qtype, w)


@pytest.mark.parametrize("qtype,K", [(Q8_0, 64), (Q8_0, 1024), (Q8_K, 256), (Q8_K, 2048)])
def test_activation_quantizer_bit_exact(ctx, oracle, golden, qtype, K):
    rng = np.random.default_rng(K + qtype)
    x = rng.normal(0, 1, size=(7, K)).astype(np.float32)
    x[1] = 0.0
    x[2, :32] = (np.arange(32) - 15.5) / np.float32(127.0)  # rounding ties
    x[3] *= 1e-6
    x[4, 5] = 9.0
    x[4, 9] = -9.0  # equal magnitudes
    x[5] = np.where(np.arange(K) % 2 == 0, 1.0, -1.0)
    got = ctx.quantize_rows(qtype, cuda(x)).cpu().numpy()
    want = oracle.quantize(qtype, x)
    assert np.array_equal(got, want)
    if qtype == Q8_0 and K == 64:
        e = golden["q8_0_edge_x"]
        assert np.array_equal(ctx.quantize_rows(Q8_0, cuda(e)).cpu().numpy(), golden["q8_0_edge_q"])


@pytest.mark.parametrize("qtype", [Q8_0, Q4_K, Q5_K, Q6_K, BF16])
def test_weight_upload_pieces_round_trip(ctx, oracle, qtype):
    rng = np.random.default_rng(qtype)
    K, N = 512, 37
    wb = rand_w(rng, qtype, N, K, oracle).reshape(-1)
    w = ctx.weight(qtype, K, N)
    cuts = sorted({0, wb.size} | set(rng.integers(1, wb.size, size=9).tolist()))
    for a, b in zip(cuts[:-1], cuts[1:]):  # pieces that split blocks, like 16 MiB pieces do
        ctx.set_weight(w, wb[a:b], offset=a)
    assert np.array_equal(ctx.get_weight(w), wb)
    assert np.array_equal(ctx.get_weight(w, offset=101, size=333), wb[101:434])
    ctx.free_weight(w)


@pytest.mark.parametrize("qtype,K", [(Q8_0, 1024), (Q8_0, 96), (Q4_K, 2048), (Q5_K, 2048), (Q6_K, 1024), (Q6_K, 6144)])
def test_block_sums_bit_exact(ctx, oracle, qtype, K):
    rng = np.random.default_rng(K)
    N = 19
    wb = rand_w(rng, qtype, N, K, oracle)
    x = rng.normal(0, 1, size=(1, K)).astype(np.float32)
    w = ctx.weight(qtype, K, N, data=wb)
    got = ctx.block_sums(w, cuda(x)).cpu().numpy()
    xq = oracle.quantize(VEC[qtype], x)[0]
    want = np.stack([oracle.block_sums(qtype, wb[n], xq, K) for n in range(N)])
    assert np.array_equal(got, want)
    ctx.free_weight(w)


SHAPES = [
    (Q8_0, 1024, 3072, 1),   # config 1
    (Q8_0, 1024, 67, 3),
    (Q8_0, 32, 5, 1),
    (Q8_0, 2048, 1024, 8),
    (Q8_0, 1024, 256, 13),
    (Q8_0, 1024, 300, 40),
    (Q4_K, 2048, 1024, 1),
    (Q4_K, 256, 33, 5),
    (Q4_K, 2048, 512, 20),
    (Q6_K, 6144, 2048, 1),
    (Q6_K, 256, 9, 2),
    (Q6_K, 2048, 300, 17),
    (BF16, 1024, 100, 1),
    (BF16, 64, 7, 4),
    (BF16, 512, 64, 24),
    (Q5_K, 2048, 1024, 1),    # Q5_K (speech.cpp's Q5_K files): the TMA GEMV and the register GEMV
    (Q5_K, 256, 33, 5),
    (Q5_K, 4096, 300, 20),    # more columns than one launch stages: column chunks
    (Q6_K, 2048, 40000, 1),   # the TMA ring wraps many times per CTA
    (Q8_0, 1024, 50000, 2),
    (Q4_K, 4096, 20000, 3),
]


@pytest.mark.parametrize("qtype,K,N,M", SHAPES)
def test_mul_mat_within_tolerance(ctx, oracle, qtype, K, N, M):
    rng = np.random.default_rng(K * 7 + N + M)
    wb = rand_w(rng, qtype, N, K, oracle)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    w = ctx.weight(qtype, K, N, data=wb)
    got = ctx.mul_mat(w, cuda(x)).cpu().numpy()
    want = oracle.mul_mat(qtype, wb, K, N, x)
    err = np.abs(got.astype(np.float64) - want)
    b = bound(oracle, qtype, wb, K, x)
    assert np.all(err <= b), f"max err/bound {np.max(err / b):.3g}"
    if M <= 16:
        # the GEMV kernels sum the block terms in double and round once, as the oracle defines the float step: equal
        # floats except where the exact sum lies within double rounding of a float32 rounding boundary (rare)
        assert np.mean(got == want) >= 0.999, f"bit-equal fraction {np.mean(got == want):.5f}"
    ctx.free_weight(w)


def test_upload_from_device_tensor_survives_reuse(ctx, oracle):
    """set_weight from a CUDA tensor: the caller may overwrite or free the tensor as soon as the call returns."""
    import torch

    rng = np.random.default_rng(8)
    K, N = 2048, 4096
    wb = rand_w(rng, Q8_0, N, K, oracle)
    w = ctx.weight(Q8_0, K, N)
    t = torch.from_numpy(wb.reshape(-1)).cuda()
    ctx.set_weight(w, t)
    t.fill_(0)  # on torch's stream, right after the call
    del t
    junk = torch.full((wb.size,), 255, dtype=torch.uint8, device="cuda")  # likely reuses the freed block
    assert np.array_equal(ctx.get_weight(w), wb.reshape(-1))
    del junk
    ctx.free_weight(w)


def test_mul_mat_rows_shard(ctx, oracle):
    rng = np.random.default_rng(3)
    K, N, M = 1024, 512, 4
    wb = rand_w(rng, Q8_0, N, K, oracle)
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    w = ctx.weight(Q8_0, K, N, data=wb)
    full = ctx.mul_mat(w, cuda(x)).cpu().numpy()
    part = ctx.mul_mat_rows(w, 128, 200, cuda(x)).cpu().numpy()
    assert np.array_equal(part, full[:, 128:328])
    ctx.free_weight(w)


def test_mul_mat_host_path(ctx, oracle):
    rng = np.random.default_rng(4)
    K, N = 1024, 3072
    wb = rand_w(rng, Q8_0, N, K, oracle)
    x = rng.normal(0, 1, size=(1, K)).astype(np.float32)
    w = ctx.weight(Q8_0, K, N, data=wb)
    got = ctx.mul_mat_host(w, x)
    want = oracle.mul_mat(Q8_0, wb, K, N, x)
    assert np.all(np.abs(got - want) <= bound(oracle, Q8_0, wb, K, x))
    ctx.free_weight(w)


@pytest.mark.parametrize("qtype", [Q8_0, Q4_K, Q5_K, Q6_K, BF16])
def test_get_rows_bit_exact(ctx, oracle, qtype):
    rng = np.random.default_rng(qtype + 1)
    K, rows = 512, 23
    tb = rand_w(rng, qtype, rows, K, oracle, sigma=0.5)
    t = ctx.weight(qtype, K, rows, data=tb)
    ids = np.array([0, 22, 5, 5, 17], dtype=np.int32)
    got = ctx.get_rows(t, cuda(ids)).cpu().numpy()
    want = oracle.get_rows(qtype, tb, K, rows, ids)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    ctx.synchronize()
    ctx.free_weight(t)


def test_get_rows_out_of_range_reports(ctx, oracle, b200):
    import torch

    rng = np.random.default_rng(9)
    tb = rand_w(rng, Q8_0, 4, 64, oracle)
    t = ctx.weight(Q8_0, 64, 4, data=tb)
    out = torch.full((2, 64), 7.0, device="cuda")
    ctx.get_rows(t, cuda(np.array([1, 4], dtype=np.int32)), out=out)
    with pytest.raises(b200.B200Error) as e:
        ctx.synchronize()
    assert e.value.status == b200.ERR_RANGE
    o = out.cpu().numpy()
    assert np.array_equal(o[0], oracle.get_rows(Q8_0, tb, 64, 4, np.array([1], dtype=np.int32))[0])
    assert np.all(o[1] == 7.0)  # the bad row is skipped
    ctx.synchronize()  # the error was cleared
    ctx.free_weight(t)


@pytest.mark.parametrize("qtype,nb1", [(Q8_0, 1), (Q8_0, 3), (Q4_K, 1), (Q6_K, 3)])
def test_mul_mat_id_within_tolerance(ctx, oracle, qtype, nb1):
    rng = np.random.default_rng(qtype * 10 + nb1)
    E, K, N, T, top_k = 12, 512, 96, 21, 3
    wb = rand_w(rng, qtype, E * N, K, oracle)
    ids = np.stack([rng.permutation(E)[:top_k] for _ in range(T)]).astype(np.int32)
    b = rng.normal(0, 1, size=(T, nb1, K)).astype(np.float32)
    w = ctx.weight(qtype, K, N, E, data=wb)
    got = ctx.mul_mat_id(w, cuda(b), cuda(ids)).cpu().numpy()
    want = oracle.mul_mat_id(qtype, wb, K, N, E, b, ids)
    for t in range(T):
        for s in range(top_k):
            e = ids[t, s]
            xb = b[t, 0 if nb1 == 1 else s][None]
            bd = bound(oracle, qtype, wb[e * N:(e + 1) * N], K, xb)[0]
            assert np.all(np.abs(got[t, s] - want[t, s]) <= bd)
    ctx.free_weight(w)


def test_mul_mat_id_bad_expert_reports(ctx, oracle, b200):
    rng = np.random.default_rng(21)
    E, K, N = 4, 64, 8
    wb = rand_w(rng, Q8_0, E * N, K, oracle)
    w = ctx.weight(Q8_0, K, N, E, data=wb)
    ids = np.array([[0, 9]], dtype=np.int32)
    ctx.mul_mat_id(w, cuda(rng.normal(0, 1, size=(1, 1, K)).astype(np.float32)), cuda(ids))
    with pytest.raises(b200.B200Error) as e:
        ctx.synchronize()
    assert e.value.status == b200.ERR_RANGE
    ctx.free_weight(w)


def test_invalid_shapes_are_errors_not_aborts(ctx, b200):
    import torch

    w = ctx.weight(Q8_0, 64, 8)
    x = torch.zeros((2, 64), device="cuda")
    with pytest.raises(b200.B200Error) as e:
        ctx.mul_mat_rows(w, 4, 8, x)  # rows past the end
    assert e.value.status == b200.ERR_INVALID
    with pytest.raises(b200.B200Error):
        ctx.weight(Q8_0, 100, 8)  # not whole blocks
    ctx.free_weight(w)


@pytest.mark.parametrize("nb1,skew", [(1, False), (4, False), (1, True)])
def test_mul_mat_id_tensor_cores(ctx, oracle, nb1, skew):
    """MUL_MAT_ID of Q8_0 experts with >= 128 (token, slot) pairs runs on the tensor cores (expert-sorted slots padded
    to 16, token tiles of <= 64 slots). N = 192 leaves a partial 128-row tile; with skew, expert 0 takes every token's
    first slot (100 pairs: two token tiles) and experts 13..15 get none."""
    rng = np.random.default_rng(77 + nb1 + 10 * skew)
    E, K, N, T, top_k = 16, 1024, 192, 100, 4
    wb = rand_w(rng, Q8_0, E * N, K, oracle)
    if skew:
        ids = np.stack([np.concatenate([[0], 1 + rng.permutation(12)[:top_k - 1]]) for _ in range(T)]).astype(np.int32)
    else:
        ids = np.stack([rng.permutation(E)[:top_k] for _ in range(T)]).astype(np.int32)
    b = rng.normal(0, 1, size=(T, nb1, K)).astype(np.float32)
    w = ctx.weight(Q8_0, K, N, E, data=wb)
    got = ctx.mul_mat_id(w, cuda(b), cuda(ids)).cpu().numpy()
    ctx.synchronize()
    want = oracle.mul_mat_id(Q8_0, wb, K, N, E, b, ids)
    for t in range(T):
        for s in range(top_k):
            e = ids[t, s]
            xb = b[t, 0 if nb1 == 1 else s][None]
            bd = bound(oracle, Q8_0, wb[e * N:(e + 1) * N], K, xb)[0]
            assert np.all(np.abs(got[t, s] - want[t, s]) <= bd), (t, s)
    ctx.free_weight(w)
