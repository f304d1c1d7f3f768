"""The integer identities behind the K-quant tensor-core products (csrc/gemm_kq_tc.cu): the expansion writes each
weight as int8 planes that carry the (sub-)block scales, and the tensor cores sum each plane over a whole super-block.
These CPU tests restate the expansion in numpy and check that the plane sums give ggml's super-block integers
exactly (Q4_K: sumi = sum_s sc_s sum_l q_l x_l, summ = sum_s m_s sum_l x_l; Q6_K: sumi = sum_g sc_g sum_l (q_l - 32)
x_l), that every plane value fits int8, and that the per-plane int32 sums cannot overflow."""

import numpy as np


def balanced_base5(sc):
    """Digits e0..e3 in -2..2 with sc = e0 + 5 e1 + 25 e2 + 125 e3 (the Q6_K expansion's digit loop)."""
    e = []
    for _ in range(4):
        d = ((sc % 5) + 5) % 5
        if d > 2:
            d -= 5
        e.append(d)
        sc = (sc - d) // 5
    assert sc == 0
    return e


def test_q6k_scale_digits_cover_int8():
    for sc in range(-128, 128):
        e = balanced_base5(sc)
        assert all(-2 <= d <= 2 for d in e)
        assert e[0] + 5 * e[1] + 25 * e[2] + 125 * e[3] == sc
        for q in (-32, 31):  # extreme q - 32 values: every plane value fits int8
            assert all(-128 <= d * q <= 127 for d in e)


def test_q4k_scale_digits_cover_six_bits():
    for sc in range(64):
        a, b = sc >> 3, sc & 7
        assert 8 * a + b == sc
        assert 0 <= a * 15 <= 127 and 0 <= b * 15 <= 127


def test_q4k_planes_give_ggml_integers():
    rng = np.random.default_rng(5)
    for _ in range(50):
        q = rng.integers(0, 16, size=256)            # nibbles of one super-block
        sc = rng.integers(0, 64, size=8)             # six-bit scales of its 8 sub-blocks
        m = rng.integers(0, 64, size=8)              # six-bit mins
        x = rng.integers(-127, 128, size=256)        # q8_K activations
        s = np.repeat(np.arange(8), 32)              # sub-block of each value
        want_sumi = sum(int(sc[j]) * int((q[s == j] * x[s == j]).sum()) for j in range(8))
        want_summ = sum(int(m[j]) * int(x[s == j].sum()) for j in range(8))
        p0, p1, p2 = (sc[s] >> 3) * q, (sc[s] & 7) * q, m[s]
        for pl in (p0, p1, p2):
            assert pl.min() >= -128 and pl.max() <= 127
        a0, a1, a2 = (int((pl * x).sum()) for pl in (p0, p1, p2))
        assert 8 * a0 + a1 == want_sumi
        assert a2 == want_summ


def test_q6k_planes_give_ggml_integers():
    rng = np.random.default_rng(6)
    for _ in range(50):
        q = rng.integers(0, 64, size=256) - 32       # q - 32 of one super-block
        sc = rng.integers(-128, 128, size=16)        # int8 scales of its 16 groups
        x = rng.integers(-127, 128, size=256)
        g = np.repeat(np.arange(16), 16)
        want = sum(int(sc[j]) * int((q[g == j] * x[g == j]).sum()) for j in range(16))
        digits = np.array([balanced_base5(int(v)) for v in sc])  # [16][4]
        acc = []
        for k in range(4):
            pl = digits[g, k] * q
            assert pl.min() >= -128 and pl.max() <= 127
            acc.append(int((pl * x).sum()))
        assert acc[0] + 5 * acc[1] + 25 * acc[2] + 125 * acc[3] == want


def test_plane_sums_fit_int32():
    # largest |plane value| x largest |activation| x 256 values, times the largest digit weight
    assert 105 * 127 * 256 * 8 + 105 * 127 * 256 < 2 ** 31          # Q4_K: 8 A0 + A1
    assert 64 * 128 * 256 * (1 + 5 + 25 + 125) < 2 ** 31            # Q6_K: A0 + 5 A1 + 25 A2 + 125 A3
