"""The graph executor's host side and the graph oracle, without a GPU: the b200_tensor records a Graph builds from
(permuted, strided) tensors, b200_graph_supports' answers (a host function), and self-checks of oracle/graph.py
against plain float64 numpy."""

import numpy as np
import pytest

from conftest import load_package


@pytest.fixture(scope="module")
def b200():
    return load_package()


def test_records_carry_ggml_shapes_and_byte_strides(b200):
    import torch

    g = b200.Graph(None)
    x = torch.zeros((5, 16, 128), dtype=torch.float32)  # [rows, heads, head_dim]
    i = g.add(t=x)
    r = g.recs[i]
    assert list(r.ne) == [128, 16, 5, 1] and list(r.nb) == [4, 512, 8192, 40960]
    v = x.permute(1, 0, 2)  # ggml_permute(q, 0, 2, 1, 3): [head_dim, rows, heads]
    r = g.recs[g.add(t=v)]
    assert list(r.ne) == [128, 5, 16, 1] and list(r.nb)[:3] == [4, 8192, 512]  # nb3 is never used with ne3 == 1
    c = torch.zeros((300, 1024), dtype=torch.float16)[10:20]  # a cache view: rows 10..19
    r = g.recs[g.add(t=c)]
    assert r.type == b200.F16 and list(r.ne)[:2] == [1024, 10] and list(r.nb)[:2] == [2, 2048]


def test_supports_answers_on_the_host(b200):
    import torch

    g = b200.Graph(None)
    x = g.add(t=torch.zeros((4, 64)))
    w = g.add(t=torch.zeros(64))
    pos = g.add(t=torch.zeros(4, dtype=torch.int32))
    n = g.add(b200.OP_RMS_NORM, torch.zeros((4, 64)), src=[x], params=[g.fbits(1e-6)])
    m = g.add(b200.OP_MUL, torch.zeros((4, 64)), src=[n, w])
    q = g.add(t=torch.zeros((4, 2, 32)))
    ok_rope = g.add(b200.OP_ROPE, torch.zeros((4, 2, 32)), src=[q, pos], params=[32, 2, g.fbits(1e6), g.fbits(1), 0, g.fbits(1)])
    bad_rope = g.add(b200.OP_ROPE, torch.zeros((4, 2, 32)), src=[q, pos], params=[32, 0, g.fbits(1e6), g.fbits(1), 0, g.fbits(1)])
    bad_add = g.add(b200.OP_ADD, torch.zeros((4, 64)), src=[x, g.add(t=torch.zeros(48))])  # 48 does not repeat to 64
    arr = g.array()
    L = b200.lib()
    assert L.b200_graph_supports(arr, len(g.recs), n) and L.b200_graph_supports(arr, len(g.recs), m)
    assert L.b200_graph_supports(arr, len(g.recs), ok_rope)
    assert not L.b200_graph_supports(arr, len(g.recs), bad_rope)  # only NEOX
    assert not L.b200_graph_supports(arr, len(g.recs), bad_add)
    assert L.b200_graph_supports(arr, len(g.recs), x)  # a leaf


def test_graph_oracle_against_float64():
    from oracle import graph as og

    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, size=(3, 7, 64)).astype(np.float32)
    y = og.rms_norm(x, 1e-6)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6)
    assert np.allclose(y, ref, rtol=1e-6, atol=1e-7)
    # rope at position 0 is the identity; rotations keep each pair's norm
    q = rng.normal(0, 1, size=(4, 2, 32)).astype(np.float32)
    r = og.rope_neox(q, np.array([0, 1, 5, 1000]), 32, 1e6)
    assert np.array_equal(r[0], q[0])
    n0 = q[..., :16] ** 2 + q[..., 16:] ** 2
    n1 = r[..., :16] ** 2 + r[..., 16:] ** 2
    assert np.allclose(n0, n1, rtol=1e-5)
    # softmax rows sum to one; masked entries get zero
    s = rng.normal(0, 1, size=(2, 3, 10)).astype(np.float32)
    mask = np.zeros((3, 10), np.float32)
    mask[:, 8:] = -np.inf
    p = og.soft_max(s, mask, 0.5)
    assert np.allclose(p.sum(-1), 1.0, rtol=1e-6) and np.all(p[..., 8:] == 0)
    # products of plain matrices, with broadcasting over heads
    a = rng.normal(0, 1, size=(2, 5, 16)).astype(np.float16)
    b = rng.normal(0, 1, size=(4, 3, 16)).astype(np.float32)
    got = og.mul_mat_plain(a, b)
    want = np.einsum("hmk,hnk->hmn", b.astype(np.float16).astype(np.float64), np.repeat(a, 2, axis=0).astype(np.float64))
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6)
    # attention equals softmax(q k^T scale + mask) v
    H, Hkv, nq, nkv, D = 4, 2, 3, 9, 16
    q = rng.normal(0, 1, size=(H, nq, D)).astype(np.float32)
    k = rng.normal(0, 1, size=(Hkv, nkv, D)).astype(np.float16)
    v = rng.normal(0, 1, size=(Hkv, nkv, D)).astype(np.float16)
    m = np.zeros((nq, nkv), np.float16)
    m[0, 5:] = -np.inf
    o = og.flash_attn(q, k, v, m, 0.25)
    for h in range(H):
        kk, vv = k[h // 2].astype(np.float64), v[h // 2].astype(np.float64)
        sc = q[h].astype(np.float16).astype(np.float64) @ kk.T * 0.25 + m.astype(np.float64)
        w = np.exp(sc - sc.max(-1, keepdims=True))
        ref = (w / w.sum(-1, keepdims=True)) @ vv
        assert np.allclose(o[:, h], ref, rtol=1e-5, atol=1e-6)
    assert np.array_equal(og.argmax(np.array([[1, 3, 3, 2]], np.float32)), [1])
