"""The routed-expert FFN block (b200_moe_ffn) against the oracle, on one GPU and as two expert shards.

Reference: TextModel::experts (src/families/drama3/text-model.cpp:198-221): gate and up MUL_MAT_ID, SwiGLU, down
MUL_MAT_ID, router-weighted sum over the chosen experts. The chain re-quantizes the SwiGLU output, so it is judged
like the decoder stack: per-token cosine similarity >= 0.9999 and a small relative error.
"""

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu


def reference(oracle, gu_b, dn_b, H, F, E, x, ids, w, tg=8, td=8):
    gu = oracle.mul_mat_id(tg, gu_b, H, 2 * F, E, x[:, None, :], ids)  # [T, k, 2F]
    g, u = gu[..., :F], gu[..., F:]
    a = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
    dn = oracle.mul_mat_id(td, dn_b, F, H, E, a, ids)  # [T, k, H]
    out = np.zeros((x.shape[0], H), dtype=np.float32)
    for s in range(ids.shape[1]):
        out = (out + dn[:, s] * w[:, s:s + 1]).astype(np.float32)
    return out


def test_moe_ffn_full_and_sharded(oracle):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    b200 = load_package()
    ctx = b200.Context(0)
    try:
        rng = np.random.default_rng(5)
        E, H, F, T, k = 16, 512, 256, 40, 4
        gu_b = oracle.quantize(8, rng.normal(0, 0.02, size=(E * 2 * F, H)).astype(np.float32))
        dn_b = oracle.quantize(8, rng.normal(0, 0.02, size=(E * H, F)).astype(np.float32))
        x = rng.normal(0, 1, size=(T, H)).astype(np.float32)
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        w = rng.random(size=(T, k)).astype(np.float32)
        w /= w.sum(1, keepdims=True)
        want = reference(oracle, gu_b, dn_b, H, F, E, x, ids, w)

        cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        gu = ctx.weight(8, H, 2 * F, E, data=gu_b)
        dn = ctx.weight(8, F, H, E, data=dn_b)
        got = ctx.moe_ffn(gu, dn, cu(x), cu(ids), cu(w)).cpu().numpy()
        ctx.synchronize()
        cos = (got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
        assert cos.min() >= 0.9999
        assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()

        # two shards of 8 experts: partial outputs sum to the full one
        half = E // 2
        rs, rd = 2 * F * H // 32 * 34, H * F // 32 * 34  # bytes per expert
        parts = []
        for sh in range(2):
            g2 = ctx.weight(8, H, 2 * F, half, data=gu_b.reshape(-1)[sh * half * rs:(sh + 1) * half * rs])
            d2 = ctx.weight(8, F, H, half, data=dn_b.reshape(-1)[sh * half * rd:(sh + 1) * half * rd])
            parts.append(ctx.moe_ffn(g2, d2, cu(x), cu(ids), cu(w), expert0=sh * half, n_expert_total=E).cpu().numpy())
            ctx.free_weight(g2)
            ctx.free_weight(d2)
        ctx.synchronize()
        assert np.abs(parts[0] + parts[1] - got).max() <= 1e-5 * np.abs(got).max()
        # an id past the last expert is reported
        bad = ids.copy()
        bad[0, 0] = E
        ctx.moe_ffn(gu, dn, cu(x), cu(bad), cu(w))
        with pytest.raises(b200.B200Error):
            ctx.synchronize()
        ctx.free_weight(gu)
        ctx.free_weight(dn)
    finally:
        ctx.close()


@pytest.mark.parametrize("tg,td", [(12, 14), (12, 12), (13, 8)])
def test_moe_ffn_kquant_experts(oracle, tg, td):
    """Drama 3 ships Q4_K files (Q4_K_M: Q4_K gate / up, Q6_K down): K-quant experts run the routed GEMV path, the
    SwiGLU rows re-quantized to q8_K for K-quant down experts. Q5_K gate|up with Q8_0 down covers the mixed case."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    b200 = load_package()
    ctx = b200.Context(0)
    try:
        rng = np.random.default_rng(7)
        E, H, F, T, k = 16, 512, 256, 40, 4
        gu_b = oracle.quantize(tg, rng.normal(0, 0.02, size=(E * 2 * F, H)).astype(np.float32))
        dn_b = oracle.quantize(td, rng.normal(0, 0.02, size=(E * H, F)).astype(np.float32))
        x = rng.normal(0, 1, size=(T, H)).astype(np.float32)
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        w = rng.random(size=(T, k)).astype(np.float32)
        w /= w.sum(1, keepdims=True)
        want = reference(oracle, gu_b, dn_b, H, F, E, x, ids, w, tg, td)
        cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
        gu = ctx.weight(tg, H, 2 * F, E, data=gu_b)
        dn = ctx.weight(td, F, H, E, data=dn_b)
        got = ctx.moe_ffn(gu, dn, cu(x), cu(ids), cu(w)).cpu().numpy()
        ctx.synchronize()
        cos = (got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
        assert cos.min() >= 0.9999
        assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()
        ctx.free_weight(gu)
        ctx.free_weight(dn)
    finally:
        ctx.close()
