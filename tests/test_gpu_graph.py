"""b200_graph_compute against the graph oracle (oracle/graph.py) on the GPU: every op of a Qwen3 decoder graph, then a
whole decoder layer with its KV cache, as Qwen3Decoder::layers / outputs builds it (src/common/qwen3-decoder.cpp:
350-438): RMS_NORM * attn_norm, the q / k / v products, the per-head q / k norms, SET_ROWS of v and of the rotated k
into the F16 cache at the rows' positions, NEOX ROPE, FLASH_ATTN over the cache with the causal mask, the o product and
residual, RMS_NORM * ffn_norm, gate and up, SWIGLU, down and residual; then the head and ARGMAX.

The device computes every float step as the oracle defines it (sums and exponentials in double, rounded once), so the
op tests expect equal floats except near rounding ties (>= 99 % bit-equal) and the layer, whose products re-quantize
their inputs, expects the same of its output.
"""

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu

F16, F32 = np.float16, np.float32


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


def cu(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def close_and_mostly_equal(got, want, rtol=1e-5, frac=0.99):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    scale = np.abs(want).max() + 1e-30
    assert np.abs(got - want).max() <= rtol * scale, f"max err {np.abs(got - want).max() / scale:.3g} of max |want|"
    same = float(np.mean(got == want))
    assert same >= frac, f"bit-equal fraction {same:.4f}"


def run(b200, ctx, build):
    import torch

    g = b200.Graph(ctx)
    out = build(g)
    g.compute()
    ctx.synchronize()
    torch.cuda.synchronize()
    return out


def test_elementwise_and_norm_ops(b200, ctx):
    import torch

    from oracle import graph as og

    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, size=(5, 16, 128)).astype(F32)
    w = rng.normal(1, 0.1, size=128).astype(F32)
    y = rng.normal(0, 1, size=(5, 16, 128)).astype(F32)
    outs = {k: torch.empty((5, 16, 128), device="cuda") for k in ("norm", "mul", "add", "swiglu", "scale")}
    outs["fill"] = cu(x)                                      # rows 2..4 set to 0 in place (a view), rows 0..1 kept
    outs["concat"] = torch.empty((5, 16, 256), device="cuda")  # along dimension 0
    outs["concat1"] = torch.empty((5, 32, 128), device="cuda")  # along dimension 1

    def build(g):
        X, W, Y = g.add(t=cu(x)), g.add(t=cu(w)), g.add(t=cu(y))
        n = g.add(b200.OP_RMS_NORM, outs["norm"], src=[X], params=[g.fbits(1e-6)])
        g.add(b200.OP_MUL, outs["mul"], src=[n, W])
        g.add(b200.OP_ADD, outs["add"], src=[X, Y])
        g.add(b200.OP_SWIGLU, outs["swiglu"], src=[X, Y])
        g.add(b200.OP_SCALE, outs["scale"], src=[X], params=[g.fbits(0.125), g.fbits(0.5)])
        g.add(b200.OP_FILL, outs["fill"][2:], params=[g.fbits(0.0)])
        g.add(b200.OP_CONCAT, outs["concat"], src=[X, Y], params=[0])
        g.add(b200.OP_CONCAT, outs["concat1"], src=[X, Y], params=[1])
        return outs

    got = {k: v.cpu().numpy() for k, v in run(b200, ctx, build).items()}
    n = og.rms_norm(x, 1e-6)
    close_and_mostly_equal(got["norm"], n)
    close_and_mostly_equal(got["mul"], og.mul(n, w))
    assert np.array_equal(got["add"], og.add(x, y))
    close_and_mostly_equal(got["swiglu"], og.swiglu(x, y))
    assert np.array_equal(got["scale"], (x * F32(0.125) + F32(0.5)).astype(F32))
    assert np.array_equal(got["fill"][:2], x[:2]) and not got["fill"][2:].any()
    assert np.array_equal(got["concat"], og.concat(x, y, 0)) and np.array_equal(got["concat1"], og.concat(x, y, 1))


def test_rope_cache_rows_softmax_attention_products(b200, ctx):
    import torch

    from oracle import graph as og

    rng = np.random.default_rng(2)
    rows, H, Hkv, D, n_past, cap = 5, 16, 8, 128, 37, 300
    q = rng.normal(0, 1, size=(rows, H, D)).astype(F32)
    pos = np.arange(n_past, n_past + rows, dtype=np.int32)
    cache = rng.normal(0, 1, size=(cap, Hkv * D)).astype(F16)
    kv = rng.normal(0, 1, size=(rows, Hkv * D)).astype(F32)
    n_kv = 64
    mask = np.full((8, n_kv), -np.inf, dtype=F16)
    for i in range(rows):
        mask[i, : n_past + i + 1] = 0
    scores = rng.normal(0, 3, size=(H, rows, n_kv)).astype(F32)
    logits = rng.normal(0, 1, size=(rows, 3000)).astype(F32)
    logits[2, 17] = logits[2, 2000] = 50.0  # a tie: the first index wins
    table = rng.normal(0, 1, size=(40, 96)).astype(F32)
    ids = np.array([3, 39, 0, 3], dtype=np.int32)

    cache_d = cu(cache)
    o = {"rope": torch.empty((rows, H, D), device="cuda"), "sm": torch.empty((H, rows, n_kv), device="cuda"),
         "attn": torch.empty((rows, H, D), device="cuda"), "kq": torch.empty((H, rows, n_kv), device="cuda"),
         "arg": torch.empty(rows, dtype=torch.int32, device="cuda"), "rows": torch.empty((4, 96), device="cuda"),
         "cpy": torch.empty((H, rows, D), dtype=torch.float16, device="cuda")}

    def build(g):
        Q, P = g.add(t=cu(q)), g.add(t=cu(pos))
        r = g.add(b200.OP_ROPE, o["rope"], src=[Q, P], params=[D, 2, g.fbits(1e6), g.fbits(1.0), 0, g.fbits(1.0)])
        C = g.add(t=cache_d)
        g.add(b200.OP_SET_ROWS, cache_d, src=[g.add(t=cu(kv)), P, C])
        keys = cache_d[:n_kv].view(n_kv, Hkv, D).permute(1, 0, 2)  # [Hkv, n_kv, D]: the cache view, permuted
        K = g.add(t=keys)
        M = g.add(t=cu(mask))
        qh = o["rope"].permute(1, 0, 2)  # [H, rows, D]
        g.add(b200.OP_FLASH_ATTN, o["attn"].permute(0, 1, 2), src=[g.add(t=qh), K, K, M], params=[g.fbits(D ** -0.5)])
        g.add(b200.OP_MUL_MAT, o["kq"], src=[K, g.add(t=qh)])  # the soft-max path's K Q product, GQA broadcast
        g.add(b200.OP_SOFT_MAX, o["sm"], src=[g.add(t=cu(scores)), M], params=[g.fbits(0.5)])
        g.add(b200.OP_ARGMAX, o["arg"], src=[g.add(t=cu(logits))])
        g.add(b200.OP_GET_ROWS, o["rows"], src=[g.add(t=cu(table)), g.add(t=cu(ids))])
        g.add(b200.OP_CPY, o["cpy"], src=[g.add(t=qh), g.add(t=o["cpy"])])
        return o

    got = {k: v.cpu().numpy() for k, v in run(b200, ctx, build).items()}
    want_rope = og.rope_neox(q, pos, D, 1e6)
    close_and_mostly_equal(got["rope"], want_rope)
    cache_w = cache.copy()
    cache_w[pos] = kv.astype(F16)
    assert np.array_equal(cache_d.cpu().numpy(), cache_w)
    keys = cache_w[:n_kv].reshape(n_kv, Hkv, D).transpose(1, 0, 2)
    qh = got["rope"].transpose(1, 0, 2)
    close_and_mostly_equal(got["attn"], og.flash_attn(qh, keys, keys, mask, D ** -0.5))
    close_and_mostly_equal(got["kq"], og.mul_mat_plain(np.repeat(keys, H // Hkv, axis=0), qh))
    close_and_mostly_equal(got["sm"], og.soft_max(scores, mask.astype(F32), 0.5))
    assert np.array_equal(got["arg"], og.argmax(logits)) and got["arg"][2] == 17
    assert np.array_equal(got["rows"], table[ids])
    assert np.array_equal(got["cpy"], qh.astype(F16))


def test_qwen3_decoder_layer_with_kv_cache(b200, ctx, oracle):
    """One decoder layer of the Qwen3-TTS 0.6B talker's shapes (hidden 1024, 16 / 8 heads of 128, ffn 3072, Q8_0) with
    37 cached positions, for a step (1 row), a verify block (5 rows: src/common/qwen3-decoder.cpp:492-510) and a
    prefill block (64 rows), then the head and argmax. From 32 rows the Q8_0 products run on the int8 tensor cores,
    whose per-block float steps are summed in a different order: that block is checked by row cosine (>= 0.99999 for
    the layer output, >= 0.9999 for the logits), its caches within one F16 rounding and its argmax wherever the top
    two logits are apart."""
    import torch

    from oracle import graph as og

    Q8 = b200.Q8_0
    hid, H, Hkv, D, ffn, vocab, n_past, cap = 1024, 16, 8, 128, 3072, 3072, 37, 512
    eps, base = 1e-6, 1e6
    rng = np.random.default_rng(3)

    def wq(n, k):
        return oracle.quantize(Q8, rng.normal(0, 0.02, size=(n, k)).astype(F32))

    Wq, Wk, Wv, Wo = wq(H * D, hid), wq(Hkv * D, hid), wq(Hkv * D, hid), wq(hid, H * D)
    Wg, Wu, Wd, Wh = wq(ffn, hid), wq(ffn, hid), wq(hid, ffn), wq(vocab, hid)
    attn_norm, ffn_norm, out_norm = (rng.normal(1, 0.1, size=hid).astype(F32) for _ in range(3))
    q_norm, k_norm = rng.normal(1, 0.1, size=D).astype(F32), rng.normal(1, 0.1, size=D).astype(F32)
    cache0_k = rng.normal(0, 1, size=(cap, Hkv * D)).astype(F16)
    cache0_v = rng.normal(0, 1, size=(cap, Hkv * D)).astype(F16)
    dev = {name: ctx.weight(Q8, k, n, data=w) for name, (w, k, n) in
           {"q": (Wq, hid, H * D), "k": (Wk, hid, Hkv * D), "v": (Wv, hid, Hkv * D), "o": (Wo, H * D, hid),
            "g": (Wg, hid, ffn), "u": (Wu, hid, ffn), "d": (Wd, ffn, hid), "h": (Wh, hid, vocab)}.items()}

    def mm(w, x, n, k):
        return oracle.mul_mat(Q8, w, k, n, x)

    for rows in (1, 5, 64):
        exact = rows < 32
        x0 = rng.normal(0, 1, size=(rows, hid)).astype(F32)
        pos = np.arange(n_past, n_past + rows, dtype=np.int32)
        n_kv = 256  # the cache rows attention reads: whole blocks, the rest masked
        mask = np.full((max(8, rows), n_kv), -np.inf, dtype=F16)
        for i in range(rows):
            mask[i, : n_past + i + 1] = 0

        # ---- the oracle ----
        h = og.mul(og.rms_norm(x0, eps), attn_norm)
        q = mm(Wq, h, H * D, hid).reshape(rows, H, D)
        k = mm(Wk, h, Hkv * D, hid).reshape(rows, Hkv, D)
        v = mm(Wv, h, Hkv * D, hid)
        q = og.mul(og.rms_norm(q, eps), q_norm)
        k = og.mul(og.rms_norm(k, eps), k_norm)
        ck, cv = cache0_k.copy(), cache0_v.copy()
        cv[pos] = v.astype(F16)
        q = og.rope_neox(q, pos, D, base)
        k = og.rope_neox(k, pos, D, base)
        ck[pos] = k.reshape(rows, Hkv * D).astype(F16)
        keys = ck[:n_kv].reshape(n_kv, Hkv, D).transpose(1, 0, 2)
        vals = cv[:n_kv].reshape(n_kv, Hkv, D).transpose(1, 0, 2)
        att = og.flash_attn(q.transpose(1, 0, 2), keys, vals, mask, D ** -0.5).reshape(rows, H * D)
        x1 = og.add(x0, mm(Wo, att, hid, H * D))
        h2 = og.mul(og.rms_norm(x1, eps), ffn_norm)
        a = og.swiglu(mm(Wg, h2, ffn, hid), mm(Wu, h2, ffn, hid))
        x2 = og.add(x1, mm(Wd, a, hid, ffn))
        logits = mm(Wh, og.mul(og.rms_norm(x2, eps), out_norm), vocab, hid)

        # ---- the same graph on the device ----
        ck_d, cv_d = cu(cache0_k), cu(cache0_v)
        T = {name: torch.empty(shape, device="cuda") for name, shape in
             {"h0": (rows, hid), "h": (rows, hid), "q": (rows, H * D), "k": (rows, Hkv * D), "v": (rows, Hkv * D),
              "qn0": (rows, H, D), "qn": (rows, H, D), "kn0": (rows, Hkv, D), "kn": (rows, Hkv, D), "qr": (rows, H, D),
              "kr": (rows, Hkv, D), "att": (rows, H, D), "o": (rows, hid), "x1": (rows, hid), "f0": (rows, hid),
              "f": (rows, hid), "gate": (rows, ffn), "up": (rows, ffn), "act": (rows, ffn), "dn": (rows, hid),
              "x2": (rows, hid), "n0": (rows, hid), "n": (rows, hid), "logits": (rows, vocab)}.items()}
        pick = torch.empty(rows, dtype=torch.int32, device="cuda")

        def build(g):
            R = lambda name: T[name]
            X = g.add(t=cu(x0))
            P = g.add(t=cu(pos))
            M = g.add(t=cu(mask))
            Wd_ = {n: g.add(weight=w) for n, w in dev.items()}
            an, fn, on = g.add(t=cu(attn_norm)), g.add(t=cu(ffn_norm)), g.add(t=cu(out_norm))
            qn_w, kn_w = g.add(t=cu(q_norm)), g.add(t=cu(k_norm))
            eps_b = g.fbits(eps)
            h0 = g.add(b200.OP_RMS_NORM, R("h0"), src=[X], params=[eps_b])
            hh = g.add(b200.OP_MUL, R("h"), src=[h0, an])
            q_ = g.add(b200.OP_MUL_MAT, R("q"), src=[Wd_["q"], hh])
            k_ = g.add(b200.OP_MUL_MAT, R("k"), src=[Wd_["k"], hh])
            v_ = g.add(b200.OP_MUL_MAT, R("v"), src=[Wd_["v"], hh])
            q3, k3 = g.add(t=R("q").view(rows, H, D)), g.add(t=R("k").view(rows, Hkv, D))  # reshape_3d: views
            qn = g.add(b200.OP_MUL, R("qn"), src=[g.add(b200.OP_RMS_NORM, R("qn0"), src=[q3], params=[eps_b]), qn_w])
            kn = g.add(b200.OP_MUL, R("kn"), src=[g.add(b200.OP_RMS_NORM, R("kn0"), src=[k3], params=[eps_b]), kn_w])
            CK, CV = g.add(t=ck_d), g.add(t=cv_d)
            g.add(b200.OP_SET_ROWS, cv_d, src=[v_, P, CV])
            rope = [D, 2, g.fbits(base), g.fbits(1.0), 0, g.fbits(1.0)]
            qr = g.add(b200.OP_ROPE, R("qr"), src=[qn, P], params=rope)
            kr = g.add(b200.OP_ROPE, R("kr"), src=[kn, P], params=rope)
            g.add(b200.OP_SET_ROWS, ck_d, src=[g.add(t=R("kr").view(rows, Hkv * D)), P, CK])
            keys = g.add(t=ck_d[:n_kv].view(n_kv, Hkv, D).permute(1, 0, 2))
            vals = g.add(t=cv_d[:n_kv].view(n_kv, Hkv, D).permute(1, 0, 2))
            qh = g.add(t=R("qr").permute(1, 0, 2))
            att = g.add(b200.OP_FLASH_ATTN, R("att"), src=[qh, keys, vals, M], params=[g.fbits(D ** -0.5)])
            o = g.add(b200.OP_MUL_MAT, R("o"), src=[Wd_["o"], g.add(t=R("att").view(rows, H * D))])
            x1 = g.add(b200.OP_ADD, R("x1"), src=[X, o])
            f = g.add(b200.OP_MUL, R("f"), src=[g.add(b200.OP_RMS_NORM, R("f0"), src=[x1], params=[eps_b]), fn])
            ga = g.add(b200.OP_MUL_MAT, R("gate"), src=[Wd_["g"], f])
            up = g.add(b200.OP_MUL_MAT, R("up"), src=[Wd_["u"], f])
            act = g.add(b200.OP_SWIGLU, R("act"), src=[ga, up])
            dn = g.add(b200.OP_MUL_MAT, R("dn"), src=[Wd_["d"], act])
            x2 = g.add(b200.OP_ADD, R("x2"), src=[x1, dn])
            nn = g.add(b200.OP_MUL, R("n"), src=[g.add(b200.OP_RMS_NORM, R("n0"), src=[x2], params=[eps_b]), on])
            lg = g.add(b200.OP_MUL_MAT, R("logits"), src=[Wd_["h"], nn])
            g.add(b200.OP_ARGMAX, pick, src=[lg])
            return T

        run(b200, ctx, build)
        if exact:
            close_and_mostly_equal(T["x2"].cpu().numpy(), x2)
            close_and_mostly_equal(T["logits"].cpu().numpy(), logits)
            assert np.array_equal(ck_d.cpu().numpy(), ck) and np.array_equal(cv_d.cpu().numpy(), cv)
            assert np.array_equal(pick.cpu().numpy(), og.argmax(logits))
            continue
        # a float difference inside a product can move an activation across a q8_0 rounding boundary of a later
        # product, which changes that element by a quantization step and the later product's whole row with it: rows
        # are compared by cosine, elements only against a bound a quantization step cannot reach past
        for got, want, bar in ((T["x2"].cpu().numpy(), x2, 0.99999), (T["logits"].cpu().numpy(), logits, 0.9999)):
            g64, w64 = got.astype(np.float64), want.astype(np.float64)
            cos = (g64 * w64).sum(-1) / np.sqrt((g64 * g64).sum(-1) * (w64 * w64).sum(-1))
            assert cos.min() >= bar, f"row cosine {cos.min():.7f}"
            assert np.abs(g64 - w64).max() <= 1e-2 * np.abs(w64).max()
        for got, want in ((ck_d, ck), (cv_d, cv)):
            g32, w32 = got.cpu().numpy().astype(F32), want.astype(F32)
            assert np.all(np.abs(g32 - w32) <= np.abs(w32) * 2.0 ** -10 + 2.0 ** -24)
        srt = np.sort(logits, axis=-1)
        apart = srt[:, -1] - srt[:, -2] > 1e-3 * np.abs(logits).max()
        assert np.array_equal(pick.cpu().numpy()[apart], og.argmax(logits)[apart]) and apart.mean() > 0.5
    for w in dev.values():
        ctx.free_weight(w)


def test_block_equals_steps(b200, ctx, oracle):
    """Blocked computation equals step-by-step computation (the property speech.cpp's qwen3-decoder-check asserts,
    checks/common/qwen3-decoder-check.cpp): a decoder layer run over a block of 6 rows, and the same 6 rows run as 6
    one-row steps that each append to the KV cache, give bit-identical outputs and caches. With fewer than 32 rows
    every product quantizes and sums each row on its own, and attention reads the same cache prefix either way."""
    import torch

    Q8 = b200.Q8_0
    hid, H, Hkv, D, ffn, n_past, cap, n_kv, rows = 256, 4, 2, 64, 512, 11, 64, 64, 6
    base = 1e6
    rng = np.random.default_rng(5)

    def wq(n, k):
        return ctx.weight(Q8, k, n, data=oracle.quantize(Q8, rng.normal(0, 0.05, size=(n, k)).astype(F32)))

    Wq, Wk, Wv, Wo, Wg, Wu, Wd = wq(H * D, hid), wq(Hkv * D, hid), wq(Hkv * D, hid), wq(hid, H * D), wq(ffn, hid), wq(ffn, hid), wq(hid, ffn)
    norms = [cu(rng.normal(1, 0.1, size=n).astype(F32)) for n in (hid, D, D, hid)]
    cache_k0 = rng.normal(0, 1, size=(cap, Hkv * D)).astype(F16)
    cache_v0 = rng.normal(0, 1, size=(cap, Hkv * D)).astype(F16)
    x_all = rng.normal(0, 1, size=(rows, hid)).astype(F32)

    def layer(x, first, ck_d, cv_d):
        n = x.shape[0]
        pos = np.arange(first, first + n, dtype=np.int32)
        mask = np.full((max(8, n), n_kv), -np.inf, dtype=F16)
        for i in range(n):
            mask[i, : first + i + 1] = 0
        T = {k: torch.empty(s, device="cuda") for k, s in
             {"h0": (n, hid), "h": (n, hid), "q": (n, H * D), "k": (n, Hkv * D), "v": (n, Hkv * D), "qn0": (n, H, D),
              "qn": (n, H, D), "kn0": (n, Hkv, D), "kn": (n, Hkv, D), "qr": (n, H, D), "kr": (n, Hkv, D),
              "att": (n, H, D), "o": (n, hid), "x1": (n, hid), "f0": (n, hid), "f": (n, hid), "g": (n, ffn),
              "u": (n, ffn), "a": (n, ffn), "d": (n, hid), "x2": (n, hid)}.items()}
        g = b200.Graph(ctx)
        e = g.fbits(1e-6)
        X, P, M = g.add(t=cu(x)), g.add(t=cu(pos)), g.add(t=cu(mask))
        W = [g.add(weight=w) for w in (Wq, Wk, Wv, Wo, Wg, Wu, Wd)]
        an, qw, kw, fw = (g.add(t=t) for t in norms)
        hh = g.add(b200.OP_MUL, T["h"], src=[g.add(b200.OP_RMS_NORM, T["h0"], src=[X], params=[e]), an])
        q_, k_, v_ = (g.add(b200.OP_MUL_MAT, T[nm], src=[W[j], hh]) for j, nm in enumerate("qkv"))
        q3, k3 = g.add(t=T["q"].view(n, H, D)), g.add(t=T["k"].view(n, Hkv, D))
        qn = g.add(b200.OP_MUL, T["qn"], src=[g.add(b200.OP_RMS_NORM, T["qn0"], src=[q3], params=[e]), qw])
        kn = g.add(b200.OP_MUL, T["kn"], src=[g.add(b200.OP_RMS_NORM, T["kn0"], src=[k3], params=[e]), kw])
        CK, CV = g.add(t=ck_d), g.add(t=cv_d)
        g.add(b200.OP_SET_ROWS, cv_d, src=[v_, P, CV])
        rope = [D, 2, g.fbits(base), g.fbits(1.0), 0, g.fbits(1.0)]
        g.add(b200.OP_ROPE, T["qr"], src=[qn, P], params=rope)
        g.add(b200.OP_ROPE, T["kr"], src=[kn, P], params=rope)
        g.add(b200.OP_SET_ROWS, ck_d, src=[g.add(t=T["kr"].view(n, Hkv * D)), P, CK])
        keys = g.add(t=ck_d[:n_kv].view(n_kv, Hkv, D).permute(1, 0, 2))
        vals = g.add(t=cv_d[:n_kv].view(n_kv, Hkv, D).permute(1, 0, 2))
        g.add(b200.OP_FLASH_ATTN, T["att"], src=[g.add(t=T["qr"].permute(1, 0, 2)), keys, vals, M], params=[g.fbits(D ** -0.5)])
        o = g.add(b200.OP_MUL_MAT, T["o"], src=[W[3], g.add(t=T["att"].view(n, H * D))])
        x1 = g.add(b200.OP_ADD, T["x1"], src=[X, o])
        f = g.add(b200.OP_MUL, T["f"], src=[g.add(b200.OP_RMS_NORM, T["f0"], src=[x1], params=[e]), fw])
        ga, up = g.add(b200.OP_MUL_MAT, T["g"], src=[W[4], f]), g.add(b200.OP_MUL_MAT, T["u"], src=[W[5], f])
        dn = g.add(b200.OP_MUL_MAT, T["d"], src=[W[6], g.add(b200.OP_SWIGLU, T["a"], src=[ga, up])])
        g.add(b200.OP_ADD, T["x2"], src=[x1, dn])
        g.compute()
        ctx.synchronize()
        return T["x2"].cpu().numpy()

    ck_b, cv_b = cu(cache_k0), cu(cache_v0)
    block = layer(x_all, n_past, ck_b, cv_b)
    ck_s, cv_s = cu(cache_k0), cu(cache_v0)
    steps = np.concatenate([layer(x_all[i : i + 1], n_past + i, ck_s, cv_s) for i in range(rows)])
    assert np.array_equal(block, steps)
    assert torch.equal(ck_b, ck_s) and torch.equal(cv_b, cv_s)
    for w in (Wq, Wk, Wv, Wo, Wg, Wu, Wd):
        ctx.free_weight(w)
