"""CPU restatement of the non-product ops of a Qwen3 decoder graph (TEST INFRASTRUCTURE ONLY: the checker of
b200_graph_compute; the product path never imports it).

ggml defines these ops in its own source, which is absent from the reference checkout; what follows restates their
documented behaviour as Qwen3Decoder::layers / outputs uses them (src/common/qwen3-decoder.cpp:350-438) — ggml_rms_norm,
ggml_mul / ggml_add with the second operand repeated, ggml_rope_ext in NEOX mode, ggml_set_rows into the F16 KV cache,
ggml_soft_max_ext with a mask, ggml_flash_attn_ext, ggml_swiglu_split, ggml_argmax, ggml_concat (the talker's code
predictor input, src/families/qwen3-tts/talker.cpp:55), ggml_mul_mat of F16 / F32 matrices — with the order-dependent reductions defined order-free, as the device computes them: sums and exponentials
in double, rounded once to float32.

Arrays are numpy arrays in torch order: shape (ne3, ne2, ne1, ne0) of the ggml tensor, innermost dimension last.
"""

import numpy as np

F32 = np.float32


def rms_norm(x, eps):
    """Rows (last axis): x * fl32(1 / sqrt(fl32(mean(x^2)) + eps)), the mean from a double sum."""
    x = np.asarray(x, dtype=F32)
    mean = (np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True) / x.shape[-1]).astype(F32)
    scale = (F32(1.0) / np.sqrt((mean + F32(eps)).astype(F32), dtype=F32)).astype(F32)
    return (x * scale).astype(F32)


def repeat_to(b, shape):
    """ggml's repeat: b tiled to `shape` (each dimension of b divides the target's)."""
    b = np.asarray(b)
    b = b.reshape((1,) * (len(shape) - b.ndim) + b.shape)
    return np.tile(b, [s // t for s, t in zip(shape, b.shape)])


def mul(a, b):
    return (np.asarray(a, F32) * repeat_to(b, np.shape(a)).astype(F32)).astype(F32)


def add(a, b):
    return (np.asarray(a, F32) + repeat_to(b, np.shape(a)).astype(F32)).astype(F32)


def concat(a, b, dim):
    """ggml_concat along ggml dimension `dim` (0 = innermost = the last numpy axis)."""
    a, b = np.asarray(a), np.asarray(b)
    return np.concatenate([a, b], axis=a.ndim - 1 - dim)


def silu(x):
    x = np.asarray(x, dtype=F32).astype(np.float64)
    return (x / (1.0 + np.exp(-x))).astype(F32)


def swiglu(a, b):
    return (silu(a) * np.asarray(b, F32)).astype(F32)


def rope_neox(x, pos, n_dims, base):
    """x [..., tokens, heads, head_dim]; pos int [tokens]. For i < n_dims / 2 the pair (x[i], x[i + n_dims / 2]) turns
    by theta = pos * base^(-2 i / n_dims), computed in double, cos and sin rounded once to float32; values past n_dims
    are copied."""
    x = np.asarray(x, dtype=F32)
    half = n_dims // 2
    i = np.arange(half, dtype=np.float64)
    theta = np.asarray(pos, dtype=np.float64)[:, None] * np.power(float(base), -2.0 * i / n_dims)[None, :]  # [tokens, half]
    c = np.cos(theta).astype(F32)[:, None, :]
    s = np.sin(theta).astype(F32)[:, None, :]
    y = x.copy()
    x0, x1 = x[..., :half], x[..., half:n_dims]
    y[..., :half] = ((x0 * c).astype(F32) - (x1 * s).astype(F32)).astype(F32)
    y[..., half:n_dims] = ((x0 * s).astype(F32) + (x1 * c).astype(F32)).astype(F32)
    return y


def soft_max(x, mask, scale):
    """Rows of softmax(x * scale + mask): v = fl(fl(x scale) + mask), e = fl32(exp(v - max)), y = fl(e / fl32(sum e))
    with the sum in double. x [..., rows, n]; mask [>= rows, n] (its row is the row's index), or None."""
    x = np.asarray(x, dtype=F32)
    v = (x * F32(scale)).astype(F32)
    if mask is not None:
        m = np.asarray(mask, F32)[: x.shape[-2], : x.shape[-1]]
        v = (v + m).astype(F32)
    mx = v.max(axis=-1, keepdims=True)
    e = np.exp((v - mx).astype(F32).astype(np.float64)).astype(F32)
    s = e.astype(np.float64).sum(axis=-1, keepdims=True).astype(F32)
    return (e / s).astype(F32)


def mul_mat_plain(a, b):
    """ggml_mul_mat of a plain matrix: a [A3, A2, N, K] (F16 or F32), b [B3, B2, M, K] F32 with B2 % A2 == B3 % A3
    == 0 -> [B3, B2, M, N]. b is rounded to a's type first (ggml's CPU converts src1 to src0's vec_dot type), each
    product is rounded to float32 (exact for F16 x F16), the products are summed exactly (double) and rounded once."""
    a4 = np.asarray(a).reshape((1,) * (4 - np.ndim(a)) + np.shape(a))
    b4 = np.asarray(b, F32).reshape((1,) * (4 - np.ndim(b)) + np.shape(b))
    if a4.dtype == np.float16:
        b4 = b4.astype(np.float16)
    r3, r2 = b4.shape[0] // a4.shape[0], b4.shape[1] // a4.shape[1]
    out = np.empty((b4.shape[0], b4.shape[1], b4.shape[2], a4.shape[2]), dtype=F32)
    for i3 in range(b4.shape[0]):
        for i2 in range(b4.shape[1]):
            A = a4[i3 // r3, i2 // r2].astype(F32)     # [N, K]
            B = b4[i3, i2].astype(F32)                 # [M, K]
            prod = (B[:, None, :] * A[None, :, :]).astype(F32)  # [M, N, K], each product rounded to float32
            out[i3, i2] = prod.astype(np.float64).sum(axis=-1).astype(F32)
    return out.reshape(b4.shape[:2] + out.shape[2:]) if np.ndim(b) == 4 else out.reshape(np.shape(b)[:-1] + (a4.shape[2],))


def flash_attn(q, k, v, mask, scale):
    """ggml_flash_attn_ext: q [H, n_q, D] F32, k and v [H_kv, n_kv, D] F16, mask [>= n_q, >= n_kv] F16 or None ->
    [n_q, H, D] F32. Per (query, head): q rounded to F16; s_j = fl32(exact sum of q k_j) * scale + mask;
    w_j = fl32(exp(s_j - max)); out = fl32(sum_j w_j v_j / sum_j w_j), sums in double. Key / value head = head /
    (H / H_kv)."""
    q = np.asarray(q, F32)
    H, nq, D = q.shape
    Hkv, nkv = k.shape[0], k.shape[1]
    out = np.empty((nq, H, D), dtype=F32)
    qh = q.astype(np.float16).astype(F32)
    for h in range(H):
        kk = np.asarray(k[h // (H // Hkv)], np.float16).astype(F32)  # [n_kv, D]
        vv = np.asarray(v[h // (H // Hkv)], np.float16).astype(F32)
        for iq in range(nq):
            prod = (kk * qh[h, iq][None, :]).astype(F32)
            s = (prod.astype(np.float64).sum(axis=-1).astype(F32) * F32(scale)).astype(F32)
            if mask is not None:
                s = (s + np.asarray(mask, np.float16)[iq, :nkv].astype(F32)).astype(F32)
            w = np.exp((s - s.max()).astype(F32).astype(np.float64)).astype(F32)
            acc = (w[:, None].astype(F32) * vv).astype(F32).astype(np.float64).sum(axis=0)
            out[iq, h] = (acc / w.astype(np.float64).sum()).astype(F32)
    return out


def argmax(x):
    """Index of the first largest value of each row (last axis), int32."""
    return np.argmax(np.asarray(x, F32), axis=-1).astype(np.int32)
