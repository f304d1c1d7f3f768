"""CPU reference of the Qwen3 decoder step's matmul stack, built on the oracle (TEST INFRASTRUCTURE ONLY).

Follows Qwen3Decoder::layers / outputs (src/common/qwen3-decoder.cpp:350-413, 422-438) for one token at the first
position of a sequence (attention output = each query head's key/value head's value row). Products go through the
oracle's ggml-CPU-semantics mul_mat; the glue is float32 as ggml's CPU computes it, with its two order-dependent reductions defined order-free: rms_norm sums
the squares in double (rounded once to float32 for the mean), scale = 1/sqrt(mean + eps) in float32, (x * scale) * w;
silu(x) = x / (1 + exp(-x)) in double, rounded once.
"""

import numpy as np

from . import oracle

Q8_0, Q4_K, Q6_K = oracle.Q8_0, oracle.Q4_K, oracle.Q6_K

# The configs of BASELINE.json: Qwen3-TTS 0.6B talker (config 2), Qwen3-ASR 1.7B-shaped decoder (config 3),
# Qwen3-TTS 1.7B talker (config 4).
CONFIGS = {
    "tts06": dict(n_layer=28, hidden=1024, n_head=16, n_kv_head=8, head_dim=128, ffn=3072, n_vocab=3072,
                  type_attn=Q8_0, type_ffn_up=Q8_0, type_ffn_down=Q8_0, type_head=Q8_0),
    "asr17": dict(n_layer=28, hidden=2048, n_head=16, n_kv_head=8, head_dim=128, ffn=6144, n_vocab=151936,
                  type_attn=Q4_K, type_ffn_up=Q4_K, type_ffn_down=Q6_K, type_head=Q6_K),
    "tts17": dict(n_layer=28, hidden=2048, n_head=16, n_kv_head=8, head_dim=128, ffn=6144, n_vocab=3072,
                  type_attn=Q8_0, type_ffn_up=Q8_0, type_ffn_down=Q8_0, type_head=Q8_0),
}

TENSORS = ["attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down"]


def tensor_shapes(c):
    """(type, ne0 = K, ne1 = N) of each matrix of one layer, and of the head."""
    attn, kv = c["n_head"] * c["head_dim"], c["n_kv_head"] * c["head_dim"]
    h, f = c["hidden"], c["ffn"]
    return {
        "attn_q": (c["type_attn"], h, attn), "attn_k": (c["type_attn"], h, kv), "attn_v": (c["type_attn"], h, kv),
        "attn_o": (c["type_attn"], attn, h), "ffn_gate": (c["type_ffn_up"], h, f), "ffn_up": (c["type_ffn_up"], h, f),
        "ffn_down": (c["type_ffn_down"], f, h), "output": (c["type_head"], h, c["n_vocab"]),
    }


def weight_bytes(c):
    sh = tensor_shapes(c)
    per_layer = sum(oracle.row_size(t, k) * n for name, (t, k, n) in sh.items() if name != "output")
    t, k, n = sh["output"]
    return per_layer * c["n_layer"] + oracle.row_size(t, k) * n


def random_model(c, seed=1234, n_layer=None, sigma=0.02, nthreads=0, normal=None):
    """GGUF bytes of random N(0, sigma) weights (quantized by the oracle) and N(1, 0.1) norm weights. `normal(shape)`,
    when given, draws the weights' N(0, 1) values instead of NumPy (the full-size configs use a faster generator)."""
    rng = np.random.default_rng(seed)
    draw = normal if normal is not None else (lambda shape: rng.normal(0, 1, size=shape))
    sh = tensor_shapes(c)
    layers = []
    for _ in range(c["n_layer"] if n_layer is None else n_layer):
        L = {}
        for name in TENSORS:
            t, k, n = sh[name]
            L[name] = oracle.quantize(t, (np.float32(sigma) * draw((n, k))).astype(np.float32), nthreads)
        L["attn_norm"] = rng.normal(1.0, 0.1, size=c["hidden"]).astype(np.float32)
        L["ffn_norm"] = rng.normal(1.0, 0.1, size=c["hidden"]).astype(np.float32)
        layers.append(L)
    t, k, n = sh["output"]
    head = oracle.quantize(t, (np.float32(sigma) * draw((n, k))).astype(np.float32), nthreads)
    out_norm = rng.normal(1.0, 0.1, size=c["hidden"]).astype(np.float32)
    return {"layers": layers, "output": head, "output_norm": out_norm}


def rms_norm(x, w, eps):
    x = x.astype(np.float32)
    mean = np.float32(np.sum(x.astype(np.float64) ** 2) / x.size)
    scale = np.float32(1.0) / np.sqrt(mean + np.float32(eps), dtype=np.float32)
    return (x * scale).astype(np.float32) * w


def silu(x):
    """x / (1 + exp(-x)) evaluated in double and rounded once to float32: the order-free definition both sides
    compute (ggml's CPU uses a float32 exp of its own; any accurate evaluation rounds to the same float32 except in
    rare near-ties)."""
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    return (x / (1.0 + np.exp(-x))).astype(np.float32)


def layer(c, L, x, eps, nthreads=0):
    sh = tensor_shapes(c)
    mm = lambda name, v: oracle.mul_mat(sh[name][0], L[name], sh[name][1], sh[name][2], v[None], nthreads)[0]
    h = rms_norm(x, L["attn_norm"], eps)
    mm("attn_q", h)
    mm("attn_k", h)  # q and k do not change the output at the first position; they are computed as a step does
    v = mm("attn_v", h)
    rep = c["n_head"] // c["n_kv_head"]
    o = np.repeat(v.reshape(c["n_kv_head"], c["head_dim"]), rep, axis=0).reshape(-1)
    x = (x + mm("attn_o", o)).astype(np.float32)
    h = rms_norm(x, L["ffn_norm"], eps)
    a = (silu(mm("ffn_gate", h)) * mm("ffn_up", h)).astype(np.float32)
    return (x + mm("ffn_down", a)).astype(np.float32)


def head(c, model, x, eps, nthreads=0):
    t, k, n = tensor_shapes(c)["output"]
    return oracle.mul_mat(t, model["output"], k, n, rms_norm(x, model["output_norm"], eps)[None], nthreads)[0]


def step(c, model, x, eps=1e-6, nthreads=0):
    x = np.asarray(x, dtype=np.float32)
    for L in model["layers"]:
        x = layer(c, L, x, eps, nthreads)
    return head(c, model, x, eps, nthreads)
