"""Writes tests/golden/gguf_blocks.npz: golden vectors for the GGUF block formats, made with gguf-py.

gguf-py 0.19.0 (the `gguf` package; gguf/quants.py) is the reference's own executable spec at the ggml quantization
boundary: checks/compare/quantize_compare.py:1-11 pins ggml's Q8_0 bytes to gguf.quants.quantize(). This script runs
it in the build container (the GPU box never needs it) on seeded inputs and stores what it returns, so the CPU oracle
(oracle/oracle.c) can be checked against it bit for bit:

  q8_0_*      gguf.quants.quantize(x, Q8_0) bytes for seeded N(0, 0.02) weights, the reference quantize-check's
              known-answer matrix (0.05 * sin(0.37 i), 16 x 256, checks/common/quantize-check.cpp:42-53), and edge
              rows (zeros, rounding ties, subnormal scales, large values, mixed signs);
  deq_*       gguf.quants.dequantize(blocks, T) floats for random valid Q8_0 / Q4_K / Q5_K / Q6_K blocks;
  bf16_*      gguf.quants.quantize(x, BF16) / dequantize for ordinary values, ties, NaN and infinities.

Run:  python tests/golden/make_golden.py
"""

import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))


def random_half_scales(rng, n, lo=-12.0, hi=-4.0):
    """Positive fp16 scales spanning normal and a few subnormal magnitudes."""
    return (2.0 ** rng.uniform(lo, hi, size=n)).astype(np.float16)


def main():
    rng = np.random.default_rng(1234)
    out = {}

    # --- Q8_0 quantization ---------------------------------------------------------------------------------------
    w = rng.normal(0.0, 0.02, size=(8, 1024)).astype(np.float32)
    out["q8_0_normal_x"] = w
    out["q8_0_normal_q"] = quants.quantize(w, T.Q8_0)

    i = np.arange(16 * 256, dtype=np.float32)
    kat = (np.sin(np.float32(0.37) * i) * np.float32(0.05)).astype(np.float32).reshape(16, 256)
    out["q8_0_kat_x"] = kat
    out["q8_0_kat_q"] = quants.quantize(kat, T.Q8_0)

    edge = np.zeros((8, 64), dtype=np.float32)
    edge[1, :32] = np.arange(-16, 16, dtype=np.float32) / 16.0 * 127.0 / 127.0  # exact multiples
    ties = (np.arange(32, dtype=np.float32) - 15.5) / np.float32(127.0)  # x * id lands on .5 boundaries
    edge[1, 32:] = ties
    edge[2, :] = rng.normal(0.0, 1e-6, size=64).astype(np.float32)  # subnormal-ish fp16 scales
    edge[3, :] = rng.normal(0.0, 3e-8, size=64).astype(np.float32)  # scale underflows in fp16
    edge[4, :] = rng.normal(0.0, 1e3, size=64).astype(np.float32)  # large values
    edge[5, :] = np.where(np.arange(64) % 2 == 0, 1.0, -1.0).astype(np.float32)  # +-amax ties
    edge[6, :32] = 0.0
    edge[6, 32:] = np.float32(1e-30)
    edge[7, :] = (rng.integers(-127, 128, size=64).astype(np.float32) + 0.5) / np.float32(127.0)
    out["q8_0_edge_x"] = edge
    out["q8_0_edge_q"] = quants.quantize(edge, T.Q8_0)

    # --- dequantization of random valid blocks --------------------------------------------------------------------
    nb = 64
    # Q8_0: fp16 d + 32 int8
    d = random_half_scales(rng, nb).view(np.uint8).reshape(nb, 2)
    qs = rng.integers(-128, 128, size=(nb, 32), dtype=np.int64).astype(np.int8).view(np.uint8)
    b = np.concatenate([d, qs], axis=1)
    out["deq_q8_0_blocks"] = b
    out["deq_q8_0_y"] = quants.dequantize(b, T.Q8_0)

    # Q4_K: d, dmin (fp16), 12 scale bytes, 128 nibble bytes
    d = random_half_scales(rng, nb).view(np.uint8).reshape(nb, 2)
    dmin = random_half_scales(rng, nb).view(np.uint8).reshape(nb, 2)
    sc = rng.integers(0, 256, size=(nb, 12), dtype=np.int64).astype(np.uint8)
    qs = rng.integers(0, 256, size=(nb, 128), dtype=np.int64).astype(np.uint8)
    b = np.concatenate([d, dmin, sc, qs], axis=1)
    out["deq_q4_K_blocks"] = b
    out["deq_q4_K_y"] = quants.dequantize(b, T.Q4_K)

    # Q6_K: 128 ql, 64 qh, 16 int8 scales, fp16 d
    ql = rng.integers(0, 256, size=(nb, 128), dtype=np.int64).astype(np.uint8)
    qh = rng.integers(0, 256, size=(nb, 64), dtype=np.int64).astype(np.uint8)
    sc = rng.integers(-128, 128, size=(nb, 16), dtype=np.int64).astype(np.int8).view(np.uint8)
    d = random_half_scales(rng, nb).view(np.uint8).reshape(nb, 2)
    b = np.concatenate([ql, qh, sc, d], axis=1)
    out["deq_q6_K_blocks"] = b
    out["deq_q6_K_y"] = quants.dequantize(b, T.Q6_K)

    # --- BF16 ----------------------------------------------------------------------------------------------------
    x = rng.normal(0.0, 1.0, size=256).astype(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 3.4e38, 1.0 + 2.0**-8, 1.0 + 3 * 2.0**-8,
                        1.0 + 2.0**-9, -(1.0 + 2.0**-8)], dtype=np.float32)
    x = np.concatenate([x, special]).astype(np.float32)
    out["bf16_x"] = x
    out["bf16_q"] = quants.quantize(x, T.BF16)
    out["bf16_y"] = quants.dequantize(out["bf16_q"], T.BF16)

    path = os.path.join(HERE, "gguf_blocks.npz")
    # Q5_K: d, dmin (fp16), 12 scale bytes, 32 high-bit bytes, 128 nibble bytes (its own generator: the entries above
    # keep their values)
    r5 = np.random.default_rng(55)
    d = random_half_scales(r5, nb).view(np.uint8).reshape(nb, 2)
    dmin = random_half_scales(r5, nb).view(np.uint8).reshape(nb, 2)
    sc = r5.integers(0, 256, size=(nb, 12), dtype=np.int64).astype(np.uint8)
    qh = r5.integers(0, 256, size=(nb, 32), dtype=np.int64).astype(np.uint8)
    qs = r5.integers(0, 256, size=(nb, 128), dtype=np.int64).astype(np.uint8)
    b = np.concatenate([d, dmin, sc, qh, qs], axis=1)
    out["deq_q5_K_blocks"] = b
    out["deq_q5_K_y"] = quants.dequantize(b, T.Q5_K)

    np.savez_compressed(path, **out)
    print(f"wrote {path}: {', '.join(sorted(out))}")


if __name__ == "__main__":
    main()
