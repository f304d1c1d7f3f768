"""Helper for tests/test_gpu_tma_geometry.py: runs products under the ring geometry given by the environment
(B200_TMA_RING_KB, B200_TMA_STAGES, B200_TMA_CTAS_PER_SM) and checks them against the oracle. Prints OK."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

from conftest import load_package  # noqa: E402
from oracle import oracle  # noqa: E402

import torch  # noqa: E402

b200 = load_package()
ctx = b200.Context(0)
for qtype, K, N in [(8, 4096, 3000), (12, 4096, 2000), (14, 2048, 2500), (30, 2048, 900)]:
    rng = np.random.default_rng(K + N)
    wb = oracle.quantize(qtype, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(1, K)).astype(np.float32)
    w = ctx.weight(qtype, K, N, data=wb)
    got = ctx.mul_mat(w, torch.from_numpy(x).cuda()).cpu().numpy()
    ctx.synchronize()
    want = oracle.mul_mat(qtype, wb, K, N, x)
    vt = {8: 8, 12: 15, 14: 15, 30: 30}[qtype]
    wd = oracle.dequantize(qtype, wb, K).astype(np.float64)
    xd = oracle.dequantize(vt, oracle.quantize(vt, x), K).astype(np.float64)
    bound = 1e-4 * (np.abs(xd) @ np.abs(wd).T)
    assert np.all(np.abs(got - want) <= bound), (qtype, K, N)
    ctx.free_weight(w)
ctx.close()
print("OK")
