"""The TMA-streamed products under ring geometries other than the default, including fewer stages than consumer
warps with slots reused many times (each slot must stay with one warp). The geometry is read once per process, so
each case runs in a child process (tests/tma_geometry_check.py)."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("ring_kb,stages,ctas", [(24, 3, 1), (48, 2, 2), (96, 16, 2), (192, 8, 1), (40, 5, 1)])
def test_products_under_ring_geometry(ring_kb, stages, ctas):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    env = dict(os.environ, B200_TMA_RING_KB=str(ring_kb), B200_TMA_STAGES=str(stages), B200_TMA_CTAS_PER_SM=str(ctas))
    r = subprocess.run([sys.executable, os.path.join(HERE, "tma_geometry_check.py")], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout[-2000:] + r.stderr[-2000:]
