"""Host logic of column-split products (speech.cpp_b200/column_parallel.py) on CPU: 2 gloo ranks, each holding half
of a weight's rows, assemble the same output as one rank. The per-rank product is the oracle's MUL_MAT (ggml's CPU
vec_dot restated) on the shard's GGUF rows; b200_mul_mat_rows on the GPU is checked in test_gpu_ops.py."""

import importlib
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, load_package

K, N, M = 256, 512, 6


def make(oracle):
    rng = np.random.default_rng(5)
    wb = oracle.quantize(oracle.Q8_0, rng.normal(0, 0.02, size=(N, K)).astype(np.float32))
    x = rng.normal(0, 1, size=(M, K)).astype(np.float32)
    return wb, x


def run(oracle, cp, rank, world, group):
    import torch

    wb, x = make(oracle)
    r0, n = cp.row_shard(N, world, rank)
    mm = lambda w, xx, out: out.copy_(torch.from_numpy(oracle.mul_mat(oracle.Q8_0, w, K, n, xx.numpy())))
    prod = cp.ColumnParallelProduct(mm, wb[r0:r0 + n], N, group=group)
    out = torch.empty((M, N))
    return prod(torch.from_numpy(x), torch.empty((M, n)), torch.empty((world, M, n)), out).numpy()


def _worker(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch.distributed as dist

    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cp = importlib.import_module(load_package().__name__ + ".column_parallel")
        q.put((rank, run(oracle, cp, rank, world, dist.group.WORLD)))
    finally:
        dist.destroy_process_group()


def test_row_shards():
    cp = importlib.import_module(load_package().__name__ + ".column_parallel")
    assert [cp.row_shard(2048, 8, r) for r in range(8)] == [(256 * r, 256) for r in range(8)]
    with pytest.raises(ValueError):
        cp.row_shard(1000, 2, 0)


def test_two_gloo_ranks_match_one(oracle):
    import torch.multiprocessing as mp

    cp = importlib.import_module(load_package().__name__ + ".column_parallel")
    want = run(oracle, cp, 0, 1, None)
    wb, x = make(oracle)
    assert np.array_equal(want, oracle.mul_mat(oracle.Q8_0, wb, K, N, x))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        assert np.array_equal(outs[r], want)
