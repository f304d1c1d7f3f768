"""Host logic of expert parallelism (speech.cpp_b200/expert_parallel.py) on CPU: 2 gloo ranks, each holding half of
every layer's experts, reproduce the single-rank MoE stack.

The per-rank expert block is a CPU stand-in with b200_moe_ffn's shard semantics (pairs routed to other ranks' experts
contribute nothing), built on the oracle's MUL_MAT_ID (ggml's CPU vec_dot restated); the GPU kernels' own shard
semantics are checked in test_gpu_moe.py. Reference: TextModel::experts (src/families/drama3/text-model.cpp:198-221).
"""

import os
import socket

import numpy as np
import pytest

from conftest import ROOT, load_package

E, H, F, T, K, L = 8, 64, 32, 6, 2, 2


class ShardFfn:
    """moe_ffn over experts [expert0, expert0 + E_local) given as GGUF Q8_0 bytes, on CPU tensors."""

    def __init__(self, oracle):
        self.o = oracle

    def moe_ffn(self, gu, dn, x, ids, w, expert0=0, n_expert_total=0, out=None):
        import torch

        o = self.o
        gu_b, dn_b, n_local = gu, dn, gu.shape[0] // (2 * F)
        ids_n, x_n, w_n = ids.numpy(), x.numpy(), w.numpy()
        local = (ids_n >= expert0) & (ids_n < expert0 + n_local)
        lid = np.where(local, ids_n - expert0, 0).astype(np.int32)
        g_u = o.mul_mat_id(o.Q8_0, gu_b, H, 2 * F, n_local, x_n[:, None, :], lid)
        g, u = g_u[..., :F], g_u[..., F:]
        a = (g / (np.float32(1.0) + np.exp(-g)) * u).astype(np.float32)
        d = o.mul_mat_id(o.Q8_0, dn_b, F, H, n_local, a, lid)
        acc = np.zeros((x_n.shape[0], H), dtype=np.float32)
        for s in range(ids_n.shape[1]):
            acc = (acc + np.where(local[:, s:s + 1], d[:, s] * w_n[:, s:s + 1], 0)).astype(np.float32)
        out.copy_(torch.from_numpy(acc))
        return out


def model(oracle):
    rng = np.random.default_rng(3)
    layers = []
    for _ in range(L):
        gu = oracle.quantize(oracle.Q8_0, rng.normal(0, 0.1, size=(E * 2 * F, H)).astype(np.float32))
        dn = oracle.quantize(oracle.Q8_0, rng.normal(0, 0.1, size=(E * H, F)).astype(np.float32))
        layers.append((gu, dn))
    ids = np.stack([np.stack([rng.permutation(E)[:K] for _ in range(T)]) for _ in range(L)]).astype(np.int32)
    w = rng.random(size=(L, T, K)).astype(np.float32)
    x = rng.normal(0, 1, size=(T, H)).astype(np.float32)
    return layers, ids, w, x


def run_stack(oracle, ep_mod, rank, world, group):
    import torch

    layers, ids, w, x = model(oracle)
    e0, n = ep_mod.expert_shard(E, world, rank)
    rs_gu, rs_dn = 2 * F, H  # rows per expert
    shard = [(gu[e0 * rs_gu:(e0 + n) * rs_gu], dn[e0 * rs_dn:(e0 + n) * rs_dn]) for gu, dn in layers]
    m = ep_mod.ExpertParallelMoe(ShardFfn(oracle), shard, e0, E, group=group)
    xs = [torch.from_numpy(x)] + [torch.empty((T, H)) for _ in range(L)]
    return m.step(xs, torch.from_numpy(ids), torch.from_numpy(w)).numpy()


def _worker(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch.distributed as dist

    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pkg = load_package()
        import importlib

        ep = importlib.import_module(pkg.__name__ + ".expert_parallel")
        out = run_stack(oracle, ep, rank, world, dist.group.WORLD)
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_expert_shard_ranges():
    pkg = load_package()
    import importlib

    ep = importlib.import_module(pkg.__name__ + ".expert_parallel")
    for world in (1, 2, 4, 8):
        got = [ep.expert_shard(128, world, r) for r in range(world)]
        assert sum(n for _, n in got) == 128
        assert [e0 for e0, _ in got] == [r * (128 // world) for r in range(world)]
    with pytest.raises(ValueError):
        ep.expert_shard(128, 3, 0)
    with pytest.raises(ValueError):
        ep.expert_shard(128, 2, 2)


def test_two_gloo_ranks_match_one(oracle):
    import torch.multiprocessing as mp

    pkg = load_package()
    import importlib

    ep = importlib.import_module(pkg.__name__ + ".expert_parallel")
    want = run_stack(oracle, ep, 0, 1, None)
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
        assert np.allclose(outs[r], want, rtol=1e-5, atol=1e-6 * np.abs(want).max())
    assert np.array_equal(outs[0], outs[1])


def test_ep_place_fewest_ranks_that_fit():
    """b200_ep_place (host code, no GPU): config 5's 48 layers of 128 Q8_0 experts (641,728,512 B a layer) with 2 GB
    of the rest on each GPU: one B200 (about 178 GiB free) holds them all; GPUs of 20 GiB need 2 ranks; of 6 GiB, 8;
    of 3 GiB, none. Uneven free memory: the first `ranks` devices must each fit."""
    from conftest import load_package

    b200 = load_package()
    layers = [641_728_512] * 48
    GiB = 1 << 30
    p = b200.ep_place([178 * GiB] * 8, layers, 128, 2 * GiB)
    assert (p.ranks, p.experts_per_rank) == (1, 128) and p.expert_bytes == 48 * 641_728_512
    assert b200.ep_place([20 * GiB] * 8, layers, 128, 2 * GiB).ranks == 2
    p = b200.ep_place([6 * GiB] * 8, layers, 128, 2 * GiB)
    assert (p.ranks, p.experts_per_rank) == (8, 16) and p.bytes_per_rank == 2 * GiB + 48 * (641_728_512 // 8)
    assert b200.ep_place([20 * GiB, 10 * GiB, 20 * GiB, 20 * GiB], layers, 128, 2 * GiB).ranks == 4  # device 1 is short
    with pytest.raises(b200.B200Error):
        b200.ep_place([3 * GiB] * 8, layers, 128, 2 * GiB)
    with pytest.raises(b200.B200Error):
        b200.ep_place([6 * GiB] * 4, layers, 128, 2 * GiB)  # would need 8 ranks, only 4 devices
    import importlib

    ep = importlib.import_module(b200.__name__ + ".expert_parallel")
    # the facade: given free memory, as place_experts reads it from every device when none is given
    p = ep.place_experts(layers, 128, 2 * GiB, free_bytes=[40 * GiB] * 2)
    assert (p.ranks, p.experts_per_rank) == (1, 128)
