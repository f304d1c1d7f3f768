"""b200_moe_ffn_ep on 2 GPUs: each rank runs half of the experts, and the combine fused with a two-shot all-reduce over
NVLink peer memory leaves the full MoE output on both ranks (TextModel::experts, src/families/drama3/text-model.cpp:
198-221, split over GPUs). Checked against b200_moe_ffn over all experts on one GPU: the partial sums are added in
another order (rank by rank), so within a float tolerance; identical on both ranks, and identical across calls (the
arrival counters carry over between calls). Skipped with fewer than 2 GPUs."""

import importlib
import os
import socket

import numpy as np
import pytest

from conftest import ROOT, load_package

pytestmark = pytest.mark.gpu

E, H, F, TMAX, K = 16, 512, 256, 48, 4


def _model(oracle):
    rng = np.random.default_rng(41)
    gu = oracle.quantize(oracle.Q8_0, rng.normal(0, 0.02, size=(E * 2 * F, H)).astype(np.float32))
    dn = oracle.quantize(oracle.Q8_0, rng.normal(0, 0.02, size=(E * H, F)).astype(np.float32))
    return gu, dn, rng


def _worker(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    from oracle import oracle

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        pkg = load_package()
        ep = importlib.import_module(pkg.__name__ + ".expert_parallel")
        ctx = pkg.Context(rank)
        gu_b, dn_b, rng = _model(oracle)
        half = E // world
        rs, rd = 2 * F * H // 32 * 34, H * F // 32 * 34
        gu_all = ctx.weight(pkg.Q8_0, H, 2 * F, E, data=gu_b)
        dn_all = ctx.weight(pkg.Q8_0, F, H, E, data=dn_b)
        gu = ctx.weight(pkg.Q8_0, H, 2 * F, half, data=gu_b.reshape(-1)[rank * half * rs:(rank + 1) * half * rs])
        dn = ctx.weight(pkg.Q8_0, F, H, half, data=dn_b.reshape(-1)[rank * half * rd:(rank + 1) * half * rd])
        peer = ep.PeerCombine(ctx, dist.group.WORLD, TMAX, H)
        results = []
        for T in (TMAX, 40, TMAX):
            x = torch.from_numpy(rng.normal(0, 1, size=(T, H)).astype(np.float32)).cuda()
            ids = torch.from_numpy(np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)).cuda()
            w = torch.from_numpy(rng.random(size=(T, K)).astype(np.float32)).cuda()
            want = ctx.moe_ffn(gu_all, dn_all, x, ids, w).cpu().numpy()
            got = ctx.moe_ffn_ep(gu, dn, x, ids, w, rank * half, E, peer.handle).cpu().numpy()
            again = ctx.moe_ffn_ep(gu, dn, x, ids, w, rank * half, E, peer.handle).cpu().numpy()
            ctx.synchronize()
            results.append((got, want, again))
        peer.close()
        q.put((rank, results))
        ctx.close()
    except Exception as e:  # reported to the test, which fails
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_moe_ffn_ep_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
    for i in range(3):
        g0, want, again0 = out[0][i]
        g1, _, again1 = out[1][i]
        assert np.array_equal(g0, g1)  # the same reduced rows on both ranks
        assert np.array_equal(g0, again0) and np.array_equal(g1, again1)  # deterministic across calls
        assert np.allclose(g0, want, rtol=1e-5, atol=1e-6 * np.abs(want).max())


def _absent_rank_worker(rank, world, port, q):
    """Rank 1 skips one call of b200_moe_ffn_ep. Rank 0's combine must give up after its short wait limit and report
    B200_ERR_TIMEOUT; the broken group refuses the next call at once; a new group on both ranks works again."""
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch
    import torch.distributed as dist

    from oracle import oracle

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    report = {}
    try:
        pkg = load_package()
        ep = importlib.import_module(pkg.__name__ + ".expert_parallel")
        ctx = pkg.Context(rank)
        gu_b, dn_b, rng = _model(oracle)
        half = E // world
        rs, rd = 2 * F * H // 32 * 34, H * F // 32 * 34
        gu = ctx.weight(pkg.Q8_0, H, 2 * F, half, data=gu_b.reshape(-1)[rank * half * rs:(rank + 1) * half * rs])
        dn = ctx.weight(pkg.Q8_0, F, H, half, data=dn_b.reshape(-1)[rank * half * rd:(rank + 1) * half * rd])
        T = 40
        x = torch.from_numpy(rng.normal(0, 1, size=(T, H)).astype(np.float32)).cuda()
        ids = torch.from_numpy(np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)).cuda()
        w = torch.from_numpy(rng.random(size=(T, K)).astype(np.float32)).cuda()
        peer = ep.PeerCombine(ctx, dist.group.WORLD, TMAX, H, timeout_us=200_000)
        if rank == 0:
            for attempt in range(2):  # the first call waits out its limit; the second finds the group broken
                ctx.moe_ffn_ep(gu, dn, x, ids, w, rank * half, E, peer.handle)
                try:
                    ctx.synchronize()
                    report[f"call{attempt}"] = "ok"
                except pkg.B200Error as e:
                    report[f"call{attempt}"] = e.status
        dist.barrier()  # rank 1 learns on the host that rank 0's calls are over; none of its kernels is in flight
        peer.close()
        fresh = ep.PeerCombine(ctx, dist.group.WORLD, TMAX, H, timeout_us=2_000_000)
        got = ctx.moe_ffn_ep(gu, dn, x, ids, w, rank * half, E, fresh.handle).cpu().numpy()
        ctx.synchronize()
        fresh.close()
        report["fresh"] = got
        q.put((rank, report))
        ctx.close()
    except Exception as e:  # reported to the test, which fails
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def test_moe_ffn_ep_absent_rank_times_out():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    b200 = load_package()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_absent_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert not isinstance(out[r], str), out[r]
    assert out[0]["call0"] == b200.ERR_TIMEOUT
    assert out[0]["call1"] == b200.ERR_TIMEOUT  # the broken group refuses without waiting
    assert np.array_equal(out[0]["fresh"], out[1]["fresh"])  # a new group combines both ranks' experts again
    assert np.all(np.isfinite(out[0]["fresh"]))
