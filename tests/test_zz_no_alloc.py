"""b200_mul_mat_id_noalloc: MUL_MAT_ID for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc: a serving runtime whose arena owns all device memory, a path where an allocation
could synchronize the device and stall other streams, a process whose weights already fill the GPU. This entry point
keeps its scratch in a static device array instead of the context's pool.

The test calls it through the C ABI several times in a row, with different inputs each time (so stale contents of the
shared array would show), and checks every result twice:
- against the CPU oracle, |err| <= 1e-4 * sum |w x| per element (the products' tolerance);
- against the allocating entry point b200_mul_mat_id: bit for bit where both run the grouped GEMV (Q4_K, and Q8_0 with
  fewer than 128 (token, slot) pairs), within the same tolerance where b200_mul_mat_id runs the tensor-core grouped
  GEMM (Q8_0 with 128 pairs or more).
It also checks that a call too large for the array is refused. It creates its own context and data, so it passes alone
in a fresh process as well as after the other tests; it is named to be collected last.
"""

import ctypes

import numpy as np
import pytest

from conftest import load_package

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q8_K = 8, 12, 15
TOL = 1e-4

#           type, E,  K,    N,   T,  top_k, nb1, bit-equal to b200_mul_mat_id
CASES = [(Q8_0, 16, 1024, 192, 40, 4, 1, False),  # 160 pairs: b200_mul_mat_id takes the tensor-core path
         (Q4_K, 12, 512, 96, 33, 3, 3, True),
         (Q8_0, 8, 512, 80, 30, 4, 1, True)]      # 120 pairs: both take the grouped GEMV


def test_mul_mat_id_noalloc_matches_allocating_entry_point(oracle):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    b200 = load_package()
    ctx = b200.Context(0)
    L = ctx.L
    stream = torch.cuda.Stream()
    try:
        for call, (qtype, E, K, N, T, top_k, nb1, bit_equal) in enumerate(CASES):
            rng = np.random.default_rng(100 + call)
            wb = oracle.quantize(qtype, rng.normal(0, 0.02, size=(E * N, K)).astype(np.float32))
            w = ctx.weight(qtype, K, N, E, data=wb)
            ids = np.stack([rng.permutation(E)[:top_k] for _ in range(T)]).astype(np.int32)
            b = rng.normal(0, 1, size=(T, nb1, K)).astype(np.float32)
            bd, idd = torch.from_numpy(b).cuda(), torch.from_numpy(ids).cuda()
            want = ctx.mul_mat_id(w, bd, idd).cpu().numpy()
            ref = oracle.mul_mat_id(qtype, wb, K, N, E, b, ids)
            out = torch.full((T, top_k, N), float("nan"), device="cuda")
            torch.cuda.synchronize()  # the upload (context stream) is complete before the call on `stream`
            status = L.b200_mul_mat_id_noalloc(ctypes.c_void_p(stream.cuda_stream), ctypes.byref(w),
                                               ctypes.c_void_p(bd.data_ptr()), nb1, ctypes.c_void_p(idd.data_ptr()),
                                               top_k, T, ctypes.c_void_p(out.data_ptr()))
            assert status == b200.OK, L.b200_last_error(None)
            stream.synchronize()
            got = out.cpu().numpy()
            assert np.all(np.isfinite(got))
            if bit_equal:
                assert np.array_equal(got, want)
            vt = Q8_0 if qtype == Q8_0 else Q8_K
            wd = oracle.dequantize(qtype, wb, K).astype(np.float64).reshape(E, N, K)
            for t in range(T):
                for s in range(top_k):
                    xd = oracle.dequantize(vt, oracle.quantize(vt, b[t, 0 if nb1 == 1 else s][None]), K)[0].astype(np.float64)
                    bound = TOL * (np.abs(wd[ids[t, s]]) @ np.abs(xd)) + 1e-30
                    assert np.all(np.abs(got[t, s].astype(np.float64) - ref[t, s]) <= bound)
                    assert np.all(np.abs(got[t, s].astype(np.float64) - want[t, s]) <= bound)
            ctx.free_weight(w)

        # a call whose activations do not fit the static array is refused with an error, not run
        K, E, N, T = 4096, 4, 32, 8192
        w = ctx.weight(Q8_0, K, N, E)
        big = torch.zeros((T, 1, K), device="cuda")
        ids = torch.zeros((T, 1), dtype=torch.int32, device="cuda")
        out = torch.zeros((T, 1, N), device="cuda")
        status = L.b200_mul_mat_id_noalloc(ctypes.c_void_p(stream.cuda_stream), ctypes.byref(w), ctypes.c_void_p(big.data_ptr()), 1,
                                           ctypes.c_void_p(ids.data_ptr()), 1, T, ctypes.c_void_p(out.data_ptr()))
        assert status == b200.ERR_INVALID
        assert b"static scratch" in L.b200_last_error(None)
        ctx.free_weight(w)
    finally:
        ctx.close()
