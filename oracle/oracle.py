"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs use it as the checker /
baseline. The product path (speech.cpp_b200, include/b200.h) never imports it.
"""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 0, 1, 8, 12, 13, 14, 15, 30
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292)}
VEC_DOT_TYPE = {Q8_0: Q8_0, Q4_K: Q8_K, Q5_K: Q8_K, Q6_K: Q8_K, BF16: BF16, F32: F32}

_lib = None


def build():
    """Compiles liboracle.so from oracle.c (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.oracle_row_size.restype = ctypes.c_size_t
        L.oracle_row_size.argtypes = [i32, i64]
        L.oracle_quantize_rows.argtypes = [i32, vp, vp, i64, i64, i32]
        L.oracle_dequantize_row.argtypes = [i32, vp, vp, i64]
        L.oracle_vec_dot.restype = ctypes.c_float
        L.oracle_vec_dot.argtypes = [i32, vp, vp, i64]
        L.oracle_block_sums.restype = i64
        L.oracle_block_sums.argtypes = [i32, vp, vp, i64, vp]
        L.oracle_mul_mat.argtypes = [i32, vp, i64, i64, vp, i64, vp, i32]
        L.oracle_mul_mat_id.argtypes = [i32, vp, i64, i64, i64, vp, i64, vp, i64, i64, vp, i32]
        L.oracle_get_rows.argtypes = [i32, vp, i64, i64, vp, i64, vp]
        L.oracle_fp32_to_fp16.restype = ctypes.c_uint16
        L.oracle_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.oracle_fp16_to_fp32.restype = ctypes.c_float
        L.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def row_size(qtype, k):
    return lib().oracle_row_size(qtype, k)


def quantize(qtype, x, nthreads=0):
    """float32 [n, k] -> uint8 [n, row_size] blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    rs = row_size(qtype, x2.shape[1])
    if rs == 0:
        raise ValueError("unsupported type or row length")
    y = np.empty((x2.shape[0], rs), dtype=np.uint8)
    if lib().oracle_quantize_rows(qtype, _p(x2), _p(y), x2.shape[1], x2.shape[0], nthreads) != 0:
        raise ValueError("quantize failed")
    return y


def dequantize(qtype, blocks, k):
    """uint8 [n, row_size(k)] -> float32 [n, k]."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, row_size(qtype, k))
    y = np.empty((b.shape[0], k), dtype=np.float32)
    for r in range(b.shape[0]):
        if lib().oracle_dequantize_row(qtype, _p(b[r]), _p(y[r]), k) != 0:
            raise ValueError("dequantize failed")
    return y


def block_sums(qtype, w_row, x_row_q, k):
    n = {Q8_0: k // 32, Q4_K: 2 * (k // 256), Q5_K: 2 * (k // 256), Q6_K: k // 256}[qtype]
    out = np.empty(n, dtype=np.int32)
    got = lib().oracle_block_sums(qtype, _p(np.ascontiguousarray(w_row)), _p(np.ascontiguousarray(x_row_q)), k, _p(out))
    assert got == n
    return out


def mul_mat(qtype, w_blocks, K, N, x, nthreads=0):
    """dst [M, N] = W[N, K] . x[M, K]^T with ggml CPU semantics."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    M = x.shape[0]
    dst = np.empty((M, N), dtype=np.float32)
    w = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    if lib().oracle_mul_mat(qtype, _p(w), K, N, _p(x), M, _p(dst), nthreads) != 0:
        raise ValueError("mul_mat failed")
    return dst


def mul_mat_id(qtype, experts, K, N, E, b, ids, nthreads=0):
    """dst [T, top_k, N]; b float32 [T, nb1, K] (nb1 1 or top_k); ids int32 [T, top_k]."""
    b = np.ascontiguousarray(b, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, top_k = ids.shape
    nb1 = b.shape[1]
    dst = np.empty((T, top_k, N), dtype=np.float32)
    r = lib().oracle_mul_mat_id(qtype, _p(np.ascontiguousarray(experts, dtype=np.uint8)), K, N, E, _p(b), nb1, _p(ids),
                                top_k, T, _p(dst), nthreads)
    if r != 0:
        raise ValueError(f"mul_mat_id failed ({r})")
    return dst


def get_rows(qtype, table, K, rows, ids):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    dst = np.empty((ids.size, K), dtype=np.float32)
    r = lib().oracle_get_rows(qtype, _p(np.ascontiguousarray(table, dtype=np.uint8)), K, rows, _p(ids), ids.size, _p(dst))
    if r != 0:
        raise ValueError(f"get_rows failed ({r})")
    return dst


def max_threads():
    return lib().oracle_max_threads()
