"""speech.cpp_b200 — Python host side of the B200 backend for speech.cpp's quantized matrix products.

A thin ctypes layer over the C ABI in include/b200.h (libb200.so, built from csrc/ for sm_100a). It mirrors the ggml
ops speech.cpp builds its graphs from — ggml_mul_mat (src/common/graph.h:15-19), ggml_mul_mat_id (graph.h:22-26),
ggml_get_rows of quantized tables (src/families/qwen3-tts/talker.cpp:131-133) — and the weight buffer's
set_tensor / get_tensor (src/common/model-file.cpp:247-268), with the same argument meaning: a weight has ne0 = K
values per row and ne1 = N rows; activations are float32 [M][K]; results [M][N].

Device memory and streams come from torch (plumbing only): every op takes torch CUDA tensors and runs on the
context's own stream. There is no CPU fallback: if libb200.so is missing or no B200 is present, calls raise.
"""

import ctypes
import os
import weakref

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200.so")

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 0, 1, 8, 12, 13, 14, 15, 30
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_K: "Q8_K", BF16: "BF16"}
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210),
         Q8_K: (256, 292)}

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_ALLOC, ERR_DEVICE, ERR_RANGE, ERR_TIMEOUT = 0, -1, -2, -3, -4, -5, -6
STATUS_NAMES = {0: "OK", -1: "INVALID", -2: "UNSUPPORTED", -3: "ALLOC", -4: "DEVICE", -5: "RANGE", -6: "TIMEOUT"}

# Every symbol include/b200.h declares (tests check the library exports each one).
EXPORTS = [
    "b200_device_count", "b200_device_info", "b200_context_create", "b200_context_destroy", "b200_context_stream",
    "b200_synchronize", "b200_last_error", "b200_malloc", "b200_free", "b200_memcpy_h2d", "b200_memcpy_d2h",
    "b200_weight_nbytes", "b200_weight_alloc", "b200_weight_free", "b200_weight_set", "b200_weight_set_device",
    "b200_weight_get", "b200_mul_mat", "b200_mul_mat_rows", "b200_mul_mat_id", "b200_get_rows", "b200_quantize_rows",
    "b200_block_sums", "b200_mul_mat_host", "b200_decoder_create", "b200_decoder_destroy", "b200_decoder_set_tensor",
    "b200_decoder_step", "b200_decoder_step_host", "b200_decoder_launches", "b200_decoder_weight_bytes",
    "b200_decoder_set_launch", "b200_mul_mat_id_noalloc", "b200_moe_ffn",
    "b200_ep_mailbox_alloc", "b200_ep_mailbox_open", "b200_ep_mailbox_close", "b200_ep_mailbox_free", "b200_ep_create",
    "b200_ep_destroy", "b200_ep_set_timeout", "b200_moe_ffn_ep", "b200_graph_compute", "b200_graph_supports",
    "b200_weight_prefetch_l2", "b200_ep_place",
]

DEC_ATTN_Q, DEC_ATTN_K, DEC_ATTN_V, DEC_ATTN_O, DEC_FFN_GATE, DEC_FFN_UP, DEC_FFN_DOWN = range(7)
DEC_ATTN_NORM, DEC_FFN_NORM, DEC_OUTPUT_NORM, DEC_OUTPUT = 7, 8, 9, 10
DEC_MODE_CHAIN, DEC_MODE_PERSISTENT = 0, 1


class B200Error(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"b200 {STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Weight(ctypes.Structure):
    """struct b200_weight (include/b200.h)."""

    _fields_ = [
        ("type", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("ne0", ctypes.c_int64),
        ("ne1", ctypes.c_int64),
        ("ne2", ctypes.c_int64),
        ("data", ctypes.c_void_p),
        ("nbytes", ctypes.c_size_t),
        ("dbytes", ctypes.c_size_t),
        ("field_off", ctypes.c_int64 * 4),
    ]


class Tensor(ctypes.Structure):
    """struct b200_tensor (include/b200.h): one ggml-shaped record of a graph for b200_graph_compute."""

    _fields_ = [
        ("op", ctypes.c_int32), ("type", ctypes.c_int32), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_int64 * 4),
        ("data", ctypes.c_void_p), ("weight", ctypes.POINTER(Weight)), ("src", ctypes.c_int32 * 4),
        ("params", ctypes.c_int32 * 8),
    ]


I32 = 26
(OP_NONE, OP_GET_ROWS, OP_MUL_MAT, OP_RMS_NORM, OP_MUL, OP_ADD, OP_ROPE, OP_SET_ROWS, OP_CPY, OP_CONT, OP_SOFT_MAX,
 OP_FLASH_ATTN, OP_SWIGLU, OP_ARGMAX, OP_SCALE, OP_FILL, OP_CONCAT) = range(17)


class EpPlan(ctypes.Structure):
    """struct b200_ep_plan (include/b200.h)."""

    _fields_ = [("ranks", ctypes.c_int32), ("experts_per_rank", ctypes.c_int32), ("bytes_per_rank", ctypes.c_uint64),
                ("expert_bytes", ctypes.c_uint64)]


def ep_place(free_bytes, expert_bytes, n_expert, rest_bytes):
    """b200_ep_place: the fewest GPUs (a power of two) whose share of the experts fits beside the rest. Returns the
    EpPlan, or raises B200Error (ALLOC) when no count fits."""
    L = lib()
    fb = (ctypes.c_size_t * len(free_bytes))(*free_bytes)
    eb = (ctypes.c_uint64 * len(expert_bytes))(*expert_bytes)
    plan = EpPlan()
    s = L.b200_ep_place(len(free_bytes), fb, len(expert_bytes), eb, n_expert, rest_bytes, ctypes.byref(plan))
    if s != OK:
        raise B200Error(s, f"{plan.expert_bytes} bytes of experts plus {rest_bytes} per GPU fit no count of the {len(free_bytes)} GPUs")
    return plan


class DecoderShape(ctypes.Structure):
    """struct b200_decoder_shape (include/b200.h)."""

    _fields_ = [
        ("n_layer", ctypes.c_int32), ("hidden", ctypes.c_int32), ("n_head", ctypes.c_int32), ("n_kv_head", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("ffn", ctypes.c_int32), ("n_vocab", ctypes.c_int64), ("eps", ctypes.c_float),
        ("type_attn", ctypes.c_int32), ("type_ffn_up", ctypes.c_int32), ("type_ffn_down", ctypes.c_int32),
        ("type_head", ctypes.c_int32),
    ]


_lib = None


def build():
    """Compiles libb200.so (nvcc, sm_100a)."""
    import importlib.util

    spec = importlib.util.spec_from_file_location("_b200_build", os.path.join(HERE, "build.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m.build()


def lib():
    """The loaded C ABI. Raises if libb200.so is missing: there is no other implementation."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run speech.cpp_b200/build.py (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, i32, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
    W = ctypes.POINTER(Weight)
    sig = {
        "b200_device_count": (i32, []),
        "b200_device_info": (i32, [i32, ctypes.c_char_p, sz, ctypes.POINTER(sz), ctypes.POINTER(sz)]),
        "b200_context_create": (i32, [i32, ctypes.POINTER(vp)]),
        "b200_context_destroy": (None, [vp]),
        "b200_context_stream": (vp, [vp]),
        "b200_synchronize": (i32, [vp]),
        "b200_last_error": (ctypes.c_char_p, [vp]),
        "b200_malloc": (i32, [vp, sz, ctypes.POINTER(vp)]),
        "b200_free": (i32, [vp, vp]),
        "b200_memcpy_h2d": (i32, [vp, vp, vp, sz]),
        "b200_memcpy_d2h": (i32, [vp, vp, vp, sz]),
        "b200_weight_nbytes": (sz, [i32, i64, i64, i64]),
        "b200_weight_alloc": (i32, [vp, i32, i64, i64, i64, W]),
        "b200_weight_free": (i32, [vp, W]),
        "b200_weight_set": (i32, [vp, W, vp, sz, sz]),
        "b200_weight_set_device": (i32, [vp, W, vp, sz, sz]),
        "b200_weight_get": (i32, [vp, W, vp, sz, sz]),
        "b200_mul_mat": (i32, [vp, W, vp, i64, vp]),
        "b200_mul_mat_rows": (i32, [vp, W, i64, i64, vp, i64, vp, i64]),
        "b200_mul_mat_id": (i32, [vp, W, vp, i64, vp, i64, i64, vp]),
        "b200_get_rows": (i32, [vp, W, vp, i64, vp]),
        "b200_quantize_rows": (i32, [vp, i32, vp, i64, i64, vp]),
        "b200_block_sums": (i32, [vp, W, vp, vp]),
        "b200_mul_mat_host": (i32, [vp, W, vp, i64, vp]),
        "b200_decoder_create": (i32, [vp, ctypes.POINTER(DecoderShape), ctypes.POINTER(vp)]),
        "b200_decoder_destroy": (None, [vp]),
        "b200_decoder_set_tensor": (i32, [vp, i32, i32, vp, i32, sz, sz]),
        "b200_decoder_step": (i32, [vp, vp, vp]),
        "b200_decoder_step_host": (i32, [vp, vp, vp]),
        "b200_decoder_launches": (i64, [vp]),
        "b200_decoder_weight_bytes": (sz, [vp]),
        "b200_decoder_set_launch": (i32, [vp, i32, i32, i32]),
        "b200_mul_mat_id_noalloc": (i32, [vp, W, vp, i64, vp, i64, i64, vp]),
        "b200_moe_ffn": (i32, [vp, W, W, i64, i64, vp, vp, vp, i64, i64, vp]),
        "b200_ep_mailbox_alloc": (i32, [vp, ctypes.c_int, i64, i64, ctypes.POINTER(vp), vp]),
        "b200_ep_mailbox_open": (i32, [vp, vp, ctypes.POINTER(vp)]),
        "b200_ep_mailbox_close": (i32, [vp, vp]),
        "b200_ep_mailbox_free": (i32, [vp, vp]),
        "b200_ep_create": (i32, [vp, ctypes.c_int, ctypes.c_int, i64, i64, ctypes.POINTER(vp), ctypes.POINTER(vp)]),
        "b200_ep_destroy": (None, [vp]),
        "b200_ep_set_timeout": (i32, [vp, ctypes.c_uint64]),
        "b200_moe_ffn_ep": (i32, [vp, W, W, i64, i64, vp, vp, vp, i64, i64, vp, vp]),
        "b200_graph_compute": (i32, [vp, ctypes.POINTER(Tensor), i64]),
        "b200_weight_prefetch_l2": (i32, [vp, W, vp]),
        "b200_ep_place": (i32, [ctypes.c_int, ctypes.POINTER(sz), ctypes.c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int,
                                ctypes.c_uint64, ctypes.POINTER(EpPlan)]),
        "b200_graph_supports": (i32, [ctypes.POINTER(Tensor), i64, i64]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def row_size(qtype, k):
    bv, bb = BLOCK[qtype]
    if k % bv:
        raise ValueError(f"{TYPE_NAMES[qtype]} rows need a multiple of {bv} values")
    return k // bv * bb


def _ptr(t):
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        if not t.is_cuda:
            raise ValueError("expected a CUDA tensor")
        if not t.is_contiguous():
            raise ValueError("expected a contiguous tensor")
        return ctypes.c_void_p(t.data_ptr())
    return ctypes.c_void_p(t)


class Context:
    """One B200 device, one stream, a scratch pool (b200_context)."""

    def __init__(self, device=0):
        self.L = lib()
        self.device = device
        h = ctypes.c_void_p()
        s = self.L.b200_context_create(device, ctypes.byref(h))
        if s != OK:
            raise B200Error(s, self.L.b200_last_error(None).decode())
        self.h = h
        self._children = weakref.WeakSet()  # decoders built on this context: closed before it

    def check(self, status):
        if status != OK:
            raise B200Error(status, self.L.b200_last_error(self.h).decode())

    @property
    def stream_handle(self):
        return self.L.b200_context_stream(self.h)

    def torch_stream(self):
        import torch

        return torch.cuda.ExternalStream(self.stream_handle, device=torch.device("cuda", self.device))

    def synchronize(self):
        self.check(self.L.b200_synchronize(self.h))

    def close(self):
        if getattr(self, "h", None):
            for child in list(getattr(self, "_children", ())):
                child.close()
            self.L.b200_context_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- weights --------------------------------------------------------------------------------------------------
    def weight(self, qtype, ne0, ne1, ne2=1, data=None):
        """Allocates a weight tensor; `data` (GGUF block bytes: numpy uint8, or a CUDA uint8 tensor) is uploaded."""
        w = Weight()
        self.check(self.L.b200_weight_alloc(self.h, qtype, ne0, ne1, ne2, ctypes.byref(w)))
        if data is not None:
            self.set_weight(w, data)
        return w

    def set_weight(self, w, data, offset=0):
        """Uploads GGUF block bytes at a byte offset: numpy (host) or a CUDA uint8 tensor. A CUDA tensor is read on the
        context's stream, ordered after torch's current stream, and torch's stream then waits for the copy, so the
        caller may free or overwrite the tensor as soon as this returns."""
        if hasattr(data, "is_cuda") and data.is_cuda:
            self._sync_in()
            self.check(self.L.b200_weight_set_device(self.h, ctypes.byref(w), _ptr(data), offset, data.numel() * data.element_size()))
            self._sync_out()
        else:
            import numpy as np

            a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
            self.check(self.L.b200_weight_set(self.h, ctypes.byref(w), a.ctypes.data_as(ctypes.c_void_p), offset, a.size))

    def get_weight(self, w, offset=0, size=None):
        import numpy as np

        size = w.nbytes - offset if size is None else size
        out = np.empty(size, dtype=np.uint8)
        self.check(self.L.b200_weight_get(self.h, ctypes.byref(w), out.ctypes.data_as(ctypes.c_void_p), offset, size))
        return out

    def free_weight(self, w):
        self.check(self.L.b200_weight_free(self.h, ctypes.byref(w)))

    # -- ops (torch CUDA tensors; run on the context's stream) ----------------------------------------------------
    def _sync_in(self):
        """Orders the context's stream after torch's current stream (inputs written by torch)."""
        import torch

        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.torch_stream().wait_event(ev)

    def _sync_out(self):
        import torch

        ev = torch.cuda.Event()
        ev.record(self.torch_stream())
        torch.cuda.current_stream(self.device).wait_event(ev)

    def mul_mat(self, w, x, out=None):
        """ggml_mul_mat(w, x): x float32 [M, K] -> [M, N]."""
        import torch

        x = x.reshape(-1, w.ne0)
        M = x.shape[0]
        out = torch.empty((M, w.ne1), dtype=torch.float32, device=x.device) if out is None else out
        self._sync_in()
        self.check(self.L.b200_mul_mat(self.h, ctypes.byref(w), _ptr(x), M, _ptr(out)))
        self._sync_out()
        return out

    def mul_mat_rows(self, w, row0, n, x, out=None):
        import torch

        x = x.reshape(-1, w.ne0)
        M = x.shape[0]
        out = torch.empty((M, n), dtype=torch.float32, device=x.device) if out is None else out
        self._sync_in()
        self.check(self.L.b200_mul_mat_rows(self.h, ctypes.byref(w), row0, n, _ptr(x), M, _ptr(out), out.stride(0)))
        self._sync_out()
        return out

    def mul_mat_id(self, experts, b, ids, out=None):
        """ggml_mul_mat_id(experts, b, ids): b float32 [T, nb1, K] (nb1 = 1 or top_k), ids int32 [T, top_k]."""
        import torch

        T, top_k = ids.shape
        nb1 = b.shape[1]
        out = torch.empty((T, top_k, experts.ne1), dtype=torch.float32, device=b.device) if out is None else out
        self._sync_in()
        self.check(self.L.b200_mul_mat_id(self.h, ctypes.byref(experts), _ptr(b), nb1, _ptr(ids), top_k, T, _ptr(out)))
        self._sync_out()
        return out

    def moe_ffn(self, gate_up, down, x, ids, w, expert0=0, n_expert_total=0, out=None):
        """The routed-expert block of TextModel::experts: x float32 [T, H], ids int32 [T, top_k], w float32 [T, top_k]
        -> [T, H] (this shard's partial sum when the experts are a shard)."""
        import torch

        T, top_k = ids.shape
        out = torch.empty((T, gate_up.ne0), dtype=torch.float32, device=x.device) if out is None else out
        self._sync_in()
        self.check(self.L.b200_moe_ffn(self.h, ctypes.byref(gate_up), ctypes.byref(down), expert0, n_expert_total, _ptr(x), _ptr(ids),
                                       _ptr(w), top_k, T, _ptr(out)))
        self._sync_out()
        return out

    def moe_ffn_ep(self, gate_up, down, x, ids, w, expert0, n_expert_total, group, out=None):
        """b200_moe_ffn_ep: this rank's experts, combined with every other rank's over NVLink peer memory; out
        [T, H] is the full sum (the same on every rank). group: a handle from expert_parallel.PeerCombine."""
        import torch

        T, top_k = ids.shape
        out = torch.empty((T, gate_up.ne0), dtype=torch.float32, device=x.device) if out is None else out
        self._sync_in()
        self.check(self.L.b200_moe_ffn_ep(self.h, ctypes.byref(gate_up), ctypes.byref(down), expert0, n_expert_total, _ptr(x),
                                          _ptr(ids), _ptr(w), top_k, T, _ptr(out), group))
        self._sync_out()
        return out

    def prefetch_l2(self, w, stream=None):
        """b200_weight_prefetch_l2: queue an L2 prefetch of the weight on `stream` (a torch stream; None: the context's)."""
        self.check(self.L.b200_weight_prefetch_l2(self.h, ctypes.byref(w), ctypes.c_void_p(stream.cuda_stream) if stream is not None else None))

    def get_rows(self, table, ids, out=None):
        import torch

        out = torch.empty((ids.numel(), table.ne0), dtype=torch.float32, device=ids.device) if out is None else out
        self._sync_in()
        self.check(self.L.b200_get_rows(self.h, ctypes.byref(table), _ptr(ids), ids.numel(), _ptr(out)))
        self._sync_out()
        return out

    def quantize_rows(self, qtype, x):
        """The CPU backend's activation quantization: float32 [M, K] -> uint8 [M, row bytes] (Q8_0 or Q8_K)."""
        import torch

        M, K = x.shape
        out = torch.empty((M, row_size(qtype, K)), dtype=torch.uint8, device=x.device)
        self._sync_in()
        self.check(self.L.b200_quantize_rows(self.h, qtype, _ptr(x), K, M, _ptr(out)))
        self._sync_out()
        return out

    def block_sums(self, w, x):
        import torch

        per_row = {Q8_0: w.ne0 // 32, Q4_K: 2 * (w.ne0 // 256), Q5_K: 2 * (w.ne0 // 256), Q6_K: w.ne0 // 256}[w.type]
        out = torch.empty((w.ne1 * w.ne2, per_row), dtype=torch.int32, device=x.device)
        self._sync_in()
        self.check(self.L.b200_block_sums(self.h, ctypes.byref(w), _ptr(x), _ptr(out)))
        self._sync_out()
        return out

    def mul_mat_host(self, w, x):
        """End-to-end host path: numpy float32 [M, K] -> numpy [M, N] (copies inside the call)."""
        import numpy as np

        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, w.ne0)
        out = np.empty((x.shape[0], w.ne1), dtype=np.float32)
        self.check(self.L.b200_mul_mat_host(self.h, ctypes.byref(w), x.ctypes.data_as(ctypes.c_void_p), x.shape[0],
                                            out.ctypes.data_as(ctypes.c_void_p)))
        return out


class Graph:
    """A list of b200_tensor records over torch CUDA tensors (or weights), computed by b200_graph_compute: the ggml
    adapter's graph_compute, driven from Python. add() appends a record and returns its index; views are leaves with
    their own strides (a permuted torch view passes its strides through)."""

    _TYPES = {"torch.float32": F32, "torch.float16": F16, "torch.int32": I32}

    def __init__(self, ctx):
        self.ctx = ctx
        self.recs = []
        self.keep = []

    def add(self, op=OP_NONE, t=None, weight=None, src=(), params=(), out=None):
        """t: the record's tensor (a torch CUDA tensor: its data, shape and strides become data / ne / nb, innermost
        dimension last in torch and first in ggml); weight: a Weight for a weight leaf; src: record indices."""
        r = Tensor()
        r.op = op
        if weight is not None:
            r.type = weight.type
            r.weight = ctypes.pointer(weight)
            r.data = weight.data
            r.ne[:] = [weight.ne0, weight.ne1, weight.ne2, 1]
            self.keep.append(weight)
        else:
            dims = list(t.shape)[::-1] + [1] * (4 - t.dim())
            strides = [st * t.element_size() for st in list(t.stride())[::-1]] + [0] * (4 - t.dim())
            for i in range(t.dim(), 4):
                strides[i] = (strides[i - 1] * dims[i - 1]) if i > 0 else t.element_size()
            r.type = self._TYPES[str(t.dtype)]
            r.ne[:] = dims[:4]
            r.nb[:] = strides[:4]
            r.data = t.data_ptr()
            self.keep.append(t)
        srcs = list(src) + [-1] * (4 - len(src))
        r.src[:] = srcs[:4]
        ps = list(params) + [0] * (8 - len(params))
        r.params[:] = [int(v) for v in ps[:8]]
        self.recs.append(r)
        return len(self.recs) - 1

    @staticmethod
    def fbits(x):
        """A float parameter's bits as the int32 params[] holds them."""
        import struct

        return struct.unpack("<i", struct.pack("<f", float(x)))[0]

    def array(self):
        return (Tensor * len(self.recs))(*self.recs)

    def supports(self, i):
        arr = self.array()
        return bool(self.ctx.L.b200_graph_supports(arr, len(self.recs), i))

    def compute(self):
        """Runs every record with an op on the context's stream, ordered after torch's current stream."""
        arr = self.array()
        self.ctx._sync_in()
        self.ctx.check(self.ctx.L.b200_graph_compute(self.ctx.h, arr, len(self.recs)))
        self.ctx._sync_out()


class Decoder:
    """The matmul stack of one Qwen3 decoder step (b200_decoder): Qwen3Decoder::layers / outputs for one token at a
    sequence's first position (src/common/qwen3-decoder.cpp:350-438)."""

    def __init__(self, ctx, n_layer, hidden, n_head, n_kv_head, head_dim, ffn, n_vocab, eps=1e-6, type_attn=Q8_0,
                 type_ffn_up=Q8_0, type_ffn_down=Q8_0, type_head=Q8_0):
        self.ctx = ctx
        self.L = ctx.L
        self.shape = DecoderShape(n_layer, hidden, n_head, n_kv_head, head_dim, ffn, n_vocab, eps, type_attn, type_ffn_up,
                                  type_ffn_down, type_head)
        h = ctypes.c_void_p()
        ctx.check(self.L.b200_decoder_create(ctx.h, ctypes.byref(self.shape), ctypes.byref(h)))
        self.h = h
        ctx._children.add(self)

    def set_tensor(self, layer, which, data, offset=0):
        """data: numpy (host) or a CUDA tensor; GGUF block bytes for matrices, float32 for norms."""
        if hasattr(data, "is_cuda") and data.is_cuda:
            n = data.numel() * data.element_size()
            self.ctx._sync_in()  # the tensor's writes (torch's stream) come first; its reuse (after return) comes after
            self.ctx.check(self.L.b200_decoder_set_tensor(self.h, layer, which, _ptr(data), 1, offset, n))
            self.ctx._sync_out()
        else:
            import numpy as np

            a = np.ascontiguousarray(data)
            self.ctx.check(self.L.b200_decoder_set_tensor(self.h, layer, which, a.ctypes.data_as(ctypes.c_void_p), 0, offset,
                                                          a.nbytes))

    def step(self, x, logits=None):
        """x: CUDA float32 [hidden]; returns CUDA float32 [n_vocab] (on the context stream, ordered after torch's)."""
        import torch

        out = torch.empty(self.shape.n_vocab, dtype=torch.float32, device=x.device) if logits is None else logits
        self.ctx._sync_in()
        self.ctx.check(self.L.b200_decoder_step(self.h, _ptr(x), _ptr(out)))
        self.ctx._sync_out()
        return out

    def step_raw(self, x_ptr, logits_ptr):
        """Enqueues one step on the context stream with no stream ordering (for timing loops)."""
        self.ctx.check(self.L.b200_decoder_step(self.h, ctypes.c_void_p(x_ptr), ctypes.c_void_p(logits_ptr) if logits_ptr else None))

    def step_host(self, x, out=None):
        import numpy as np

        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.shape.n_vocab, dtype=np.float32) if out is None else out
        self.ctx.check(self.L.b200_decoder_step_host(self.h, x.ctypes.data_as(ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p)))
        return out

    @property
    def launches(self):
        return self.L.b200_decoder_launches(self.h)

    @property
    def weight_bytes(self):
        return self.L.b200_decoder_weight_bytes(self.h)

    def set_launch(self, mode=-1, pdl=True, ctas_per_sm=2):
        """mode: -1 automatic, DEC_MODE_CHAIN (one launch per product) or DEC_MODE_PERSISTENT (one kernel)."""
        self.ctx.check(self.L.b200_decoder_set_launch(self.h, mode, int(bool(pdl)), ctas_per_sm))

    def close(self):
        # a decoder's memory belongs to its context: destroy it only while the context is alive
        if getattr(self, "h", None):
            if getattr(self.ctx, "h", None):
                self.L.b200_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_count():
    return lib().b200_device_count()


def device_info(device: int):
    """b200_device_info: (name, free bytes, total bytes) of one device, as ggml_backend_dev_memory reports them."""
    name = ctypes.create_string_buffer(256)
    free, total = ctypes.c_size_t(), ctypes.c_size_t()
    s = lib().b200_device_info(device, name, 256, ctypes.byref(free), ctypes.byref(total))
    if s != OK:
        raise B200Error(s, f"device_info({device})")
    return name.value.decode(), free.value, total.value
