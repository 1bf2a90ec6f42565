"""ctypes binding of libopure_cuda.so (include/opure_cuda.h).

There is no fallback: if the library is missing or fails to load, every entry point
raises. Device memory is owned through the ABI's own allocator (DeviceBuffer).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG, "libopure_cuda.so")

OK, ERR_INVALID_ARG, ERR_NO_DEVICE, ERR_CUDA, ERR_OOM = 0, 1, 2, 3, 4
ERR_TIMEOUT, ERR_DEVICE_TIMEOUT, ERR_UNSUPPORTED, ERR_INJECTED, ERR_DEVICE_BOUNDS = 5, 6, 7, 8, 9
W_F16, W_Q8 = 0, 1
PRO_NONE, PRO_RMSNORM = 0, 1
EPI_STORE, EPI_ADD, EPI_SWIGLU, EPI_ARGMAX = 0, 1, 2, 3
SPEC_GREEDY, SPEC_REJECTION = 0, 1

P, u8, u32, u64, f32, i32, sz = (C.c_void_p, C.c_uint8, C.c_uint32, C.c_uint64, C.c_float,
                                 C.c_int32, C.c_size_t)


class OpureError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {_strerror(status)} (status {status})")


class KvLayout(C.Structure):
    _fields_ = [("pool", P), ("page_table", P), ("n_pages", u32), ("max_pages", u32),
                ("page_size", u32), ("n_kv", u32), ("head_dim", u32), ("ring", u32)]


class AttnArgs(C.Structure):
    _fields_ = [("q", P), ("out", P), ("seq", P), ("seq_len", P), ("n", u32), ("n_q", u32),
                ("n_heads", u32), ("scale", f32), ("max_ctx", u32), ("split_tokens", u32),
                ("scratch", P), ("scratch_bytes", sz), ("kv", KvLayout), ("out_packed", P)]


class GemvArgs(C.Structure):
    _fields_ = [("w", P), ("w_dtype", u32), ("scale_w", f32), ("scale_x", f32),
                ("scale_w2", f32), ("rows", u32),
                ("cols", u32), ("nvec", u32), ("x", P), ("x_stride", u32), ("y", P),
                ("y_stride", u32), ("prologue", u32), ("norm_gain", P), ("eps", f32),
                ("epilogue", u32), ("residual", P), ("argmax_keys", P),
                ("x_packed", P), ("x_sumsq", P), ("y_packed", P), ("y_pack_gain", P), ("y_sumsq", P)]


class StepIO(C.Structure):
    _fields_ = [("nvec", u32), ("seq", P), ("pos", P), ("seq_len", P), ("known", P),
                ("flags", P), ("in_tokens", P), ("tokens", P), ("max_len", u32), ("keys", P),
                ("embed", P),
                ("vocab", u32), ("hidden", u32), ("x", P)]


class SpecArgs(C.Structure):
    _fields_ = [("mode", u32), ("n_seq", u32), ("k", u32), ("vocab", u32),
                ("target_logits", P), ("draft_logits", P), ("draft", P), ("u_accept", P),
                ("u_final", P), ("out_tokens", P), ("out_accepted", P)]


class SampleArgs(C.Structure):
    _fields_ = [("logits", P), ("vocab", u32), ("rows", u32), ("stride", sz),
                ("temperature", f32), ("top_k", u32), ("top_p", f32), ("rep_penalty", f32),
                ("hist", P), ("max_len", u32), ("seq", P), ("hist_len", P), ("u", P),
                ("out", P), ("keys", P)]


class DeviceInfo(C.Structure):
    _fields_ = [("device", i32), ("sm_count", i32), ("cc_major", i32), ("cc_minor", i32),
                ("hbm_bytes", u64), ("l2_bytes", u64), ("smem_per_block_optin", u32),
                ("clock_mhz_max", u32), ("name", C.c_char * 96)]


_lib = None

_SIGS = {
    "opure_init": [i32, P], "opure_shutdown": [P], "opure_get_device_info": [P, P],
    "opure_last_error": [P], "opure_alloc": [P, sz, P], "opure_free": [P, P],
    "opure_alloc_host": [P, sz, P], "opure_free_host": [P, P],
    "opure_h2d": [P, P, P, sz], "opure_d2h": [P, P, P, sz], "opure_d2d": [P, P, P, sz],
    "opure_fill": [P, P, u8, sz], "opure_sync": [P, u32],
    "opure_graph_begin": [P], "opure_graph_end": [P, P], "opure_graph_launch": [P, P],
    "opure_graph_free": [P], "opure_event_create": [P, P], "opure_event_record": [P, P],
    "opure_event_elapsed_ms": [P, P, P], "opure_event_free": [P],
    "opure_embedding": [P, P, u32, P, u32, u32, P],
    "opure_rmsnorm": [P, P, P, P, u32, u32, f32],
    "opure_swiglu": [P, P, P, P, u32], "opure_add": [P, P, P, P, u32],
    "opure_argmax": [P, P, u32, u32, P, P],
    "opure_rope_kv_append": [P, P, u32, P, P, P, u32, u32, C.c_double, P],
    "opure_attention": [P, P], "opure_gemv": [P, P], "opure_argmax_decode": [P, P, u32, P, P],
    "opure_spec_accept": [P, P], "opure_sample_softmax": [P, P, u32, u32, P, P],
    "opure_debug_inject_failure": [P, u32, u32],
    "opure_step_begin": [P, P], "opure_step_end": [P, P],
    "opure_attention_static": [P, P],
    "opure_last_error_detail": [P, P, P],
    "opure_sample_keys": [P, P, u32, u32, P, P, P, sz],
    "opure_spec_gather": [P, P, u32, P, P, u32, u32, P, P],
    "opure_kv_synth": [P, P, u32, u32, u32, u32, u64],
    "opure_comm_init": [P, u32, u32, P, u32, P], "opure_comm_destroy": [P],
    "opure_comm_info": [P, P, P],
    "opure_allreduce_sum_f32": [P, P, P, sz], "opure_allreduce_max_u64": [P, P, P, sz],
    "opure_argmax_key_offset": [P, P, u32, u32],
    "opure_sample_filtered": [P, P], "opure_logit_stats": [P, P, u32, u32, sz, P],
    "opure_peer_create": [P, P, u32, u32, P], "opure_peer_destroy": [P, P, P],
    "opure_peer_info": [P, P, P, P], "opure_gemv_allreduce": [P, P, P],
    "opure_peer_argmax": [P, P, P, u32, u32],
}


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is not built: run __graft_entry__.build() "
                          "(make -C opure-voxelengine_b200)")
        L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        for name, args in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = C.c_int
        L.opure_strerror.argtypes = [C.c_int]
        L.opure_strerror.restype = C.c_char_p
        L.opure_stream.argtypes = [P]
        L.opure_stream.restype = P
        L.opure_comm_unique_id.argtypes = [P]
        L.opure_comm_unique_id.restype = C.c_int
        L.opure_attention_scratch_bytes.argtypes = [u32, u32, u32, u32, u32, u32, u32]
        L.opure_attention_scratch_bytes.restype = sz
        L.opure_packed_bytes.argtypes = [u32, u32]
        L.opure_packed_bytes.restype = sz
        _lib = L
    return _lib


def _strerror(status: int) -> str:
    try:
        return lib().opure_strerror(status).decode()
    except OSError:
        return "library not loaded"


def argmax_key(value: float, index: int) -> int:
    """The kernels' packed argmax key: (orderable fp32 bits << 32) | (0xffffffff - index)."""
    b = int(np.float32(value).view(np.uint32))
    b = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (b << 32) | (0xFFFFFFFF - index)


def argmax_key_index(key: int) -> int:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


def check(status: int, what: str) -> None:
    if status != OK:
        raise OpureError(status, what)


def attention_scratch_bytes(n, n_q, n_heads, n_kv, head_dim, max_ctx, split_tokens=0) -> int:
    return int(lib().opure_attention_scratch_bytes(n, n_q, n_heads, n_kv, head_dim, max_ctx,
                                                   split_tokens))


def packed_bytes(nvec: int, length: int) -> int:
    """Bytes of a chained tensor-core operand (fp16 hi/lo pairs of nvec vectors)."""
    return int(lib().opure_packed_bytes(nvec, length))


class DeviceBuffer:
    """Device memory from opure_alloc, freed with its context."""

    def __init__(self, ctx: "Ctx", nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = C.c_void_p()
        check(lib().opure_alloc(ctx.h, self.nbytes, C.byref(p)), "opure_alloc")
        self.ptr = p.value or 0
        ctx._bufs.append(self)

    def free(self):
        if self.ptr:
            lib().opure_free(self.ctx.h, C.c_void_p(self.ptr))
            self.ptr = 0

    def upload(self, arr: np.ndarray, offset: int = 0) -> "DeviceBuffer":
        a = np.ascontiguousarray(arr)
        assert offset + a.nbytes <= self.nbytes
        check(lib().opure_h2d(self.ctx.h, C.c_void_p(self.ptr + offset), a.ctypes.data_as(P),
                              a.nbytes), "opure_h2d")
        self.ctx.sync()
        return self

    def download(self, dtype, shape, offset: int = 0) -> np.ndarray:
        out = np.empty(shape, dtype)
        assert offset + out.nbytes <= self.nbytes
        check(lib().opure_d2h(self.ctx.h, out.ctypes.data_as(P), C.c_void_p(self.ptr + offset),
                              out.nbytes), "opure_d2h")
        self.ctx.sync()
        return out

    def fill(self, byte: int = 0) -> "DeviceBuffer":
        check(lib().opure_fill(self.ctx.h, C.c_void_p(self.ptr), byte, self.nbytes), "opure_fill")
        return self

    def __int__(self):
        return self.ptr


class Ctx:
    """One GPU, one stream (opure_ctx)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().opure_init(device, C.byref(h)), "opure_init")
        self.h = h
        self._bufs: list[DeviceBuffer] = []

    def close(self):
        if self.h:
            for b in self._bufs:
                b.free()
            self._bufs.clear()
            lib().opure_shutdown(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def info(self) -> DeviceInfo:
        d = DeviceInfo()
        check(lib().opure_get_device_info(self.h, C.byref(d)), "opure_get_device_info")
        return d

    def sync(self, timeout_ms: int = 60000):
        check(lib().opure_sync(self.h, timeout_ms), "opure_sync")

    def last_error(self) -> int:
        return int(lib().opure_last_error(self.h))

    def buffer(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def to_device(self, arr: np.ndarray) -> DeviceBuffer:
        a = np.ascontiguousarray(arr)
        return DeviceBuffer(self, max(a.nbytes, 16)).upload(a)

    # ---- kernels ------------------------------------------------------------
    def gemv(self, args: GemvArgs):
        check(lib().opure_gemv(self.h, C.byref(args)), "opure_gemv")

    def attention(self, args: AttnArgs):
        check(lib().opure_attention(self.h, C.byref(args)), "opure_attention")

    def spec_accept(self, args: SpecArgs):
        check(lib().opure_spec_accept(self.h, C.byref(args)), "opure_spec_accept")

    def sample_filtered(self, args: SampleArgs):
        check(lib().opure_sample_filtered(self.h, C.byref(args)), "opure_sample_filtered")

    def call(self, name: str, *args):
        check(getattr(lib(), name)(self.h, *args), name)


COMM_ID_BYTES = 128


def comm_unique_id() -> bytes:
    """NCCL unique id (created on one rank; send it to the others out of band)."""
    buf = (C.c_uint8 * COMM_ID_BYTES)()
    check(lib().opure_comm_unique_id(buf), "opure_comm_unique_id")
    return bytes(buf)


class Comm:
    """Tensor-parallel communicator (opure_comm) of rank `rank` of `n_ranks` on `ctx`."""

    def __init__(self, ctx: Ctx, n_ranks: int, rank: int, uid: bytes, timeout_ms: int = 60000):
        idbuf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        check(lib().opure_comm_init(ctx.h, n_ranks, rank, idbuf, timeout_ms, C.byref(h)), "opure_comm_init")
        self.h, self.ctx, self.n_ranks, self.rank = h, ctx, n_ranks, rank

    def allreduce_sum(self, buf: "DeviceBuffer", n: int):
        check(lib().opure_allreduce_sum_f32(self.ctx.h, self.h, buf.ptr, n), "opure_allreduce_sum_f32")

    def allreduce_max_u64(self, buf: "DeviceBuffer", n: int):
        check(lib().opure_allreduce_max_u64(self.ctx.h, self.h, buf.ptr, n), "opure_allreduce_max_u64")

    def close(self):
        if getattr(self, "h", None):
            lib().opure_comm_destroy(self.h)
            self.h = None


class Peer:
    """NVLink peer mailboxes of the ranks of `comm` (opure_peer): collective creation,
    GEMVs all-reduced inside the kernel, and the argmax-key max over vocabulary shards."""

    def __init__(self, comm: Comm, max_rows: int, timeout_ms: int = 2000):
        h = C.c_void_p()
        check(lib().opure_peer_create(comm.ctx.h, comm.h, max_rows, timeout_ms, C.byref(h)), "opure_peer_create")
        self.h, self.comm, self.ctx = h, comm, comm.ctx

    def gemv_allreduce(self, a: "GemvArgs"):
        check(lib().opure_gemv_allreduce(self.ctx.h, self.h, C.byref(a)), "opure_gemv_allreduce")

    def argmax(self, keys: "DeviceBuffer", n: int, offset: int):
        check(lib().opure_peer_argmax(self.ctx.h, self.h, keys.ptr, n, offset), "opure_peer_argmax")

    def close(self, collective: bool = True):
        if getattr(self, "h", None):
            check(lib().opure_peer_destroy(self.ctx.h, self.comm.h if collective else None, self.h),
                  "opure_peer_destroy")
            self.h = None


class Graph:
    def __init__(self, ctx: Ctx):
        self.ctx = ctx
        self.h = None

    def __enter__(self):
        check(lib().opure_graph_begin(self.ctx.h), "opure_graph_begin")
        return self

    def __exit__(self, et, ev, tb):
        g = C.c_void_p()
        st = lib().opure_graph_end(self.ctx.h, C.byref(g))
        if et is None:
            check(st, "opure_graph_end")
        self.h = g

    def launch(self):
        check(lib().opure_graph_launch(self.ctx.h, self.h), "opure_graph_launch")

    def free(self):
        if self.h:
            lib().opure_graph_free(self.h)
            self.h = None


class Event:
    def __init__(self, ctx: Ctx):
        self.ctx = ctx
        h = C.c_void_p()
        check(lib().opure_event_create(ctx.h, C.byref(h)), "opure_event_create")
        self.h = h

    def record(self):
        check(lib().opure_event_record(self.ctx.h, self.h), "opure_event_record")

    def elapsed_ms(self, later: "Event") -> float:
        ms = C.c_float()
        check(lib().opure_event_elapsed_ms(self.h, later.h, C.byref(ms)), "opure_event_elapsed_ms")
        return float(ms.value)

    def free(self):
        if self.h:
            lib().opure_event_free(self.h)
            self.h = None
