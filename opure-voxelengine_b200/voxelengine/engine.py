"""ctypes binding of libopure_engine.so (include/opure_engine.h): the C++20 host engine
and the seeded synthetic-input generators. No fallback: a missing library raises."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import cuda

LIB_PATH = os.path.join(cuda.PKG, "libopure_engine.so")
P, u32, u64, f32, i32, f64 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_float, C.c_int32, C.c_double


class EngineOptions(C.Structure):
    _fields_ = [("max_new_tokens", u32), ("max_batch", u32), ("max_len", u32), ("page_size", u32),
                ("page_seed", u64), ("use_graphs", u32), ("attn_scale", f32), ("path", u32),
                ("phase_trace", u32), ("prefill_chunk", u32), ("kv_window", u32),
                ("tp_allreduce", u32)]


PATH_AUTO, PATH_UNFUSED, PATH_FUSED, PATH_FUSED_LAYERS = 0, 1, 2, 3
TP_AUTO, TP_NCCL, TP_PEER = 0, 1, 2


class EngineInfo(C.Structure):
    _fields_ = [("vocab", u32), ("hidden", u32), ("inter", u32), ("layers", u32), ("heads", u32),
                ("kv_heads", u32), ("head_dim", u32), ("max_pos", u32), ("max_len", u32),
                ("max_batch", u32), ("page_size", u32), ("w_dtype", u32), ("weight_bytes", u64),
                ("stream_bytes", u64), ("kv_bytes_per_token", u64), ("tp_ranks", u32),
                ("tp_peer", u32)]


class Timing(C.Structure):
    _fields_ = [("prefill_ms", f64), ("decode_ms", f64), ("prefill_steps", u32),
                ("decode_steps", u32)]


class Metrics(C.Structure):
    _fields_ = [("kv_occupancy", f32), ("tokens_per_sec", f32), ("memory_pressure", f32),
                ("speculative_acceptance", f32), ("position", u32)]


class SpecOptions(C.Structure):
    _fields_ = [("k", u32), ("mode", u32), ("seed", u64), ("draft_log", P), ("draft_log_rounds", u32)]


class SpecStats(C.Structure):
    _fields_ = [("rounds", u32), ("drafted", u64), ("accepted", u64), ("draft_ms", f64),
                ("verify_ms", f64), ("total_ms", f64)]


SPEC_GREEDY, SPEC_REJECTION = 0, 1


class SampleOptions(C.Structure):
    _fields_ = [("temperature", f32), ("top_k", u32), ("top_p", f32), ("rep_penalty", f32),
                ("seed", u64)]


class SynthSpec(C.Structure):
    _fields_ = [("vocab", u32), ("hidden", u32), ("inter", u32), ("layers", u32), ("heads", u32),
                ("kv_heads", u32), ("max_pos", u32), ("eps", f32), ("theta", f64), ("tied", u32),
                ("seed", u64), ("std", f32), ("int8", u32), ("noise_seed", u64),
                ("noise_std", f32)]


# SmolLM-135M shape (BASELINE configs 0/2/3) and the 1.7B shape (config 4).
SMOLLM_135M = dict(vocab=49152, hidden=576, inter=1536, layers=30, heads=9, kv_heads=3,
                   max_pos=2048, eps=1e-5, theta=10000.0)
LLAMA_1_7B = dict(vocab=49152, hidden=2048, inter=8192, layers=24, heads=32, kv_heads=32,
                  max_pos=8192, eps=1e-5, theta=10000.0)

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        cuda.lib()  # libopure_cuda first (RTLD_GLOBAL)
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is not built: run __graft_entry__.build()")
        L = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        sigs = {
            "opure_engine_create": [C.c_char_p, C.c_int, P, P],
            "opure_engine_create_shared": [C.c_char_p, P, P, P],
            "opure_engine_create_tp": [C.c_char_p, P, P, P, P],
            "opure_engine_spec_generate": [P, P, P, u32, u32, u32, P, P, P, u32, P],
            "opure_engine_sample_generate": [P, P, u32, u32, u32, P, P, P, P],
            "opure_engine_destroy": [P],
            "opure_engine_get_info": [P, P],
            "opure_engine_generate": [P, P, P, u32, u32, P, P],
            "opure_engine_generate_stop": [P, P, P, u32, u32, P, P, P, P],
            "opure_engine_snapshot_metrics": [P, P],
            "opure_engine_prefill": [P, P, u32, P],
            "opure_engine_decode_step": [P, P, P, u32, P],
            "opure_engine_forward_logits": [P, P, u32, P],
            "opure_engine_run_steps": [P, u32, u32],
            "opure_engine_set_positions": [P, P, u32],
            "opure_engine_sync": [P],
            "opure_engine_forward_argmax": [P, P, u32, P],
            "opure_engine_trace": [P, i32, u32, P],
            "opure_engine_poison": [P, f32],
            "opure_engine_load_kv": [P, u32, P, u32],
            "opure_engine_synth_context": [P, u32, u32, u32, u64, P],
            "opure_engine_phase_trace": [P, P, C.c_size_t, P],
            "opure_engine_read_tokens": [P, u32, u32, u32, P],
            "opure_synth_kv": [u64, u32, u32, u32, u32, u32, P],
            "opure_server_start": [C.c_char_p, P, u32, C.c_uint16, P, P],
            "opure_server_stop": [P],
            "opure_server_parse_generate": [C.c_char_p, C.c_size_t, u32, P, u32, P, P, P, C.c_char_p, C.c_size_t],
            "opure_model_inspect": [C.c_char_p, P, C.c_char_p, C.c_size_t],
            "opure_synth_model": [C.c_char_p, P],
            "opure_synth_normal_f16": [u64, f32, u64, P],
            "opure_synth_prompt": [u64, u32, u32, P],
            "opure_synth_permutation": [u64, u32, P],
            "opure_synth_uniforms": [u64, u64, P],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = C.c_int
        L.opure_engine_last_error.argtypes = [P]
        L.opure_engine_last_error.restype = C.c_char_p
        L.opure_engine_ctx.argtypes = [P]
        L.opure_engine_ctx.restype = P
        L.opure_server_port.argtypes = [P]
        L.opure_server_port.restype = C.c_uint16
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


def _check(status, what, h=None):
    if status != 0:
        msg = lib().opure_engine_last_error(h) or b""
        raise cuda.OpureError(status, f"{what}: {msg.decode(errors='replace')}")


# ---- synthetic inputs ---------------------------------------------------------
def synth_model(path: str, seed: int = 0, std: float = 0.02, int8: bool = False, tied: bool = True,
                noise_seed: int = 0, noise_std: float = 0.0, **shape) -> str:
    """Writes config.json + model.safetensors to `path` (skipped when already present with
    the same spec, recorded in a marker file)."""
    dims = dict(SMOLLM_135M)
    dims.update(shape)
    spec = SynthSpec(dims["vocab"], dims["hidden"], dims["inter"], dims["layers"], dims["heads"],
                     dims["kv_heads"], dims["max_pos"], dims["eps"], dims["theta"], int(tied), seed,
                     std, int(int8), noise_seed, noise_std)
    marker = os.path.join(path, ".synth")
    want = repr(sorted(dict(dims, seed=seed, std=std, int8=int8, tied=tied, noise_seed=noise_seed,
                            noise_std=noise_std).items()))
    if os.path.exists(marker) and open(marker).read() == want and \
            os.path.exists(os.path.join(path, "model.safetensors")):
        return path
    _check(lib().opure_synth_model(path.encode(), C.byref(spec)), "opure_synth_model")
    with open(marker, "w") as f:
        f.write(want)
    return path


def normal_f16(seed: int, std: float, n: int) -> np.ndarray:
    out = np.empty(n, np.uint16)
    _check(lib().opure_synth_normal_f16(seed, std, n, _p(out)), "opure_synth_normal_f16")
    return out


def prompt(seed: int, vocab: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    _check(lib().opure_synth_prompt(seed, vocab, n, _p(out)), "opure_synth_prompt")
    return out


def permutation(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    _check(lib().opure_synth_permutation(seed, n, _p(out)), "opure_synth_permutation")
    return out


def uniforms(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    _check(lib().opure_synth_uniforms(seed, n, _p(out)), "opure_synth_uniforms")
    return out


def synth_kv(seed: int, slot: int, layers: int, n_kv: int, length: int, head_dim: int) -> np.ndarray:
    """Host form of the device's synthetic KV context: [layers][2][n_kv][length][head_dim] fp16 bits."""
    out = np.empty((layers, 2, n_kv, length, head_dim), np.uint16)
    _check(lib().opure_synth_kv(seed, slot, layers, n_kv, length, head_dim, _p(out)), "opure_synth_kv")
    return out


def inspect(model_dir: str) -> EngineInfo:
    """Plans a model without a GPU; raises with the engine's reason on refusal."""
    info = EngineInfo()
    err = C.create_string_buffer(4096)
    st = lib().opure_model_inspect(model_dir.encode(), C.byref(info), err, 4096)
    if st != 0:
        raise cuda.OpureError(st, "opure_model_inspect: " + err.value.decode(errors="replace"))
    return info


# ---- engine ----------------------------------------------------------------------
class Engine:
    """engine::VoxelEngine on one GPU."""

    def __init__(self, model_dir: str, device: int = 0, max_batch: int = 1, max_len: int = 0,
                 page_size: int = 64, page_seed: int = 3, use_graphs: bool = True,
                 attn_scale: float = 1.0, max_new_tokens: int = 256, path: int = PATH_AUTO,
                 share: "Engine | None" = None, comm: "cuda.Comm | None" = None,
                 phase_trace: bool = False, prefill_chunk: int = 0, kv_window: int = 0,
                 tp_allreduce: int = TP_AUTO):
        """With `share`, the engine runs on that engine's ctx (stream), as the draft of a
        speculative pair must; it keeps a reference so the owner outlives it. With `comm`
        it is that communicator's tensor-parallel shard, on the communicator's ctx, whose
        all-reduces run as NCCL calls (`tp_allreduce` TP_NCCL, and TP_AUTO at 2 ranks) or
        as NVLink peer kernels (TP_PEER, and TP_AUTO at any rank count, when every pair of GPUs
        can map each other's memory)."""
        o = EngineOptions(max_new_tokens, max_batch, max_len, page_size, page_seed,
                          int(use_graphs), attn_scale, path, int(phase_trace), prefill_chunk, kv_window,
                          tp_allreduce)
        h = C.c_void_p()
        if comm is not None:
            st = lib().opure_engine_create_tp(model_dir.encode(), comm.ctx.h, comm.h, C.byref(o), C.byref(h))
        elif share is None:
            st = lib().opure_engine_create(model_dir.encode(), device, C.byref(o), C.byref(h))
        else:
            st = lib().opure_engine_create_shared(model_dir.encode(), share.h, C.byref(o), C.byref(h))
        _check(st, "opure_engine_create", None)
        self.share = share
        self.comm = comm
        self.h = h
        self.info = EngineInfo()
        _check(lib().opure_engine_get_info(self.h, C.byref(self.info)), "get_info", self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().opure_engine_destroy(self.h)
            self.h = None
        self.share = None
        self.comm = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def ctx(self):
        return lib().opure_engine_ctx(self.h)

    def generate(self, prompts, budget: int):
        """prompts: list of token-id sequences; returns (tokens [n][budget], Timing)."""
        ps = [np.asarray(p, np.int32) for p in prompts]
        flat = np.ascontiguousarray(np.concatenate(ps), np.int32)
        lens = np.array([p.size for p in ps], np.uint32)
        out = np.zeros((len(ps), budget), np.int32)
        t = Timing()
        _check(lib().opure_engine_generate(self.h, _p(flat), _p(lens), len(ps), budget, _p(out),
                                           C.byref(t)), "generate", self.h)
        return out, t

    def generate_stop(self, prompts, budget: int):
        """generate with the per-sequence results of the reference's stop rules: returns
        (tokens [n][budget] with -1 after each sequence's last token, counts [n],
        hit_stop [n] bool, Timing)."""
        ps = [np.asarray(p, np.int32) for p in prompts]
        flat = np.ascontiguousarray(np.concatenate(ps), np.int32)
        lens = np.array([p.size for p in ps], np.uint32)
        out = np.zeros((len(ps), budget), np.int32)
        counts = np.zeros(len(ps), np.uint32)
        hit = np.zeros(len(ps), np.uint32)
        t = Timing()
        _check(lib().opure_engine_generate_stop(self.h, _p(flat), _p(lens), len(ps), budget, _p(out), _p(counts),
                                                _p(hit), C.byref(t)), "generate_stop", self.h)
        return out, counts, hit.astype(bool), t

    def metrics(self) -> Metrics:
        m = Metrics()
        _check(lib().opure_engine_snapshot_metrics(self.h, C.byref(m)), "metrics", self.h)
        return m

    def spec_generate(self, draft: "Engine", prompts, budget: int, k: int = 4, mode: int = SPEC_GREEDY,
                      seed: int = 0, log_rounds: int = 0, draft_log: bool = False):
        """Speculative decoding with `draft` (created with share=self). prompts: equal-length
        sequences. Returns (tokens [n][budget], SpecStats, accept log [rounds][n] or None), and
        with draft_log=True also the drafted tokens [rounds][n][k] (log_rounds rounds)."""
        ps = np.ascontiguousarray(np.stack([np.asarray(p, np.int32) for p in prompts]), np.int32)
        n, plen = ps.shape
        out = np.zeros((n, budget), np.int32)
        dlog = np.zeros((log_rounds, n, k), np.int32) if draft_log else None
        o = SpecOptions(k, mode, seed, _p(dlog) if dlog is not None else None, log_rounds if draft_log else 0)
        st = SpecStats()
        log = np.zeros((log_rounds, n), np.int32) if log_rounds else None
        _check(lib().opure_engine_spec_generate(self.h, draft.h, _p(ps), plen, n, budget, C.byref(o),
                                                _p(out), _p(log), log_rounds, C.byref(st)),
               "spec_generate", self.h)
        if log is not None:
            log = log[: min(log_rounds, st.rounds)]
        if draft_log:
            return out, st, log, dlog[: min(log_rounds, st.rounds)]
        return out, st, log

    def sample_generate(self, prompts, budget: int, temperature: float = 1.0, top_k: int = 0,
                        top_p: float = 1.0, rep_penalty: float = 1.0, seed: int = 0, stats: bool = False,
                        logits: bool = False):
        """Sampled generation (equal-length prompts). Returns tokens [n][budget], or a tuple
        with, when asked for, the logit statistics [n][budget][4] (max, L2 norm, entropy,
        log-sum-exp) and the logits [n][budget][vocab] each token was drawn from."""
        ps = np.ascontiguousarray(np.stack([np.asarray(p, np.int32) for p in prompts]), np.int32)
        n, plen = ps.shape
        out = np.zeros((n, budget), np.int32)
        st = np.zeros((n, budget, 4), np.float32) if stats else None
        lg = np.zeros((n, budget, self.info.vocab), np.float32) if logits else None
        o = SampleOptions(temperature, top_k, top_p, rep_penalty, seed)
        _check(lib().opure_engine_sample_generate(self.h, _p(ps), plen, n, budget, C.byref(o), _p(out), _p(st),
                                                  _p(lg)), "sample_generate", self.h)
        if not stats and not logits:
            return out
        return (out,) + ((st,) if stats else ()) + ((lg,) if logits else ())

    def prefill(self, tokens) -> int:
        """Prefill slot 0; returns the first generated token."""
        t = np.ascontiguousarray(tokens, np.int32)
        nxt = C.c_int32()
        _check(lib().opure_engine_prefill(self.h, _p(t), t.size, C.byref(nxt)), "prefill", self.h)
        return int(nxt.value)

    def decode_step(self, tokens, positions) -> np.ndarray:
        t = np.ascontiguousarray(np.atleast_1d(tokens), np.int32)
        p = np.ascontiguousarray(np.atleast_1d(positions), np.int32)
        nxt = np.zeros(t.size, np.int32)
        _check(lib().opure_engine_decode_step(self.h, _p(t), _p(p), t.size, _p(nxt)), "decode_step",
               self.h)
        return nxt

    def forward_logits(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        out = np.zeros(self.info.vocab, np.float32)
        _check(lib().opure_engine_forward_logits(self.h, _p(t), t.size, _p(out)), "forward_logits",
               self.h)
        return out

    def forward_argmax(self, tokens) -> int:
        t = np.ascontiguousarray(tokens, np.int32)
        out = C.c_int32()
        _check(lib().opure_engine_forward_argmax(self.h, _p(t), t.size, C.byref(out)),
               "forward_argmax", self.h)
        return int(out.value)

    def trace(self, token: int, n_layers: int) -> np.ndarray:
        out = np.zeros((n_layers, self.info.hidden), np.float32)
        _check(lib().opure_engine_trace(self.h, token, n_layers, _p(out)), "trace", self.h)
        return out

    def poison(self, value: float):
        _check(lib().opure_engine_poison(self.h, value), "poison", self.h)

    def phase_trace(self) -> np.ndarray:
        """The last persistent step's stamps [sm_count][3 layers + 2][2] (ns), or an empty array."""
        cap = 4096 * (3 * self.info.layers + 2) * 2
        out = np.zeros(cap, np.uint64)
        n = C.c_size_t()
        _check(lib().opure_engine_phase_trace(self.h, _p(out), cap, C.byref(n)), "phase_trace", self.h)
        rows = 3 * self.info.layers + 2
        return out[: n.value].reshape(-1, rows, 2) if n.value else out[:0]

    def synth_context(self, n: int, length: int, reserve: int, seed: int, first_tokens):
        """Slots 0..n-1: `length` cached positions of seeded KV values, then self-driving
        decode from position `length` with first_tokens[v] as input (run_steps)."""
        f = np.ascontiguousarray(first_tokens, np.int32)
        _check(lib().opure_engine_synth_context(self.h, n, length, reserve, seed, _p(f)), "synth_context",
               self.h)

    def run_steps(self, n: int, steps: int):
        _check(lib().opure_engine_run_steps(self.h, n, steps), "run_steps", self.h)

    def sync(self):
        _check(lib().opure_engine_sync(self.h), "sync", self.h)

    def read_tokens(self, slot: int, pos: int, count: int) -> np.ndarray:
        out = np.zeros(count, np.int32)
        _check(lib().opure_engine_read_tokens(self.h, slot, pos, count, _p(out)), "read_tokens", self.h)
        return out

    def load_kv(self, seq: int, kv: np.ndarray, length: int):
        kv = np.ascontiguousarray(kv, np.uint16)
        _check(lib().opure_engine_load_kv(self.h, seq, _p(kv), length), "load_kv", self.h)


# ---- serving front end -------------------------------------------------------------
class Server:
    """The HTTP front end (GET /health, POST /generate, GET /metrics) on 127.0.0.1 with one
    engine per device in `devices` (none: the routes answer, /generate with 503)."""

    def __init__(self, model_dir: str | None = None, devices=(), port: int = 0, **engine_opts):
        devs = np.ascontiguousarray(list(devices), np.int32)
        o = EngineOptions(engine_opts.get("max_new_tokens", 256), engine_opts.get("max_batch", 1),
                          engine_opts.get("max_len", 0), engine_opts.get("page_size", 64),
                          engine_opts.get("page_seed", 3), 1, 1.0, engine_opts.get("path", PATH_AUTO), 0, 0, 0, 0)
        h = C.c_void_p()
        _check(lib().opure_server_start(model_dir.encode() if model_dir else None, _p(devs) if devs.size else None,
                                        int(devs.size), port, C.byref(o), C.byref(h)), "opure_server_start")
        self.h = h
        self.port = int(lib().opure_server_port(h))

    def close(self):
        if getattr(self, "h", None):
            lib().opure_server_stop(self.h)
            self.h = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def parse_generate(body: bytes, vocab: int = 0):
    """The server's /generate body parser: (tokens, max_tokens, temperature), or raises
    ValueError with the message a client would get."""
    toks = np.zeros(4096, np.int32)
    n, mt, t = C.c_uint32(), C.c_uint32(), C.c_float()
    err = C.create_string_buffer(512)
    st = lib().opure_server_parse_generate(body, len(body), vocab, _p(toks), toks.size, C.byref(n), C.byref(mt),
                                           C.byref(t), err, 512)
    if st != 0:
        raise ValueError(err.value.decode(errors="replace"))
    return toks[: n.value].tolist(), int(mt.value), float(t.value)
