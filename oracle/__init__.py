"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference legs use this as the parity checker. The product never imports
it. See oracle.h for what each function restates and how the oracle is pinned.
"""
from __future__ import annotations

import ctypes as C
import json
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32, F16, BF16, I8 = 0, 1, 2, 3
EMBED, FINAL_NORM, LM_HEAD, IN_NORM, POST_NORM = 0, 1, 2, 3, 4
WQ, WK, WV, WO, GATE, UP, DOWN = 5, 6, 7, 8, 9, 10, 11


class OrcSynth(C.Structure):
    _fields_ = [("seed", C.c_uint64), ("std", C.c_float), ("tied", C.c_uint32), ("int8", C.c_uint32),
                ("noise_seed", C.c_uint64), ("noise_std", C.c_float)]


# SmolLM-135M shape (BASELINE configs 0/2/3).
SMOLLM_135M = dict(vocab=49152, hidden=576, inter=1536, layers=30, heads=9, kv_heads=3,
                   max_pos=2048, eps=1e-5, theta=10000.0)


class OrcConfig(C.Structure):
    _fields_ = [
        ("vocab", C.c_uint32), ("hidden", C.c_uint32), ("inter", C.c_uint32),
        ("layers", C.c_uint32), ("heads", C.c_uint32), ("kv_heads", C.c_uint32),
        ("max_pos", C.c_uint32), ("eps", C.c_float), ("theta", C.c_double),
        ("attn_scale", C.c_float), ("rope_cpu_literal", C.c_int32),
    ]


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        P, u32, u64, f32, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_float, C.c_int
        sig = {
            "orc_rng_u32_stream": (None, [u64, u64, P]),
            "orc_f32_to_f16": (C.c_uint16, [f32]),
            "orc_f16_to_f32": (f32, [C.c_uint16]),
            "orc_f32_to_f16_n": (None, [P, P, u64]),
            "orc_f16_to_f32_n": (None, [P, P, u64]),
            "orc_gemv_f16": (None, [P, P, P, u32, u32, u32]),
            "orc_gemv_f32": (None, [P, P, P, u32, u32, u32]),
            "orc_gemv_q8": (None, [P, f32, f32, P, P, u32, u32, u32]),
            "orc_quantize_q8": (None, [P, u64, P, P]),
            "orc_rmsnorm": (None, [P, P, P, u32, f32]),
            "orc_rope": (None, [P, u32, u32, u32, C.c_double, i32]),
            "orc_swiglu": (None, [P, P, P, u32]),
            "orc_argmax": (None, [P, u32, u32, P, P]),
            "orc_attention_paged": (None, [P, P, P, P, u32, u32, u32, u32, u32, u32, u32, f32, P]),
            "orc_attention_f32": (None, [P, P, P, u32, u32, u32, u32, u32, f32, P]),
            "orc_sample_softmax": (u32, [P, u32, f32]),
            "orc_sample_filtered": (u32, [P, u32, f32, u32, f32, f32, P, u32, f32]),
            "orc_logit_stats": (None, [P, u32, P]),
            "orc_spec_accept_greedy": (i32, [P, P, u32, u32, P]),
            "orc_spec_accept_rejection": (i32, [P, P, P, P, f32, u32, u32, P]),
            "orc_model_create": (P, [P]),
            "orc_model_set_tensor": (i32, [P, i32, i32, i32, P, u64, f32]),
            "orc_model_ready": (i32, [P]),
            "orc_model_free": (None, [P]),
            "orc_state_create": (P, [P, u32]),
            "orc_state_free": (None, [P]),
            "orc_state_len": (u32, [P]),
            "orc_state_truncate": (None, [P, u32]),
            "orc_state_set_window": (None, [P, u32, u32]),
            "orc_state_load_kv": (i32, [P, P, u32]),
            "orc_forward": (i32, [P, P, u32, P, P]),
            "orc_generate": (i32, [P, P, u32, u32, u32, P, P]),
            "orc_set_threads": (None, [i32]),
            "orc_get_threads": (i32, []),
            "orc_thread_serial": (None, [i32]),
            "orc_generate_stop": (i32, [P, P, u32, u32, u32, C.c_int64, P, P, P]),
            "orc_generate_batch": (i32, [P, P, P, u32, u32, u32, C.c_int64, i32, P, P, P, P]),
            "orc_synth_normal_f16": (None, [u64, f32, u64, P]),
            "orc_synth_prompt": (None, [u64, u32, u32, P]),
            "orc_synth_permutation": (None, [u64, u32, P]),
            "orc_synth_uniforms": (None, [u64, u64, P]),
            "orc_model_create_synth": (P, [P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# ---- data ----------------------------------------------------------------
def rng_u32(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().orc_rng_u32_stream(seed, n, _p(out))
    return out


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16_n(_p(x), _p(out), x.size)
    return out


def f16_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_f16_to_f32_n(_p(h), _p(out), h.size)
    return out


def thread_serial(on: bool = True) -> None:
    """The calling thread computes serially (never the shared worker pool): for callers
    that run independent sequences on Python threads of their own (ctypes releases the
    GIL during each call)."""
    lib().orc_thread_serial(int(on))


# ---- seeded synthetic inputs (the same bytes as the engine's generators) ----
def normal_f16(seed: int, std: float, n: int) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_synth_normal_f16(seed, std, n, _p(out))
    return out


def prompt(seed: int, vocab: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().orc_synth_prompt(seed, vocab, n, _p(out))
    return out


def permutation(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    lib().orc_synth_permutation(seed, n, _p(out))
    return out


def uniforms(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_synth_uniforms(seed, n, _p(out))
    return out


# ---- kernels -------------------------------------------------------------
def gemv_f16(w_f16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """w [rows, cols] uint16 (fp16 bits); x [cols] or [n, cols] float32."""
    w = np.ascontiguousarray(w_f16, np.uint16)
    xs = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    rows, cols = w.shape
    y = np.empty((xs.shape[0], rows), np.float32)
    lib().orc_gemv_f16(_p(w), _p(xs), _p(y), rows, cols, xs.shape[0])
    return y if np.ndim(x) == 2 else y[0]


def gemv_f32(w: np.ndarray, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    xs = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    rows, cols = w.shape
    y = np.empty((xs.shape[0], rows), np.float32)
    lib().orc_gemv_f32(_p(w), _p(xs), _p(y), rows, cols, xs.shape[0])
    return y if np.ndim(x) == 2 else y[0]


def gemv_q8(q: np.ndarray, scale_w: float, x: np.ndarray, scale_x: float = 1.0) -> np.ndarray:
    q = np.ascontiguousarray(q, np.int8)
    xs = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    rows, cols = q.shape
    y = np.empty((xs.shape[0], rows), np.float32)
    lib().orc_gemv_q8(_p(q), scale_w, scale_x, _p(xs), _p(y), rows, cols, xs.shape[0])
    return y if np.ndim(x) == 2 else y[0]


def quantize_q8(w_f16: np.ndarray) -> tuple[np.ndarray, float]:
    w = np.ascontiguousarray(w_f16, np.uint16)
    q = np.empty(w.shape, np.int8)
    s = C.c_float()
    lib().orc_quantize_q8(_p(w), w.size, _p(q), C.byref(s))
    return q, float(s.value)


def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(g), _p(y), x.size, eps)
    return y


def rope(vec: np.ndarray, nheads: int, hd: int, pos: int, theta: float, cpu_literal=False):
    v = np.array(vec, np.float32, copy=True)
    lib().orc_rope(_p(v), nheads, hd, pos, theta, int(cpu_literal))
    return v


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    h = np.empty_like(g)
    lib().orc_swiglu(_p(g), _p(u), _p(h), g.size)
    return h


def argmax(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
    rows, n = x.shape
    idx = np.empty(rows, np.uint32)
    val = np.empty(rows, np.float32)
    lib().orc_argmax(_p(x), n, rows, _p(idx), _p(val))
    return idx, val


def attention_paged(q, pool, page_table, seq_lens, page_size, n_heads, n_kv, hd, scale=1.0):
    """q [nseq, nq, nH, hd] f32; pool uint16 in the documented page layout;
    page_table [nseq, max_pages] int32; seq_lens [nseq] uint32."""
    q = np.ascontiguousarray(q, np.float32)
    nseq, nq = q.shape[0], q.shape[1]
    pool = np.ascontiguousarray(pool, np.uint16)
    pt = np.ascontiguousarray(page_table, np.int32)
    sl = np.ascontiguousarray(seq_lens, np.uint32)
    out = np.empty_like(q)
    lib().orc_attention_paged(_p(q), _p(pool), _p(pt), _p(sl), nseq, nq, pt.shape[1],
                              page_size, n_heads, n_kv, hd, scale, _p(out))
    return out


def attention_f32(q, k_plane, v_plane, n_heads, n_kv, hd, max_seq, seq_len, scale=1.0):
    """Reference cache layout: k_plane/v_plane [n_kv, max_seq, hd] f32; q [n_heads, hd]."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k_plane, np.float32)
    v = np.ascontiguousarray(v_plane, np.float32)
    out = np.empty_like(q)
    lib().orc_attention_f32(_p(q), _p(k), _p(v), n_heads, n_kv, hd, max_seq, seq_len, scale,
                            _p(out))
    return out


def sample_softmax(logits: np.ndarray, u: float) -> int:
    lg = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample_softmax(_p(lg), lg.size, u))


def sample_filtered(logits: np.ndarray, u: float, temperature: float = 1.0, top_k: int = 0,
                    top_p: float = 1.0, rep_penalty: float = 1.0, hist=None) -> int:
    lg = np.ascontiguousarray(logits, np.float32)
    h = None if hist is None else np.ascontiguousarray(hist, np.int32)
    return int(lib().orc_sample_filtered(_p(lg), lg.size, temperature, top_k, top_p, rep_penalty, _p(h),
                                         0 if h is None else h.size, u))


def logit_stats(logits: np.ndarray) -> np.ndarray:
    """{max, L2 norm, entropy (nats), log-sum-exp} of one row."""
    lg = np.ascontiguousarray(logits, np.float32)
    out = np.zeros(4, np.float32)
    lib().orc_logit_stats(_p(lg), lg.size, _p(out))
    return out


def spec_accept_greedy(target_logits: np.ndarray, draft: np.ndarray):
    tl = np.ascontiguousarray(target_logits, np.float32)
    d = np.ascontiguousarray(draft, np.uint32)
    out = np.zeros(d.size + 1, np.uint32)
    a = lib().orc_spec_accept_greedy(_p(tl), _p(d), d.size, tl.shape[1], _p(out))
    return a, out[: a + 1]


def spec_accept_rejection(target_logits, draft_logits, draft, u_accept, u_final):
    tl = np.ascontiguousarray(target_logits, np.float32)
    dl = np.ascontiguousarray(draft_logits, np.float32)
    d = np.ascontiguousarray(draft, np.uint32)
    ua = np.ascontiguousarray(u_accept, np.float32)
    out = np.zeros(d.size + 1, np.uint32)
    a = lib().orc_spec_accept_rejection(_p(tl), _p(dl), _p(d), _p(ua), float(u_final),
                                        d.size, tl.shape[1], _p(out))
    return a, out[: a + 1]


# ---- whole model ----------------------------------------------------------
_DT = {"F32": F32, "F16": F16, "BF16": BF16, "I8": I8}
_NP = {"F32": np.float32, "F16": np.uint16, "BF16": np.uint16, "I8": np.int8}


def read_safetensors(path: str) -> dict:
    """name -> (dtype string, shape, numpy view, scale) over a memory map."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    hlen = int(raw[:8].view(np.uint64)[0])
    header = json.loads(bytes(raw[8:8 + hlen]).decode("utf-8"))
    base = 8 + hlen
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        b, e = meta["data_offsets"]
        arr = raw[base + b: base + e].view(_NP[meta["dtype"]]).reshape(meta["shape"])
        out[name] = (meta["dtype"], meta["shape"], arr, float(meta.get("scale", 1.0)))
    return out


def _config_from(cfg: dict, attn_scale: float, rope_cpu_literal: bool) -> OrcConfig:
    c = OrcConfig()
    c.vocab = cfg["vocab_size"]
    c.hidden = cfg["hidden_size"]
    c.inter = cfg["intermediate_size"]
    c.layers = cfg["num_hidden_layers"]
    c.heads = cfg["num_attention_heads"]
    c.kv_heads = cfg.get("num_key_value_heads", c.heads)
    c.max_pos = cfg["max_position_embeddings"]
    c.eps = cfg["rms_norm_eps"]
    c.theta = cfg.get("rope_theta", 10000.0)
    c.attn_scale = attn_scale
    c.rope_cpu_literal = int(rope_cpu_literal)
    return c


def _eos_of(cfg: dict) -> int:
    """The stop id: config.json's eos_token_id (the first when it is a list), -1 when absent."""
    e = cfg.get("eos_token_id")
    if isinstance(e, list):
        e = e[0] if e else None
    return int(e) if isinstance(e, int) and e >= 0 else -1


class Model:
    """A model directory (config.json + model.safetensors) loaded into the oracle, or
    (Model.synth) a seeded random-init model built in memory."""

    @classmethod
    def synth(cls, seed: int = 0, std: float = 0.02, int8: bool = False, tied: bool = True,
              noise_seed: int = 0, noise_std: float = 0.0, eos: int = -1, **shape) -> "Model":
        """The model the engine's synth_model writes for the same arguments (same draw order,
        same bytes), without touching the product's libraries or the file system."""
        dims = dict(SMOLLM_135M)
        dims.update(shape)
        cfg = {"vocab_size": dims["vocab"], "hidden_size": dims["hidden"], "intermediate_size": dims["inter"],
               "num_hidden_layers": dims["layers"], "num_attention_heads": dims["heads"],
               "num_key_value_heads": dims["kv_heads"], "max_position_embeddings": dims["max_pos"],
               "rms_norm_eps": dims["eps"], "rope_theta": dims["theta"], "tie_word_embeddings": bool(tied)}
        if eos >= 0:
            cfg["eos_token_id"] = int(eos)
        self = cls.__new__(cls)
        self.cfg = cfg
        self.c = _config_from(cfg, 1.0, False)
        self.eos = _eos_of(cfg)
        sp = OrcSynth(seed, std, int(tied), int(int8), noise_seed, noise_std)
        self.h = lib().orc_model_create_synth(C.byref(self.c), C.byref(sp))
        if not self.h:
            raise ValueError("oracle rejected the synthetic model")
        return self

    def __init__(self, model_dir: str, attn_scale: float = 1.0, rope_cpu_literal: bool = False):
        cfg = json.load(open(os.path.join(model_dir, "config.json")))
        self.cfg = cfg
        c = _config_from(cfg, attn_scale, rope_cpu_literal)
        self.c = c
        self.eos = _eos_of(cfg)
        self.h = lib().orc_model_create(C.byref(c))
        if not self.h:
            raise ValueError("oracle rejected the model configuration")
        tensors = read_safetensors(os.path.join(model_dir, "model.safetensors"))

        def put(role, layer, name):
            dt, _shape, arr, scale = tensors[name]
            a = np.ascontiguousarray(arr)
            rc = lib().orc_model_set_tensor(self.h, role, layer, _DT[dt], _p(a), a.size, scale)
            if rc != 0:
                raise ValueError(f"oracle rejected tensor {name}")

        put(EMBED, 0, "model.embed_tokens.weight")
        put(FINAL_NORM, 0, "model.norm.weight")
        if not cfg.get("tie_word_embeddings", True) and "lm_head.weight" in tensors:
            put(LM_HEAD, 0, "lm_head.weight")
        roles = [(IN_NORM, "input_layernorm"), (POST_NORM, "post_attention_layernorm"),
                 (WQ, "self_attn.q_proj"), (WK, "self_attn.k_proj"), (WV, "self_attn.v_proj"),
                 (WO, "self_attn.o_proj"), (GATE, "mlp.gate_proj"), (UP, "mlp.up_proj"),
                 (DOWN, "mlp.down_proj")]
        for layer in range(c.layers):
            for role, nm in roles:
                put(role, layer, f"model.layers.{layer}.{nm}.weight")
        if lib().orc_model_ready(self.h) != 0:
            raise ValueError("oracle model incomplete")

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None

    def generate(self, prompt, budget: int, max_pos: int | None = None):
        p = np.ascontiguousarray(prompt, np.uint32)
        mp = max_pos or self.c.max_pos
        out = np.zeros(budget, np.uint32)
        margins = np.zeros(budget, np.float32)
        n = lib().orc_generate(self.h, _p(p), p.size, budget, mp, _p(out), _p(margins))
        if n < 0:
            raise ValueError("oracle generate failed")
        return out[:n], margins[:n]

    def generate_stop(self, prompt, budget: int, max_pos: int | None = None, eos: int | None = None):
        """Generate with the reference's stop rules (stop id = config.json's eos_token_id
        unless `eos` is given; -1: none). Returns (tokens, margins, hit_stop)."""
        p = np.ascontiguousarray(prompt, np.uint32)
        mp = max_pos or self.c.max_pos
        out = np.zeros(budget, np.uint32)
        margins = np.zeros(budget, np.float32)
        hit = C.c_int(0)
        n = lib().orc_generate_stop(self.h, _p(p), p.size, budget, mp, self.eos if eos is None else eos,
                                    _p(out), _p(margins), C.byref(hit))
        if n < 0:
            raise ValueError("oracle generate failed")
        return out[:n], margins[:n], bool(hit.value)

    def generate_batch(self, prompts, budget: int, threads: int, max_pos: int | None = None,
                       eos: int | None = None):
        """Independent sequences on `threads` host threads (one sequence per thread at a
        time, serial arithmetic inside). Returns (tokens [n][budget] (unused entries 0),
        counts [n], margins [n][budget], runner-up tokens [n][budget])."""
        ps = [np.asarray(p, np.uint32) for p in prompts]
        flat = np.ascontiguousarray(np.concatenate(ps), np.uint32)
        lens = np.array([p.size for p in ps], np.uint32)
        n = len(ps)
        out = np.zeros((n, budget), np.uint32)
        counts = np.zeros(n, np.uint32)
        margins = np.zeros((n, budget), np.float32)
        second = np.zeros((n, budget), np.uint32)
        rc = lib().orc_generate_batch(self.h, _p(flat), _p(lens), n, budget, max_pos or self.c.max_pos,
                                      self.eos if eos is None else eos, int(threads), _p(out), _p(counts),
                                      _p(margins), _p(second))
        if rc != 0:
            raise ValueError("oracle generate_batch failed")
        return out, counts, margins, second

    def state(self, max_pos: int | None = None) -> "State":
        return State(self, max_pos or self.c.max_pos)


class State:
    def __init__(self, model: Model, max_pos: int):
        self.m = model
        self.h = lib().orc_state_create(model.h, max_pos)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_state_free(self.h)
            self.h = None

    def __len__(self):
        return int(lib().orc_state_len(self.h))

    def truncate(self, n: int):
        lib().orc_state_truncate(self.h, n)

    def set_window(self, page_size: int, ring: int):
        """Sliding window of `ring` pages (orc_state_set_window); 0 turns it off."""
        lib().orc_state_set_window(self.h, page_size, ring)

    def load_kv(self, kv: np.ndarray, length: int):
        kv = np.ascontiguousarray(kv, np.uint16)
        if lib().orc_state_load_kv(self.h, _p(kv), length) != 0:
            raise ValueError("load_kv failed")

    def forward(self, token: int, logits=True, trace=False):
        c = self.m.c
        lg = np.empty(c.vocab, np.float32) if logits else None
        tr = np.empty((c.layers, c.hidden), np.float32) if trace else None
        if lib().orc_forward(self.m.h, self.h, int(token), _p(lg), _p(tr)) != 0:
            raise ValueError("oracle forward failed")
        return lg, tr
