"""Decode benchmark: BASELINE config 0 (SmolLM-135M shape greedy decode) on B200.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

A step is one greedy decode step of B independent sequences (one token each) at the
config-0 contexts: a 32-token prompt (seed 1 + sequence index) is prefilled once, then
decode positions run 32..159 (the 128 decode steps of config 0) and wrap back to 32, so
any K keeps the config-0 context lengths. Weights are random-init N(0, 0.02) fp16 from
seed 0 (synthetic: no checkpoint is downloaded).

  value     tokens/s over all ranks, inputs resident in HBM, steps replayed from a CUDA
            graph with no host round trip, device-timed (CUDA events on the engine's
            stream, max over ranks).
  e2e       the same metric through the engine's C ABI (opure_engine_decode_step): each
            step copies the tokens and positions in from pinned host memory and reads the
            8-byte argmax results back, as the reference's DecodeStep does.
  roofline  algorithmic HBM bytes of one decode step (every weight once + the KV rows
            read and written) / step time, against MEASURED_PEAKS.json.
  cpu_baseline / --impl reference: the CPU oracle (a port of the reference's scalar
            C++ forward) on the host cores, same workload, bounded sample.

Under torchrun (N > 1) every rank drives its own GPU with its own B sequences (sequence
sharding, no collective on the data path); ranks meet only at the timing barriers.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "opure-voxelengine_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "decode tok/s (bs1, bs64) at SmolLM-135M shape; GEMV+attn HBM GB/s as % of peak"
PROMPT_LEN, DECODE_STEPS = 32, 128
FALLBACK_PEAK = 6650.0  # GB/s, used only when MEASURED_PEAKS.json is absent
# DRAM bytes (read + write) of one decode step, from ncu captures of this build (cold caches:
# ncu serialises launches). Batch 1, the persistent step kernel, mean of two launches:
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#     --clock-control none -k regex:persistent_step -s 33 -c 2
#     python bench.py --quick --no-cpu --steps 2 --warmup 3 --bs64-steps 0 --int8 0
# -> 269.92 MB read + 1.0-3.5 MB written per launch.
# Batch 64 (chained operands: six kernels per layer), layers 0 and 1 of one step, with layer
# 1's kernels taken for every layer, plus layer 0's pack kernel and the lm_head GEMM:
#   ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum
#     --clock-control none -k "regex:gemm_tc_kernel|pack_kernel|attn_tma_kernel|rope_kv_kernel"
#     -s 6552 -c 13 python bench.py --quick --no-cpu --batch 64 --steps 2 --warmup 3
#     --bs64-steps 0 --int8 0
# -> 11.03 MB per layer, 331.0 MB for 30 layers + 0.16 MB pack + 56.8 MB lm_head (the lm_head
# GEMM's figure, its 56.6 MB of weights, from the capture of the build before the chained
# operands) = 388.0 MB per step. ncu flushes the caches before every captured launch, so at
# batch 64 each kernel's activation inputs count as DRAM reads too (an upper bound; at batch
# 1 the step is one launch). Both captures ran at a mean context of about 37 positions;
# step_traffic() moves the K/V share to the timed steps' mean context.
NCU_STEP_TRAFFIC = {1: 272.2e6, 64: 388.0e6}
NCU_CAPTURE_CTX = 37.0


def step_traffic(info, batch: int, positions):
    """The captured DRAM bytes of one step, with the K/V reads moved from the capture's mean
    context to the mean context of `positions`; None without a capture for this batch."""
    t = NCU_STEP_TRAFFIC.get(batch)
    if t is None:
        return None
    mean_ctx = float(np.mean([p + 1 for p in positions]))
    return t + batch * info.kv_bytes_per_token * (mean_ctx - NCU_CAPTURE_CTX)


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_PEAK, "fallback"


def model_dir():
    from voxelengine import engine as ve
    d = os.path.join(os.environ.get("OPURE_BENCH_DIR", "/tmp/opure_bench"), "smollm135m_seed0")
    return ve.synth_model(d, seed=0)


def step_bytes(info, batch: int, positions) -> float:
    """Algorithmic HBM bytes of one decode step: every weight byte once, plus per sequence
    the K/V rows attended (23,040 B per position at the SmolLM shape), the new K/V row and
    the embedding row gathered."""
    kv_row = info.kv_bytes_per_token
    mean_ctx = float(np.mean([p + 1 for p in positions]))
    return info.stream_bytes + batch * (kv_row * mean_ctx + kv_row + info.hidden * 2)


def smi_index(local: int) -> int:
    """nvidia-smi's index of this rank's GPU (CUDA_VISIBLE_DEVICES maps CUDA ordinals)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if vis:
        parts = [v.strip() for v in vis.split(",")]
        if local < len(parts) and parts[local].isdigit():
            return int(parts[local])
    return local


class ClockSampler:
    """nvidia-smi samples of ONE GPU (clocks, power, throttle reasons), each stamped on
    arrival; stop() keeps only those inside the window marked by mark_begin/mark_end."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.rows, self.proc, self.gpu = [], None, gpu_index
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def mark_begin(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [c.strip() for c in line.split(",")]))

    def stop(self, window: str):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        self.t.join(timeout=2)
        rows = [r for t, r in self.rows if len(r) >= 9 and r[0] == str(self.gpu)
                and self.t0 is not None and self.t0 <= t <= (self.t1 or t)]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "gpu_index": self.gpu, "window": window, "reasons": reasons}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """This rank's contiguous share (first, count) of `total` independent sequences; the
    first total % world ranks take one more. No collective: sequences never interact."""
    base, rem = divmod(total, world)
    return rank * base + min(rank, rem), base + (1 if rank < rem else 0)


def allreduce_sum(world, x: float) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_objects(world, obj):
    """Every rank's `obj`, in rank order (a list of one at world 1)."""
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def allreduce_max(world, x: float) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---- CPU side (the oracle: a port of the reference's scalar C++ forward) ----------------
# Everything here uses the oracle alone (test infrastructure): its own seeded model and
# prompts, byte-identical to the engine's, so the reference arm loads no product library.
def cpu_model():
    import oracle
    oracle.set_threads(os.cpu_count() or 1)
    return oracle.Model.synth(seed=0)


def cpu_decode(m, steps: int, warmup: int, threads: int):
    """Config 0 at batch 1 on the CPU oracle: the 32-token prompt (seed 1) prefilled, then
    `steps` timed greedy tokens after `warmup` untimed ones at positions 32..159 (cyclic, as
    the GPU arm), with the GEMV rows spread over `threads` host threads (rows are
    independent; the results equal the one-thread ones). Returns (tok/s, tokens, seconds)."""
    import oracle
    oracle.set_threads(threads)
    st = m.state(PROMPT_LEN + DECODE_STEPS + 1)
    prompt = oracle.prompt(1, 49152, PROMPT_LEN)
    logits = None
    for i, t in enumerate(prompt):
        logits, _ = st.forward(int(t), logits=(i == PROMPT_LEN - 1))
    tok = int(np.argmax(logits))
    done, t0 = 0, None
    for s in range(warmup + steps):
        if s == warmup:
            t0 = time.perf_counter()
        if len(st) >= PROMPT_LEN + DECODE_STEPS:
            st.truncate(PROMPT_LEN)
        logits, _ = st.forward(tok)
        tok = int(np.argmax(logits))
        done += s >= warmup
    dt = time.perf_counter() - t0
    return done / dt, done, dt


def cpu_decode_sequences(m, n_seq: int, steps: int):
    """The reference's CPU path as a server would run it on this host: `n_seq` independent
    config-0 sequences (prompt seeds 1..n_seq), one per host thread, each computing
    serially. All threads prefill, meet at a barrier, then time `steps` greedy tokens each.
    Returns (aggregate tok/s, seconds)."""
    import oracle
    oracle.set_threads(1)
    bar = threading.Barrier(n_seq + 1)
    err = []

    def worker(b):
        try:
            oracle.thread_serial(True)
            st = m.state(PROMPT_LEN + steps + 2)
            logits = None
            for i, t in enumerate(oracle.prompt(1 + b, 49152, PROMPT_LEN)):
                logits, _ = st.forward(int(t), logits=(i == PROMPT_LEN - 1))
            tok = int(np.argmax(logits))
            bar.wait()
            for _ in range(steps):
                logits, _ = st.forward(tok)
                tok = int(np.argmax(logits))
            bar.wait()
        except Exception as e:  # keep the barrier from hanging the others
            err.append(e)
            bar.abort()

    ts = [threading.Thread(target=worker, args=(b,)) for b in range(n_seq)]
    for t in ts:
        t.start()
    bar.wait()
    t0 = time.perf_counter()
    bar.wait()
    dt = time.perf_counter() - t0
    for t in ts:
        t.join()
    if err:
        raise err[0]
    return n_seq * steps / dt, dt


def cpu_baseline_record(m, steps: int, warmup: int):
    """The CPU baseline of the config-0 line: batch 1 with the GEMV rows over every host
    thread (the line's value), the same on one thread, and independent sequences, one per
    host thread (the reference CPU path's throughput on this host)."""
    threads = os.cpu_count() or 1
    tps, done, dt = cpu_decode(m, steps, warmup, threads)
    one, done1, _ = cpu_decode(m, max(4, min(steps, 8)), 1, 1)
    seq_tps, _ = cpu_decode_sequences(m, threads, 4)
    return {"value": tps, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{done} config-0 decode tokens of one sequence (positions 32..159 cyclic) after a "
                      f"{PROMPT_LEN}-token prefill and {warmup} untimed tokens, GEMV rows over {threads} threads",
            "one_thread": {"value": one, "unit": "tok/s", "cores": 1, "sample": f"{done1} tokens, batch 1"},
            "independent_sequences": {"value": seq_tps, "unit": "tok/s", "cores": threads, "batch": threads,
                                      "sample": f"{threads} config-0 sequences (prompt seeds 1..{threads}), one per "
                                                "thread, 4 timed tokens each after their prefills"}}


def run_reference(args, world, rank):
    """The reference arm: the CPU oracle (a port of the reference's scalar C++ forward; its
    own CPU reference includes <windows.h> and cannot be built here) on this host's cores,
    same metric, unit and config-0 workload as the GPU arm, batch 1."""
    if rank != 0:
        return
    m = cpu_model()
    rec = cpu_baseline_record(m, args.steps, args.warmup)
    tps = rec["value"]
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / tps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64 accumulate, f16 weights/KV",
        "data": "synthetic",
        "config": {"workload": "cfg0 greedy decode, SmolLM-135M shape, bs1, 32-token prompt, decode positions "
                               "32..159 cyclic", "global_batch": 1, "seq_len": PROMPT_LEN + DECODE_STEPS},
        "cpu_baseline": rec,
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- GPU side ---------------------------------------------------------------------------
def phase_stats(t: np.ndarray, n_layers: int) -> dict:
    """Per-phase timing of one persistent decode step from its per-CTA stamps (ns):
    work = a CTA's arrival at a barrier minus its release from the previous one; release =
    first release minus last arrival (the barrier's own latency). Medians over layers of
    the median / max over CTAs, in microseconds."""
    t = t.astype(np.int64)
    start = t[:, 3 * n_layers, 1]
    end = t[:, 3 * n_layers + 1, 0]
    t0 = start.min()
    arrive = t[:, :3 * n_layers, 0] - t0
    leave = t[:, :3 * n_layers, 1] - t0
    prev = start - t0
    rows = []
    for k in range(3 * n_layers):
        work = arrive[:, k] - prev
        rows.append((np.median(work), work.max(), leave[:, k].min() - arrive[:, k].max()))
        prev = leave[:, k]
    rows = np.array(rows, np.float64) / 1e3
    out = {"kernel_us": float((end.max() - t0) / 1e3), "lm_head_us": float((end.max() - t0) / 1e3 - leave[:, -1].min() / 1e3)}
    for ph, name in enumerate(("qkv_rope_kv", "attention_oproj", "mlp")):
        r = rows[ph::3]
        out[name] = {"work_median_us": float(np.median(r[:, 0])), "work_max_us": float(np.median(r[:, 1])),
                     "barrier_release_us": float(np.median(r[:, 2]))}
    return out


def device_steps(eng, B: int, steps: int, warmup: int, world: int, sample_clocks: bool, local: int = 0):
    """Times `steps` device-resident decode steps of sequences 0..B-1 (graph replays, no host
    round trip; positions rewound to 32 every 128 steps, so every step has config-0 context
    lengths) after `warmup` untimed ones. Returns (device ms, max over ranks; clock record).

    The clock record holds the nvidia-smi samples of this GPU taken from the start of the
    timed steps to the end of an untimed continuation of the same steps lasting at least
    0.5 s: a short timed region (tens of steps of ~0.5 ms) ends before the next sample."""
    import ctypes as C

    from voxelengine import cuda as cu
    from voxelengine import engine as ve
    L = cu.lib()
    ctx = eng.ctx
    eng_lib = ve.lib()
    pos_rewind = np.full(B, PROMPT_LEN, np.int32)

    def reset_positions():
        # pos := 32 for every sequence; tokens 32.. are already in the history from the
        # generate before, so the replayed steps redo the same config-0 work.
        cu.check(eng_lib.opure_engine_set_positions(eng.h, pos_rewind.ctypes.data_as(C.c_void_p), B),
                 "set_positions")

    def run(n_steps):
        left = n_steps
        while left:
            chunk = min(left, run.remaining)
            cu.check(eng_lib.opure_engine_run_steps(eng.h, B, chunk), "run_steps")
            run.remaining -= chunk
            left -= chunk
            if run.remaining == 0:
                reset_positions()
                run.remaining = DECODE_STEPS
    run.remaining = DECODE_STEPS
    reset_positions()

    ev0, ev1 = _events(ctx)
    run(warmup)
    cu.check(L.opure_sync(ctx, 600000), "sync")
    sampler = ClockSampler(smi_index(local)) if sample_clocks else None
    barrier(world)
    if sampler:
        sampler.start()
        time.sleep(0.3)  # nvidia-smi's first sample
        sampler.mark_begin()
    cu.check(L.opure_event_record(ctx, ev0), "event")
    run(steps)
    cu.check(L.opure_event_record(ctx, ev1), "event")
    if sampler:
        # Keep the GPU on the same work, untimed, until the sampler has seen it.
        t_soak = time.monotonic()
        while time.monotonic() - t_soak < 0.5:
            run(64)
            cu.check(L.opure_sync(ctx, 600000), "sync")
        sampler.mark_end()
    cu.check(L.opure_sync(ctx, 600000), "sync")
    ms = C.c_float()
    cu.check(L.opure_event_elapsed_ms(ev0, ev1, C.byref(ms)), "elapsed")
    clocks = sampler.stop("timed steps + >= 0.5 s of the same steps right after") if sampler else None
    barrier(world)
    L.opure_event_free(ev0)
    L.opure_event_free(ev1)
    return allreduce_max(world, float(ms.value)), clocks


def measure_bs64(args, world, rank, local, mp):
    """The metric's second batch size: 64 independent config-0 sequences per GPU (prompt
    seeds 1..64), device-resident steps, same accounting as the bs1 line."""
    from voxelengine import engine as ve
    B = 64
    eng = ve.Engine(mp, device=local, max_batch=B, max_len=PROMPT_LEN + DECODE_STEPS + 8, page_size=64,
                    page_seed=3)
    info = eng.info
    eng.generate([ve.prompt(1 + rank * B + b, 49152, PROMPT_LEN) for b in range(B)], DECODE_STEPS)
    dev_ms, _ = device_steps(eng, B, args.bs64_steps, 8, world, False)
    eng.close()
    positions = [PROMPT_LEN + (i % DECODE_STEPS) for i in range(DECODE_STEPS)]
    sbytes = step_bytes(info, B, positions)
    step_ms = dev_ms / args.bs64_steps
    achieved = sbytes / (step_ms * 1e-3) / 1e9
    peak, _ = peaks()
    return {"value": world * B * args.bs64_steps / (dev_ms * 1e-3), "unit": "tok/s", "steps": args.bs64_steps,
            "warmup": 8, "ms_per_step": step_ms, "global_batch": world * B,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": step_traffic(info, B, positions),
                         "bytes_per_step": sbytes},
            "gpu_launches": launches_per_step(info, B) * args.bs64_steps}


def measure_int8(args, world, rank, local):
    """Config 0 at batch 1 with GEMV_Quant weights: the same model quantised per tensor to
    int8 (absmax / 127; embedding and lm_head stay fp16), on the persistent step kernel.
    Device-resident steps, same accounting as the bs1 line (algorithmic bytes from the
    int8 weight stream)."""
    from voxelengine import engine as ve
    root = os.environ.get("OPURE_BENCH_DIR", "/tmp/opure_bench")
    mp = ve.synth_model(os.path.join(root, "smollm135m_seed0_int8"), seed=0, int8=True)
    eng = ve.Engine(mp, device=local, max_batch=1, max_len=PROMPT_LEN + DECODE_STEPS + 8, page_size=64, page_seed=3)
    info = eng.info
    eng.generate([ve.prompt(1 + rank, 49152, PROMPT_LEN)], DECODE_STEPS)
    steps = args.steps
    dev_ms, _ = device_steps(eng, 1, steps, args.warmup, world, False, local)
    eng.close()
    positions = [PROMPT_LEN + (i % DECODE_STEPS) for i in range(DECODE_STEPS)]
    sbytes = step_bytes(info, 1, positions)
    step_ms = dev_ms / steps
    achieved = sbytes / (step_ms * 1e-3) / 1e9
    peak, _ = peaks()
    return {"value": world * steps / (dev_ms * 1e-3), "unit": "tok/s", "steps": steps, "ms_per_step": step_ms,
            "weights": "int8 per-tensor (q/k/v/o/gate/up/down), fp16 embedding and lm_head",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "bytes_per_step": sbytes}}


def run_ours(args, world, rank, local):
    import ctypes as C

    from voxelengine import cuda as cu
    from voxelengine import engine as ve

    mp = model_dir() if rank == 0 else None
    barrier(world)
    if mp is None:
        mp = model_dir()
    B = args.batch
    max_len = PROMPT_LEN + DECODE_STEPS + 8
    path = {"auto": ve.PATH_AUTO, "layers": ve.PATH_FUSED_LAYERS, "unfused": ve.PATH_UNFUSED}[args.path]
    eng = ve.Engine(mp, device=local, max_batch=B, max_len=max_len, page_size=64, page_seed=3, path=path,
                    phase_trace=args.phase_trace)
    info = eng.info
    L = cu.lib()
    ctx = eng.ctx
    prompts = [ve.prompt(1 + rank * B + b, 49152, PROMPT_LEN) for b in range(B)]

    # Parity gate on this rank's first sequence: the engine's 128 config-0 tokens.
    # (--quick, for profiler launch lists, generates one token: the launches before the
    # timed region are then (PROMPT_LEN + 1 + warmup) * launches_per_step.)
    # Quick runs generate only as far as their steps reach (each step needs its KV page
    # reserved by the generate before).
    gen, _ = eng.generate(prompts, min(DECODE_STEPS, args.steps + args.warmup + 2) if args.quick else DECODE_STEPS)
    parity = {"tokens_checked": 0}

    dev_ms, clocks = device_steps(eng, B, args.steps, args.warmup, world, not args.quick, local)
    clocks_per_rank = gather_objects(world, clocks)
    cu.check(L.opure_last_error(ctx), "device status")
    phases = None
    if args.phase_trace:
        tr = eng.phase_trace()
        phases = phase_stats(tr, info.layers) if tr.size else {"unavailable": "step is not the persistent kernel"}

    positions = [PROMPT_LEN + (i % DECODE_STEPS) for i in range(DECODE_STEPS)]
    sbytes = step_bytes(info, B, positions)
    step_ms = dev_ms / args.steps
    achieved = sbytes / (step_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    value = world * B * args.steps / (dev_ms * 1e-3)

    # e2e: host-driven steps through the C ABI with pinned host buffers.
    e2e_steps = 0 if args.quick else min(args.steps, 512)
    toks = gen[:, 0].copy()
    barrier(world)
    t0 = time.perf_counter()
    pos = np.full(B, PROMPT_LEN, np.int32)
    for i in range(e2e_steps):
        toks = eng.decode_step(toks, pos)
        pos = pos + 1
        if pos[0] >= PROMPT_LEN + DECODE_STEPS:
            pos[:] = PROMPT_LEN
    wall = max(time.perf_counter() - t0, 1e-9)
    wall = allreduce_max(world, wall)
    e2e = {"value": world * B * e2e_steps / wall, "unit": "tok/s", "h2d_bytes_per_step": 8 * B,
           "d2h_bytes_per_step": 8 * B, "steps": e2e_steps,
           "path": "opure_engine_decode_step (H2D tokens+positions, one step, D2H argmax keys)"}

    # Parity: the first sequence's config-0 tokens against the CPU oracle (rank 0 only).
    cpu = None
    if rank == 0 and not args.no_cpu and not args.quick:
        import oracle
        oracle.set_threads(os.cpu_count() or 1)
        m = oracle.Model(mp)
        want, margins = m.generate(prompts[0], DECODE_STEPS)
        parity = {"tokens_checked": int(want.size), "tokens_equal": bool(np.array_equal(want, gen[0])),
                  "min_top2_margin": float(margins.min())}
        cpu = cpu_baseline_record(m, args.cpu_steps, 4)

    line_launches = launches_per_step(info, B, args.path)
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 weights/KV, f32 accumulate", "data": "synthetic",
        "config": {"workload": f"cfg0 greedy decode, SmolLM-135M shape, bs{B} per GPU, 32-token "
                               "prompt, decode positions 32..159 cyclic",
                   "global_batch": world * B, "seq_len": PROMPT_LEN + DECODE_STEPS,
                   "parallelism": f"sequence-sharded x{world}",
                   "l2": "inputs larger than L2: every step streams 269 MB of weights (L2 126 MB)"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": step_traffic(info, B, positions),
                     "kernel": ("the persistent decode-step kernel (one launch per step)"
                                if line_launches == 3 else "whole decode step (GEMV dominant)"),
                     "peak_kind": peak_kind,
                     "bytes_per_step": sbytes},
        "e2e": e2e,
        "gpu_launches": line_launches * args.steps,
        "clocks": clocks,
        **({"clocks_per_rank": clocks_per_rank} if world > 1 else {}),
        "parity": parity,
        "launches_before_timed": (PROMPT_LEN + (min(DECODE_STEPS, args.steps + args.warmup + 2) if args.quick
                                                else DECODE_STEPS) + args.warmup)
        * line_launches,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if B == 1 and not args.quick:
        # Time to first token: the 32-token prompt one token per step (the reference's way)
        # against one chunked tensor-core step; best of 3 after a graph-capturing warm-up.
        pre = {}
        for name, chunk in (("per_token_steps", 0), ("chunked", PROMPT_LEN)):
            with ve.Engine(mp, device=local, max_len=max_len, prefill_chunk=chunk) as e2:
                e2.generate([prompts[0]], 1)
                pre[name + "_ms"] = min(e2.generate([prompts[0]], 1)[1].prefill_ms for _ in range(3))
        line["prefill"] = {"prompt_tokens": PROMPT_LEN, **pre}
    if phases:
        line["phases"] = phases
    eng.close()
    if B == 1 and args.bs64_steps > 0 and not args.quick:
        line["bs64"] = measure_bs64(args, world, rank, local, mp)
    if B == 1 and args.int8 and not args.quick:
        line["int8"] = measure_int8(args, world, rank, local)
    if rank == 0:
        print(json.dumps(line), flush=True)


def launches_per_step(info, B: int, path: str = "auto") -> int:
    """Kernel launches of one decode step: step_begin + step_end, then
    fused path (fp16, B in 1/2/4/8): one persistent kernel (path auto, head_dim 64, <= 48
    layers) or 3 per layer + lm_head (path layers);
    per-op path: per layer the q;k;v, o, gate;up and down GEMVs (+ RoPE/KV append and
    attention), each GEMV one launch per 9-vector pass on the CUDA cores (int8 q;k;v as 3
    GEMVs) or pack + tcgen05 GEMM per 256-vector pass from 16 vectors up, + the lm_head GEMV;
    with chained operands (fp16, 16..256 vectors, head_dim 64 or 128) one tcgen05 GEMM per
    projection and a single pack kernel (layer 0's q;k;v input)."""
    from voxelengine import cuda as cu
    if info.w_dtype == cu.W_F16 and B in (1, 2, 4, 8) and path != "unfused":
        if path == "auto" and info.head_dim == 64 and info.layers <= 48:
            return 3
        return 2 + 3 * info.layers + 1
    if info.w_dtype == cu.W_F16 and 16 <= B <= 256 and info.head_dim in (64, 128):
        return 2 + 1 + info.layers * 6 + 1
    if info.w_dtype == cu.W_F16 and B >= 16:
        gemv = 2 * -(-B // 256)
    else:
        gemv = -(-B // 9)
    qkv = gemv if info.w_dtype == cu.W_F16 else 3 * gemv
    return 2 + info.layers * (qkv + 3 * gemv + 2) + gemv


def _events(ctx):
    import ctypes as C

    from voxelengine import cuda as cu
    L = cu.lib()
    a, b = C.c_void_p(), C.c_void_p()
    cu.check(L.opure_event_create(ctx, C.byref(a)), "event")
    cu.check(L.opure_event_create(ctx, C.byref(b)), "event")
    return a, b


# ---- kernel workloads: BASELINE configs 1 (attention sweep) and 2 (GEMV shapes) ----------
def _time_events(ctx, fn, iters, warm=3):
    """Average device ms of fn() over `iters` launches (CUDA events on the ctx stream)."""
    import ctypes as C

    from voxelengine import cuda as cu
    L = cu.lib()
    for _ in range(warm):
        fn(0)
    cu.check(L.opure_sync(ctx.h, 600000), "sync")
    a, b = _events(ctx.h)
    cu.check(L.opure_event_record(ctx.h, a), "event")
    for i in range(iters):
        fn(i)
    cu.check(L.opure_event_record(ctx.h, b), "event")
    ms = C.c_float()
    cu.check(L.opure_event_elapsed_ms(a, b, C.byref(ms)), "elapsed")
    L.opure_event_free(a)
    L.opure_event_free(b)
    return ms.value / iters


def run_attention_sweep(args):
    """Config 1: paged flash-decode, 9 q heads / 3 kv heads, hd 64, fp16 Q/K/V N(0, 1) from
    seed 2 (stream order: the queries [B][9][64], then the page pool in memory order
    [page][K|V][kv head][slot][dim]), page size 64, page table a seeded permutation (seed 3)
    of the physical pages: the inputs the config-1 parity tests check."""
    from voxelengine import cuda as cu
    from voxelengine import engine as ve
    peak, kind = peaks()
    nh, nkv, hd, P = 9, 3, 64, 64
    out = []
    with cu.Ctx(0) as ctx:
        for B in (1, 8, 64):
            for ctxlen in (512, 2048, 8192, 32768):
                if (args.attn_b and B != args.attn_b) or (args.attn_ctx and ctxlen != args.attn_ctx):
                    continue
                pages = B * (ctxlen // P)
                pool_elems = pages * 2 * nkv * P * hd
                draws = ve.normal_f16(2, 1.0, B * nh * hd + pool_elems)
                pool = ctx.to_device(draws[B * nh * hd:])
                perm = ve.permutation(3, pages).reshape(B, ctxlen // P)
                q = oracle_free_f16_to_f32(draws[: B * nh * hd])
                del draws
                dq, dpt = ctx.to_device(q), ctx.to_device(perm.astype(np.int32))
                dseq = ctx.to_device(np.arange(B, dtype=np.int32))
                dlen = ctx.to_device(np.full(B, ctxlen, np.int32))
                dout = ctx.buffer(B * nh * hd * 4)
                bytes_ = B * ctxlen * 2 * nkv * hd * 2 + B * nh * hd * 8 + B * (ctxlen // P) * 4
                for split in args.attn_splits:
                    sb = cu.attention_scratch_bytes(B, 1, nh, nkv, hd, ctxlen, split)
                    scratch = ctx.buffer(sb).fill(0)
                    a = cu.AttnArgs()
                    a.q, a.out, a.seq, a.seq_len = dq.ptr, dout.ptr, dseq.ptr, dlen.ptr
                    a.n, a.n_q, a.n_heads, a.scale, a.max_ctx = B, 1, nh, 1.0, ctxlen
                    a.split_tokens, a.scratch, a.scratch_bytes = split, scratch.ptr, sb
                    a.kv = cu.KvLayout(pool.ptr, dpt.ptr, pages, ctxlen // P, P, nkv, hd)
                    iters = max(5, min(200, int(2e9 / bytes_)))
                    ms = _time_events(ctx, lambda i: ctx.attention(a), iters)
                    gbs = bytes_ / (ms * 1e-3) / 1e9
                    pt = {"B": B, "ctx": ctxlen, "us": ms * 1e3, "bytes": bytes_, "GB/s": gbs, "frac": gbs / peak,
                          "l2": "pool > L2" if bytes_ > 126e6 else "pool fits L2 (upper bound)"}
                    if split:
                        pt["split_tokens"] = split
                    out.append(pt)
                    scratch.free()
                for b in (pool, dq, dpt, dseq, dlen, dout):
                    b.free()
    line = {"metric": "paged flash-decode attention HBM GB/s (config 1)", "unit": "GB/s",
            "peak": peak, "peak_kind": kind, "points": out}
    print(json.dumps(line), flush=True)


def oracle_free_f16_to_f32(h):
    return np.asarray(h, np.uint16).view(np.float16).astype(np.float32)


def run_gemv_sweep(args):
    """Config 2: GEMV at the projection shapes, fp16 and int8 (GEMV_Quant) weights derived
    from N(0, 0.02) seed 4, x fp16 N(0,1), n = 1, 5, 9 vectors. Each timed launch reads a
    different weight copy from a rotating set of >= 256 MB so the bytes come from HBM."""
    from voxelengine import cuda as cu
    from voxelengine import engine as ve
    peak, kind = peaks()
    out = []
    with cu.Ctx(0) as ctx:
        for rows, cols in args.gemv_shapes:
            w16 = ve.normal_f16(4, 0.02, rows * cols)
            wf = oracle_free_f16_to_f32(w16)
            amax = float(np.abs(wf).max())
            sq = amax / 127.0
            q8 = np.clip(np.rint(wf / sq), -127, 127).astype(np.int8)
            for dtype, wh, eb, scale in ((cu.W_F16, w16, 2, 1.0), (cu.W_Q8, q8, 1, sq)):
                wbytes = rows * cols * eb
                copies = max(2, -(-256 * (1 << 20) // wbytes))
                pool = ctx.buffer(copies * wbytes)
                for c in range(copies):
                    pool.upload(wh, offset=c * wbytes)
                for n in args.gemv_n:
                    x = oracle_free_f16_to_f32(ve.normal_f16(4 + n, 1.0, n * cols))
                    dx, dy = ctx.to_device(x), ctx.buffer(n * rows * 4)
                    a = cu.GemvArgs()
                    a.w_dtype, a.scale_w, a.scale_x = dtype, scale, 1.0
                    a.rows, a.cols, a.nvec = rows, cols, n
                    a.x, a.x_stride, a.y, a.y_stride = dx.ptr, cols, dy.ptr, rows

                    def launch(i, a=a):
                        a.w = pool.ptr + (i % copies) * wbytes
                        ctx.gemv(a)
                    iters = max(copies, 50)
                    ms = _time_events(ctx, launch, iters)
                    bytes_ = wbytes + n * cols * 2 + n * rows * 4 + (4 if dtype == cu.W_Q8 else 0)
                    gbs = bytes_ / (ms * 1e-3) / 1e9
                    out.append({"shape": f"{rows}x{cols}", "dtype": "f16" if dtype == cu.W_F16 else "q8",
                                "n": n, "us": ms * 1e3, "bytes": bytes_, "GB/s": gbs, "frac": gbs / peak})
                    dx.free()
                    dy.free()
                pool.free()
    print(json.dumps({"metric": "weight-streaming GEMV HBM GB/s (config 2)", "unit": "GB/s", "peak": peak,
                      "peak_kind": kind, "points": out}), flush=True)


def run_cfg4(args, world, rank, local):
    """Config 4: 1.7B-shape batched decode (24 layers, hidden 2048, 32/32 heads, ff 8192,
    vocab 49152, fp16 weights N(0, 0.02) seed 5, tied embeddings). 512 independent sequences
    (--seqs) with 4096-token contexts each decode 64 tokens, sharded by sequence across the
    ranks (no collective on the data path) and run in waves of at most --wave sequences per
    GPU. Contexts are seeded synthetic KV values written on the device (opure_kv_synth,
    seed 5 + wave index) instead of a 4096-step prefill; each sequence's first input token
    is seeded. Device time of the 64 steps of every wave, summed, max over ranks."""
    import ctypes as C

    from voxelengine import cuda as cu
    from voxelengine import engine as ve
    root = os.environ.get("OPURE_BENCH_DIR", "/tmp/opure_bench")
    path = os.path.join(root, "llama1p7b_seed5")
    if rank == 0:
        ve.synth_model(path, seed=5, **ve.LLAMA_1_7B)
    barrier(world)
    mp = ve.synth_model(path, seed=5, **ve.LLAMA_1_7B)
    ctx_len, steps = 4096, 64
    first_seq, count = shard(args.seqs, world, rank)
    per_rank = -(-args.seqs // world)           # the largest share: sizes every rank's engine
    wave = min(args.wave, per_rank)
    eng = ve.Engine(mp, device=local, max_batch=wave, max_len=ctx_len + steps + 8, page_size=64, page_seed=3)
    info = eng.info
    L = cu.lib()
    ev0, ev1 = _events(eng.ctx)
    dev_ms, tokens, waves = 0.0, 0, 0
    warm = 3  # graph capture + 2 replays; positions are rewound before the timed steps
    for w0 in range(0, count, wave):
        n = min(wave, count - w0)
        first = ve.prompt(1000 + first_seq + w0, info.vocab, n)
        eng.synth_context(n, ctx_len, ctx_len + steps + 4, 5 + waves, first)
        eng.run_steps(n, warm)                      # captures the step graph
        eng.sync()
        cu.check(ve.lib().opure_engine_set_positions(
            eng.h, np.full(n, ctx_len, np.int32).ctypes.data_as(C.c_void_p), n), "set_positions")
        cu.check(L.opure_event_record(eng.ctx, ev0), "event")
        eng.run_steps(n, steps)
        cu.check(L.opure_event_record(eng.ctx, ev1), "event")
        eng.sync()
        ms = C.c_float()
        cu.check(L.opure_event_elapsed_ms(ev0, ev1, C.byref(ms)), "elapsed")
        dev_ms += ms.value
        tokens += n * steps
        waves += 1
    barrier(world)
    dev_ms = allreduce_max(world, dev_ms)
    total_tokens = allreduce_sum(world, float(tokens))
    kv = info.kv_bytes_per_token
    step_bytes_ = info.stream_bytes + wave * (kv * (ctx_len + steps / 2 + 1) + kv)
    step_ms = dev_ms / (max(waves, 1) * steps)
    achieved = step_bytes_ / (step_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    line = {"metric": "config-4 batched decode tok/s (1.7B shape, 4096-token contexts, 64 steps)",
            "value": total_tokens / (dev_ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
            "dtype": "f16 weights/KV, f32 accumulate", "data": "synthetic",
            "config": {"workload": f"cfg4: {args.seqs} sequences x 4096-token synthetic context, 64 decode "
                                   f"steps, up to {per_rank} per GPU in waves of {wave}",
                       "global_batch": args.seqs, "seq_len": ctx_len + steps,
                       "parallelism": f"sequence-sharded x{world}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                         "bytes_per_step": step_bytes_, "kernel": "whole decode step (attention dominant)"}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()


def run_tp(args, world, rank, local):
    """Config 4, second variant: batch-1 greedy decode of the 1.7B shape with world-way tensor
    parallelism, one rank per GPU. Every step all-reduces the o_proj and down_proj partial
    sums of each layer (48 x 8 KB fp32 per token) and the vocabulary shards' argmax keys
    (8 B): as NCCL calls, or inside the producing kernels over NVLink peer memory
    (opure_gemv_allreduce / opure_peer_argmax) with --tp-allreduce peer (auto: the peer
    kernels when every GPU pair maps each other's memory). 32-token prompt (seed 1) prefilled, then device-resident steps
    (graph replays, NCCL inside the graph) at positions 32..159 (cyclic). Device time, max
    over ranks. `comm_us` is one 2048-float all-reduce timed on its own (100-call average)."""
    import ctypes as C

    import torch.distributed as dist

    from voxelengine import cuda as cu
    from voxelengine import engine as ve
    root = os.environ.get("OPURE_BENCH_DIR", "/tmp/opure_bench")
    path = os.path.join(root, "llama1p7b_seed5")
    if rank == 0:
        ve.synth_model(path, seed=5, **ve.LLAMA_1_7B)
    barrier(world)
    mp = ve.synth_model(path, seed=5, **ve.LLAMA_1_7B)
    obj = [cu.comm_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(obj, src=0)
    ctx = cu.Ctx(local)
    comm = cu.Comm(ctx, world, rank, obj[0], timeout_ms=120000)
    tp_mode = {"auto": ve.TP_AUTO, "nccl": ve.TP_NCCL, "peer": ve.TP_PEER}[args.tp_allreduce]
    eng = ve.Engine(mp, max_len=PROMPT_LEN + DECODE_STEPS + 8, comm=comm, tp_allreduce=tp_mode)
    info = eng.info
    L = cu.lib()
    eng.generate([ve.prompt(1, info.vocab, PROMPT_LEN)], DECODE_STEPS)
    pos_rewind = np.full(1, PROMPT_LEN, np.int32)

    def rewind():
        cu.check(ve.lib().opure_engine_set_positions(eng.h, pos_rewind.ctypes.data_as(C.c_void_p), 1),
                 "set_positions")

    def run(n_steps):
        left = n_steps
        while left:
            chunk = min(left, run.remaining)
            eng.run_steps(1, chunk)
            run.remaining -= chunk
            left -= chunk
            if run.remaining == 0:
                rewind()
                run.remaining = DECODE_STEPS
    run.remaining = DECODE_STEPS
    rewind()
    ev0, ev1 = _events(ctx.h)
    run(args.warmup)
    eng.sync()
    barrier(world)
    cu.check(L.opure_event_record(ctx.h, ev0), "event")
    run(args.steps)
    cu.check(L.opure_event_record(ctx.h, ev1), "event")
    eng.sync()
    ms = C.c_float()
    cu.check(L.opure_event_elapsed_ms(ev0, ev1, C.byref(ms)), "elapsed")
    barrier(world)
    dev_ms = allreduce_max(world, float(ms.value))
    # One o_proj-sized all-reduce on its own: 100 of them captured in a CUDA graph (as the
    # decode step runs them), replayed and timed on the device.
    buf = ctx.buffer(info.hidden * 4).fill(0)
    g = cu.Graph(ctx)
    with g:
        for _ in range(100):
            comm.allreduce_sum(buf, info.hidden)
    for _ in range(3):
        g.launch()
    ctx.sync()
    barrier(world)
    cu.check(L.opure_event_record(ctx.h, ev0), "event")
    g.launch()
    cu.check(L.opure_event_record(ctx.h, ev1), "event")
    ctx.sync()
    g.free()
    cu.check(L.opure_event_elapsed_ms(ev0, ev1, C.byref(ms)), "elapsed")
    comm_us = allreduce_max(world, float(ms.value) * 10.0)
    # The fused alternative: an o_proj-shaped peer GEMV all-reduce (this shard's 2048 x
    # 2048/world fp16 block, partial sums exchanged over NVLink and added to the residual),
    # 100 per graph. Every rank takes this path or none (the engine's flag is collective).
    peer_us = None
    if info.tp_peer:
        peer = cu.Peer(comm, info.hidden)
        cols = info.hidden // world
        w = ctx.buffer(info.hidden * cols * 2).fill(0)
        x = ctx.buffer(cols * 4).fill(0)
        a = cu.GemvArgs()
        a.w, a.w_dtype, a.rows, a.cols, a.nvec = w.ptr, cu.W_F16, info.hidden, cols, 1
        a.x, a.x_stride, a.y, a.y_stride = x.ptr, cols, buf.ptr, info.hidden
        a.epilogue, a.residual = cu.EPI_ADD, buf.ptr
        g = cu.Graph(ctx)
        with g:
            for _ in range(100):
                peer.gemv_allreduce(a)
        for _ in range(3):
            g.launch()
        ctx.sync()
        barrier(world)
        cu.check(L.opure_event_record(ctx.h, ev0), "event")
        g.launch()
        cu.check(L.opure_event_record(ctx.h, ev1), "event")
        ctx.sync()
        g.free()
        cu.check(L.opure_event_elapsed_ms(ev0, ev1, C.byref(ms)), "elapsed")
        peer_us = allreduce_max(world, float(ms.value) * 10.0)
        cu.check(ctx.last_error(), "peer all-reduce")
        peer.close()
    step_ms = dev_ms / args.steps
    positions = [PROMPT_LEN + (i % DECODE_STEPS) for i in range(DECODE_STEPS)]
    sbytes = step_bytes(info, 1, positions)   # this shard's weights and KV heads
    achieved = sbytes / (step_ms * 1e-3) / 1e9
    peak, peak_kind = peaks()
    line = {"metric": "config-4 TP decode tok/s (1.7B shape, batch 1, tensor-parallel)",
            "value": args.steps / (dev_ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "strong",
            "dtype": "f16 weights/KV, f32 accumulate", "data": "synthetic",
            "config": {"workload": f"cfg4 TP-{world}: 1.7B shape, bs1, 32-token prompt, positions 32..159 cyclic",
                       "global_batch": 1, "seq_len": PROMPT_LEN + DECODE_STEPS, "parallelism": f"tp{world}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                         "bytes_per_step": sbytes, "kernel": "whole decode step, per GPU (its shard)"},
            "comm": {"path": "nvlink peer kernels" if info.tp_peer else "nccl",
                     "allreduce_us_2048_f32": comm_us, "allreduces_per_step": 2 * info.layers + 1,
                     "nccl_est_ms_per_step": comm_us * (2 * info.layers + 1) / 1000.0,
                     "peer_gemv_allreduce_us": peer_us}}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()
    comm.close()
    ctx.close()


def run_spec(args):
    """Config 3: speculative decoding. Target = the config-0 model; draft = the same weights
    plus seeded N(0, 0.004) noise on every matrix element (noise seed 6); k = 4 and 8;
    batch 1 and 16 (prompt seeds 1..B); greedy and rejection sampling (temperature 1,
    uniform seed 3); 256 generated tokens per sequence. Reports the acceptance rate,
    generated tok/s (wall clock of the whole loop, host round trip per round included, and
    device time) and the verify pass's algorithmic HBM GB/s (weights once + the KV rows of
    the B(k+1) verify positions) over its device time (verify + accept)."""
    from voxelengine import engine as ve
    peak, kind = peaks()
    tgt = model_dir()
    root = os.environ.get("OPURE_BENCH_DIR", "/tmp/opure_bench")
    drf = ve.synth_model(os.path.join(root, "smollm135m_seed0_draft6"), seed=0, noise_seed=6, noise_std=0.004)
    budget = args.spec_budget
    points = []
    for k in args.spec_k:
        for B in args.spec_b:
            max_len = PROMPT_LEN + budget + k + 8
            t = ve.Engine(tgt, max_batch=B * (k + 1), max_len=max_len)
            d = ve.Engine(drf, max_batch=B, max_len=max_len, share=t)
            info = t.info
            prompts = [ve.prompt(1 + b, 49152, PROMPT_LEN) for b in range(B)]
            for mode, name in ((ve.SPEC_GREEDY, "greedy"), (ve.SPEC_REJECTION, "rejection")):
                t.spec_generate(d, prompts, 16, k=k, mode=mode, seed=3)  # captures the step graphs
                t0 = time.perf_counter()
                _, st, _ = t.spec_generate(d, prompts, budget, k=k, mode=mode, seed=3)
                wall = time.perf_counter() - t0
                kv = info.kv_bytes_per_token
                mean_p = PROMPT_LEN + budget / 2
                vbytes = info.stream_bytes + B * (k + 1) * (kv * (mean_p + k / 2 + 1) + kv)
                vgbs = vbytes * st.rounds / (st.verify_ms * 1e-3) / 1e9
                points.append({"k": k, "B": B, "mode": name, "acceptance": st.accepted / max(st.drafted, 1),
                               "rounds": st.rounds, "tok_s_wall": B * budget / wall,
                               "tok_s_device": B * budget / (st.total_ms * 1e-3),
                               "draft_ms": st.draft_ms, "verify_ms": st.verify_ms,
                               "verify_GB_s": vgbs, "verify_frac": vgbs / peak})
            d.close()
            t.close()
    line = {"metric": "speculative decode (config 3): generated tok/s and acceptance", "unit": "tok/s",
            "peak": peak, "peak_kind": kind, "budget": budget, "points": points}
    if not args.no_cpu:
        import oracle
        from oracle import spec
        oracle.set_threads(os.cpu_count() or 1)
        om_t, om_d = oracle.Model(tgt), oracle.Model(drf)
        t0 = time.perf_counter()
        spec.spec_generate(om_t, om_d, [ve.prompt(1, 49152, PROMPT_LEN)], 32, 4, rejection=False)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": 32 / dt, "unit": "tok/s", "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": "B=1, k=4, greedy: the first 32 generated tokens (prefill included) "
                                          "of the oracle's speculative loop"}
    print(json.dumps(line), flush=True)


def run_window(args):
    """Sliding-window KV cache (ring of pages): config-0 model, bs1, 1024 greedy tokens
    after the 32-token prompt, with a 256-token window (4 pages of 64 as a ring) and without
    one. Device time of the decode steps (the engine's Timing); with the window the KV held per
    sequence stays at 4 pages and each step attends to at most 256 positions."""
    from voxelengine import engine as ve
    mp = model_dir()
    budget, window = 1024, 256
    points = []
    for w in (0, window):
        with ve.Engine(mp, max_batch=1, max_len=PROMPT_LEN + budget + 8, page_size=64, kv_window=w) as eng:
            p = [ve.prompt(1, 49152, PROMPT_LEN)]
            eng.generate(p, 16)
            _, t = eng.generate(p, budget)
            kvb = eng.info.kv_bytes_per_token
        points.append({"kv_window": w, "tok_s_device": t.decode_steps / (t.decode_ms * 1e-3),
                       "decode_ms": t.decode_ms, "kv_bytes_per_sequence": kvb * (w or PROMPT_LEN + budget)})
    line = {"metric": "greedy decode tok/s over 1024 tokens with and without a sliding-window KV cache (bs1, config 0)",
            "unit": "tok/s", "points": points}
    print(json.dumps(line), flush=True)


def run_sample(args):
    """Sampling: the opure_sample_filtered and opure_logit_stats kernels
    on seeded N(0, 3) logits of the config-0 vocabulary (device time per call, CUDA events
    over 50 calls after 5 warm-up ones), and sampled generation through the engine at the
    reference chat defaults (temperature 0.8, top-k 50, top-p 0.95, Opure_Chat.cpp:69;
    repetition penalty 1.1) against greedy generation of the same config-0 model: 128
    tokens after the 32-token prompt, wall clock of the whole call (prefill included)."""
    import ctypes as C

    from voxelengine import cuda as cu
    from voxelengine import engine as ve
    V = 49152
    points = []
    ctx = cu.Ctx(0)
    L = cu.lib()
    rng = np.random.default_rng(5)
    for rows in (1, 64):
        lg = ctx.to_device((rng.standard_normal((rows, V)) * 3).astype(np.float32))
        u = ctx.to_device(rng.random(rows).astype(np.float32))
        out, st = ctx.buffer(rows * 4), ctx.buffer(rows * 16)
        for name, T, k, p in (("top-k 50 + top-p 0.95", 0.8, 50, 0.95), ("top-p 0.9 (whole vocabulary)", 1.0, 0, 0.9),
                              ("temperature only", 1.0, 0, 1.0), ("logit stats", None, 0, 1.0)):
            a = cu.SampleArgs()
            a.logits, a.vocab, a.rows, a.stride = lg.ptr, V, rows, V
            a.temperature, a.top_k, a.top_p, a.rep_penalty = (T or 1.0), k, p, 1.0
            a.u, a.out = u.ptr, out.ptr

            def call():
                if T is None:
                    ctx.call("opure_logit_stats", C.c_void_p(lg.ptr), V, rows, V, C.c_void_p(st.ptr))
                else:
                    ctx.sample_filtered(a)
            for _ in range(5):
                call()
            e0, e1 = cu.Event(ctx), cu.Event(ctx)
            e0.record()
            for _ in range(50):
                call()
            e1.record()
            ctx.sync()
            points.append({"rows": rows, "kernel": name, "us_per_call": e0.elapsed_ms(e1) * 1e3 / 50})
            e0.free()
            e1.free()
    ctx.close()
    mp = model_dir()
    budget = 128
    gen = {}
    with ve.Engine(mp, max_batch=1, max_len=PROMPT_LEN + budget + 8) as eng:
        prompts = [ve.prompt(1, V, PROMPT_LEN)]
        eng.generate(prompts, 8)
        eng.sample_generate(prompts, 8, temperature=0.8, top_k=50, top_p=0.95, rep_penalty=1.1, seed=1)
        t0 = time.perf_counter()
        eng.generate(prompts, budget)
        gen["greedy_tok_s"] = budget / (time.perf_counter() - t0)
        t0 = time.perf_counter()
        eng.sample_generate(prompts, budget, temperature=0.8, top_k=50, top_p=0.95, rep_penalty=1.1, seed=1)
        gen["sampled_tok_s"] = budget / (time.perf_counter() - t0)
    line = {"metric": "sampling kernels (us per call) and sampled generation tok/s (bs1, config 0)",
            "unit": "us", "points": points, "generate": gen}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2560)
    ap.add_argument("--warmup", type=int, default=128)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-steps", type=int, default=128)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", choices=["decode", "attn", "gemv", "spec", "cfg4", "tp", "sample", "window"], default="decode")
    ap.add_argument("--path", choices=["auto", "layers", "unfused"], default="auto",
                    help="decode: step kernels (auto = one persistent kernel per step when eligible, "
                         "layers = three fused kernels per layer, unfused = per-op kernels)")
    ap.add_argument("--phase-trace", action="store_true",
                    help="decode: record the persistent step's per-CTA phase stamps and report "
                         "per-phase times (last timed step) under \"phases\"")
    ap.add_argument("--bs64-steps", type=int, default=256,
                    help="decode at --batch 1: also time this many bs64 steps (the metric's second "
                         "batch size) and report them under \"bs64\"; 0 skips")
    ap.add_argument("--int8", type=int, default=1,
                    help="decode at --batch 1: also time the int8 (GEMV_Quant) config-0 model and report it "
                         "under \"int8\"; 0 skips")
    ap.add_argument("--gemv-n", type=lambda v: [int(x) for x in v.split(",")], default=[1, 5, 9],
                    help="gemv: comma-separated vector counts (16 and more run on the tensor cores)")
    ap.add_argument("--gemv-shapes", type=lambda v: [tuple(int(d) for d in x.split("x")) for x in v.split(",")],
                    default=[(576, 576), (192, 576), (1536, 576), (576, 1536), (49152, 576)],
                    help="gemv: comma-separated ROWSxCOLS shapes")
    ap.add_argument("--spec-k", type=lambda v: [int(x) for x in v.split(",")], default=[4, 8],
                    help="spec: comma-separated draft lengths")
    ap.add_argument("--spec-b", type=lambda v: [int(x) for x in v.split(",")], default=[1, 16],
                    help="spec: comma-separated batch sizes")
    ap.add_argument("--spec-budget", type=int, default=256, help="spec: generated tokens per sequence")
    ap.add_argument("--seqs", type=int, default=512, help="cfg4: total sequences over all ranks")
    ap.add_argument("--wave", type=int, default=128, help="cfg4: sequences per GPU per wave")
    ap.add_argument("--attn-b", type=int, default=0, help="attn: only this batch size (1, 8 or 64)")
    ap.add_argument("--attn-ctx", type=int, default=0, help="attn: only this context length")
    ap.add_argument("--attn-splits", type=lambda v: [int(x) for x in v.split(",")], default=[0],
                    help="attn: comma-separated keys per split to time (0: the library's choice)")
    ap.add_argument("--tp-allreduce", choices=["auto", "nccl", "peer"], default="auto",
                    help="tp: NCCL or NVLink peer kernels (auto: the peer kernels when every GPU pair maps)")
    ap.add_argument("--quick", action="store_true",
                    help="minimal run for profiler launch lists: no parity, e2e or CPU legs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_init()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.workload == "attn":
            run_attention_sweep(args)
        elif args.workload == "gemv":
            run_gemv_sweep(args)
        elif args.workload == "spec":
            run_spec(args)
        elif args.workload == "sample":
            run_sample(args)
        elif args.workload == "window":
            run_window(args)
        elif args.workload == "cfg4":
            run_cfg4(args, world, rank, local)
        elif args.workload == "tp":
            run_tp(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
