#!/usr/bin/env python3
"""Benchmark of the B200 LFM3 backbone step (one JSON line on rank 0).

Workload (steady state; configs[1] is a parity
case): per GPU, 8 sessions of the graded synthetic LFM3 geometry (Q8_0,
hidden 2048, FFN 8192, 16/4 heads, vocab 65536, 24 layers) with prompt
lengths uniform in [64, 4096] (seed 1, + rank), prefilled through 512-row
prompt passes; then decode rounds of all 8 ragged rows. A "step" is one
decode round (8 tokens per GPU); `value` is whole-job decode tok/s with every
input resident on the device (ForwardBatchInputs, logits left in HBM), `e2e`
is the same through the host API with token selection on the device
(ForwardBatchSample: pinned tokens in, the reference runner's sampler
applied on the device, selected tokens out), `e2e_logits` through
ForwardBatch (every session's logits to pinned host memory, greedy selection
on the host). Prefill tok/s of the workload's 512-row passes and of a
standalone 512-row pass go beside it, and `config3_job` runs BASELINE config
3 whole: arrivals 0-2 rounds apart, prompt passes between decode rounds,
256 sampled tokens per session.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun: one process per GPU, each an independent model
replica with its own sessions (no collective on the data path); timing is the
maximum over ranks.
"""
import argparse
import concurrent.futures
import ctypes
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
METRIC = "decode tok/s (8 ragged sessions, Q8_0) + 512-chunk prefill tok/s; % roofline"
SESSIONS = 8
PROMPT_RANGE = (64, 4096)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prompt-max", type=int, default=PROMPT_RANGE[1])
    ap.add_argument("--profile", action="store_true",
                    help="no timing: a fixed launch sequence for ncu captures "
                         "(see profile_sequence)")
    ap.add_argument("--profile-bf16", action="store_true",
                    help="no timing: the same sequence over BF16 weights "
                         "(config 4's matrix type)")
    ap.add_argument("--configs", nargs="?", const="2,5,4", default=None,
                    help="BASELINE configs 2, 4 and a one-GPU slice of 5 (a comma "
                         "list selects), one JSON line each (see config_runs); not "
                         "the headline")
    ap.add_argument("--profile-workload", action="store_true",
                    help="no timing: the bench's own sessions, then decode rounds "
                         "for ncu captures (see profile_workload)")
    return ap.parse_args()


# ---- roofline arithmetic ------------------------------------------------------------
def layer_counts(cfg):
    kinds = [cfg.layer_type[i] for i in range(cfg.n_layers)]
    return kinds.count(0), kinds.count(1), kinds.count(2)  # conv, global, sliding


def matrix_elements(cfg):
    """Q8_0 matrix elements read by one decode round (all layers + LM head)."""
    H, F, A = cfg.hidden, cfg.intermediate, cfg.heads * 128
    total = 0
    for i in range(cfg.n_layers):
        total += 3 * F * H
        if cfg.layer_type[i] == 0:
            total += 3 * H * H + H * H
        else:
            kv = cfg.kv_heads[i] * 128
            total += A * H + 2 * kv * H + cfg.heads * H + H * A
    return total + cfg.vocab * H


def small_tensor_bytes(cfg):
    """F32 norm, convolution and RoPE weights read by one round."""
    H = cfg.hidden
    total = 4 * H * 4 * cfg.n_layers + H * 4 + 64 * 4
    for i in range(cfg.n_layers):
        total += H * cfg.conv_width * 4 if cfg.layer_type[i] == 0 else 2 * 128 * 4
    return total


def decode_round_bytes(cfg, depths, bf16=False):
    """Algorithmic HBM bytes of one decode round whose rows sit at `depths`
    keys before them: Q8 (or BF16) weights once, plus per row the K/V rows
    attention reads, the new K/V row, convolution state read+write, logits
    and the embedding row."""
    conv, full, sliding = layer_counts(cfg)
    W = matrix_elements(cfg) * 2 if bf16 else matrix_elements(cfg) * 34 // 32
    kv_key = {i: 2 * cfg.kv_heads[i] * 128 * 2 for i in range(cfg.n_layers)}
    per_key = max(kv_key.values()) if kv_key else 0
    total = W + small_tensor_bytes(cfg)
    for d in depths:
        keys = d + 1
        for i in range(cfg.n_layers):
            t = cfg.layer_type[i]
            if t == 1:
                total += kv_key[i] * keys + kv_key[i]
            elif t == 2:
                total += kv_key[i] * min(keys, cfg.window) + kv_key[i]
            else:
                total += 2 * cfg.hidden * (cfg.conv_width - 1) * 4
        total += cfg.vocab * 4 + (cfg.hidden * 2 if bf16 else cfg.hidden * 34 // 32)
    del per_key
    return total


def prefill_flops(cfg, n, position, logits=True):
    """Dense FLOPs of one prompt pass of n rows at position, with the
    engine's live-row pruning after the last full-attention layer; attention
    counts QK and PV over the keys each live query sees; dequantisation and
    per-block scaling are not counted."""
    H, F, A, L = cfg.hidden, cfg.intermediate, cfg.heads * 128, cfg.n_layers
    live_in, live_out = [n] * L, [n] * L
    need = 1
    for i in reversed(range(L)):
        t = cfg.layer_type[i]
        if t == 2:
            break
        live_out[i] = min(n, need)
        if t == 1:
            break
        need = min(n, need + cfg.conv_width - 1)
        live_in[i] = need
    flops = 0
    for i in range(L):
        rin, rout = live_in[i], live_out[i]
        if cfg.layer_type[i] == 0:
            flops += 2 * rin * 3 * H * H + 2 * rout * H * H
        else:
            kv = cfg.kv_heads[i] * 128
            flops += 2 * n * (A * H + 2 * kv * H + cfg.heads * H)
            keys = 0
            for q in range(n - rout, n):
                k = position + q + 1
                keys += min(k, cfg.window) if cfg.layer_type[i] == 2 else k
            flops += 4 * cfg.heads * 128 * keys + 2 * rout * H * A
        flops += 2 * rout * 3 * F * H
    if logits:
        flops += 2 * cfg.vocab * H
    return flops


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained"), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


def committed_traffic(kernel="decode_gemv_round"):
    """DRAM bytes (read + write) per launch of a kernel from one ncu capture,
    kept in profiles/traffic.json beside the summary it comes from."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return float(json.load(f)[kernel]["dram_bytes_per_launch"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


# ---- clocks ---------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and clock-event reasons sampled during a timed region (read
    only): NVML every 5 ms when the bindings load, else nvidia-smi every
    200 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40}

    def __init__(self, index):
        self.index, self.lines, self.proc = index, [], None
        self.samples, self.max_mhz, self.reasons = [], None, set()
        self.stop, self.thread, self.nvml = None, None, None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            import torch
            props = torch.cuda.get_device_properties(self.index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        return pynvml, handle

    def _sample(self):
        nv, h = self.nvml
        reasons_of = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
        bits = reasons_of(h)
        for name, bit in self.REASONS.items():
            if bits & bit:
                self.reasons.add(name)

    def _poll(self):
        while not self.stop.wait(0.005):
            self._sample()

    def _query(self):
        # one nvidia-smi reading (short timed regions end between its -lms ticks)
        try:
            out = subprocess.run(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index)], capture_output=True, text=True, timeout=10).stdout
            self.lines += [l.strip() for l in out.splitlines() if l.strip()]
        except (OSError, subprocess.SubprocessError):
            pass

    def __enter__(self):
        # a reading at each end of the region, and the poller in between
        try:
            self.nvml = self._nvml_handle()
            nv, h = self.nvml
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._sample()
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        self._query()
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.nvml:
            self.stop.set()
            self.thread.join(5)
            try:
                self._sample()
            except Exception:
                pass
            return
        self._query()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.nvml:
            if not self.samples:
                return None
            return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(self.reasons), "samples": len(self.samples),
                    "source": "nvml 5 ms"}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 200 ms"}


# ---- CPU baseline ------------------------------------------------------------------------
def cpu_decode_rate(weights, threads, tokens_per_session, warm_steps, prefer_reference=True):
    """Decode tok/s of `threads` independent sessions, one per host thread,
    on the reference's CPU oracle (oracle/_ref, compiled reference.cpp) when
    present, else on the oracle's C restatement. Each session first advances
    warm_steps tokens (depth), then times tokens_per_session logits steps."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    kind = "reference" if prefer_reference and oracle.reference_available() else "port"
    make = (lambda: oracle.ReferenceOracle(weights, 256)) if kind == "reference" else (
        lambda: oracle.Oracle(weights, 256, threads=1))
    sessions = [make() for _ in range(threads)]
    barrier = threading.Barrier(threads)
    times = [0.0] * threads

    def run(i):
        s = sessions[i]
        for t in range(warm_steps):
            s.step((7 * i + t) % weights.config.vocab, False)
        barrier.wait()
        t0 = time.perf_counter()
        for t in range(tokens_per_session):
            s.step((11 * i + t) % weights.config.vocab, True)
        times[i] = time.perf_counter() - t0

    with concurrent.futures.ThreadPoolExecutor(threads) as pool:
        list(pool.map(run, range(threads)))
    for s in sessions:
        s.close()
    elapsed = max(times)
    return threads * tokens_per_session / elapsed, elapsed, kind


def cpu_depth_note(cfg, depth, steps):
    """How much the CPU sample's shallow rows understate the work of the GPU
    rows (multiply-adds per token: weights plus attention over the keys)."""
    H, A = cfg.hidden, cfg.heads * 128
    weights = matrix_elements(cfg)

    def macs(d):
        keys = 0
        for i in range(cfg.n_layers):
            if cfg.layer_type[i] == 1:
                keys += d + 1
            elif cfg.layer_type[i] == 2:
                keys += min(d + 1, cfg.window)
        return weights + 2 * A * keys

    lengths, _ = rank_workload(0, PROMPT_RANGE[1], cfg.vocab)
    gpu = float(np.mean([macs(int(n)) for n in lengths]))
    return (f"CPU rows at depths {depth}..{depth + steps - 1}; the GPU rows (prompts "
            f"{int(lengths.min())}..{int(lengths.max())} tokens) need "
            f"{100 * (gpu / macs(depth + steps // 2) - 1):.1f}% more multiply-adds per token "
            f"(attention over their keys; {H}-wide weights dominate)")


def reference_arm(args):
    """The reference's own CPU implementation of the path on this host."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # weights from the oracle library's copy of the generator: this arm
    # loads no library of this package (the reference's code and its shim
    # only, oracle/_ref)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    weights = oracle.SyntheticWeights(seed=0, prefer_reference=True)
    threads = max(1, min(SESSIONS, os.cpu_count() or 1))
    # one step = one decode token per session; warm-up steps deepen the rows
    rate, elapsed, kind = cpu_decode_rate(weights.weights, threads, args.steps,
                                          args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{threads} sessions on {threads} host threads, one decode "
                               f"token per session per step after {args.warmup} warm-up "
                               "tokens (the CPU cannot prefill 4096-token prompts in minutes)",
                   "depth_note": cpu_depth_note(weights.config, args.warmup, args.steps),
                   "model": "LFM3 synthetic 24L h2048 f8192 16/4x128 v65536 Q8_0",
                   "parallelism": "threads"},
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": kind,
                         "sample": f"{threads} sessions x {args.steps} decode tokens"},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- ranks (one process per GPU under torchrun) ------------------------------------------------
class Ranks:
    """Rank plumbing of a replicas-only job: RANK / WORLD_SIZE / LOCAL_RANK from
    the torchrun environment, a MAX over ranks and a barrier. Only timings
    cross ranks: each rank runs its own model replica and sessions."""

    def __init__(self, backend="nccl"):
        import torch
        import torch.distributed as dist
        self.dist, self.torch = dist, torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.device = torch.device("cuda", self.local) if backend == "nccl" else torch.device("cpu")
        if backend == "nccl":
            torch.cuda.set_device(self.local)
        if self.world > 1:
            from datetime import timedelta
            extra = {"device_id": self.device} if backend == "nccl" else {}
            dist.init_process_group(backend, timeout=timedelta(seconds=300), **extra)

    def sync_max(self, value):
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sync_sum(self, value):
        if self.world == 1:
            return value
        t = self.torch.tensor([value], dtype=self.torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return float(t.item())

    def barrier(self):
        if self.device.type == "cuda":
            self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def rank_workload(rank, prompt_max, vocab):
    """This rank's 8 sessions: prompt lengths U[64, prompt_max] and tokens, from
    seed (1, rank), so ranks hold different sessions."""
    rng = np.random.default_rng([1, rank])
    lengths = rng.integers(PROMPT_RANGE[0], prompt_max + 1, SESSIONS)
    prompts = [rng.integers(0, vocab, int(n)).astype(np.uint32) for n in lengths]
    return lengths, prompts


SAMPLER = (0.1, 50, 1.1)  # the reference runner's defaults (runner.cpp:31-35)
GOLDEN64 = np.uint64(0x9E3779B97F4A7C15)


class SampledRounds:
    """Decode rounds of a fixed batch through the host API with selection on
    the device (lfm3_session_forward_batch_sample): the reference runner's
    sampler (temperature 0.1, top-k 50, repeat penalty 1.1) over each
    session's last 64 tokens, kept as a ring in one host table that is
    updated in place; a fresh seed per draw from (session seed, position).
    Pinned token buffers in and out, as a C++ host would hold them."""

    def __init__(self, lfm3, sessions, tokens, histories, seed):
        import torch
        n = len(sessions)
        self.lfm3, self.lib, self.n = lfm3, lfm3.library(), n
        self.handles = (ctypes.c_void_p * n)(*[s.handle for s in sessions])
        self.sampler = lfm3.sampler(*SAMPLER)
        self.table = np.zeros((n, 64), np.uint32)
        self.count = np.zeros(n, np.uint32)
        self.ring = np.zeros(n, np.int64)
        for r, h in enumerate(histories):
            h = np.asarray(h, np.uint32)[-64:]
            self.table[r, :h.size] = h
            self.count[r] = h.size
            self.ring[r] = h.size % 64
        self.tokens = torch.empty(n, dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
        self.out = torch.empty(n, dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
        self.tokens[:] = tokens
        self.base = np.array([(seed << 8) + r for r in range(n)], np.uint64)
        self.positions = np.array([s.position for s in sessions], np.uint64)
        self.seeds = np.zeros(n, np.uint64)
        self.rows = np.arange(n)
        ptr = lambda a: ctypes.c_void_p(a.ctypes.data)  # noqa: E731
        self.args = (self.handles, ptr(self.tokens), n, ctypes.byref(self.sampler),
                     ptr(self.table), ptr(self.count), ptr(self.seeds), ptr(self.out))
        # bytes each round sends to the device: the round's row table
        # (DecodeRows) and the selection's per-row tables (kernel parameters)
        self.h2d_bytes = 136 + n * (64 * 4 + 4 + 8)
        self.d2h_bytes = 4 * n

    def round(self):
        # the token this round consumes joins its session's penalty window
        self.table[self.rows, self.ring] = self.tokens
        self.ring = (self.ring + 1) % 64
        np.minimum(self.count + 1, 64, out=self.count)
        with np.errstate(over="ignore"):
            self.seeds[:] = self.base ^ (self.positions * GOLDEN64)
        self.lfm3.check(self.lib.lfm3_session_forward_batch_sample(*self.args))
        self.positions += 1
        self.tokens[:] = self.out


CONFIG5_PROMPTS = (512, 32768)


def config5_workload(rank, vocab):
    """This rank's share of BASELINE config 5 (64 sessions over 8 GPUs = 8 per
    GPU): prompt lengths log-uniform in [512, 32768] and tokens, from seed
    (5, rank), so ranks hold different sessions."""
    rng = np.random.default_rng([5, rank])
    lo, hi = CONFIG5_PROMPTS
    lengths = np.exp(rng.uniform(np.log(lo), np.log(hi), SESSIONS)).astype(int)
    prompts = [rng.integers(0, vocab, int(n)).astype(np.uint32) for n in lengths]
    return lengths, prompts


def config5_rank(lfm3, model, cfg, rank, rounds, warmup=3):
    """Config 5 on this rank's GPU: prefill its 8 sessions (512-row passes,
    device-timed per session), then `rounds` decode rounds of the 8 ragged
    rows (ForwardBatchInputs, logits on the device), device-timed."""
    import torch
    lengths, prompts = config5_workload(rank, cfg.vocab)
    sessions = [model.session(int(n) + rounds + warmup + 16) for n in lengths]
    prefill_ms = 0.0
    for sess, p in zip(sessions, prompts):
        st = torch.cuda.ExternalStream(sess.stream)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        sess.forward(p, logits=False)
        b.record(st)
        b.synchronize()
        prefill_ms += a.elapsed_time(b)
    tokens = [int(t) for t in np.random.default_rng([6, rank]).integers(0, cfg.vocab, SESSIONS)]

    def run(k):
        for step in range(k):
            lfm3.Session.forward_batch_inputs(
                sessions, [(t + step) % cfg.vocab for t in tokens], logits=True)

    run(warmup)
    depths = [sess.position for sess in sessions]
    st = torch.cuda.ExternalStream(sessions[0].stream)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    run(rounds)
    b.record(st)
    b.synchronize()
    decode_ms = a.elapsed_time(b)
    for sess in sessions:
        sess.close()
    return {"prefill_tokens": int(lengths.sum()), "prefill_ms": prefill_ms,
            "decode_ms": decode_ms, "depths": depths,
            "lengths": [int(n) for n in lengths]}


def config3_job(lfm3, model, cfg, rank, prompt_max, decode_tokens=256, trace=None):
    """BASELINE config 3 as one whole job on this GPU, through the library's
    continuous-batching scheduler (lfm3_scheduler): 8 requests (prompts
    U[64, prompt_max], seed (1, rank)) admitted 0-2 steps apart (seed
    (2, rank)); each scheduler step runs one prompt pass of at most 512 rows
    (first come, first served) and one decode round of every decoding
    request, tokens selected on the device with the reference runner's
    sampler. Every request selects `decode_tokens` tokens (the first from its
    last prompt pass). Pass and round times are the scheduler's host times
    (each part returns with its results on the host). `trace`, when given,
    receives (step, "pass", request) and (step, "round", rows) in order."""
    lengths, prompts = rank_workload(rank, prompt_max, cfg.vocab)
    rng = np.random.default_rng([2, rank])
    arrive = np.concatenate([[0], np.cumsum(rng.integers(0, 3, SESSIONS - 1))])
    sched = lfm3.Scheduler(model, lfm3.sampler(*SAMPLER))
    ids = {}
    t_prefill = t_decode = 0.0
    prefill_tokens = decode_rows = rounds = passes = 0
    step = 0
    t_job = time.perf_counter()
    while len(ids) < SESSIONS or not sched.idle:
        for i in range(SESSIONS):
            if arrive[i] == step:
                ids[i] = sched.admit(prompts[i], decode_tokens,
                                     ((1000 + rank) << 40) ^ (i << 32),
                                     int(lengths[i]) + decode_tokens + 8)
        st = sched.step()
        if st.pass_request >= 0:
            passes += 1
            prefill_tokens += st.pass_rows
            t_prefill += st.pass_ms / 1e3
            if trace is not None:
                trace.append((step, "pass", int(st.pass_request)))
        if st.round_rows:
            rounds += 1
            decode_rows += st.round_rows
            t_decode += st.round_ms / 1e3
            if trace is not None:
                trace.append((step, "round", int(st.round_rows)))
        step += 1
    t_job = time.perf_counter() - t_job
    for i in range(SESSIONS):
        if len(sched.tokens(ids[i])) != decode_tokens:
            raise RuntimeError(f"request {i} ended early")
    sched.close()
    return {"decode_tokens": decode_rows, "decode_s": t_decode,
            "prefill_tokens": prefill_tokens, "prefill_s": t_prefill,
            "job_s": t_job, "rounds": rounds, "passes": passes,
            "steps": step, "arrivals": [int(a) for a in arrive]}


def job_rate(tokens_per_rank, world, max_ms):
    """Whole-job throughput: every rank's tokens over the slowest rank's time."""
    return tokens_per_rank * world / (max_ms / 1e3)


# ---- profiling sequence ----------------------------------------------------------------------
PROFILE_PROMPT = 64
PROFILE_WARM_ROUNDS = 3


def profile_sequence(matrix_type=None):
    """A fixed, untimed launch sequence for ncu: 8 sessions prefilled with
    64-token prompts (one prompt pass each, whose last row's logits take one
    LM-head decode_gemv launch), 3 warm decode rounds, then the captured work: one
    decode round of the 8 rows, then one 512-row prompt pass on session 0.
    Before the captured round: 8 + 3 x 97 = 299 decode_gemv launches and
    8 x 96 = 768 q8_prefill_tc_kernel launches (24 layers: 4 projection
    launches per layer). With matrix_type BF16 (--profile-bf16) the weights
    are BF16: the decode rounds run decode_gemv_kernel's BF16 instantiations
    and each prompt projection is split_bf16_rows_kernel then
    q8_prefill_tc_kernel<1>."""
    import torch
    lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
    weights = (lfm3.SyntheticWeights(seed=0) if matrix_type is None else
               lfm3.SyntheticWeights(seed=0, matrix_type=matrix_type))
    cfg = weights.config
    model = lfm3.Model(weights.weights)
    rng = np.random.default_rng([1, 0])
    sessions = [model.session(1024) for _ in range(SESSIONS)]
    for s in sessions:
        s.forward(rng.integers(0, cfg.vocab, PROFILE_PROMPT).astype(np.uint32))
    tokens = [int(t) for t in rng.integers(0, cfg.vocab, SESSIONS)]
    for _ in range(PROFILE_WARM_ROUNDS + 1):
        lfm3.Session.forward_batch_inputs(sessions, tokens, logits=True)
    sessions[0].forward(rng.integers(0, cfg.vocab, 512).astype(np.uint32))
    torch.cuda.synchronize()
    print(json.dumps({"profile_sequence": "done", "sessions": SESSIONS,
                      "prompt": PROFILE_PROMPT, "warm_rounds": PROFILE_WARM_ROUNDS}))


def profile_workload(prompt_max):
    """A fixed, untimed launch sequence over the bench's own rank-0 workload for
    ncu: the 8 sessions' prompts U[64, prompt_max] (seed 1) prefilled, then
    PROFILE_WARM_ROUNDS + 1 decode rounds of the 8 rows. Before the last round
    the sequence has launched PROFILE_WARM_ROUNDS x 11 decode_attention_kernel
    launches (the prompts' passes use the prompt attention kernel)."""
    import torch
    lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
    weights = lfm3.SyntheticWeights(seed=0)
    cfg = weights.config
    model = lfm3.Model(weights.weights)
    lengths, prompts = rank_workload(0, prompt_max, cfg.vocab)
    sessions = [model.session(int(n) + PROFILE_WARM_ROUNDS + 2) for n in lengths]
    for s, p in zip(sessions, prompts):
        s.forward(p, logits=False)
    tokens = [int(t) for t in np.random.default_rng([2, 0]).integers(0, cfg.vocab, SESSIONS)]
    for _ in range(PROFILE_WARM_ROUNDS + 1):
        lfm3.Session.forward_batch_inputs(sessions, tokens, logits=True)
    torch.cuda.synchronize()
    print(json.dumps({"profile_workload": "done", "depths": [s.position for s in sessions]}))


# ---- our arm ---------------------------------------------------------------------------------
def config_runs(which="2,5,4"):
    """The BASELINE configs besides the headline, on one GPU, one JSON line
    each (printed as each finishes):
      config2: Q8_0, one session, 2048-token prompt in four 512-row passes,
        then 128 greedy tokens through Forward (host logits, host argmax);
      config5: a one-GPU slice of the box-scale config, 8 sessions with
        prompts log-uniform in [512, 32768] (seed 5), prefilled in 512-row
        passes, then 512 decode rounds of the 8 rows with logits on the device;
      config4: BF16 weights, 8 sessions at depth 8192, each prefilled from
        its own 8192 random tokens in 512-row passes, then 128 decode rounds
        with logits on the device.
    Device time with CUDA events on the session streams (max with the host's
    wall time for calls that return to the host)."""
    import torch
    lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
    hbm_peak, tensor_peak, _, peak_source = measured_peaks()

    def timed(stream, fn):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        start.record(stream)
        fn()
        end.record(stream)
        end.synchronize()
        return max(start.elapsed_time(end), (time.perf_counter() - t0) * 1e3)

    def emit(line):
        line["peak_source"] = peak_source
        print(json.dumps(line), flush=True)

    chosen = {c.strip() for c in which.split(",")}
    rng = np.random.default_rng(2)
    if chosen & {"2", "5"}:
        w = lfm3.SyntheticWeights(seed=0)
        model = lfm3.Model(w.weights)
        if "2" in chosen:
            config2_run(lfm3, w.config, model, rng, timed, emit, tensor_peak, hbm_peak)
        if "5" in chosen:
            config5_run(lfm3, w.config, model, rng, timed, emit, hbm_peak)
        model.close()
        w.close()
    if "4" in chosen:
        wb = lfm3.SyntheticWeights(seed=0, matrix_type=lfm3.abi.BF16)
        mb = lfm3.Model(wb.weights)
        config4_run(lfm3, wb.config, mb, rng, timed, emit, hbm_peak)
        mb.close()
        wb.close()


def config2_run(lfm3, cfg, model, rng, timed, emit, tensor_peak, hbm_peak):
    """Config 2 (see config_runs)."""
    import torch
    prompt = rng.integers(0, cfg.vocab, 2048).astype(np.uint32)
    warm = model.session(600)
    warm.forward(prompt[:512])
    warm.forward(prompt[512:513])
    warm.close()
    s = model.session(2048 + 128 + 8)
    st = torch.cuda.ExternalStream(s.stream)
    state = {}
    prefill_ms = timed(st, lambda: state.update(logits=s.forward(prompt)))

    def greedy():
        tok = int(np.argmax(state["logits"]))
        for _ in range(128):
            tok = int(np.argmax(s.forward([tok])))

    decode_ms = timed(st, greedy)
    flops = sum(prefill_flops(cfg, 512, 512 * i, logits=i == 3) for i in range(4))
    per_token = decode_ms / 128
    emit({"config": "config2", "prefill_tok_s": 2048 / (prefill_ms / 1e3),
          "prefill_tflops": flops / (prefill_ms * 1e-3) / 1e12,
          "prefill_frac_of_tensor_peak": flops / (prefill_ms * 1e-3) / 1e12 / tensor_peak,
          "decode_tok_s": 128 / (decode_ms / 1e3), "decode_ms_per_token": per_token,
          "decode_frac_of_hbm_peak": decode_round_bytes(cfg, [2048 + 64])
          / (per_token * 1e-3) / 1e9 / hbm_peak,
          "path": "Forward: four 512-row passes, then 128 one-token calls with host "
                  "logits and host argmax"})
    s.close()


def config5_run(lfm3, cfg, model, rng, timed, emit, hbm_peak):
    """One GPU's share of config 5 (see config_runs)."""
    import torch
    lengths = np.exp(rng.uniform(np.log(512), np.log(32768), SESSIONS)).astype(int)
    prompts = [rng.integers(0, cfg.vocab, int(n)).astype(np.uint32) for n in lengths]
    sessions = [model.session(int(n) + 512 + 16) for n in lengths]
    prefill_ms = 0.0
    flops = 0.0
    for sess, p in zip(sessions, prompts):
        prefill_ms += timed(torch.cuda.ExternalStream(sess.stream),
                            lambda: sess.forward(p, logits=False))
        flops += sum(prefill_flops(cfg, min(512, len(p) - a), a, logits=False)
                     for a in range(0, len(p), 512))
    tokens = [int(t) for t in rng.integers(0, cfg.vocab, SESSIONS)]
    fst = torch.cuda.ExternalStream(sessions[0].stream)

    def rounds(k):
        for step in range(k):
            lfm3.Session.forward_batch_inputs(
                sessions, [(t + step) % cfg.vocab for t in tokens], logits=True)

    rounds(3)
    depths = [sess.position for sess in sessions]
    decode_ms = timed(fst, lambda: rounds(512))
    per_round = decode_ms / 512
    bytes_round = decode_round_bytes(cfg, [d + 256 for d in depths])
    emit({"config": "config5_one_gpu", "prompt_lengths": [int(n) for n in lengths],
          "prefill_tok_s": int(lengths.sum()) / (prefill_ms / 1e3),
          "prefill_tflops": flops / (prefill_ms * 1e-3) / 1e12,
          "decode_tok_s": SESSIONS * 512 / (decode_ms / 1e3),
          "decode_ms_per_round": per_round,
          "decode_frac_of_hbm_peak": bytes_round / (per_round * 1e-3) / 1e9 / hbm_peak,
          "path": "Forward 512-row passes per session, then 512 ForwardBatchInputs "
                  "rounds of the 8 rows (logits on the device)"})
    for sess in sessions:
        sess.close()


def config4_run(lfm3, cfg, mb, rng, timed, emit, hbm_peak):
    """Config 4 (see config_runs)."""
    import torch
    depth = 8192
    sessions = [mb.session(depth + 128 + 16) for _ in range(SESSIONS)]
    first = sessions[0]
    prefill_ms = 0.0
    for sess in sessions:
        prompt = rng.integers(0, cfg.vocab, depth).astype(np.uint32)
        prefill_ms += timed(torch.cuda.ExternalStream(sess.stream),
                            lambda: sess.forward(prompt, logits=False))
    tokens = [int(t) for t in rng.integers(0, cfg.vocab, SESSIONS)]
    fst = torch.cuda.ExternalStream(first.stream)

    def rounds(k):
        for step in range(k):
            lfm3.Session.forward_batch_inputs(
                sessions, [(t + step) % cfg.vocab for t in tokens], logits=True)

    rounds(3)
    decode_ms = timed(fst, lambda: rounds(128))
    per_round = decode_ms / 128
    bytes_round = decode_round_bytes(cfg, [depth + 3 + 64] * SESSIONS, bf16=True)
    emit({"config": "config4", "depth": depth,
          "prefill_tok_s": SESSIONS * depth / (prefill_ms / 1e3),
          "decode_tok_s": SESSIONS * 128 / (decode_ms / 1e3),
          "decode_ms_per_round": per_round, "bytes_per_round": bytes_round,
          "decode_frac_of_hbm_peak": bytes_round / (per_round * 1e-3) / 1e9 / hbm_peak,
          "path": "8 sessions each prefilled in 512-row BF16 passes (tcgen05, "
                  "inputs as three exact bf16 planes); 128 ForwardBatchInputs "
                  "rounds (packed BF16 decode copies, mma.sync)"})
    for sess in sessions:
        sess.close()


def main():
    args = parse()
    if args.configs:
        config_runs(args.configs)
        return
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.profile:
        profile_sequence()
        return
    if args.profile_bf16:
        profile_sequence(importlib.import_module(
            "lfm3-gufo-extension_b200").abi.BF16)
        return
    if args.profile_workload:
        profile_workload(args.prompt_max)
        return
    import torch

    ranks = Ranks("nccl")
    world, rank, local = ranks.world, ranks.rank, ranks.local
    sync_max, barrier = ranks.sync_max, ranks.barrier

    lfm3 = importlib.import_module("lfm3-gufo-extension_b200")
    weights = lfm3.SyntheticWeights(seed=0)
    cfg = weights.config
    t_load = time.perf_counter()
    model = lfm3.Model(weights.weights)  # upload + the decode copies' packing
    load_s = time.perf_counter() - t_load
    lengths, prompts = rank_workload(rank, args.prompt_max, cfg.vocab)
    total_steps = args.warmup * 2 + args.steps * 3 + 8
    sessions = [model.session(int(n) + total_steps + 16) for n in lengths]

    def stream_of(s):
        return torch.cuda.ExternalStream(s.stream)

    # ---- prefill of the workload (512-row passes), device-timed per session
    prefill_ms, prefill_tokens, prefill_fl = 0.0, 0, 0.0
    launches0 = lfm3.launch_count()
    for s, p in zip(sessions, prompts):
        st = stream_of(s)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(st)
        s.forward(p)
        end.record(st)
        end.synchronize()
        prefill_ms += start.elapsed_time(end)
        prefill_tokens += len(p)
        for first in range(0, len(p), 512):
            n = min(512, len(p) - first)
            prefill_fl += prefill_flops(cfg, n, first, logits=first + n == len(p))
    # ---- a standalone 512-row pass at position 0 (reference's pp512 unit)
    probe = model.session(1024)
    pass_tokens = np.random.default_rng(5).integers(0, cfg.vocab, 512).astype(np.uint32)
    st = stream_of(probe)
    pass_times = []
    for rep in range(4):
        probe.reset()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(st)
        probe.forward(pass_tokens)
        end.record(st)
        end.synchronize()
        if rep:
            pass_times.append(start.elapsed_time(end))
    pass_ms = min(pass_times)
    pass_flops = prefill_flops(cfg, 512, 0)
    probe.close()

    hbm_peak, tensor_peak, tensor_sustained, peak_source = measured_peaks()
    front = sessions[0]
    fst = stream_of(front)
    tokens = [int(np.argmax(s.read_logits())) for s in sessions]

    def device_rounds(k):
        for step in range(k):
            lfm3.Session.forward_batch_inputs(
                sessions, [(t + step) % cfg.vocab for t in tokens], logits=True)

    # ---- warm-up, then the device-resident timed region
    device_rounds(args.warmup)
    depths = [s.position for s in sessions]
    barrier()
    sampler = ClockSampler(local)
    with sampler:
        launches_before = lfm3.launch_count()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(fst)
        device_rounds(args.steps)
        end.record(fst)
        end.synchronize()
        launches = lfm3.launch_count() - launches_before
        decode_ms = start.elapsed_time(end)
    barrier()
    decode_ms_max = sync_max(decode_ms)
    step_bytes = decode_round_bytes(cfg, [d + args.steps // 2 for d in depths])

    # ---- end to end through the host API: pinned token/logit buffers
    # one pinned [sessions][vocab] block; each session's logits are a row view
    logit_block = torch.empty((SESSIONS, cfg.vocab), dtype=torch.float32,
                              pin_memory=True).numpy()
    pinned_logits = [logit_block[r] for r in range(SESSIONS)]
    pinned_tokens = torch.empty(SESSIONS, dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    for r, s in enumerate(sessions):
        pinned_logits[r][:] = s.read_logits()
    pinned_tokens[:] = logit_block.argmax(axis=1)

    def host_rounds(k):
        for _ in range(k):
            lfm3.Session.forward_batch(sessions, pinned_tokens, outs=pinned_logits)
            pinned_tokens[:] = logit_block.argmax(axis=1)  # greedy, on the host

    host_rounds(args.warmup)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record(fst)
    host_rounds(args.steps)
    end.record(fst)
    end.synchronize()
    e2e_ms = max(start.elapsed_time(end), (time.perf_counter() - t0) * 1e3)
    barrier()
    e2e_ms_max = sync_max(e2e_ms)

    # ---- end to end with token selection on the device: the same rounds
    # through ForwardBatchSample (pinned tokens in, selected tokens out)
    rounds = SampledRounds(lfm3, sessions, pinned_tokens,
                           [p[-64:] for p in prompts], seed=1000 + rank)
    for _ in range(args.warmup):
        rounds.round()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    start.record(fst)
    for _ in range(args.steps):
        rounds.round()
    end.record(fst)
    end.synchronize()
    sampled_ms = max(start.elapsed_time(end), (time.perf_counter() - t0) * 1e3)
    barrier()
    sampled_ms_max = sync_max(sampled_ms)

    # ---- profiled pass (events around each kernel; not the headline timing)
    front.set_profiling(True)
    front.take_profile()
    device_rounds(min(args.steps, 10))
    prof = front.take_profile()
    front.set_profiling(False)
    proj_ms, proj_launches = prof["decode_projection"]
    profiled_rounds = min(args.steps, 10)
    proj_bytes = matrix_elements(cfg) * 34 // 32 * profiled_rounds
    gemv_gbs = proj_bytes / (proj_ms * 1e-3) / 1e9 if proj_ms else 0.0
    traffic = committed_traffic()
    launches_per_round = proj_launches / profiled_rounds if profiled_rounds else 0
    weight_bytes = matrix_elements(cfg) * 34 // 32
    step_s = decode_ms_max / args.steps * 1e-3

    # ---- CPU baseline (rank 0, one GPU only; bounded sample)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = max(1, min(SESSIONS, os.cpu_count() or 1))
        rate, elapsed, kind = cpu_decode_rate(weights.weights, threads, 6, 3)
        cpu = {"value": rate, "unit": "tok/s", "cores": threads, "kind": kind,
               "sample": f"{threads} sessions x 6 decode tokens at depth 3, one session "
                         f"per host thread ({elapsed:.1f} s)"}

    # ---- this GPU's 8 sessions of the 64 (prompts
    # log-uniform [512, 32768]), prefill then decode rounds
    c5_rounds = 64
    c5 = config5_rank(lfm3, model, cfg, rank, c5_rounds)
    c5_prefill_ms = sync_max(c5["prefill_ms"])
    c5_decode_ms = sync_max(c5["decode_ms"])
    c5_prefill_tokens = ranks.sync_sum(c5["prefill_tokens"])

    # ---- BASELINE config 3 as a whole job (arrivals, passes between rounds)
    job = config3_job(lfm3, model, cfg, rank, args.prompt_max)
    job_decode_s = sync_max(job["decode_s"])
    job_prefill_s = sync_max(job["prefill_s"])
    job_s = sync_max(job["job_s"])

    value = job_rate(SESSIONS * args.steps, world, decode_ms_max)
    e2e = job_rate(SESSIONS * args.steps, world, sampled_ms_max)
    e2e_logits = job_rate(SESSIONS * args.steps, world, e2e_ms_max)
    prefill_rate = ranks.sync_sum(prefill_tokens) / (sync_max(prefill_ms) / 1e3)
    load_s_max = sync_max(load_s)
    if rank != 0:
        ranks.close()
        return
    clocks = sampler.summary()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": decode_ms_max / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q8_0 codes x fp16 pairs -> fp32",
        "data": "synthetic",
        "config": {
            "workload": "config3 steady decode: 8 sessions/GPU, prompts U[64,4096] "
                        "(seed 1) prefilled in 512-row passes, then decode rounds of the "
                        "8 ragged rows; logits on device each round",
            "model": "LFM3 synthetic 24L h2048 f8192 16/4x128 v65536 Q8_0 (random init)",
            "global_batch": SESSIONS * world,
            "depths": [int(d) for d in depths],
            "parallelism": f"replicas x{world} (sessions partitioned, no collective)",
            "l2": "inputs larger than L2: each round streams 1.78 GB of weights",
        },
        "roofline": {
            "bound": "hbm", "kernel": "decode_gemv_kernel (decode projections + LM head)",
            "achieved": weight_bytes / step_s / 1e9, "peak": hbm_peak, "unit": "GB/s",
            "frac": weight_bytes / step_s / 1e9 / hbm_peak,
            "traffic": traffic * launches_per_round if traffic else None,
            "traffic_unit": "bytes per round (ncu, all decode_gemv launches of one round)",
            "peak_source": f"{peak_source} hbm_gbs",
            "how": "Q8 weight bytes of one round (read once by the round's decode_gemv "
                   "launches) / the timed ms_per_step: the whole round is charged to "
                   "the projections, so this is a lower bound of their bandwidth",
        },
        "serialised_gemv": {
            "achieved": gemv_gbs, "unit": "GB/s", "frac": gemv_gbs / hbm_peak,
            "how": f"Q8 weight bytes of {profiled_rounds} rounds / summed CUDA-event "
                   f"time of their {proj_launches} decode_gemv launches in a separate "
                   "profiled pass (events serialise the launches: not the headline)",
        },
        "step_roofline": {
            "bound": "hbm", "bytes_per_step": step_bytes,
            "achieved": step_bytes / (decode_ms_max / args.steps * 1e-3) / 1e9,
            "peak": hbm_peak, "unit": "GB/s",
            "frac": step_bytes / (decode_ms_max / args.steps * 1e-3) / 1e9 / hbm_peak,
        },
        "prefill": {
            "value": prefill_rate, "unit": "tok/s",
            "tflops": prefill_fl / (prefill_ms * 1e-3) / 1e12,
            "pass512_ms": pass_ms, "pass512_tok_s": 512 / (pass_ms * 1e-3) * world,
            "pass512_tflops": pass_flops / (pass_ms * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "achieved": pass_flops / (pass_ms * 1e-3) / 1e12,
                         "peak": tensor_peak, "unit": "TFLOP/s",
                         "frac": pass_flops / (pass_ms * 1e-3) / 1e12 / tensor_peak,
                         "peak_source": f"{peak_source} bf16_tflops (dense, burst)"},
        },
        "kernel_ms_per_round": {k: v[0] / profiled_rounds for k, v in prof.items() if v[1]},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e, "unit": "tok/s",
                "h2d_bytes_per_step": rounds.h2d_bytes,
                "d2h_bytes_per_step": rounds.d2h_bytes,
                "path": "lfm3_session_forward_batch_sample: pinned tokens in, the "
                        "tokens selected on the device out (temperature 0.1, top-k 50, "
                        "repeat penalty 1.1 over each session's last 64 tokens)"},
        "e2e_logits": {"value": e2e_logits, "unit": "tok/s", "h2d_bytes_per_step": 136,
                       "d2h_bytes_per_step": 4 * cfg.vocab * SESSIONS,
                       "path": "lfm3_session_forward_batch: pinned tokens in, every "
                               "session's logits out, greedy selection on the host"},
        "config3_job": {
            "decode_tok_s": job["decode_tokens"] * world / job_decode_s,
            "prefill_tok_s": job["prefill_tokens"] * world / job_prefill_s,
            "job_s": job_s, "rounds": job["rounds"], "passes": job["passes"],
            "decode_tokens": job["decode_tokens"] * world,
            "prefill_tokens": job["prefill_tokens"] * world,
            "arrivals_rank0": job["arrivals"],
            "how": "lfm3_scheduler: 8 requests/GPU, prompts U[64,4096], admitted 0-2 "
                   "steps apart; each step one <=512-row prompt pass (FIFO) then one "
                   "decode round of every decoding request with device sampling; 256 "
                   "tokens per request; host times of the scheduler's parts, max over "
                   "ranks"},
        "config5": {
            "sessions": SESSIONS * world, "per_gpu": SESSIONS,
            "prefill_tok_s": c5_prefill_tokens / (c5_prefill_ms / 1e3),
            "decode_tok_s": job_rate(SESSIONS * c5_rounds, world, c5_decode_ms),
            "decode_ms_per_round": c5_decode_ms / c5_rounds,
            "rounds": c5_rounds, "prompt_lengths_rank0": c5["lengths"],
            "how": "each rank its 8 sessions (prompts log-uniform [512, 32768], seed "
                   "(5, rank)), prefilled in 512-row passes (device-timed per "
                   "session), then 64 ForwardBatchInputs rounds of the 8 rows; "
                   "aggregate tokens over the max time over ranks"},
        "load": {"seconds": load_s_max, "weight_bytes": int(model.weight_bytes),
                 "host_to_device_gb_s": model.weight_bytes / load_s_max / 1e9,
                 "how": "Model::Load from host memory (pinned staging, 4 reader "
                        "threads) plus packing the decode copies on the device; max "
                        "over ranks"},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    ranks.close()


if __name__ == "__main__":
    main()
