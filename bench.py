"""Benchmark: paged MLA decode serving step on 1..N GPUs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)

Workload (config 5): 512 concurrent sequences, lengths log-uniform in
[128, 65536] (seeded), 8 layers, Q8_0 paged KV with block size 64, 20 heads,
576-wide latent rows N(0,1) with 1% x20 outliers.  Sequences are sharded
across ranks by greedy LPT on their token counts; each GPU owns its pool.
A step appends one token per sequence per layer and runs decode attention on
every layer.  No collective runs inside the timed region.

Printed JSON (rank 0): value = ctx-tokens/s of the whole job (sum over ranks of
the context tokens attended, / max-over-ranks device time); `e2e` = the same
through the host-buffer API (kvcache_append_batch / kvcache_mla_decode with
pinned host buffers, copies inside); `roofline` for the decode kernel (HBM,
algorithmic bytes = 612 B per context token + q + out + tables); the CPU
oracle timed on a bounded sample as `cpu_baseline`.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mobile-moe.zig_b200"))

R, P, W, H = 512, 64, 576, 20
N_SEQS, N_LAYERS, BS = 512, 8, 64
LEN_LO, LEN_HI = 128, 65536
SEED = 5
OUTLIER_P = 0.01
SCALE = float(np.float32(1.0 / math.sqrt(192.0)))
Q8_ROW_BYTES = 18 * 34  # 612
METRIC = "paged MLA decode ctx-tokens/s (config 5 serving step, Q8_0 KV)"
# what the decode computes in: Q8_0 KV; QK exact in int8 (q as two int8 digits,
# int32 per Q8_0 block); V and P in f16; f32 accumulation and softmax
DTYPE = "q8_0 KV; int8 QK exact; f16 PV; f32 accumulate"
CPU_DTYPE = "q8_0 KV dequantized to f32; f32 arithmetic"
UNIT = "ctx-tokens/s"


def config5_lengths(seed=SEED, n=N_SEQS):
    rng = np.random.default_rng(seed)
    u = rng.uniform(math.log(LEN_LO), math.log(LEN_HI), n)
    return np.minimum(np.floor(np.exp(u)).astype(np.int64), LEN_HI)


from sharding import aggregate_throughput, lpt_partition  # noqa: E402


def read_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def read_traffic_profile():
    """Per-context-token DRAM bytes of the decode kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "decode_tc_config5_ncu.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_ctx_token:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []  # (host arrival time, csv line)
        self.window = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def mark(self, t0, t1):
        """Host-time bounds of the timed region: only samples inside it are summarised
        (plus one sampling period after it, for a sample taken inside but read late)."""
        self.window = (t0, t1 + 0.03)

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=5)

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for t, ln in self.lines:
            if self.window and not (self.window[0] <= t <= self.window[1]):
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline (oracle)
def cpu_sample(n_threads, target_tokens, seed=SEED):
    """A bounded sample of the config-5 workload for the CPU restatement:
    sequences drawn from the same length distribution, one layer, Q8_0."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import kvoracle

    lens_all = config5_lengths(seed + 1000, 4096)
    lens, tot = [], 0
    for L in lens_all:
        if tot >= target_tokens:
            break
        lens.append(int(L))
        tot += int(L)
    nb = sum((L + BS - 1) // BS for L in lens)
    pool = kvoracle.Pool(1, nb, BS, R, P, True)
    offs, tabs, k = [0], [], 0
    for s, L in enumerate(lens):
        need = (L + BS - 1) // BS
        tabs.extend(range(k, k + need))
        k += need
        offs.append(len(tabs))
        rows = kvoracle.gen_rows(seed, 0, np.full(L, s, np.uint32), np.arange(L, dtype=np.uint32), W,
                                 OUTLIER_P, n_threads=n_threads)
        t = np.arange(L)
        pool.put_rows(0, np.array(tabs[offs[s]:offs[s + 1]], np.uint32)[t // BS], t % BS, rows)
    q = np.random.default_rng(seed).standard_normal((len(lens), H, W)).astype(np.float32)
    return pool, np.array(offs, np.uint32), np.array(tabs, np.uint32), np.array(lens, np.uint32), q


def cpu_time(sample, n_threads):
    pool, offs, tabs, lens, q = sample
    t0 = time.perf_counter()
    pool.attention_batch(0, offs, tabs, lens, q, SCALE, n_threads=n_threads)
    return time.perf_counter() - t0, int(lens.sum())


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    cores = host_cores()
    sample = cpu_sample(cores, args.cpu_sample_tokens)
    for _ in range(args.warmup):
        cpu_time(sample, cores)
    dt, toks = 0.0, 0
    for _ in range(args.steps):
        d, t = cpu_time(sample, cores)
        dt += d
        toks += t
    value = toks / dt
    desc = (f"one layer of {len(sample[3])} sequences drawn from the config-5 length distribution "
            f"({int(sample[3].sum())} ctx tokens, 20 heads, Q8_0), oracle C restatement of "
            f"src/inference.zig:572-660 on a pthread mutex/cond FIFO pool (src/thread_pool.zig)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": CPU_DTYPE,
        "data": "synthetic (seeded N(0,1), 1% x20 outliers)",
        "config": {"workload": "config5_sharded_serving_step", "kv_dtype": "q8_0", "heads": H,
                   "kv_rank": R, "rope_dim": P, "sample": desc},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the Zig reference cannot be built here (no zig toolchain); its CPU path is timed "
                "through the C restatement in oracle/",
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm
APPEND_ROWS = 1 << 17
QK_NOPE, V_DIM = 128, 128  # DeepSeek2-Lite head dims (head_dim 192 = 128 + 64 rope)


def measure_mla_step(cache, ids, lens_before, NL, steps, torch, dev, st):
    """Whole MLA decode steps (kvcache_mla_step_dev) on the same cache, all layers:
    RMSNorm + RoPE + k_b absorption, the append, a plan, the decode with LSE over
    the history, the newest-token merge and v_b. One untimed step, then `steps`
    timed with CUDA events per layer. Random f32 weights of the model's shapes."""
    n = ids.size
    g = torch.Generator(device=dev).manual_seed(SEED + 7)
    with torch.cuda.stream(st):
        q = torch.randn((NL, n, H, QK_NOPE + P), device=dev, generator=g)
        kv_a = torch.randn((NL, n, W), device=dev, generator=g)
        norm_w = 1.0 + 0.1 * torch.randn((NL, R), device=dev, generator=g)
        k_b = torch.randn((NL, H * QK_NOPE, R), device=dev, generator=g) / R ** 0.5
        v_b = torch.randn((NL, H * V_DIM, R), device=dev, generator=g) / R ** 0.5
        attn = torch.empty((NL, n, H, V_DIM), device=dev)
    st.synchronize()
    times, tokens = [], 0
    for k in range(1 + steps):
        pos = (lens_before + k).astype(np.uint32)
        for layer in range(NL):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            cache.mla_step_dev(layer, ids, pos, q[layer], kv_a[layer], norm_w[layer], 1e-6, 10000.0, k_b[layer],
                               v_b[layer], QK_NOPE, V_DIM, SCALE, attn[layer], st)
            e1.record(st)
            if k:
                times.append((e0, e1))
                tokens += int((pos.astype(np.int64) + 1).sum())
    st.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in times) / len(times)
    return {"ms_per_layer": ms, "ctx_tokens_per_s": tokens / (ms * 1e-3 * len(times)), "layers": NL,
            "steps": steps, "what": "kvcache_mla_step_dev per layer: RMSNorm, RoPE, k_b absorption, append, "
                                    "plan, decode with LSE over the history, newest-token merge, v_b "
                                    "(q, kv_a after their projections; random f32 weights)"}


def measure_append(kvcu, torch, dev, local_rank, reps=5):
    """Append GB/s on one prefill-sized batch: APPEND_ROWS f32 rows (302 MB,
    larger than L2) quantized into a fresh Q8_0 pool through a block table."""
    nb = APPEND_ROWS // BS
    pool = kvcu.DevicePool(local_rank, 1, nb, BS, R, P, True)
    rows = torch.randn((APPEND_ROWS, W), dtype=torch.float32, device=dev)
    seq = torch.zeros(APPEND_ROWS, dtype=torch.int32, device=dev)
    pos = torch.arange(APPEND_ROWS, dtype=torch.int32, device=dev)
    toff = torch.tensor([0, nb], dtype=torch.int32, device=dev)
    tables = torch.randperm(nb, device=dev).to(torch.int32)
    st = torch.cuda.current_stream(dev)
    pool.append(0, rows, seq, pos, toff, tables, stream=st)  # warm-up
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        pool.append(0, rows, seq, pos, toff, tables, stream=st)
    e1.record(st)
    torch.cuda.synchronize(dev)
    dt = e0.elapsed_time(e1) / 1e3 / reps
    # gather/dequant of the same rows back to f32 (getKVCompressed + getKPe for
    # every position): 612 B in (+8 B of row indices) and 2,304 B out per row
    out = torch.empty_like(rows)
    pool.gather_rows(0, seq, pos, toff, tables, out, stream=st)  # warm-up
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(st)
    for _ in range(reps):
        pool.gather_rows(0, seq, pos, toff, tables, out, stream=st)
    g1.record(st)
    torch.cuda.synchronize(dev)
    gdt = g0.elapsed_time(g1) / 1e3 / reps
    status = pool.status()
    pool.close()
    if status:
        raise RuntimeError(f"append/gather benchmark hit device status {status:#x}")
    return (APPEND_ROWS * (2304 + Q8_ROW_BYTES + 8) / dt / 1e9,
            APPEND_ROWS * (Q8_ROW_BYTES + 8 + 2304) / gdt / 1e9)

# ------------------------------------------------------------------ config 4 (second bench figure)
C4_SEQS, C4_LAYERS, C4_LO, C4_HI, C4_SEED = 64, 4, 8192, 32768, 4


def measure_config4(kvcu, torch, dev, local_rank, peak, steps=10, warmup=3):
    """BASELINE config 4 on this GPU: 64 sequences with lengths uniform in
    [8192, 32768], 4 layers, Q8_0, block size 64, 20 heads; a step appends one
    token per sequence per layer, then decodes (fused Q8_0 dequant) each layer.
    Device-resident inputs, CUDA events around `steps` steps after `warmup`."""
    lens0 = np.random.default_rng(C4_SEED).integers(C4_LO, C4_HI + 1, C4_SEQS).astype(np.int64)
    n, NL = C4_SEQS, C4_LAYERS
    total = warmup + steps
    nb = int(sum((int(L) + total + BS - 1) // BS for L in lens0)) + 8
    cache = kvcu.KVCache.with_blocks(NL, R, P, nb, BS, quantized=True, device=local_rank)
    for _ in range(n - 1):
        cache.seq_create()
    ids = np.arange(n, dtype=np.uint32)
    for i in range(n):
        cache.seq_ensure_capacity(i, int(lens0[i]) + total)
    for layer in range(NL):
        cache.prefill_synthetic(layer, ids, lens0, C4_SEED, OUTLIER_P)
    st = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        pos_dev = torch.stack([torch.from_numpy((lens0 + k).astype(np.int32)) for k in range(total)]).to(dev)
        ids_dev = torch.from_numpy(ids.astype(np.int32)).to(dev)
        rows = torch.empty((total, NL, n, W), dtype=torch.float32, device=dev)
        for k in range(total):
            for layer in range(NL):
                kvcu.synth_rows(C4_SEED, layer, ids_dev, pos_dev[k], W, rows[k, layer], OUTLIER_P, st)
        qs = torch.randn((NL, n, H, W), device=dev, generator=torch.Generator(device=dev).manual_seed(C4_SEED))
        outs = torch.empty((NL, n, H, R), dtype=torch.float32, device=dev)
    st.synchronize()
    dec = []

    def step(k, timed):
        pos_h = (lens0 + k).astype(np.uint32)
        for layer in range(NL):
            cache.appendBatch_dev(layer, ids, pos_h, ids_dev, pos_dev[k], rows[k, layer], st)
            if timed:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(st)
            cache.mlaDecode_dev(layer, ids, qs[layer], SCALE, outs[layer], st)
            if timed:
                e1.record(st)
                dec.append((e0, e1))

    for k in range(warmup):
        step(k, False)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx = 0
    st.synchronize()
    t0.record(st)
    for k in range(warmup, total):
        step(k, True)
        ctx += int((lens0 + k + 1).sum()) * NL
    t1.record(st)
    st.synchronize()
    status = cache.pool().status()
    secs = t0.elapsed_time(t1) / 1e3
    avg_dec = sum(a.elapsed_time(b) for a, b in dec) / len(dec) / 1e3
    per_launch = ctx / len(dec)
    dec_bytes = per_launch * Q8_ROW_BYTES + n * H * W * 4 + n * H * R * 4 + 4 * nb / NL
    cache.close()
    if status:
        raise RuntimeError(f"config 4 hit device status {status:#x}")
    return {"workload": "config4_long_context_q8_step", "n_seqs": n, "layers": NL, "block_size": BS, "heads": H,
            "lengths": f"uniform[{C4_LO},{C4_HI}] seed {C4_SEED}", "steps": steps, "warmup": warmup,
            "ctx_tokens_per_step": ctx // steps, "ms_per_step": 1e3 * secs / steps,
            "ctx_tokens_per_s": ctx / secs,
            "decode": {"GB/s": dec_bytes / avg_dec / 1e9, "frac": dec_bytes / avg_dec / 1e9 / peak,
                       "avg_launch_ms": avg_dec * 1e3, "algorithmic_bytes_per_launch": dec_bytes},
            "what": "per step and layer: append 1 token per sequence (k_append_rows), decode (k_plan when the "
                    "batch changes, k_decode_tc, k_combine); device-resident inputs; KV larger than L2"}


# ------------------------------------------------------------------ prefill (causal multi-query attention)
PREFILL_LEN = 4096


def measure_config3(kvcu, torch, dev, local_rank, peak, reps=20):
    """MLA decode over an f32 paged cache, 16 sequences with
    context lengths uniform in [1, 4096], block size 16, 20 heads, one layer
    (the CUDA-core kernel; f32 pools have no tensor-core path).  2,304 B per
    context token; the 75 MB of KV fit in L2, so this is a latency-sized case."""
    lens = np.random.default_rng(3).integers(1, 4097, 16).astype(np.int64)
    n = lens.size
    nb = int(sum((int(L) + 15) // 16 for L in lens)) + 4
    c = kvcu.KVCache.with_blocks(1, R, P, nb, 16, quantized=False, device=local_rank)
    for _ in range(n - 1):
        c.seq_create()
    ids = np.arange(n, dtype=np.uint32)
    for i in range(n):
        c.seq_ensure_capacity(i, int(lens[i]))
    c.prefill_synthetic(0, ids, lens, 3, 0.0)
    st = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        q = torch.randn((n, H, W), device=dev, generator=torch.Generator(device=dev).manual_seed(3))
        out = torch.empty((n, H, R), device=dev)
    st.synchronize()
    c.mlaDecode_dev(0, ids, q, SCALE, out, st)  # plan + warm-up
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        c.mlaDecode_dev(0, ids, q, SCALE, out, st)
    e1.record(st)
    st.synchronize()
    status = c.pool().status()
    c.close()
    if status:
        raise RuntimeError(f"config 3 hit device status {status:#x}")
    secs = e0.elapsed_time(e1) / 1e3 / reps
    ctx = int(lens.sum())
    gbs = (ctx * 2304 + n * H * (W + R) * 4) / secs / 1e9
    return {"workload": "config3_f32_decode", "n_seqs": n, "ctx_tokens": ctx, "ms_per_decode": secs * 1e3,
            "ctx_tokens_per_s": ctx / secs, "GB/s": gbs, "frac": gbs / peak,
            "kernel": "k_decode (CUDA cores, f32 pool) + k_combine",
            "note": "the KV (75 MB) is smaller than L2: a latency-sized case"}


def measure_prefill(kvcu, torch, dev, local_rank, reps=5):
    """mlaAttentionBatch over a 4,096-token prompt of one sequence (one layer,
    Q8_0, block size 64, 20 heads): the prompt's rows are appended, then every
    position attends causally to itself and the positions before it, in one
    call (kvcache_mla_attention_batch_dev).  Prompt tokens/s and the context
    tokens attended (sum of 1..4096) per second."""
    L = PREFILL_LEN
    c = kvcu.KVCache.with_blocks(1, R, P, (L + BS - 1) // BS + 2, BS, quantized=True, device=local_rank)
    c.seq_ensure_capacity(0, L)
    c.prefill_synthetic(0, [0], [L], SEED + 9, OUTLIER_P)
    st = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        q = torch.randn((L, H, W), device=dev, generator=torch.Generator(device=dev).manual_seed(SEED + 9))
        out = torch.empty((L, H, R), device=dev)
    st.synchronize()
    c.mlaAttentionBatch_dev(0, 0, 0, q, SCALE, out, st)  # warm-up
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        c.mlaAttentionBatch_dev(0, 0, 0, q, SCALE, out, st)
    e1.record(st)
    st.synchronize()
    status = c.pool().status()
    c.close()
    if status:
        raise RuntimeError(f"prefill hit device status {status:#x}")
    secs = e0.elapsed_time(e1) / 1e3 / reps
    ctx = L * (L + 1) // 2
    return {"prompt_tokens": L, "prompt_tokens_per_s": L / secs, "ms_per_prompt_layer": secs * 1e3,
            "ctx_tokens_per_s": ctx / secs,
            "what": "one layer of a 4,096-token prompt: every position attends causally (one causal plan, one "
                    "decode launch, one combine; the prefix re-reads are served from L2)"}


# ------------------------------------------------------------------ checkpoint round trip (config 5)
class _DeviceBytes:
    """Zero-copy view of device memory the library owns, for torch."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (int(nbytes),), "typestr": "|u1", "data": (int(ptr), False),
                                         "version": 3}


def _pool_views(cache, torch, dev):
    d = cache.pool().describe()
    rows = d.n_layers * d.num_blocks * d.block_size
    return (torch.as_tensor(_DeviceBytes(d.qs, rows * 32 * d.nblk), device=dev),
            torch.as_tensor(_DeviceBytes(d.sc, rows * 2 * d.nblk), device=dev))


def checkpoint_roundtrip(kvcu, torch, dev, cache, local_rank, rank, NL, nb, n, directory, serve=None):
    """saveToFile / loadFromFile of this rank's whole cache (the v2 container:
    header, every sequence's length and block table, the full Q8_0 pool in the
    reference's 34-byte block order) into a fresh cache, compared bit for bit:
    the payload and scale pools on the device, lengths and tables on the host.
    The save runs in the background (kvcache_save_to_file_v2_async) while
    `serve()` keeps issuing decode steps, which are timed (wall clock)."""
    import shutil
    import tempfile

    directory = directory or tempfile.gettempdir()
    need = cache.pool().describe().checkpoint_bytes + 64 * 1024 * 1024
    free = shutil.disk_usage(directory).free
    if free < need:
        return {"skipped": f"{free / 1e9:.1f} GB free in {directory}, the file needs {need / 1e9:.1f} GB"}
    path = os.path.join(directory, f"kvcache_ckpt_rank{rank}_{os.getpid()}.bin")
    torch.cuda.synchronize()
    served, t_served = 0, 0.0
    try:
        t0 = time.perf_counter()
        job = cache.saveToFileV2Async(path)
        while not job.done():
            if serve is None:
                time.sleep(0.01)
                continue
            ts = time.perf_counter()
            serve()
            t_served += time.perf_counter() - ts
            served += 1
        job.wait()
        t_save = time.perf_counter() - t0
        size = os.path.getsize(path)
        fresh = kvcu.KVCache.with_blocks(NL, R, P, nb, BS, quantized=True, device=local_rank)
        t0 = time.perf_counter()
        fresh.loadFromFileV2(path)
        t_load = time.perf_counter() - t0
    finally:
        if os.path.exists(path):
            os.remove(path)
    same_meta = fresh.num_seqs == cache.num_seqs and all(
        fresh.seq_len(i) == cache.seq_len(i) and np.array_equal(fresh.seq_block_table(i), cache.seq_block_table(i))
        for i in range(cache.num_seqs))
    qa, sa = _pool_views(cache, torch, dev)
    qb, sb = _pool_views(fresh, torch, dev)
    same_pool = bool(torch.equal(qa, qb)) and bool(torch.equal(sa, sb))
    pool_bytes = qa.numel() + sa.numel()
    del qa, sa, qb, sb
    fresh.close()
    return {"bytes": size, "pool_bytes": pool_bytes, "sequences": n, "bit_exact": bool(same_meta and same_pool),
            "save_GB/s": size / t_save / 1e9, "load_GB/s": size / t_load / 1e9, "save_s": t_save, "load_s": t_load,
            "save": "in the background (kvcache_save_to_file_v2_async) while decode steps kept running",
            "decode_steps_during_save": served,
            "ms_per_decode_step_during_save": (1e3 * t_served / served) if served else None,
            "what": "kvcache_save_to_file_v2 -> kvcache_load_from_file_v2 into a fresh cache; pools compared on the "
                    "device, lengths and block tables on the host; outside the timed region"}


# ------------------------------------------------------------------ multi-GPU output check
def multi_gpu_check(kvcu, torch, dist, dev, local_rank, rank, world, parts, lens_all, n_appended, layer, outs_layer):
    """Outputs of the last timed step for a sample of every rank's sequences
    (its shortest and its median-length one), gathered to rank 0 with an NCCL
    all-gather, against the same sequences decoded alone in a fresh cache on
    rank 0's GPU (rebuilt from the seeded generator).  Returns the max relative
    error per (sequence, head) row on rank 0, None elsewhere."""
    per_rank = 2
    picks = []
    for p in parts:
        o = sorted(p, key=lambda s: (int(lens_all[s]), s))
        picks.append([o[0], o[len(o) // 2]] if o else [])
    mine = [parts[rank].index(s) for s in picks[rank]]
    local = torch.zeros((per_rank, H, R), dtype=torch.float32, device=dev)
    if mine:
        local[:len(mine)] = outs_layer[torch.tensor(mine, device=dev)]
    if world > 1:
        bufs = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(bufs, local)
    else:
        bufs = [local]
    if rank != 0:
        return None
    sample = [s for p in picks for s in p]
    got = torch.cat([bufs[r][:len(picks[r])] for r in range(world)])
    L = np.array([int(lens_all[s]) + n_appended for s in sample], np.int64)
    m = len(sample)
    nb = int(sum((int(x) + BS - 1) // BS for x in L)) + 4
    ref = kvcu.KVCache.with_blocks(layer + 1, R, P, nb, BS, quantized=True, device=local_rank)
    for _ in range(m - 1):
        ref.seq_create()
    ids = np.arange(m, dtype=np.uint32)
    for i in range(m):
        ref.seq_ensure_capacity(i, int(L[i]))
    ref.prefill_synthetic(layer, ids, L, SEED, OUTLIER_P, seq_tags=np.array(sample, np.int64))
    qtag = (np.array(sample, np.int64) * 64)[:, None] + np.arange(H)[None, :]
    qb = torch.from_numpy(qtag.reshape(-1).astype(np.int32)).to(dev)
    qc = torch.zeros(m * H, dtype=torch.int32, device=dev)
    q = torch.empty((m, H, W), dtype=torch.float32, device=dev)
    kvcu.synth_rows(SEED + 1, 100 + layer, qb, qc, W, q.view(m * H, W), 0.0)
    want = torch.empty((m, H, R), dtype=torch.float32, device=dev)
    ref.mlaDecode_dev(layer, ids, q, SCALE, want)
    torch.cuda.synchronize()
    status = ref.pool().status()
    ref.close()
    g, w = got.double(), want.double()
    den = w.abs().amax(dim=-1)
    err = ((g - w).abs().amax(dim=-1) / torch.where(den > 0, den, torch.ones_like(den))).max().item()
    return {"max_rel_err": err, "tolerance": 1e-3, "ok": bool(err <= 1e-3 and status == 0), "layer": layer,
            "sequences": m, "ctx_tokens": int(L.sum()),
            "gather": "NCCL all_gather of each rank's sample rows to rank 0" if world > 1 else "single rank",
            "reference": "the same sequences decoded alone in a fresh cache on rank 0's GPU, rebuilt from the "
                         "seeded generator"}


def bind_to_gpu_node(torch, dev_index):
    """Run this process on the CPUs of the NUMA node that the GPU's PCIe root
    hangs off, so that the pinned host buffers it touches first afterwards (q,
    out, rows, the cache's staging) are local to the GPU: with 8 ranks, buffers
    on the other socket send every host<->device byte over the socket link.
    Best effort; returns (node, previous CPU set) or (None, None)."""
    try:
        prev = os.sched_getaffinity(0)
        p = torch.cuda.get_device_properties(dev_index)
    except (OSError, AttributeError, RuntimeError, AssertionError):
        return None, None
    node, cpus = None, set()
    try:  # the kernel's view: the device's NUMA node and that node's CPUs
        bus = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node >= 0:
            with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
                for part in f.read().strip().split(","):
                    lo, _, hi = part.partition("-")
                    cpus.update(range(int(lo), int(hi or lo) + 1))
    except (OSError, ValueError):
        node, cpus = None, set()
    if not cpus:  # else the driver's view (a read-only NVML query): the device's ideal CPU set
        try:
            import pynvml

            pynvml.nvmlInit()
            try:
                h = pynvml.nvmlDeviceGetHandleByPciBusId(
                    f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")
                words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
                for w, word in enumerate(words):
                    cpus.update(64 * w + b for b in range(64) if (int(word) >> b) & 1)
                node = "nvml"
            finally:
                pynvml.nvmlShutdown()
        except Exception:  # no NVML binding or no answer: leave the process as it is
            return None, None
    cpus &= prev
    if not cpus or cpus == prev:
        return (node if cpus else None), None
    os.sched_setaffinity(0, cpus)
    return node, prev


def physical_gpu(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import kvcu

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    numa_node, all_cpus = bind_to_gpu_node(torch, local_rank)
    kvcu.init(local_rank)
    NL = args.layers
    lens_all = config5_lengths(n=args.seqs)
    parts, loads = lpt_partition(lens_all, world)
    mine = np.array(parts[rank], np.int64)
    lens0 = lens_all[mine]
    n = mine.size
    # step indices: timed layered steps, per-layer steps (2 warm + steps), e2e
    # (layered then per-layer), then the MLA steps
    total_steps = (args.warmup + args.steps + 2 + args.steps + args.e2e_warmup + 2 * args.e2e_steps + 1 + 1
                   + args.mla_steps)
    nb = int(sum((int(L) + total_steps + BS - 1) // BS for L in lens0)) + 8
    cache = kvcu.KVCache.with_blocks(NL, R, P, nb, BS, quantized=True, device=local_rank)
    for _ in range(n - 1):
        cache.seq_create()
    ids = np.arange(n, dtype=np.uint32)
    for i in range(n):
        cache.seq_ensure_capacity(i, int(lens0[i]) + total_steps)
    # ---- prefill (device generator + batched append); also the large-append measurement
    t_pre = time.perf_counter()
    for layer in range(NL):
        cache.prefill_synthetic(layer, ids, lens0, SEED, OUTLIER_P, seq_tags=mine)
    torch.cuda.synchronize()
    t_pre = time.perf_counter() - t_pre

    st = torch.cuda.Stream(device=dev)
    W_steps = args.warmup + args.steps
    # per-step inputs, resident in HBM before timing
    with torch.cuda.stream(st):
        pos_dev = torch.empty((total_steps, n), dtype=torch.int32, device=dev)
        for k in range(total_steps):
            pos_dev[k] = torch.from_numpy((lens0 + k).astype(np.int32)).to(dev)
        ids_dev = torch.from_numpy(ids.astype(np.int32)).to(dev)
        tags_dev = torch.from_numpy(mine.astype(np.int32)).to(dev)
        rows = torch.empty((W_steps, NL, n, W), dtype=torch.float32, device=dev)
        for k in range(W_steps):
            for layer in range(NL):
                kvcu.synth_rows(SEED, layer, tags_dev, pos_dev[k], W, rows[k, layer], OUTLIER_P, st)
        qs = torch.empty((NL, n, H, W), dtype=torch.float32, device=dev)
        qtag = (mine.astype(np.int64) * 64)[:, None] + np.arange(H)[None, :]
        qb = torch.from_numpy(qtag.reshape(-1).astype(np.int32)).to(dev)
        qc = torch.zeros(n * H, dtype=torch.int32, device=dev)
        for layer in range(NL):
            kvcu.synth_rows(SEED + 1, 100 + layer, qb, qc, W, qs[layer].view(n * H, W), 0.0, st)
        outs = torch.empty((NL, n, H, R), dtype=torch.float32, device=dev)
    st.synchronize()

    ev = {"dec": [], "launches": 0}

    def step(k, timed, per_layer=False):
        """One serving step: append one token per sequence in every layer, then
        decode every layer.  Default: all layers in one append launch and one
        persistent decode launch (the layers' inputs of this synthetic step are
        all known up front); per_layer: the call sequence a model's layer loop
        makes (append + decode per layer)."""
        pos_h = (lens0 + k).astype(np.uint32)
        rk = rows[k % W_steps]
        if per_layer:
            for layer in range(NL):
                cache.appendBatch_dev(layer, ids, pos_h, ids_dev, pos_dev[k], rk[layer], st)
                ev["launches"] += cache.last_launches
                if timed:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                cache.mlaDecode_dev(layer, ids, qs[layer], SCALE, outs[layer], st)
                ev["launches"] += cache.last_launches
                if timed:
                    e1.record(st)
                    ev["dec"].append((e0, e1, 1))
            return
        cache.appendLayers_dev(0, ids, pos_h, ids_dev, pos_dev[k], rk, st)
        ev["launches"] += cache.last_launches
        if timed:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
        cache.mlaDecodeLayers_dev(0, ids, qs, SCALE, outs, st)
        ev["launches"] += cache.last_launches
        if timed:
            e1.record(st)
            ev["dec"].append((e0, e1, NL))

    def barrier():
        if world > 1:
            dist.barrier()

    def timed_steps(k0, count, per_layer):
        """`count` steps from step index k0 between CUDA events on the stream;
        returns (seconds, ctx tokens attended over all layers)."""
        ev["dec"].clear()
        ev["launches"] = 0
        toks = 0
        t_a, t_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t_a.record(st)
        for k in range(k0, k0 + count):
            step(k, True, per_layer)
            toks += int((lens0 + k + 1).sum()) * NL
        t_b.record(st)
        st.synchronize()
        return t_a, t_b, toks

    # the clock sampler runs from before the warm-up (nvidia-smi takes a moment to
    # start); only the samples that arrive inside the timed region are kept
    with ClockSampler(physical_gpu(local_rank)) as clk:
        for k in range(args.warmup):
            step(k, False)
        st.synchronize()
        barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        torch.cuda.nvtx.range_push("timed")
        t_start, t_end, ctx_tokens = timed_steps(args.warmup, args.steps, False)
        torch.cuda.nvtx.range_pop()
        clk.mark(h0, time.perf_counter())
    barrier()
    torch.cuda.synchronize()
    elapsed = t_start.elapsed_time(t_end) / 1e3
    launches = ev["launches"]
    # decode kernel roofline: one launch covers `nl` layers of one step
    dec_ms = [e0.elapsed_time(e1) for e0, e1, _ in ev["dec"]]
    layers_per_launch = ev["dec"][0][2]
    avg_dec = sum(dec_ms) / len(dec_ms) / 1e3
    avg_ctx_per_launch = ctx_tokens / len(dec_ms)
    tables_bytes = 4 * sum((int(L) + BS - 1) // BS for L in lens0)
    dec_bytes = (avg_ctx_per_launch * Q8_ROW_BYTES + layers_per_launch * (n * H * W * 4 + n * H * R * 4)
                 + tables_bytes)
    # outputs of the last timed step, checked outside the timed region: a sample
    # of every rank's sequences gathered to rank 0 (NCCL) against the same
    # sequences decoded alone there
    mg_check = multi_gpu_check(kvcu, torch, dist, dev, local_rank, rank, world, parts, lens_all, W_steps, NL - 1,
                               outs[NL - 1])

    # ---- cross-rank aggregation (outside the timed region)
    job_tokens, job_time = aggregate_throughput(ctx_tokens, elapsed, dist if world > 1 else None, dev)
    # per-GPU decode bandwidth, averaged over ranks
    dec_gbs = aggregate_throughput(dec_bytes / avg_dec, 0.0, dist if world > 1 else None, dev)[0] / world / 1e9
    value = job_tokens / job_time

    # ---- the same steps as a model's layer loop issues them (append + decode per layer)
    k_pl = W_steps
    for k in range(k_pl, k_pl + 2):
        step(k, False, True)
    barrier()
    torch.cuda.synchronize()
    pl_a, pl_b, pl_tokens = timed_steps(k_pl + 2, args.steps, True)
    pl_dec = sum(e0.elapsed_time(e1) for e0, e1, _ in ev["dec"]) / len(ev["dec"]) / 1e3
    pl_tok, pl_time = aggregate_throughput(pl_tokens, pl_a.elapsed_time(pl_b) / 1e3, dist if world > 1 else None,
                                           dev)
    per_layer = {"value": pl_tok / pl_time, "unit": UNIT, "ms_per_step": 1e3 * pl_time / args.steps,
                 "avg_decode_layer_ms": pl_dec * 1e3,
                 "what": "the same config-5 steps issued per layer (append launch, decode + combine per layer), as "
                         "a model's layer loop calls the cache"}

    # ---- e2e through the host-buffer API (pinned host memory, copies inside)
    # Measured on this pool's 8-GPU boxes (config 5, e2e ctx-tokens/s): N=4 in place 10.6 G, q by DMA
    # 9.8 G; N=8 in place 8.5 G, q by DMA 13.2 G, both by DMA 10.8 G. With 8 ranks the kernels' own
    # reads of q over the shared host links fall behind one large DMA per step.
    host_io = args.host_io if args.host_io != "scale" else ("copy_in" if world >= 8 else "auto")
    cache.set_host_io({"auto": cache.HOST_IO_AUTO, "copy": cache.HOST_IO_COPY,
                       "copy_in": cache.HOST_IO_COPY_IN}[host_io])
    q_host = qs.cpu().pin_memory()
    out_host = torch.empty((NL, n, H, R), dtype=torch.float32).pin_memory()
    rows_host = torch.empty((NL, n, W), dtype=torch.float32).pin_memory()
    rows_host.copy_(rows[0])  # same distribution; content does not change the work
    base = k_pl + 2 + args.steps

    def e2e_step(k, per_layer=False):
        pos_h = (lens0 + base + k).astype(np.uint32)
        if per_layer:
            for layer in range(NL):
                cache.appendBatch(layer, ids, pos_h, rows_host[layer].numpy())
                cache.mlaDecode_ptr(layer, n, ids, q_host[layer].data_ptr(), H, SCALE, out_host[layer].data_ptr())
                _ = out_host[layer, 0, 0, 0].item()
            return
        # one call for the whole step: appends and decodes of every layer, one synchronise
        cache.appendDecodeLayers_ptr(0, NL, n, ids, pos_h, rows_host.data_ptr(), q_host.data_ptr(), H, SCALE,
                                     out_host.data_ptr())
        _ = out_host[NL - 1, 0, 0, 0].item()

    def e2e_run(k0, count, per_layer):
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        toks = 0
        for k in range(k0, k0 + count):
            e2e_step(k, per_layer)
            toks += int((lens0 + base + k + 1).sum()) * NL
        torch.cuda.synchronize()
        secs = time.perf_counter() - t0
        tok, tm = aggregate_throughput(toks, secs, dist if world > 1 else None, dev)
        return tok / tm if tm > 0 else None

    for k in range(args.e2e_warmup):
        e2e_step(k)
    e2e_value = e2e_run(args.e2e_warmup, args.e2e_steps, False)
    e2e_mapped = cache.last_decode_mapped
    kk = args.e2e_warmup + args.e2e_steps
    e2e_step(kk, True)  # warm the per-layer host path
    per_layer["e2e"] = e2e_run(kk + 1, args.e2e_steps, True)
    h2d = NL * n * (W * 4 + 8 + H * W * 4)
    d2h = NL * n * H * R * 4
    e2e_end = kk + 1 + args.e2e_steps

    mla = measure_mla_step(cache, ids, lens0 + base + e2e_end, NL, args.mla_steps,
                           torch, dev, st)
    append_gbs, gather_gbs = measure_append(kvcu, torch, dev, local_rank)
    clk_sum = clk.summary()

    peak, peak_kind = read_peaks()
    c4 = None if args.no_config4 else measure_config4(kvcu, torch, dev, local_rank, peak)
    prefill = measure_prefill(kvcu, torch, dev, local_rank)
    c3 = measure_config3(kvcu, torch, dev, local_rank, peak)
    def serve_decode():
        # one decode step of every layer (reads only, so the pool stays as saved), finished
        cache.mlaDecodeLayers_dev(0, ids, qs, SCALE, outs, st)
        st.synchronize()

    ckpt = None if args.no_checkpoint else checkpoint_roundtrip(kvcu, torch, dev, cache, local_rank, rank, NL, nb, n,
                                                                args.ckpt_dir, serve_decode)
    if world > 1 and ckpt is not None:
        # every rank's round trip must be exact
        ok = torch.tensor([1.0 if ckpt.get("bit_exact") else 0.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        ckpt["all_ranks_bit_exact"] = bool(ok.item() == 1.0)
    traffic_per_tok = read_traffic_profile()
    if rank == 0:
        if all_cpus:
            os.sched_setaffinity(0, all_cpus)  # the CPU baseline uses every host core
        cores = host_cores()
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            sample = cpu_sample(cores, args.cpu_sample_tokens)
            dt, toks = cpu_time(sample, cores)
            # the reference's default pool size (src/inference.zig:149), same sample
            dt4, toks4 = cpu_time(sample, 4)
            cpu = {"value": toks / dt, "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"one layer, {len(sample[3])} sequences from the config-5 length "
                             f"distribution ({toks} ctx tokens, 20 heads, Q8_0); oracle C "
                             f"restatement on a pthread FIFO pool, {cores} threads",
                   "reference_default_threads": {"threads": 4, "value": toks4 / dt4}}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * job_time / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": DTYPE,
            "data": "synthetic (seeded N(0,1) rows with 1% x20 outliers, random q)",
            "config": {"workload": ("config5_sharded_serving_step" if (args.seqs, NL) == (N_SEQS, N_LAYERS)
                                    else f"config5_reduced_{args.seqs}seqs_{NL}layers"), "n_seqs": args.seqs,
                       "layers": NL, "block_size": BS, "heads": H, "kv_rank": R, "rope_dim": P,
                       "kv_dtype": "q8_0", "lengths": f"log-uniform[{LEN_LO},{LEN_HI}] seed {SEED}",
                       "ctx_tokens_per_step": int(job_tokens / args.steps),
                       "parallelism": f"sequence-sharded x{world} (LPT by tokens), no collective",
                       "shard_tokens": loads, "l2": "inputs larger than L2 (>=0.4 GB of KV per layer per GPU)"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "call": "kvcache_append_decode_layers: one host-buffer call per step (all layers), one "
                            "synchronise",
                    "host_numa_node": numa_node,
                    "host_io": host_io,
                    "host_buffers": ("pinned; q copied in by DMA, out written over PCIe by the kernels"
                                     if host_io == "copy_in" else
                                     "pinned; q read and out written over PCIe by the kernels"
                                     if e2e_mapped else "copied in and out around the kernels")},
            "step_form": ("all layers of a step in one append launch and one persistent decode launch "
                          "(kvcache_append_layers_dev + kvcache_mla_decode_layers_dev); per_layer below is the same "
                          "work issued layer by layer"),
            "per_layer": per_layer,
            "roofline": {"kernel": (f"multi-layer decode call ({layers_per_launch} layers: k_decode_tc + k_combine, "
                                    "k_decode_tc ~99.8% of the device time)"),
                         "layers_per_launch": layers_per_launch,
                         "bound": "hbm", "achieved": dec_gbs, "peak": peak, "unit": "GB/s",
                         "frac": dec_gbs / peak, "peak_source": peak_kind,
                         "traffic": (traffic_per_tok * avg_ctx_per_launch if traffic_per_tok else None),
                         "traffic_source": ("not measured in this run: DRAM bytes per ctx token from the ncu "
                                            "capture in profiles/decode_tc_config5_ncu.md (64-sequence, "
                                            "1-layer case larger than L2), scaled by this launch's tokens"),
                         "algorithmic_bytes_per_launch": dec_bytes,
                         "avg_launch_ms": avg_dec * 1e3},
            "gpu_launches": launches,
            "clocks": clk_sum,
            "append": {"GB/s": append_gbs, "rows": APPEND_ROWS,
                       "bytes_per_row": 2304 + Q8_ROW_BYTES + 8, "frac": append_gbs / peak,
                       "what": "one batched f32->Q8_0 append through the block table (prefill-sized)"},
            "gather": {"GB/s": gather_gbs, "rows": APPEND_ROWS, "bytes_per_row": Q8_ROW_BYTES + 8 + 2304,
                       "frac": gather_gbs / peak,
                       "what": "batched Q8_0 -> f32 gather/dequant through the block table (k_gather), "
                               "302 MB out, larger than L2"},
            "mla_step": mla,
            "prefill_s": t_pre,
            "multi_gpu_check": mg_check,
            "prefill": prefill,
            "config3": c3,
        }
        if c4 is not None:
            line["config4"] = c4
        if ckpt is not None:
            line["checkpoint_roundtrip"] = ckpt
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    cache.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--host-io", choices=["scale", "auto", "copy", "copy_in"], default="scale",
                    help="how the host-buffer calls of the e2e figure move q / out (kvcache_set_host_io); "
                         "scale: q read in place by the kernels below 8 ranks, copied by DMA from 8 on")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-warmup", type=int, default=1)
    ap.add_argument("--mla-steps", type=int, default=2, help="timed whole-MLA-step passes (after one untimed)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-sample-tokens", type=int, default=400_000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seqs", type=int, default=N_SEQS, help="sequences (config 5: 512)")
    ap.add_argument("--layers", type=int, default=N_LAYERS, help="layers (config 5: 8)")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 measurement")
    ap.add_argument("--no-checkpoint", action="store_true", help="skip the checkpoint round trip")
    ap.add_argument("--ckpt-dir", default=None, help="directory for the checkpoint file (default: temp dir)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
