#!/usr/bin/env python3
"""Benchmark of the LazyRecall KV-management hot path on B200.

Metric: managed KV tokens/s (score + evict + compact) and the
per-decode-step overhead.  A managed token is one resident (layer, KV head,
position) row that goes through one score -> pool -> select -> compact pass.

Workload: configs[1], a Llama-3-8B-shaped single request (32 layers x 8 KV
heads x head_dim 128, GQA group 4, bf16 K/V ~N(0,1)) at the steady state of
its 8000-step run: a 32768-token protected prompt per head plus the
generation rows the budget allows (budget 2000 -> wall 512,000 slots,
staging 2,048), temporal window 250, protect_recent 32.  One step = one audit
pass at that state:
  scoring of every candidate row of every (layer, head) exactly as
  scoring.py:152-195 composes it (g V^T and Q K^T on cuBLAS, then the
  temporal probability and risk kernels per query chunk), Pool7, the
  allocation-preserving selection of immediate + 250*256 references, and the
  eviction of the immediate prefix (one compaction per layer).
Per-decode-step overhead (reported as decode_overhead_us): the append of one
token to all 32 layers plus the lazy eviction of a 2048-row queue prefix
every 8 steps, amortised: the median 8-step interval over 8 (the mean over
every step is decode_overhead_mean_us).

Inputs are synthetic and seeded; all K/V state (4.6 GB per request) is larger
than L2, so no flush is needed between steps.  Multi-GPU: one independent
request per rank (request sharding, weak scaling), no collective inside the
timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

LAYERS, HEADS, GROUPS, DIM = 32, 8, 4, 128
PROMPT = 32768
BUDGET, AUDIT_PERIOD, WINDOW, EVICT_INTERVAL, PROTECT_RECENT = 2000, 250, 250, 8, 32
SLOTS_PER_STEP = LAYERS * HEADS
WALL = BUDGET * SLOTS_PER_STEP
STAGING = EVICT_INTERVAL * SLOTS_PER_STEP
RETAINED = WALL - STAGING
IMMEDIATE = 2 * SLOTS_PER_STEP  # steady state: audits fall 2 steps after an eviction batch
QUEUED = AUDIT_PERIOD * SLOTS_PER_STEP
GENERATED = 4000  # tokens generated before the measured audit (mid-run)
METRIC = "managed KV tokens/s (score+pool+select+evict audit pass)"


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--decode-steps", type=int, default=64)
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--skip-side", action="store_true",
                        help="skip the configs[2] batch_append and configs[3] recall measurements (N=1 only)")
    parser.add_argument("--skip-large", action="store_true", help="skip the configs[4] measurements")
    parser.add_argument("--large-requests", type=int, default=8, help="configs[4] requests per GPU")
    parser.add_argument("--large-steps", type=int, default=2, help="configs[4] timed passes")
    parser.add_argument("--large-warmup", type=int, default=2, help="configs[4] warm-up passes")
    parser.add_argument("--scoring", choices=["fused", "dropin"], default="fused",
                        help="fused: lrk_temporal_scores per layer; dropin: the reference's per-head composition of "
                             "temporal_probabilities + temporal_risk")
    return parser.parse_args()


def measured_traffic_ratio():
    """DRAM bytes per fused scoring call over its algorithmic bytes, from the
    committed ncu summary of one configs[1] layer call (None when absent)."""
    path = ROOT / "profiles" / "temporal_scores_traffic.json"
    if path.exists():
        return float(json.loads(path.read_text())["traffic_over_algorithmic"])
    return None


def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- workload


def generation_lengths(rng: np.random.Generator) -> np.ndarray:
    """Generation rows per (layer, head) at the audit: RETAINED + IMMEDIATE in
    total, unevenly spread across heads as evictions leave them."""
    total = RETAINED + IMMEDIATE
    weights = rng.uniform(0.7, 1.3, size=LAYERS * HEADS)
    lengths = np.floor(weights / weights.sum() * total).astype(np.int64)
    lengths[: total - lengths.sum()] += 1
    return lengths.reshape(LAYERS, HEADS)


def head_positions(rng: np.random.Generator, generated: int) -> np.ndarray:
    """Prompt positions 0..PROMPT-1, then `generated` surviving generation
    positions: the last PROTECT_RECENT tokens plus an ordered sample of older ones."""
    recent = np.arange(PROMPT + GENERATED - PROTECT_RECENT, PROMPT + GENERATED)
    older = np.sort(rng.choice(np.arange(PROMPT, PROMPT + GENERATED - PROTECT_RECENT), generated - PROTECT_RECENT,
                               replace=False))
    return np.concatenate([np.arange(PROMPT), older, recent]).astype(np.float32)


def build_request(device, seed: int):
    """One request's cache and audit inputs, generated on the device."""
    import torch

    from code_for_iclr27_b200.kvcache import PackedCache

    rng = np.random.default_rng(seed)
    lengths = generation_lengths(rng)
    cache = PackedCache()
    g = torch.Generator(device=device).manual_seed(seed)
    for layer in range(LAYERS):
        head_lens = [PROMPT + int(n) for n in lengths[layer]]
        rows = sum(head_lens)
        keys = torch.randn(rows, DIM, generator=g, device=device).to(torch.bfloat16)
        values = torch.randn(rows, DIM, generator=g, device=device).to(torch.bfloat16)
        positions = torch.from_numpy(np.concatenate([head_positions(rng, int(n)) for n in lengths[layer]]))
        cache.add_layer(keys, values, positions.to(device), head_lens, [PROMPT] * HEADS)
    cache.seen_tokens = PROMPT + GENERATED
    queries = [(torch.randn(WINDOW, HEADS * GROUPS, DIM, generator=g, device=device) * 2).to(torch.bfloat16)
               for _ in range(LAYERS)]
    gradients = [torch.randn(HEADS * GROUPS, DIM, generator=g, device=device) / math.sqrt(DIM)
                 for _ in range(LAYERS)]
    query_positions = torch.arange(PROMPT + GENERATED - WINDOW, PROMPT + GENERATED, dtype=torch.int64,
                                   device=device)
    margin = torch.tensor([1.0], device=device)
    return cache, queries, query_positions, gradients, margin


def config_cfg1(world: int, scoring: str) -> dict:
    """The bench line's config: the configs[1] workload (both arms report it)."""
    return {"workload": "configs[1] llama-3-8b single request, steady-state audit pass",
            "scoring": scoring,
            "layers": LAYERS, "kv_heads": HEADS, "gqa_group": GROUPS, "head_dim": DIM,
            "prompt_rows_per_head": PROMPT, "generation_rows": RETAINED + IMMEDIATE, "budget": BUDGET,
            "temporal_window": WINDOW, "selected_per_audit": IMMEDIATE + QUEUED, "evicted_per_audit": IMMEDIATE,
            "managed_rows_per_request": LAYERS * HEADS * PROMPT + RETAINED + IMMEDIATE,
            "requests_per_gpu": 1,
            "parallelism": f"request-sharded x{world}" if world > 1 else "single request",
            "l2": "no flush: 4.6 GB of K/V per request, larger than L2"}


# ------------------------------------------------------------ instruments


class KernelTimer:
    """CUDA events around one operator's launches, on the launching stream."""

    def __init__(self):
        self.pairs, self.bytes = [], 0

    def wrap(self, function, bytes_of):
        import torch

        def timed(*args):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            result = function(*args)
            end.record()
            self.pairs.append((start, end))
            self.bytes += bytes_of(*args)
            return result

        return timed

    def total_ms(self):
        return sum(a.elapsed_time(b) for a, b in self.pairs)


class LaunchCounter:
    """Counts liblrk kernel launches made through the operator module."""

    KERNELS = {"temporal_probabilities": 1, "temporal_risk": 1, "pool": 1, "compact": 1, "append": 1, "merge": 1,
               "pack": 1}

    def __init__(self, module):
        self.module, self.count = module, 0

    def __getattr__(self, name):
        attribute = getattr(self.module, name)
        if not callable(attribute):
            return attribute

        def counted(*args):
            self.count += self.kernels(name, args)
            return attribute(*args)

        return counted

    def kernels(self, name, args):
        if name == "refine":
            n, segments = args[0].numel(), args[2].numel()
            segment_bits = ((max(1, int(segments - 1).bit_length()) + 7) // 8) * 8 if segments > 1 else 0
            count = args[4]
            bitonic = 1 if 2 <= count <= 32 else 0
            # keys, 4 raw passes x3, pick passes x3, 4+ segment passes x3, picks, scan, fixup, transplant, stats
            return 1 + 12 + 3 * (segment_bits // 8) + 3 * ((32 + segment_bits) // 8) + bitonic + 5
        if name == "batch_append":
            return max(1, math.ceil(len(args[0]) * args[3].shape[1] / 64))
        return self.KERNELS.get(name, 1)


_NVML_SAMPLER = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
key = sys.argv[1]
h = pynvml.nvmlDeviceGetHandleByUUID(key) if key.startswith("GPU-") else pynvml.nvmlDeviceGetHandleByIndex(int(key))
print("ready", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
while True:
    print(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), pynvml.nvmlDeviceGetCurrentClocksEventReasons(h),
          flush=True)
    time.sleep(0.01)
"""


class Clocks:
    """SM clock and throttle reasons sampled during the timed region: NVML
    every 10 ms from a child process (read-only queries; a thread here would
    wait for the interpreter lock the audit's host code holds), plus one
    in-process NVML sample at each end of the region; if the child cannot
    start, an in-process thread samples instead, and without NVML nvidia-smi
    every 200 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index: int):
        self.index, self.process, self.sampler, self.thread, self.handle = index, None, None, None, None
        self.samples, self.nvml, self.maximum, self.error, self.errors = [], [], None, None, None

    def _device_key(self):
        import torch

        uuid = getattr(torch.cuda.get_device_properties(self.index), "uuid", None)
        if uuid is None:
            return str(self.index)
        text = str(uuid)
        return text if text.startswith("GPU-") else "GPU-" + text

    def _sample_here(self):
        import pynvml

        self.nvml.append((pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM), self.maximum,
                          pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)))

    def __enter__(self):
        import tempfile
        import threading

        key = self._device_key()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.handle = (pynvml.nvmlDeviceGetHandleByUUID(key) if key.startswith("GPU-")
                           else pynvml.nvmlDeviceGetHandleByIndex(int(key)))
            self.maximum = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # no NVML: nvidia-smi below
            self.handle, self.error = None, f"nvml: {e}"
        if self.handle is not None:
            try:
                self.errors = tempfile.TemporaryFile(mode="w+")
                self.sampler = subprocess.Popen([sys.executable, "-c", _NVML_SAMPLER, key], stdout=subprocess.PIPE,
                                                stderr=self.errors, text=True)
                first = self.sampler.stdout.readline().split()
                if not (len(first) == 2 and first[0] == "ready"):
                    self.sampler.kill()
                    self.sampler.wait()
                    self.errors.seek(0)
                    lines = self.errors.read().strip().splitlines()
                    self.error = "sampler: " + (lines[-1] if lines else f"exit {self.sampler.returncode}")
                    self.sampler = None
            except OSError as e:
                self.sampler, self.error = None, f"sampler: {e}"
            if self.sampler is None:
                self.stop = threading.Event()

                def sample():
                    while True:
                        try:
                            self._sample_here()
                        except Exception:
                            return
                        if self.stop.wait(0.01):
                            return

                self.thread = threading.Thread(target=sample, daemon=True)
                self.thread.start()
            self._sample_here()
            return self
        try:
            self.process = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                             "--format=csv,noheader,nounits", "-lms", "200"],
                                            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.process = None
        return self

    def __exit__(self, *exc):
        if self.handle is not None:
            try:
                self._sample_here()
            except Exception:
                pass
            if self.thread is not None:
                self.stop.set()
                self.thread.join(timeout=5)
            if self.sampler is not None:
                self.sampler.terminate()
                try:
                    out, _ = self.sampler.communicate(timeout=5)
                except subprocess.TimeoutExpired:
                    self.sampler.kill()
                    out, _ = self.sampler.communicate()
                for line in out.splitlines():
                    parts = line.split()
                    if len(parts) == 2 and parts[0].isdigit() and parts[1].isdigit():
                        self.nvml.append((int(parts[0]), self.maximum, int(parts[1])))
            if self.errors is not None:
                self.errors.close()
            return
        if self.process is None:
            return
        self.process.terminate()
        try:
            out, _ = self.process.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.process.kill()
            out, _ = self.process.communicate()
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.samples.append(parts)

    def summary(self):
        if self.nvml:
            sm = [float(clock) for clock, _, _ in self.nvml]
            reasons = sorted({name for _, _, mask in self.nvml for name, bit in self.REASONS if mask & bit})
            out = {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(self.nvml[0][1]), "reasons": reasons,
                   "samples": len(self.nvml),
                   "source": "nvml, 10 ms, " + ("child process" if self.thread is None else "in-process thread")}
            if self.error:
                out["sampler_error"] = self.error
            return out
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(p[1]) for p in self.samples if p[1].replace(".", "").isdigit()]
        names = [name for name, _ in self.REASONS]
        reasons = sorted({names[i] for p in self.samples for i in range(4) if p[4 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": float(self.samples[0][2]),
                "reasons": reasons, "samples": len(self.samples), "source": "nvidia-smi, 200 ms"}


# --------------------------------------------------------------- CPU side


def cpu_baseline(seed: int = 0):
    """The oracle's restatement of the reference's CPU math path on a bounded
    sample, extrapolated to one full audit pass: one (layer, head) scored by
    temporal_head_scores_reference's algorithm (scoring.py:75-149) at the
    workload's head length, Pool7 + selection over the whole table, and one
    layer's index_select compaction (cache.py:162-167)."""
    from oracle import lrk_oracle as O

    rng = np.random.default_rng(seed)
    lengths = generation_lengths(rng)
    generated = int(lengths[0, 0])
    length = PROMPT + generated
    keys = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((length, DIM), dtype=np.float32)))
    values = O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((length, DIM), dtype=np.float32)))
    queries = rng.standard_normal((WINDOW, GROUPS, DIM), dtype=np.float32) * 2
    grad = rng.standard_normal((GROUPS, DIM), dtype=np.float32) / math.sqrt(DIM)
    kpos = head_positions(rng, generated)
    qpos = np.arange(PROMPT + GENERATED - WINDOW, PROMPT + GENERATED)
    t0 = time.perf_counter()
    O.temporal_head_scores_cpu_path(queries, qpos, keys, kpos, values, PROMPT, length - PROTECT_RECENT, grad, 1.0,
                                    1e-6, 250)
    t_head = time.perf_counter() - t0
    candidates = lengths.reshape(-1) - PROTECT_RECENT
    raw = rng.random(int(candidates.sum()), dtype=np.float32)
    ends = np.cumsum(candidates)
    t0 = time.perf_counter()
    bounds = np.concatenate(([0], ends))
    pooled = O.pool(raw, bounds, 7)
    O.refine(raw, pooled, ends, np.full(len(ends), PROMPT), IMMEDIATE + QUEUED)
    t_select = time.perf_counter() - t0
    rows = HEADS * length
    k16 = rng.integers(0, 65535, size=(rows, DIM), dtype=np.uint16)
    removed = np.sort(rng.choice(rows, IMMEDIATE // LAYERS, replace=False))
    t0 = time.perf_counter()
    O.compact(k16, k16, np.zeros(rows, np.float32), removed)
    t_compact = time.perf_counter() - t0
    total = SLOTS_PER_STEP * t_head + t_select + LAYERS * t_compact
    managed = LAYERS * HEADS * PROMPT + RETAINED + IMMEDIATE
    try:
        from threadpoolctl import threadpool_info

        cores = max([int(info.get("num_threads", 1)) for info in threadpool_info()] or [1])
    except Exception:  # noqa: BLE001
        cores = 1
    return {"value": managed / total, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": (f"numpy oracle: 1 of {SLOTS_PER_STEP} heads scored (Lh={length}, W={WINDOW}, G={GROUPS}, "
                       f"D={DIM}) x{SLOTS_PER_STEP} + full Pool7/selection ({raw.size} scores) + 1 of {LAYERS} "
                       f"layer compactions x{LAYERS}; BLAS threads={cores}, elementwise single-threaded"),
            "seconds": {"head": t_head, "select": t_select, "compact_layer": t_compact,
                        "extrapolated_pass": total}}


def host_cores() -> dict:
    """The host's CPU: logical cores, torch's intra-op threads, model name."""
    import torch

    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads(), "cpu_model": model}


def reference_cpu_sample(seed: int):
    """The reference's own CPU path -- its unchanged Python package installed
    with LAZY_RECALL_BUILD_CUDA=0 (oracle/_ref/py, made by
    oracle/install_ref_py.py) -- on a bounded sample of one configs[1] audit
    pass, extrapolated to the pass:
      * one layer's 8 heads scored by temporal_head_scores_reference
        (scoring.py:75-149: bf16 Q K^T, softmax, risk), x32 layers;
      * pool_score_table's CPU branch (scoring.py:336-353) and refine_arrays
        (selection.py:52-88) over the whole 502,272-score table;
      * one layer's compaction by the CPU branch of remove_positions
        (cache.py:162-167: keep mask, compact_flattened_kv, index_select), x32
        (the immediate prefix touches every layer).
    Returns None when the package is not installed."""
    from oracle.install_ref_py import installed

    where = installed()
    if where is None:
        return None
    if str(where) not in sys.path:
        sys.path.insert(0, str(where))
    import torch
    from lazy_recall._core.cuda_ops import compact_flattened_kv
    from lazy_recall._core.scoring import ScoreSegment, ScoreTable
    from lazy_recall.scoring import pool_score_table, temporal_head_scores_reference
    from lazy_recall.selection import refine_arrays

    rng = np.random.default_rng(seed)
    lengths = generation_lengths(rng)
    g = torch.Generator().manual_seed(seed)
    qpos = torch.arange(PROMPT + GENERATED - WINDOW, PROMPT + GENERATED)
    margin = torch.tensor(1.0)
    t_layer = 0.0
    for head in range(HEADS):
        generated = int(lengths[0, head])
        length = PROMPT + generated
        keys = torch.randn(length, DIM, generator=g).to(torch.bfloat16)
        values = torch.randn(length, DIM, generator=g).to(torch.bfloat16)
        queries = (torch.randn(WINDOW, GROUPS, DIM, generator=g) * 2).to(torch.bfloat16)
        grad = torch.randn(GROUPS, DIM, generator=g) / math.sqrt(DIM)
        kpos = torch.from_numpy(head_positions(rng, generated))
        t0 = time.perf_counter()
        temporal_head_scores_reference(queries, qpos, keys, kpos, values, PROMPT, length - PROTECT_RECENT, grad,
                                       margin, 1e-6, WINDOW)
        t_layer += time.perf_counter() - t0
    candidates = lengths.reshape(-1) - PROTECT_RECENT
    ends = np.cumsum(candidates).tolist()
    segments = [ScoreSegment(l, h, PROMPT, int(c)) for (l, h), c in
                zip(((l, h) for l in range(LAYERS) for h in range(HEADS)), candidates)]
    table = ScoreTable(torch.rand(int(candidates.sum()), generator=g), segments, ends, 0.0)
    t0 = time.perf_counter()
    pooled = pool_score_table(table, 7)
    t_pool = time.perf_counter() - t0
    t0 = time.perf_counter()
    refine_arrays(table, pooled, IMMEDIATE + QUEUED)
    t_select = time.perf_counter() - t0
    rows = int(sum(PROMPT + int(n) for n in lengths[0]))
    keys = torch.randn(rows, DIM, generator=g).to(torch.bfloat16)
    values = torch.randn(rows, DIM, generator=g).to(torch.bfloat16)
    position_rows = torch.arange(rows, dtype=torch.float32).reshape(-1, 1)
    absolute = torch.from_numpy(np.sort(rng.choice(rows, IMMEDIATE // LAYERS, replace=False)))
    t0 = time.perf_counter()
    keep_mask = torch.ones(position_rows.shape[0], dtype=torch.bool)
    keep_mask[absolute] = False
    keep_indices = torch.nonzero(keep_mask, as_tuple=False).reshape(-1)
    compact_flattened_kv(keys, values, keep_indices)
    position_rows.index_select(0, keep_indices)
    t_compact = time.perf_counter() - t0
    total = LAYERS * t_layer + t_pool + t_select + LAYERS * t_compact
    managed = LAYERS * HEADS * PROMPT + RETAINED + IMMEDIATE
    return {"value": managed / total, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": (f"reference package (oracle/_ref/py, LAZY_RECALL_BUILD_CUDA=0): 1 of {LAYERS} layers scored by "
                       f"temporal_head_scores_reference ({HEADS} heads, Lh~{PROMPT + int(lengths[0].mean())}, "
                       f"W={WINDOW}, G={GROUPS}, D={DIM}) x{LAYERS} + pool_score_table + refine_arrays over "
                       f"{table.scores.numel()} scores + 1 of {LAYERS} layer compactions x{LAYERS}"),
            "host": host_cores(),
            "seconds": {"layer_scores": t_layer, "pool": t_pool, "select": t_select, "compact_layer": t_compact,
                        "extrapolated_pass": total}}


def reference_arm(args, rank: int):
    """--impl reference: the reference's own CPU implementation of the path
    (its unchanged Python package, CPU math path), timed on the host cores
    with all of torch's threads; each step is one bounded sample
    (reference_cpu_sample), after --warmup untimed samples.  Falls back to the
    numpy port (cpu_baseline) when the package is not installed.  Under
    torchrun only rank 0 runs."""
    if rank != 0:
        return
    import torch

    torch.set_num_threads(os.cpu_count() or 1)
    sample = reference_cpu_sample if reference_cpu_sample(args.seed) is not None else cpu_baseline
    for i in range(args.warmup):
        sample(args.seed + 100 + i)
    runs = [sample(args.seed + i) for i in range(max(1, args.steps))]
    value = float(np.median([r["value"] for r in runs]))
    first = runs[0]
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": float(np.median([r["seconds"]["extrapolated_pass"] for r in runs]))
            * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded): bf16 K/V ~N(0,1), queries ~N(0,4), margin gradient ~N(0,1/D)",
            "impl": "reference", "config": config_cfg1(args.gpus, "reference CPU path"),
            "cpu_baseline": {k: first[k] for k in ("cores", "kind", "sample")} | {"value": value, "unit": "tokens/s",
                                                                                   "host": host_cores()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm


def fused_bytes(logits, projected_values, key_positions, first, last, query_positions, margin, scale, eps,
                query_chunks=None):
    """The fused scorer's algorithmic bytes: the logits read once, projected
    values and key positions once, the scores written."""
    total = 0
    for lg, f, l in zip(logits, first, last):
        w, g, length = lg.shape
        total += w * g * length * lg.element_size() + g * length * 4 + length * 4 + (l - f) * 4
    return total


def probability_bytes(logits, projected_values, query_positions, key_positions, scale):
    # read logits, write probabilities, read projected values and key positions
    w, g, length = logits.shape
    return w * g * length * (logits.element_size() + 4) + g * length * 4 + length * 4


def measure_cfg1(args, device, world: int, rank: int, distributed: bool, barrier, layer_groups: bool,
                 steps: int, warmup: int, with_e2e: bool):
    """configs[1] audit passes: one request per rank (request sharding), or
    one request split into per-rank layer groups (layer_groups).  Returns the
    raw measurements of this rank."""
    import torch

    from code_for_iclr27_b200 import audit as audit_module
    from code_for_iclr27_b200 import kvcache as kvcache_module
    from code_for_iclr27_b200 import operators
    from code_for_iclr27_b200 import selection as selection_module
    from code_for_iclr27_b200.audit import audit_pass, evict_prefix
    from code_for_iclr27_b200.distributed import lazy_prefix_share, layer_group_audit_pass
    from code_for_iclr27_b200.kvcache import PackedCache

    cache, queries, qpos, gradients, margin = build_request(device, args.seed + (0 if layer_groups else 1000 * rank))
    managed = cache.total_rows()
    if layer_groups:
        # Every rank built the same request; each keeps its contiguous group of layers.
        if LAYERS % world:
            raise SystemExit(f"layer groups need the {LAYERS} layers to split evenly over {world} GPUs")
        mine = slice(rank * (LAYERS // world), (rank + 1) * (LAYERS // world))
        cache = PackedCache(layers=cache.layers[mine], seen_tokens=cache.seen_tokens)
        queries, gradients = queries[mine], gradients[mine]
    C = operators()
    counter = LaunchCounter(C)
    timer = KernelTimer()
    fused = args.scoring == "fused"
    timed_name = "temporal_scores" if fused else "temporal_probabilities"
    patched = (audit_module, kvcache_module, selection_module)
    originals = [module.operators for module in patched]

    def route(provider):
        for module in patched:
            module.operators = provider

    gathers = []

    def one_pass(q=queries, g=gradients, timings=None):
        if layer_groups:
            return layer_group_audit_pass(cache, q, qpos, g, margin, IMMEDIATE, QUEUED, protect_recent=PROTECT_RECENT,
                                          timings=timings)
        return audit_pass(cache, q, qpos, g, margin, IMMEDIATE, QUEUED, PROTECT_RECENT, fused=fused)

    route(lambda: counter)
    try:
        for _ in range(warmup):
            last = one_pass()
        barrier()
        counter.count = 0
        wrapped = timer.wrap(getattr(C, timed_name), fused_bytes if fused else probability_bytes)

        class Timed:
            def __getattr__(self, name):
                if name == timed_name:
                    return wrapped
                return getattr(counter, name)

        timed_ops = Timed()
        route(lambda: timed_ops)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(torch.cuda.current_device()) as clocks:
            barrier()
            start.record()
            for _ in range(steps):
                last = one_pass(timings=gathers)
            end.record()
            barrier()
        elapsed_ms = start.elapsed_time(end)
        # lrk_temporal_scores: visibility, statistics and risk kernels per call (<= 48 segments);
        # layer groups add 3 histogram + 3 pick launches per pass.
        launches = counter.count + len(timer.pairs) * (3 if fused else 1) + (6 * steps if layer_groups else 0)
    finally:
        for module, function in zip(patched, originals):
            module.operators = function

    # Per-decode-step overhead: append one token to every layer, evict a
    # staging-sized queue prefix every EVICT_INTERVAL steps.  With layer
    # groups each rank appends to its own layers and takes its share of each
    # request-wide queue prefix (lazy_prefix_share: one all-gather of the
    # ranks' next queue scores per batch); the audit already evicted its share
    # of the immediate prefix, the first slots of its local queue.
    # The lazy queue follows the immediate prefix, whose rows are already gone
    # (controller.py:154-156: removed_at_audit starts as that prefix).
    first = lazy_prefix_share(last.references.scores, IMMEDIATE) if layer_groups else IMMEDIATE
    queue = last.references[first:]
    removed_at_audit = last.references[:first].groups()
    layers_here = len(cache.layers)
    g = torch.Generator(device=device).manual_seed(args.seed + 7)
    new_keys = torch.randn(EVICT_INTERVAL + args.decode_steps, layers_here, 1, HEADS, 1, DIM, generator=g,
                           device=device).to(torch.bfloat16)

    def decode_step(step):
        nonlocal queue, removed_at_audit
        for layer in range(layers_here):
            cache.append(layer, new_keys[step, layer], new_keys[step, layer], cache.seen_tokens)
        cache.seen_tokens += 1
        if (step + 1) % EVICT_INTERVAL == 0:
            if layer_groups:
                share = lazy_prefix_share(queue.scores, STAGING)
                if share:
                    queue, removed_at_audit = evict_prefix(cache, queue, removed_at_audit, share)
            elif len(queue) >= STAGING:
                queue, removed_at_audit = evict_prefix(cache, queue, removed_at_audit, STAGING)

    for step in range(EVICT_INTERVAL):  # warm-up: one eviction interval, untimed
        decode_step(step)
    barrier()
    # One event per eviction interval (EVICT_INTERVAL steps: the appends and one
    # lazy batch): the step overhead is the median interval over EVICT_INTERVAL,
    # which keeps a stalled interval (the caching allocator mapping a new
    # segment, clocks ramping after the host work) from setting the figure; the
    # mean over all steps is reported beside it.
    marks = [torch.cuda.Event(enable_timing=True)]
    marks[0].record()
    for step in range(EVICT_INTERVAL, EVICT_INTERVAL + args.decode_steps):
        decode_step(step)
        if (step + 1) % EVICT_INTERVAL == 0:
            marks.append(torch.cuda.Event(enable_timing=True))
            marks[-1].record()
    d0, d1 = marks[0], torch.cuda.Event(enable_timing=True)
    d1.record()
    barrier()
    if with_e2e:
        out_arena = measure_arena(args, cache, queries, qpos, gradients, margin, steps, warmup, barrier, g)
    windows = sorted(a.elapsed_time(b) for a, b in zip(marks[:-1], marks[1:]))
    decode_median_ms = (windows[len(windows) // 2] / EVICT_INTERVAL * args.decode_steps if windows
                        else d0.elapsed_time(d1))
    out = {"managed": managed, "elapsed_ms": elapsed_ms, "decode_ms": d0.elapsed_time(d1),
           "decode_median_ms": decode_median_ms, "launches": launches,
           "kernel_ms": timer.total_ms(), "kernel_bytes": timer.bytes, "kernel_launches": len(timer.pairs),
           "timed_name": timed_name, "clocks": clocks.summary(),
           "gather_us": [a.elapsed_time(b) * 1e3 for a, b in gathers]}
    if with_e2e:
        out["arena"] = out_arena
        # End to end through the public API: audit inputs copied from pinned
        # host memory each step, the queue read back (refine_arrays returns
        # host arrays).
        host_queries = [q.cpu().pin_memory() for q in queries]
        host_gradients = [x.cpu().pin_memory() for x in gradients]
        out["h2d"] = sum(q.numel() * q.element_size() for q in host_queries) + sum(x.numel() * 4 for x in host_gradients)
        out["d2h"] = (IMMEDIATE + QUEUED) * (4 + 8 + 8) + 2 * 8

        def e2e_pass():
            one_pass([q.to(device, non_blocking=True) for q in host_queries],
                     [x.to(device, non_blocking=True) for x in host_gradients])

        e2e_pass()  # warm-up
        barrier()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record()
        out["e2e_steps"] = max(1, steps)
        for _ in range(out["e2e_steps"]):
            e2e_pass()
        e_end.record()
        barrier()
        out["e2e_ms"] = e_start.elapsed_time(e_end)
    return out


def measure_arena(args, cache, queries, qpos, gradients, margin, steps: int, warmup: int, barrier, generator):
    """The same request in the gapped per-head arena (arena.ArenaCache): audit
    passes that evict in place, then decode steps whose appends are one
    launch for all layers and whose lazy evictions run on the device from the
    audit's queue (no host round trip) and shift only the touched heads' rows.
    Returns this rank's times."""
    import torch

    from code_for_iclr27_b200.arena import ArenaCache
    from code_for_iclr27_b200.audit import audit_pass

    arena = ArenaCache.from_packed(cache, margin=args.decode_steps + 256)
    torch.cuda.empty_cache()
    for _ in range(warmup):
        last = audit_pass(arena, queries, qpos, gradients, margin, IMMEDIATE, QUEUED, PROTECT_RECENT)
    barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(steps):
        last = audit_pass(arena, queries, qpos, gradients, margin, IMMEDIATE, QUEUED, PROTECT_RECENT)
    a1.record()
    barrier()
    layers = len(arena.head_lens)
    new_keys = torch.randn(EVICT_INTERVAL + args.decode_steps, layers * HEADS, DIM, generator=generator,
                           device=arena.device).to(torch.bfloat16)
    # Lazy batches straight from the device queue: each slot's (head, logical
    # position) was gathered at the audit (AuditResult.lazy).
    flat, logical = last.lazy
    start = IMMEDIATE

    def decode_step(step):
        nonlocal start
        arena.append_all(new_keys[step], new_keys[step], arena.seen_tokens)
        arena.seen_tokens += 1
        if (step + 1) % EVICT_INTERVAL == 0 and start + STAGING <= flat.numel():
            arena.evict_logical(flat[start:start + STAGING], logical[start:start + STAGING])
            start += STAGING

    for step in range(EVICT_INTERVAL):  # warm-up: one eviction interval, untimed
        decode_step(step)
    barrier()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for step in range(EVICT_INTERVAL, EVICT_INTERVAL + args.decode_steps):
        decode_step(step)
    d1.record()
    barrier()
    arena.check_flags()
    return {"pass_ms": a0.elapsed_time(a1), "decode_ms": d0.elapsed_time(d1), "capacity": arena.capacity,
            "bytes": (arena.keys.numel() + arena.values.numel()) * arena.keys.element_size()
            + arena.positions.numel() * 4}


def max_over_ranks(values, distributed: bool, device):
    """Elementwise maximum over ranks of a list of floats."""
    import torch
    import torch.distributed as dist

    local = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if distributed:
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
    return local.tolist()


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank)

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    distributed = world > 1
    if distributed:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)

    def barrier():
        if distributed:
            dist.barrier()
        torch.cuda.synchronize()

    head = measure_cfg1(args, device, world, rank, distributed, barrier, layer_groups=False, steps=args.steps,
                        warmup=args.warmup, with_e2e=True)
    elapsed_ms, decode_ms, e2e_ms, decode_median_ms = max_over_ranks(
        [head["elapsed_ms"], head["decode_ms"], head["e2e_ms"], head["decode_median_ms"]],
                                                   distributed, device)
    value = world * head["managed"] * args.steps / (elapsed_ms / 1e3)
    e2e_value = world * head["managed"] * head["e2e_steps"] / (e2e_ms / 1e3)
    candidates = RETAINED + IMMEDIATE - LAYERS * HEADS * PROTECT_RECENT
    peak, peak_kind = measured_peaks()
    traffic_ratio = measured_traffic_ratio()
    kernel_ms = head["kernel_ms"]
    achieved = head["kernel_bytes"] / (kernel_ms / 1e3) / 1e9 if kernel_ms > 0 else 0.0
    per_launch = head["kernel_bytes"] / max(1, head["kernel_launches"])
    result = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "impl": "ours",
        "data": "synthetic (seeded): bf16 K/V ~N(0,1), queries ~N(0,4), margin gradient ~N(0,1/D)",
        "config": config_cfg1(world, args.scoring),
        "candidate_rows_per_s": world * candidates * args.steps / (elapsed_ms / 1e3),
        "decode_overhead_us": decode_median_ms * 1e3 / args.decode_steps,
        "decode_overhead_mean_us": decode_ms * 1e3 / args.decode_steps,
        "roofline": {"kernel": head["timed_name"], "bound": "hbm", "achieved": achieved, "peak": peak,
                     "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                     "share_of_step": kernel_ms / head["elapsed_ms"],
                     "traffic": None if traffic_ratio is None else traffic_ratio * per_launch,
                     "traffic_source": "profiles/temporal_scores_traffic.json (ncu dram bytes / algorithmic bytes)",
                     "bytes_per_launch": per_launch, "launches": head["kernel_launches"]},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": head["h2d"],
                "d2h_bytes_per_step": head["d2h"]},
        "gpu_launches": head["launches"],
        "clocks": head["clocks"],
    }
    pass_ms, arena_decode_ms = max_over_ranks([head["arena"]["pass_ms"], head["arena"]["decode_ms"]], distributed,
                                              device)
    result["arena"] = {
        "layout": "gapped per-head arena (K, V [layers*heads, capacity, D]): decode appends are one launch for all "
                  "layers, evictions shift only the touched heads' rows in place (lrk_arena_append, "
                  "lrk_arena_compact); FlashAttention reads it through flash_attn_with_kvcache",
        "capacity_rows_per_head": head["arena"]["capacity"], "bytes": head["arena"]["bytes"],
        "ms_per_pass": pass_ms / args.steps,
        "tokens_per_s": world * head["managed"] * args.steps / (pass_ms / 1e3),
        "decode_overhead_us": arena_decode_ms * 1e3 / args.decode_steps,
        "decode_steps": args.decode_steps,
    }
    del head
    torch.cuda.empty_cache()
    if distributed:
        # One request split into per-rank layer groups (strong scaling); the
        # request-wide selection is the NCCL histogram all-gathers.
        lg = measure_cfg1(args, device, world, rank, distributed, barrier, layer_groups=True, steps=args.steps,
                          warmup=args.warmup, with_e2e=False)
        gather = lg["gather_us"]
        ms, dec = max_over_ranks([lg["elapsed_ms"], lg["decode_median_ms"]], distributed, device)
        rounds = max_over_ranks(gather, distributed, device) if gather else []
        result["layer_groups"] = {
            "config": f"configs[1], one request split into {world} groups of {LAYERS // world} layers",
            "scaling": "strong", "steps": args.steps, "warmup": args.warmup,
            "ms_per_pass": ms / args.steps, "tokens_per_s": lg["managed"] * args.steps / (ms / 1e3),
            "decode_overhead_us": dec * 1e3 / args.decode_steps,
            "allgather_us_per_round": rounds[:3],
            "allgather_us_per_pass": sum(rounds) / max(1, args.steps),
            "allgather_share_of_pass": sum(rounds) / 1e3 / ms if ms else None,
            "allgather_note": "each round's span starts when this rank's histogram is ready, so round 0 also "
                              "holds the wait for the slower rank's scoring",
            "gpu_launches": lg["launches"],
        }
        del lg
        torch.cuda.empty_cache()
    if not args.skip_large:
        from code_for_iclr27_b200.workloads import measure_large, measure_large_layer_groups

        big = measure_large(device, requests=args.large_requests, steps=args.large_steps, warmup=args.large_warmup,
                            rank=rank, barrier=barrier, peak_gbs=peak)
        ms, kms = max_over_ranks([big["ms_per_pass"], big["temporal_scores_ms_per_pass"]], distributed, device)
        big["ms_per_pass"] = ms
        big["tokens_per_s"] = world * args.large_requests * big["managed_rows_per_request"] / (ms / 1e3)
        big["n_gpus"], big["scaling"] = world, "weak"
        big["temporal_scores_share_of_pass"] = big.pop("temporal_scores_ms_per_pass") / ms
        result["configs4"] = big
        torch.cuda.empty_cache()
        if distributed:
            lgb = measure_large_layer_groups(device, world, rank, requests=args.large_requests,
                                             steps=args.large_steps, warmup=args.large_warmup, barrier=barrier)
            ms, = max_over_ranks([lgb["ms_per_pass"]], distributed, device)
            rounds = lgb["allgather_us_per_round"]
            rounds = max_over_ranks(rounds, distributed, device) if rounds else []
            lgb["ms_per_pass"] = ms
            lgb["tokens_per_s"] = args.large_requests * big["managed_rows_per_request"] / (ms / 1e3)
            lgb["allgather_us_per_round"] = rounds[:3]
            # The rounds of the last timed pass.
            lgb["allgather_share_of_pass"] = sum(rounds) / 1e3 / ms if ms else None
            lgb["n_gpus"], lgb["scaling"] = world, "strong"
            result["configs4_layer_groups"] = lgb
            torch.cuda.empty_cache()
    if world == 1 and not args.skip_side:
        # The other configurations' hot operators, measured on the same GPU.
        from code_for_iclr27_b200.workloads import measure_batch_append, measure_recall, measure_small

        result["configs0"] = measure_small(device, peak_gbs=peak)
        torch.cuda.empty_cache()
        result["batch_append"] = measure_batch_append(device)
        torch.cuda.empty_cache()
        result["recall"] = measure_recall(device)
    if distributed:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1:
            import torch

            torch.set_num_threads(os.cpu_count() or 1)
            result["cpu_baseline"] = reference_cpu_sample(args.seed) or cpu_baseline(args.seed)
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
