"""Decode throughput of the B200 paged-attention path (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg2|cfg4|cfg1] [--impl ours|reference]

Workload (default ``cfg2``): GPT-2 124M architecture,
random-init N(0, 0.02) fp32 weights, 64 sequences with contexts uniform in
[16, 512], block size 16, fragmented block tables, consecutive greedy decode
steps.  A *step* is one paged forward over the 64 sequences plus the greedy
argmax that feeds the next step.  Config 2's pool of 1,024 blocks cannot hold
its contexts, so it runs on 2,048 blocks (the reference case does the same).

Multi-GPU: one process per GPU (torchrun), each an independent engine replica
with its own sequences and KV pool; no collective on the data path.  Timing is
the max over ranks; ``value`` is the tokens of all ranks over that time.

Reported on one JSON line (rank 0):
  value        device-resident loop: step plans already in HBM, each step's
               input tokens are the previous step's argmax (CUDA events)
  e2e          the public API: ``paged_greedy_decode`` over the K steps (configs
               1, 2: each step's host plan, pinned host->device plan copy,
               graph replay and greedy tokens back to the host, pipelined one
               step ahead) or ``paged_greedy_step`` per step (config 4)
  roofline     the paged-attention kernel (+ its split-K combine): algorithmic
               bytes (K/V rows read + q read + output write + split scratch) per
               launch over its CUDA-event duration, vs the measured HBM copy peak
  cpu_baseline the numpy oracle (the reference algorithm: dense gather + masked
               softmax) on the host cores, on a bounded sample of the workload

``--impl reference`` times that CPU implementation as the main line (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_PATH = ROOT / "MEASURED_PEAKS.json"
# ncu captures of the dominant kernel on each workload's shape: DRAM traffic
# (read + write) over algorithmic bytes, with the capture command of each,
# scaled here to this run's launches.
TRAFFIC_PATH = ROOT / "profiles" / "dram_traffic.json"
FALLBACK_HBM_GBS = 6650.0
L2_BYTES = 126 * 2**20

WORKLOADS = {
    "cfg2": dict(n_seqs=64, ctx_range=(16, 512), block_size=16, num_blocks=2048, grow=True,
                 desc="BASELINE config 2: 64 seqs, ctx U[16,512], bs 16, 2048 blocks, consecutive greedy decode steps"),
    "cfg4": dict(n_seqs=512, ctx_range=(256, 1024), block_size=32, pool_bytes=150e9, grow=False, strong=True,
                 desc="BASELINE config 4: 512 seqs, ctx U[256,1024], bs 32, ~150 GB pool, repeated decode step"),
    "cfg1": dict(n_seqs=8, ctx_range=(16, 256), block_size=16, num_blocks=1024, grow=True,
                 desc="BASELINE config 1: 8 seqs, ctx U[16,256], bs 16, 1024 blocks, greedy decode steps"),
}  # fmt: skip


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------------------ modules
def _standalone(name: str, rel: str):
    """A pure-Python module of this repository loaded from its file, without
    importing the ``tokquay_b200`` package (so none of its native code loads)."""
    import importlib.util

    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, ROOT / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


# One replica per GPU (tokquay_b200/replicas.py, plain torch.distributed): no
# collective on the data path, host reductions only for the barrier and the
# max-over-ranks timing.
_replicas = _standalone("tq_bench_replicas", "tokquay_b200/replicas.py")
ReplicaInfo, barrier, replica_seed = _replicas.ReplicaInfo, _replicas.barrier, _replicas.replica_seed
max_over_ranks, sum_over_ranks, all_over_ranks = (_replicas.max_over_ranks, _replicas.sum_over_ranks,
                                                  _replicas.all_over_ranks)  # fmt: skip
_lib = None  # tokquay_b200._lib, imported by _load_library() for this build's arms


def _load_library():
    global _lib
    from tokquay_b200 import _lib as lib

    _lib = lib
    return lib


def reference_package():
    """The unmodified reference, installed next to this file by
    baseline/install_ref.sh (importable as ``tokquay``); None if absent."""
    path = ROOT / "baseline" / "_ref"
    if (path / "tokquay" / "__init__.py").is_file() and str(path) not in sys.path:
        sys.path.append(str(path))
    try:
        import tokquay.engine  # noqa: F401
        import tokquay.generate  # noqa: F401
    except ImportError:
        return None
    import tokquay

    return tokquay


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples the SM clock and throttle reasons through NVML every 10 ms."""

    REASONS = {
        "sw_power_cap": 0x4,
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            try:  # the CUDA device's own GPU, whatever CUDA_VISIBLE_DEVICES remaps
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:  # noqa: BLE001
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            log(f"clock sampling unavailable: {e}")
            self._nvml = None

    def _run(self):
        n = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
                get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    n.nvmlDeviceGetCurrentClocksThrottleReasons
                bits = get(self._h)
                for name, mask in self.REASONS.items():
                    if bits & mask:
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            self._stop.wait(0.01)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self) -> dict:
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


def traffic_source(workload: str) -> str | None:
    r = traffic_ratio(workload)
    if r is None:
        return None
    return (f"{TRAFFIC_PATH.relative_to(ROOT)} entry {workload!r}: ncu DRAM read+write / algorithmic bytes = {r} "
            "on a captured launch, times this run's average algorithmic bytes per launch")


def traffic_ratio(workload: str) -> float | None:
    """ncu DRAM bytes over algorithmic bytes of the workload's dominant kernel."""
    if not TRAFFIC_PATH.exists():
        return None
    entry = json.loads(TRAFFIC_PATH.read_text())["entries"].get(workload)
    return float(entry["ratio"]) if entry else None


def kernel_table(model, a, seqs, spec, steps: int = 10) -> str:
    """Per-kernel device time over `steps` public-API decode steps (CUPTI via
    torch.profiler, kernels back to back as in the run)."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    from tokquay_b200 import paged_greedy_step

    # Algorithmic bytes of the table's attention launches: contexts grow by one per step.
    ctx0 = [s.num_cached_tokens + 1 for s in seqs]
    bytes_per_launch = sum(attn_bytes([c + (k if spec["grow"] else 0) for c in ctx0], model.cfg.n_head,
                                      model.cfg.n_embd // model.cfg.n_head, 0) for k in range(steps)) / steps
    def step():
        toks = paged_greedy_step(model, a, seqs)
        for s, t in zip(seqs, toks):
            s.append_token(t)
            if spec["grow"]:
                a.append_slot(s)
            else:
                s.num_cached_tokens -= 1
                s.output_token_ids.pop()

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    spans = []
    for e in prof.events():
        if e.device_type == torch.autograd.DeviceType.CUDA:
            k = e.name.split("(")[0][:90]
            agg[k][0] += 1
            agg[k][1] += getattr(e, "device_time", None) or e.cuda_time
            spans.append((e.time_range.start, e.time_range.end, k))
    tot = sum(v[1] for v in agg.values())
    # The attention launch's exposed time: from the later of its own start and
    # the end of the operation before it to its end.  A programmatic dependent
    # starts its CTAs during the kernel before it, so its own duration counts
    # time that kernel also spends; the exposed time is what the step pays.
    spans.sort()
    exposed, n_attn, prev_end = 0.0, 0, None
    for t0, t1, k in spans:
        if "paged_attention_kernel" in k and prev_end is not None:
            exposed += t1 - max(t0, prev_end)
            n_attn += 1
        prev_end = t1 if prev_end is None else max(prev_end, t1)
    # Idle device time between consecutive operations of one step (gaps under
    # 20 us; longer ones are the host's turn between steps).
    gaps = [b[0] - a[1] for a, b in zip(spans, spans[1:])]
    idle = sum(g for g in gaps if 0 < g < 20)
    lines = [f"device time per step: {tot / steps:.1f} us; idle between operations inside a step: "
             f"{idle / steps:.1f} us",
             f"attention exposed (end - max(own start, previous operation's end)): "
             f"{exposed / max(n_attn, 1):.2f} us per launch over {n_attn} launches, "
             f"{bytes_per_launch / 1e6:.1f} MB algorithmic per launch = "
             f"{bytes_per_launch / (exposed / max(n_attn, 1)) / 1e3:.0f} GB/s exposed",
             "| kernel | us/step | share | launches/step | avg us |",
             "|---|---|---|---|---|"]  # fmt: skip
    for k, (n, t) in sorted(agg.items(), key=lambda x: -x[1][1])[:20]:
        lines.append(f"| {k} | {t / steps:.1f} | {100 * t / tot:.1f}% | {n / steps:.1f} | {t / n:.2f} |")
    return "\n".join(lines)


# ------------------------------------------------------------------------------ setup
def workload_spec(args) -> dict:
    """The workload, with the --num-seqs / --pool-gb overrides used for small
    profiling cases of the same shape (the defaults are the BASELINE configs)."""
    spec = dict(WORKLOADS[args.workload])
    if args.num_seqs:
        spec["n_seqs"] = args.num_seqs
        spec["desc"] += f" [num_seqs overridden: {args.num_seqs}]"
    if args.pool_gb:
        spec["pool_gb"] = args.pool_gb
        spec["desc"] += f" [pool overridden: {args.pool_gb} GB]"
    return spec


def make_model(device, seed=0):
    from tokquay_b200 import GPT2, GPT2Config
    from tokquay_b200 import workloads as W

    cfg = GPT2Config(**W.GPT2_SMALL)
    with torch.device("meta"):
        m = GPT2(cfg)
    m = m.to_empty(device=device)
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0.0, 0.02, generator=g)  # BASELINE random init: every parameter N(0, 0.02)
    return m.eval()


def make_allocator(spec, cfg, device):
    from tokquay_b200 import BlockAllocator

    bs = spec["block_size"]
    if spec.get("pool_gb"):
        nb = int(spec["pool_gb"] * 1e9 // (cfg.n_layer * 2 * cfg.n_head * bs * cfg.d_head * 4))
    elif "num_blocks" in spec:
        nb = spec["num_blocks"]
    else:
        per_block = cfg.n_layer * 2 * cfg.n_head * bs * cfg.d_head * 4
        free = torch.cuda.mem_get_info(device)[0]
        nb = int(min(spec["pool_bytes"], free - 8e9) // per_block)
    a = BlockAllocator(cfg, nb, bs, device=device)
    g = torch.Generator(device=device).manual_seed(1234)
    a.pool.normal_(generator=g)  # BASELINE: K/V pool filled N(0, 1)
    return a


def reset_allocator(a):
    a._free = list(range(a.num_blocks - 1, -1, -1))
    a.ref_counts = [0] * a.num_blocks


def make_case(spec, a, seed, rank=0, world=1):
    """The workload's decode batch on this replica: a copy of the whole batch
    (weak scaling), or with ``strong`` its share of one batch of ``n_seqs``
    sequences split by sequence over the replicas (config 4)."""
    from tokquay_b200 import Sequence
    from tokquay_b200 import workloads as W

    reset_allocator(a)
    shard = (rank, world) if spec.get("strong") else (0, 1)
    return W.decode_case(Sequence, a, spec["n_seqs"], spec["ctx_range"], a.cfg.vocab_size, seed=seed, shard=shard)


def attn_bytes(ctx_list, n_head, d, num_partials):
    """Algorithmic bytes of one attention launch (one layer): every sequence's
    K and V rows of all heads read once, q read, output written, split-K
    partials written and read back."""
    kv = sum(ctx_list) * n_head * d * 4 * 2
    qo = len(ctx_list) * n_head * d * 4 * 2
    part = num_partials * (d + 2) * 4 * 2
    return kv + qo + part


# ------------------------------------------------------------------------------ attention timing
def eager_attention_times(model, a, spec, seed, warmup, total_steps, rank=0,
                          world=1) -> tuple[list[float], list[float], list[float]]:  # fmt: skip
    """Attention times (ms per launch) over the same steps, eager, three ways:

    * stream: after each step's forward, its 12 attention launches (one per
      layer) again back to back, one event before the first and one after the
      last; the interval / 12 is one launch as a stream of launches runs it
      (the kernel plus the GPU's gap to the next launch);
    * evented: the same 12 launches with an event between consecutive launches
      (each interval one launch; a timing event between two launches also
      keeps the GPU from starting the next launch before it is recorded);
    * single: events around each attention launch inside the forward itself,
      each after a device sleep, so the interval also holds the GPU's launch
      and CTA start-up of a kernel that follows an idle stream."""
    from tokquay_b200.kv_cache import DevicePagedBatch

    case = make_case(spec, a, seed, rank, world)
    seqs = case.seqs
    B = len(seqs)
    pairs: list = []
    bursts: list = []
    streams: list = []
    C = model.cfg.n_embd
    q = torch.randn(B, C, device=a.pool.device, generator=torch.Generator(a.pool.device).manual_seed(0))
    out = torch.empty_like(q)

    def timer(layer: int, start: bool) -> None:
        if start:
            torch.cuda._sleep(200_000)  # ~0.1 ms of device work: the host gets ahead
            pairs.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
        pairs[-1][0 if start else 1].record()

    try:
        for k in range(total_steps):
            starts = [s.num_cached_tokens for s in seqs]
            ids = [s.token_ids[st:st + 1][0] for s, st in zip(seqs, starts)]
            b = DevicePagedBatch(a, [list(s.block_table) for s in seqs], starts, [1] * B, ids)
            if k == warmup:
                torch.cuda.synchronize()
                pairs.clear()
                bursts.clear()
                streams.clear()
            model.attention_timer = timer
            model.forward_paged(b, last_only=True)
            model.attention_timer = None
            L = model.cfg.n_layer
            sid = torch.cuda.current_stream().cuda_stream
            torch.cuda._sleep(1_000_000)  # ~0.5 ms: the host queues all 12 launches before the first runs
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record()
            for layer in range(L):
                b.attend_rows(layer, q, out, sid)
            g1.record()
            streams.append((g0, g1, L))
            torch.cuda._sleep(200_000)
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(L + 1)]
            evs[0].record()
            for layer in range(L):
                b.attend_rows(layer, q, out, sid)
                evs[layer + 1].record()
            bursts.append(evs)
            if spec["grow"]:
                for s in seqs:
                    s.num_cached_tokens += 1
                    s.append_token(0)
                    a.append_slot(s)
        torch.cuda.synchronize()
    finally:
        model.attention_timer = None
    stream_ms = [g0.elapsed_time(g1) / n for g0, g1, n in streams for _ in range(n)]
    evented = [e0.elapsed_time(e1) for evs in bursts for e0, e1 in zip(evs, evs[1:])]
    return stream_ms, evented, [e0.elapsed_time(e1) for e0, e1 in pairs]


# ------------------------------------------------------------------------------ our arm
def run_ours(args, world, rank, local):
    from tokquay_b200 import kv_cache as KV
    from tokquay_b200 import paged_greedy_decode, paged_greedy_step
    from tokquay_b200.kv_cache import DevicePagedBatch, plan_step_host

    spec = workload_spec(args)
    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    model = make_model(device)
    model.fused_lm_head = args.fused_lm_head
    cfg = model.cfg
    a = make_allocator(spec, cfg, device)
    # Every replica decodes its own copy of the same batch (own sequence objects,
    # own pool): per-GPU work is identical as N grows (weak scaling), so the
    # max over ranks measures the replicas, not the spread of random contexts.
    # Config 4 instead splits its one batch of 512 sequences over the replicas
    # by sequence (strong scaling).
    seed = 2
    K, Wm = args.steps, args.warmup
    total_steps = K + Wm
    strong = bool(spec.get("strong"))
    B = len(range(rank, spec["n_seqs"], world)) if strong else spec["n_seqs"]
    runner = None if args.no_graphs else model.use_cuda_graphs(a)
    bucket = runner.bucket_for(B) if runner else None

    # ---- plan every step first (bookkeeping only; the plans go to HBM) ------------
    case = make_case(spec, a, seed, rank, world)
    seqs = case.seqs
    plans, batches, ctx_per_step, nparts_per_step = [], [], [], []
    if runner:
        caps = runner.graph(bucket)[1].caps  # captures the bucket's graph
    t_plan = time.perf_counter()
    for k in range(total_steps):
        starts = [s.num_cached_tokens for s in seqs]
        ids = [s.token_ids[st:st + 1][0] for s, st in zip(seqs, starts)]
        tables = [list(s.block_table) for s in seqs]
        if runner:
            plan, lay = plan_step_host(a.block_size, a.num_blocks, cfg.n_head, tables, starts, [1] * B, ids,
                                       cfg.vocab_size, KV.sm_count(device), KV.MIN_SPLIT_CHUNKS,
                                       caps=caps)  # fmt: skip
            plans.append(torch.from_numpy(plan).to(device))
            nparts_per_step.append(int(lay[_lib.PLAN_NUM_PARTIALS]))
        else:
            batches.append(DevicePagedBatch(a, tables, starts, [1] * B, ids))
            nparts_per_step.append(batches[-1].num_partials)
        ctx_per_step.append([st + 1 for st in starts])
        if spec["grow"]:
            for s in seqs:
                s.num_cached_tokens += 1
                s.append_token(0)  # placeholder; the device loop feeds the real argmax
                a.append_slot(s)
    plan_ms = (time.perf_counter() - t_plan) * 1e3 / total_steps  # host planning + packing per step
    torch.cuda.synchronize(device)

    prev = [None]

    def device_step(k):
        if runner:
            prev[0] = runner.replay_plan(bucket, plans[k], ids=prev[0][:B] if prev[0] is not None else None)
        else:
            logits = model.forward_paged(batches[k], last_only=True)[:, 0]
            tok = logits.argmax(-1)
            if k + 1 < total_steps:
                batches[k + 1].token_ids.copy_(tok)

    for k in range(Wm):
        device_step(k)
    torch.cuda.synchronize(device)
    launches0 = model.kernel_launches
    stream = torch.cuda.current_stream(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for k in range(Wm, total_steps):
            device_step(k)
        end.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    ms = start.elapsed_time(end)
    launches = model.kernel_launches - launches0
    tokens = B * K
    ms_max = max_over_ranks(ms, world)
    tokens_all = sum_over_ranks(tokens, world)

    # ---- attention kernel timing: CUDA events around every attention launch ----------
    # The same steps eager (events cannot bracket a node of the timed graph
    # without changing it), a short device sleep before each bracketed launch
    # keeping host launch latency out of the interval.
    bytes_per_launch = [attn_bytes(ctx_per_step[k], cfg.n_head, cfg.d_head, nparts_per_step[k])
                        for k in range(Wm, total_steps) for _ in range(cfg.n_layer)]  # fmt: skip
    attn_ms, evented_ms, single_ms = eager_attention_times(model, a, spec, seed, Wm, total_steps, rank, world)
    attn_timing = ("CUDA events on the launching stream, eager pass over the same steps: after each step's "
                   "forward its 12 attention launches (one per layer) run again back to back between two "
                   "events; average launch = the interval / 12 (the kernel plus the GPU's gap to the next "
                   "launch)")
    del plans, batches

    # ---- end to end through the public API -----------------------------------------
    case = make_case(spec, a, seed, rank, world)
    seqs = case.seqs
    h2d = []

    def api_step():
        # Plans on the host, copies the plan, replays the graph; the step's greedy
        # tokens (the graph's own argmax) are its one device->host read.
        toks = paged_greedy_step(model, a, seqs)
        for s, t in zip(seqs, toks):
            s.append_token(t)
            if spec["grow"]:
                a.append_slot(s)
            else:
                s.num_cached_tokens -= 1  # repeat the same step
                s.output_token_ids.pop()
        return toks

    # A growing workload (configs 1, 2) runs its K steps as one fixed-batch
    # greedy decode (paged_greedy_decode: graph steps pipelined one ahead of
    # the host); a repeated step (config 4) goes step by step.
    pipelined = spec["grow"] and runner is not None
    if pipelined:
        paged_greedy_decode(model, a, seqs, Wm)
        for s in seqs:
            a.append_slot(s)
    else:
        for _ in range(Wm):
            api_step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    e0.record(stream)
    if pipelined:
        paged_greedy_decode(model, a, seqs, K)
        h2d = list(runner.step_h2d_bytes) or [model.last_h2d_bytes]
        for s in seqs:  # blocks for a following step (the kernel table's)
            a.append_slot(s)
    else:
        for _ in range(K):
            api_step()
            h2d.append(model.last_h2d_bytes)
    e1.record(stream)
    torch.cuda.synchronize(device)
    wall_ms = (time.perf_counter() - t0) * 1e3
    barrier(world)
    e2e_ms = max(e0.elapsed_time(e1), 0.0)
    e2e_ms_max = max_over_ranks(e2e_ms, world)
    # Every rank's own figures: the job's time is the slowest rank's, and the
    # spread says what limits it (host planning, the launch stream, the GPU).
    per_rank = {"ms_per_step": [x / K for x in all_over_ranks(ms, world)],
                "e2e_ms_per_step": [x / K for x in all_over_ranks(e2e_ms, world)],
                "host_plan_ms_per_step": all_over_ranks(plan_ms, world)}  # fmt: skip
    # Bytes copied per step: the packed step plan (host->device, token ids
    # included) and the B int64 sampled tokens back.
    h2d_bytes = sum(h2d) / len(h2d)
    d2h_bytes = len(seqs) * 8

    result = None
    if rank == 0:
        peaks = json.loads(PEAKS_PATH.read_text()) if PEAKS_PATH.exists() else {}
        peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
        avg_attn_ms = sum(attn_ms) / len(attn_ms)
        avg_bytes = sum(bytes_per_launch) / len(bytes_per_launch)
        achieved = avg_bytes / (avg_attn_ms * 1e-3) / 1e9
        result = {
            "metric": "decode tok/s",
            "value": tokens_all / (ms_max * 1e-3),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": K,
            "warmup": Wm,
            "ms_per_step": ms_max / K,
            "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {
                "workload": spec["desc"] + (f" [sequences split over {world} replicas]" if strong and world > 1 else ""),
                "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32, TF32 off",
                "global_batch": spec["n_seqs"] if strong else B * world,
                "seq_len": f"ctx U{list(spec['ctx_range'])}",
                "block_size": spec["block_size"],
                "num_blocks": a.num_blocks,
                "parallelism": f"replicas{world} (one engine + KV pool per GPU, no collective)",
                "cuda_graphs": runner is not None,
                "lm_head": ("opt-in fused ln_f + LM head + greedy argmax (tq_lm_head_argmax, fp32 CUDA cores)"
                            if args.fused_lm_head and B <= _lib.LM_HEAD_MAX_ROWS else
                            "torch fp32 matmul (TF32 off) + tq_argmax_rows, as the north star keeps it"),
                "l2": "inputs larger than L2: each step reads the whole weight set (0.5 GB) and every "
                      "context's K/V of 12 layers (> 1 GB), so no step finds the previous step's data in L2",
            },  # fmt: skip
            "roofline": {
                "bound": "hbm",
                "kernel": "paged_attention_kernel (split-K merge fused)",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": (traffic_ratio(args.workload) or float("nan")) * avg_bytes
                if traffic_ratio(args.workload) else None,
                "traffic_source": traffic_source(args.workload),
                "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "fallback",
                "algorithmic_bytes_per_launch": avg_bytes,
                "avg_launch_ms": avg_attn_ms,
                "launches_timed": len(attn_ms),
                "timing": attn_timing,
                "evented_launch_ms": sum(evented_ms) / len(evented_ms),
                "evented_launch_achieved": avg_bytes / (sum(evented_ms) / len(evented_ms) * 1e-3) / 1e9,
                "evented_launch_timing": "the same launches with an event between consecutive ones: each "
                                         "event also holds back the next launch until it is recorded",
                "single_launch_ms": sum(single_ms) / len(single_ms),
                "single_launch_achieved": avg_bytes / (sum(single_ms) / len(single_ms) * 1e-3) / 1e9,
                "single_launch_timing": "events around each attention launch inside the forward, each after "
                                        "a device sleep: adds the GPU's launch and CTA start-up after an idle "
                                        "stream",
                "attention_ms_per_step": avg_attn_ms * cfg.n_layer,
            },  # fmt: skip
            "e2e": {
                "value": tokens_all / (e2e_ms_max * 1e-3),
                "unit": "tok/s",
                "h2d_bytes_per_step": h2d_bytes,
                "d2h_bytes_per_step": d2h_bytes,
                "ms_per_step": e2e_ms_max / K,
                "wall_ms_per_step_rank0": wall_ms / K,
            },
            "gpu_launches": launches,
            "clocks": clocks.summary(),
            "per_rank": {**per_rank, "note": "device-timed step, end-to-end step and host planning time of "
                                             "each rank (rank order); value uses the slowest rank"},
        }
        if strong and world > 1:
            result["config"]["scaling_limit"] = (
                f"strong scaling: {B} of the batch's {spec['n_seqs']} sequences per replica; the fp32 linears "
                "(torch SIMT SGEMM, kept by the north star) take about as long at 64 rows as at 512, so the step "
                "time does not fall in proportion to the sequences per GPU")
    if args.kernel_table and rank == 0:
        log(kernel_table(model, a, seqs, spec))
    return result


# ------------------------------------------------------------------------------ the reference itself
def _reference_case(spec, tq, W, device, seed=2):
    """The workload's decode batch on the reference's own allocator and
    sequences (config 4: its 64-sequence subset, every 8th sequence)."""
    from tokquay.kv_cache import BlockAllocator
    from tokquay.model import GPT2Config
    from tokquay.sequence import Sequence

    cfg = GPT2Config(**W.GPT2_SMALL)
    bs = spec["block_size"]
    shard, n_seqs, note = (0, 1), spec["n_seqs"], ""
    if "num_blocks" in spec:
        nb = spec["num_blocks"]
    else:  # config 4: the subset the parity fixtures use, on a pool sized to it
        shard, nb = tuple(W.CFG4_SUBSET["shard"]), W.CFG4_SUBSET["num_blocks"]
        n_seqs = len(range(0, spec["n_seqs"], shard[1]))
        note = f" [{n_seqs}-sequence subset: every {shard[1]}th sequence, {nb}-block pool]"
    a = BlockAllocator(cfg, nb, bs, device=device)
    a.pool.normal_(generator=torch.Generator(device=device).manual_seed(1234))  # BASELINE: pool N(0, 1)
    case = W.decode_case(Sequence, a, spec["n_seqs"], spec["ctx_range"], cfg.vocab_size, seed=seed, shard=shard)
    return cfg, a, case.seqs, note


def _reference_model(cfg, device):
    from tokquay.model import GPT2

    gen = torch.Generator(device=device).manual_seed(0)
    with torch.device(device):
        m = GPT2(cfg)
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0.0, 0.02, generator=gen)  # BASELINE random init: every parameter N(0, 0.02)
    return m.eval()


def reference_rate(spec, steps: int, warmup: int, budget_s: float, device="cpu", threads: int | None = None):
    """The unmodified reference's own step -- ``tokquay.generate.paged_forward``
    (tokquay/generate.py:63-87: ``BlockAllocator.batch_for``, the padded ids,
    ``GPT2.forward`` with its dense gather and masked softmax) and the greedy
    ``argmax(-1).tolist()`` + append / ``append_slot`` of its decode loop
    (tokquay/generate.py:109-119) -- over the workload's whole batch, timed
    step by step after ``warmup`` steps, until ``steps`` steps or ``budget_s``
    seconds of timed steps.  Returns (tok/s, steps timed, batch size, sample
    note, threads)."""
    tq = reference_package()
    if tq is None:
        return None
    from tokquay.generate import paged_forward

    W = _standalone("tq_bench_workloads", "tokquay_b200/workloads.py")
    if device == "cpu" and threads:
        torch.set_num_threads(threads)
    cfg, a, seqs, note = _reference_case(spec, tq, W, device)
    model = _reference_model(cfg, device)
    sync = torch.cuda.synchronize if device != "cpu" else (lambda: None)
    times = []
    with torch.no_grad():
        for k in range(warmup + steps):
            sync()
            t0 = time.perf_counter()
            toks = paged_forward(model, a, seqs).argmax(-1).tolist()
            for s, t in zip(seqs, toks):
                s.append_token(t)
                if spec["grow"]:
                    a.append_slot(s)
                else:  # config 4 repeats its one step
                    s.num_cached_tokens -= 1
                    s.output_token_ids.pop()
            dt = time.perf_counter() - t0
            if k >= warmup:
                times.append(dt)
                if sum(times) > budget_s:
                    break
    del a
    rate = len(seqs) * len(times) / sum(times)
    return rate, len(times), len(seqs), note, torch.get_num_threads()


# ------------------------------------------------------------------------------ CPU oracle
def cpu_oracle_rate(spec, n_seqs, steps, warmup, seed=2, budget_s=None):
    """The numpy oracle (reference algorithm) on the host: decode steps over
    ``n_seqs`` sequences of the workload, with every host core (torchrun sets
    OMP_NUM_THREADS=1 per rank; the reference arm runs on rank 0 alone).
    Returns (tok/s, sample description, threads)."""
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    if threadpool_limits is not None:
        with threadpool_limits(limits=os.cpu_count()):
            return _cpu_oracle_rate(spec, n_seqs, steps, warmup, seed, budget_s)
    return _cpu_oracle_rate(spec, n_seqs, steps, warmup, seed, budget_s)


def _cpu_oracle_rate(spec, n_seqs, steps, warmup, seed, budget_s):
    import oracle
    from tokquay_b200 import BlockAllocator, GPT2Config, Sequence
    from tokquay_b200 import workloads as W

    cfg = GPT2Config(**W.GPT2_SMALL)
    rng = np.random.default_rng(0)
    weights = {n: (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)) for n, s in W.param_specs(cfg)}
    bs = spec["block_size"]
    max_ctx = spec["ctx_range"][1] + steps + warmup + 1
    nb = n_seqs * (-(-max_ctx // bs)) + 1
    a = BlockAllocator(cfg, nb, bs, device="cpu")  # bookkeeping only
    a.pool = torch.empty(0)
    case = W.decode_case(Sequence, a, n_seqs, spec["ctx_range"], cfg.vocab_size, seed=seed)
    pool = np.zeros((nb, cfg.n_layer, 2, cfg.n_head, bs, cfg.d_head), np.float32)
    seqs = case.seqs
    times = []
    for k in range(warmup + steps):
        t0 = time.perf_counter()
        logits = oracle.paged_forward(weights, cfg, pool, bs, seqs)
        dt = time.perf_counter() - t0
        if k >= warmup:
            times.append(dt)
        for s, t in zip(seqs, logits.argmax(-1).tolist()):
            s.append_token(int(t))
            if spec["grow"]:
                a.append_slot(s)
            else:
                s.num_cached_tokens -= 1
                s.output_token_ids.pop()
        if budget_s and sum(times) > budget_s:
            break
    try:
        from threadpoolctl import threadpool_info

        threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:  # noqa: BLE001
        threads = os.cpu_count()
    rate = n_seqs * len(times) / sum(times)
    sample = f"{len(times)} decode steps x {n_seqs} sequences of {spec['desc']} (numpy oracle, float32)"
    return rate, sample, threads


# ------------------------------------------------------------------------------ config 3
def mixed_case(a, seed):
    """BASELINE config 3 on allocator ``a``: 4 fresh prompts (U[16,256], start 0)
    and 60 decoding sequences (contexts U[16,256]) in a seeded interleaved order."""
    from tokquay_b200 import Sequence
    from tokquay_b200 import workloads as W

    c = W.CONFIGS[3]
    reset_allocator(a)
    return W.mixed_case(Sequence, a, c["n_prefill"], c["n_decode"], c["len_range"], a.cfg.vocab_size, seed=seed)


def run_mixed(args, world, rank, local) -> dict | None:
    """one mixed step -- 4 prompts prefilled from position 0
    next to 60 decode rows -- through the paged forward, one attention launch
    per layer covering the causal prefill rows and the decode rows together.
    A step is that forward (+ greedy argmax) over the same batch again: every
    sequence's cached count goes back, so each step writes the same K/V rows
    and reads the same contexts.  ``value`` is the query rows (prompt tokens +
    decode tokens) processed per second."""
    from tokquay_b200 import BlockAllocator, paged_greedy_step
    from tokquay_b200.kv_cache import DevicePagedBatch
    from tokquay_b200.model import argmax_rows

    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    model = make_model(device)
    cfg = model.cfg
    bs = args.block_size or 16
    a = BlockAllocator(cfg, 1024, bs, device=device)
    a.pool.normal_(generator=torch.Generator(device=device).manual_seed(1234))  # BASELINE: pool N(0, 1)
    seed = replica_seed(3, 0)  # the same mixed batch on every replica (weak scaling)
    case = mixed_case(a, seed)
    seqs, new_lens = case.seqs, case.new_lens
    starts = [s.num_cached_tokens for s in seqs]
    ids = [t for s, st, n in zip(seqs, starts, new_lens) for t in s.token_ids[st:st + n]]
    batch = DevicePagedBatch(a, [list(s.block_table) for s in seqs], starts, new_lens, ids)
    N, B = batch.N, batch.B
    K, Wm = args.steps, args.warmup

    def device_step():
        logits = model.forward_paged(batch, last_only=True)[:, 0]
        return argmax_rows(logits)

    for _ in range(Wm):
        device_step()
    torch.cuda.synchronize(device)
    launches0 = model.kernel_launches
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(K):
            device_step()
        e1.record(stream)
        torch.cuda.synchronize(device)
    barrier(world)
    ms = e0.elapsed_time(e1)
    launches = model.kernel_launches - launches0 + K  # + one argmax per step
    ms_max = max_over_ranks(ms, world)
    rows_all = sum_over_ranks(N * K, world)

    # Attention alone: each timed step's 12 launches again, back to back between two events.
    q = torch.randn(N, cfg.n_embd, device=device, generator=torch.Generator(device).manual_seed(0))
    out = torch.empty_like(q)
    sid = stream.cuda_stream
    groups = []
    for k in range(Wm + K):
        torch.cuda._sleep(1_000_000)
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for layer in range(cfg.n_layer):
            batch.attend_rows(layer, q, out, sid)
        g1.record(stream)
        if k >= Wm:
            groups.append((g0, g1))
    torch.cuda.synchronize(device)
    attn_ms = sum(g0.elapsed_time(g1) for g0, g1 in groups) / (len(groups) * cfg.n_layer)
    ctx = [st + n for st, n in zip(starts, new_lens)]
    abytes = attn_bytes(ctx, cfg.n_head, cfg.d_head, batch.num_partials) + (N - B) * cfg.n_head * cfg.d_head * 4 * 2

    # End to end: the public API with host planning and the plan copy inside.
    def api_step():
        toks = paged_greedy_step(model, a, seqs, new_lens)
        for s, st in zip(seqs, starts):
            s.num_cached_tokens = st
        return toks

    for _ in range(Wm):
        api_step()
    torch.cuda.synchronize(device)
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(device)
    h0.record(stream)
    for _ in range(K):
        api_step()
    h1.record(stream)
    torch.cuda.synchronize(device)
    barrier(world)
    e2e_ms_max = max_over_ranks(h0.elapsed_time(h1), world)
    h2d_bytes = model.last_h2d_bytes
    if rank != 0:
        return None
    peaks = json.loads(PEAKS_PATH.read_text()) if PEAKS_PATH.exists() else {}
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    achieved = abytes / (attn_ms * 1e-3) / 1e9
    n_prefill = sum(1 for n in new_lens if n > 1)
    return {
        "metric": "mixed prefill+decode step rows/s",
        "value": rows_all / (ms_max * 1e-3),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": K,
        "warmup": Wm,
        "ms_per_step": ms_max / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": f"BASELINE config 3: {n_prefill} prompts U[16,256] prefilled + {B - n_prefill} decodes, "
                        f"ctx U[16,256], bs {bs}, 1024 blocks, one mixed paged forward per step",
            "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32, TF32 off",
            "rows_per_step": N,
            "sequences": B,
            "block_size": bs,
            "parallelism": f"replicas{world} (one engine + KV pool per GPU, no collective)",
            "cuda_graphs": False,
            "l2": "each step reads the whole weight set (0.5 GB, larger than L2)",
        },
        "roofline": {
            "bound": "hbm",
            "kernel": "paged_attention_kernel (causal prefill + decode rows, one launch per layer)",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": traffic_ratio("cfg3") * abytes if traffic_ratio("cfg3") else None,
            "traffic_source": traffic_source("cfg3"),
            "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "fallback",
            "algorithmic_bytes_per_launch": abytes,
            "avg_launch_ms": attn_ms,
            "timing": "CUDA events on the launching stream: each timed step's 12 attention launches back to back "
                      "between two events, average launch = the interval / 12; algorithmic bytes = every "
                      "sequence's K/V rows read once + q read + output written",
        },
        "e2e": {
            "value": rows_all / (e2e_ms_max * 1e-3),
            "unit": "rows/s",
            "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": B * 8,
            "ms_per_step": e2e_ms_max / K,
        },
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }


def run_kvwrite(args, world, rank, local) -> dict | None:
    """The KV-write kernels alone at a prefill-sized step: --num-seqs prompts
    (default 64) of 256 tokens each (16,384 new rows) written into a shuffled
    pool of 16-token blocks, GPT-2 124M shapes.  Two kernels, each timed as a
    stream of launches between two CUDA events (12 layers per step, L2 flushed
    by a 512 MB read before each step):
      * tq_qkv_bias_kv_write (the model's c_attn epilogue): reads the c_attn
        output rows [N, 3C], writes q [N, C] and the K/V rows into the pool;
      * tq_kv_write (the plain scatter): reads K/V from the [N, 3C] rows and
        writes them into the pool.
    ``value`` is the fused kernel's algorithmic HBM GB/s."""
    from tokquay_b200 import BlockAllocator
    from tokquay_b200.kv_cache import DevicePagedBatch

    from tokquay_b200 import GPT2Config
    from tokquay_b200 import workloads as W

    device = torch.device("cuda", local)
    model_cfg = GPT2Config(**W.GPT2_SMALL)
    C = model_cfg.n_embd
    n_prompts, plen, bs = (args.num_seqs or 64), 256, 16
    N = n_prompts * plen
    a = BlockAllocator(model_cfg, n_prompts * plen // bs + 8, bs, device=device)
    import random as _random

    _random.Random(7).shuffle(a._free)
    tables = [a._take(plen // bs) for _ in range(n_prompts)]
    batch = DevicePagedBatch(a, tables, [0] * n_prompts, [plen] * n_prompts)
    g = torch.Generator(device=device).manual_seed(0)
    qkv = torch.randn(N, 3 * C, device=device, generator=g)
    bias = torch.randn(3 * C, device=device, generator=g)
    q = torch.empty(N, C, device=device)
    flush = torch.ones(128 << 20, device=device)
    sid = torch.cuda.current_stream(device).cuda_stream
    K, Wm, L = args.steps, args.warmup, model_cfg.n_layer

    def timed(fn):
        per = []
        for k in range(Wm + K):
            flush.sum()
            torch.cuda._sleep(1_000_000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for layer in range(L):
                fn(layer)
            e1.record()
            torch.cuda.synchronize(device)
            if k >= Wm:
                per.append(e0.elapsed_time(e1) / L)
        return sum(per) / len(per)

    with ClockSampler(local) as clocks:
        fused_ms = timed(lambda layer: batch.write_qkv_rows(layer, qkv, 1, 0, bias, q, sid))
        plain_ms = timed(lambda layer: batch.write_rows(layer, qkv, C, 2 * C, sid))
    assert _lib.device_status() == 0
    # Algorithmic bytes: fused -- rows [N, 3C] read, q [N, C] and K/V [N, 2C] written (bias once);
    # plain -- K/V [N, 2C] read and written.
    fused_bytes = N * 3 * C * 4 + N * C * 4 + N * 2 * C * 4 + 3 * C * 4
    plain_bytes = 2 * N * 2 * C * 4
    peaks = json.loads(PEAKS_PATH.read_text()) if PEAKS_PATH.exists() else {}
    peak = float(peaks.get("hbm_gbs", FALLBACK_HBM_GBS))
    fused = fused_bytes / (fused_ms * 1e-3) / 1e9
    plain = plain_bytes / (plain_ms * 1e-3) / 1e9
    if rank != 0:
        return None
    traffic = traffic_ratio("kvwrite")
    return {
        "metric": "KV-write HBM GB/s (fused c_attn epilogue)",
        "value": fused,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": K,
        "warmup": Wm,
        "ms_per_step": fused_ms * L,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"KV write of {n_prompts} prompts x {plen} tokens ({N} rows), GPT-2 124M shapes, "
                               f"bs {bs}, shuffled blocks",
                   "l2": "a 512 MB read before each step's 12 launches; each launch moves > 200 MB"},  # fmt: skip
        "roofline": {
            "bound": "hbm",
            "kernel": "qkv_bias_kv_write_kernel",
            "achieved": fused,
            "peak": peak,
            "unit": "GB/s",
            "frac": fused / peak,
            "traffic": traffic * fused_bytes if traffic else None,
            "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "fallback",
            "algorithmic_bytes_per_launch": fused_bytes,
            "avg_launch_ms": fused_ms,
            "timing": "CUDA events around 12 back-to-back launches (one per layer), interval / 12",
        },
        "kv_write_plain": {"kernel": "kv_write_kernel", "achieved": plain, "frac": plain / peak,
                           "algorithmic_bytes_per_launch": plain_bytes, "avg_launch_ms": plain_ms},
        "e2e": None,
        "gpu_launches": 2 * L * (Wm + K),
        "clocks": clocks.summary(),
    }


def cpu_oracle_mixed_rate(bs: int, reps: int, seed: int) -> tuple[float, str, int]:
    """The numpy oracle on config 3's mixed step (every host core)."""
    import oracle
    from tokquay_b200 import BlockAllocator, GPT2Config
    from tokquay_b200 import workloads as W

    try:
        from threadpoolctl import threadpool_info, threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = threadpool_info = None
    cfg = GPT2Config(**W.GPT2_SMALL)
    rng = np.random.default_rng(0)
    weights = {n: (rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)) for n, s in W.param_specs(cfg)}
    a = BlockAllocator(cfg, 1024, bs, device="cpu")  # bookkeeping only
    a.pool = torch.empty(0)
    case = mixed_case(a, seed)
    pool = np.zeros((1024, cfg.n_layer, 2, cfg.n_head, bs, cfg.d_head), np.float32)
    starts = [s.num_cached_tokens for s in case.seqs]
    times = []
    ctx = threadpool_limits(limits=os.cpu_count()) if threadpool_limits else None
    if ctx:
        ctx.__enter__()
    try:
        for _ in range(reps):  # ~20-40 s per step: the oracle pads every row to the longest prompt
            t0 = time.perf_counter()
            oracle.paged_forward(weights, cfg, pool, bs, case.seqs, case.new_lens)
            times.append(time.perf_counter() - t0)
            for s, st in zip(case.seqs, starts):
                s.num_cached_tokens = st
        threads = max((i.get("num_threads", 1) for i in threadpool_info()), default=1) if threadpool_info else 1
    finally:
        if ctx:
            ctx.__exit__(None, None, None)
    rows = sum(case.new_lens)
    sample = f"{len(times)} mixed steps of BASELINE config 3 ({rows} rows, bs {bs}; numpy oracle, float32)"
    return rows * len(times) / sum(times), sample, threads


# ------------------------------------------------------------------------------ config 5
def run_serving(args, world, rank, local) -> dict | None:
    """BASELINE config 5, shortened: the first --trace-requests requests of the
    serving workload (prompts and outputs U[16,256], Poisson arrivals at
    --rate req/s, or all at t=0 with --rate inf), round-robined over the
    replicas, each replica an Engine with 16,384 KV slots (1,024 blocks of 16)
    and CUDA-graph decode steps, driven open loop in real time."""
    import math

    from tokquay_b200 import BlockAllocator
    from tokquay_b200.engine import Engine
    from tokquay_b200.scheduler import SchedulerConfig
    from tokquay_b200.serving import make_workload, round_robin, run_trace, summarize

    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    model = make_model(device)
    a = BlockAllocator(model.cfg, 1024, 16, device=device)
    runner = model.use_cuda_graphs(a)
    P = args.mixed_tokens
    if P > 0:  # mixed-step graphs sized for P prompt tokens per step
        runner.mixed_extra = sorted({max(1, P // 4), max(1, P // 2), P})
    for b in runner.buckets:  # capture every graph the engine can use before the clock starts
        if b <= 64:
            runner.graph(b)
            for e in runner.mixed_extra if P > 0 else ():
                runner.graph((b, b + e))
    sched_cfg = SchedulerConfig(max_model_len=model.cfg.n_positions, mixed_prefill_tokens=P)
    rate = math.inf if args.rate == "inf" else float(args.rate)
    workload = make_workload(rate, args.trace_requests, seed=0)
    mine = round_robin(workload, world, rank)
    warm = Engine(model, a, sched_cfg)
    for spec in make_workload(math.inf, 8, seed=99, output_len=(4, 8)):  # warm the prefill shapes too
        warm.add_request(list(spec.prompt_ids))
    warm.run_until_done()
    torch.cuda.synchronize(device)
    eng = Engine(model, a, sched_cfg)
    barrier(world)
    records, steps, wall = run_trace(eng, mine)
    torch.cuda.synchronize(device)
    barrier(world)
    out = summarize(records, steps)
    tokens_all = sum_over_ranks(out["output_tokens"], world)
    dur_max = max_over_ranks(out["duration_s"], world)
    if rank != 0:
        return None
    return {
        "metric": "serving tok/s (config 5 trace)",
        "value": tokens_all / dur_max,
        "unit": "tok/s",
        "n_gpus": world,
        "higher_is_better": True,
        "scaling": "weak" if math.isinf(rate) else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"BASELINE config 5, first {args.trace_requests} requests at rate {args.rate} req/s "
                               f"(seed 0), round-robin over {world} replica(s), 1,024 x 16 KV slots each",
                   "scheduler": ("the reference's (prefill and decode steps alternate)" if P == 0 else
                                 f"opt-in chunked prefill: decodes + up to {P} prompt tokens per step"),
                   "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32, TF32 off",
                   "parallelism": f"replicas{world}"},  # fmt: skip
        "rank0": {k: out[k] for k in ("requests", "output_tokens", "duration_s", "throughput_tok_s", "ttft_ms",
                                      "itl_ms", "latency_ms", "steps", "prefill_steps", "decode_step_ms")},
        "preemptions_rank0": eng.stats.num_preemptions,
        "mixed_steps_rank0": eng.mixed_steps,
        "wall_s_rank0": wall,
    }


def run_serving_http(args) -> dict:
    """Config 5 through the serving front end: the same trace as --workload
    cfg5, sent by an HTTP client (aiohttp, open loop in real time) to
    ``tokquay_b200.frontend`` (uvicorn, one process) over --gpus N replica
    processes, one per GPU, round robin (--front-ends K: K server processes on
    one port, each over its share of the replicas).  With streaming (the default) every
    token arrives as a server-sent event and TTFT / ITL are the client's
    clock; with --http-json each request gets one JSON body (throughput and
    end-to-end latency only)."""
    import asyncio
    import math
    import socket

    import aiohttp
    import uvicorn

    from tokquay_b200.frontend import FrontEnds, RandomGPT2Engine, ReplicaRouter, create_app
    from tokquay_b200.serving import RequestRecord, make_workload, summarize

    n = args.gpus
    P = args.mixed_tokens
    rate = math.inf if args.rate == "inf" else float(args.rate)
    workload = make_workload(rate, args.trace_requests, seed=0)
    stream = not args.http_json
    factory = RandomGPT2Engine(num_blocks=1024, block_size=16, mixed_prefill_tokens=P, seed=0, warm=True)
    K = args.front_ends
    router = ReplicaRouter(factory, list(range(n))) if K == 1 else None
    app = create_app(router) if K == 1 else None

    async def one(session, url, spec, t0, rec):
        await asyncio.sleep(max(0.0, spec.arrival - (time.perf_counter() - t0)))
        body = {"prompt_token_ids": list(spec.prompt_ids), "max_tokens": spec.output_len, "ignore_eos": True,
                "stream": stream}  # fmt: skip
        async with session.post(url, json=body) as resp:
            if resp.status != 200:
                raise RuntimeError(f"HTTP {resp.status}: {await resp.text()}")
            if stream:
                async for line in resp.content:
                    if line.startswith(b"data: "):
                        rec.token_times.append(time.perf_counter() - t0)
            else:
                out = await resp.json()
                rec.token_times.extend([time.perf_counter() - t0] * len(out["token_ids"]))

    async def client(url):
        records = [RequestRecord(spec.arrival, len(spec.prompt_ids), spec.output_len) for spec in workload]
        timeout = aiohttp.ClientTimeout(total=None)
        async with aiohttp.ClientSession(connector=aiohttp.TCPConnector(limit=0), timeout=timeout) as session:
            t0 = time.perf_counter()
            await asyncio.gather(*(one(session, url, sp, t0, r) for sp, r in zip(workload, records)))
            return records, time.perf_counter() - t0

    async def main():
        sock = socket.socket()
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
        server = uvicorn.Server(uvicorn.Config(app, log_level="warning", timeout_keep_alive=600))
        task = asyncio.create_task(server.serve(sockets=[sock]))
        t_ready = time.perf_counter()
        while not server.started:  # the replicas are built and warmed in the app's start-up
            if task.done():
                task.result()
                raise RuntimeError("the front end failed to start (its log is above)")
            await asyncio.sleep(0.1)
        log(f"front end up with {n} replica(s) in {time.perf_counter() - t_ready:.1f} s")
        url = f"http://127.0.0.1:{port}/generate"
        records, wall = await client(url)
        health = router.stats()
        server.should_exit = True
        await task
        return records, wall, health

    if K == 1:
        records, wall, health = asyncio.run(main())
    else:
        fe = FrontEnds(factory, list(range(n)), K)
        t_ready = time.perf_counter()
        fe.start()
        log(f"{K} front ends up with {n} replica(s) in {time.perf_counter() - t_ready:.1f} s")
        try:
            records, wall = asyncio.run(client(f"http://127.0.0.1:{fe.port}/generate"))
        finally:
            fe.stop()
        health = {"preemptions": None}  # each front end answers for its own replicas only
    out = summarize(records, [])
    if not stream:  # one body per request: no per-token times
        out["ttft_ms"] = out["itl_ms"] = None
    return {
        "metric": "serving tok/s over HTTP (config 5 trace)",
        "value": out["throughput_tok_s"],
        "unit": "tok/s",
        "n_gpus": n,
        "higher_is_better": True,
        "scaling": "weak" if math.isinf(rate) else "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"BASELINE config 5, first {args.trace_requests} requests at rate {args.rate} "
                               f"req/s (seed 0), HTTP {'SSE streams' if stream else 'JSON bodies'} to {K} "
                               f"server process(es) on one port, round robin over {n} replica process(es), "
                               f"1,024 x 16 KV slots each",
                   "scheduler": ("the reference's (prefill and decode steps alternate)" if P == 0 else
                                 f"opt-in chunked prefill: decodes + up to {P} prompt tokens per step"),
                   "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32, TF32 off",
                   "parallelism": f"replicas{n} (processes)"},  # fmt: skip
        "client": {k: out[k] for k in ("requests", "output_tokens", "duration_s", "ttft_ms", "itl_ms",
                                       "latency_ms")},
        "preemptions": health["preemptions"],
        "wall_s": wall,
    }


def cpu_baseline(spec) -> dict:
    """The reference's own CPU step on the host cores, a bounded sample (about
    20 s of steps over the whole batch); the numpy port when the reference is
    not installed."""
    threads = os.cpu_count()
    got = reference_rate(spec, 30, 1, budget_s=20.0, threads=threads)
    if got is None:
        rate, sample, threads = cpu_oracle_rate(spec, 16, 2, 1)
        return {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}
    rate, timed, n, note, threads = got
    return {"value": rate, "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"{timed} decode steps x {n} sequences{note}: the reference's own paged_forward "
                      f"(baseline/_ref) on the host, float32"}  # fmt: skip


def reference_gpu_line(spec, args, local) -> dict | None:
    """The unmodified reference on this GPU, after this build's arm (N = 1):
    the "reference on B200" figure beside the main line."""
    device = torch.device("cuda", local)
    got = reference_rate(spec, args.steps, args.warmup, budget_s=60.0, device=device)
    if got is None:
        return None
    rate, timed, n, note, _ = got
    torch.cuda.empty_cache()
    return {"value": rate, "unit": "tok/s", "ms_per_step": n / rate * 1e3, "steps": timed,
            "sample": f"{timed} greedy decode steps x {n} sequences{note}: the reference's own GPT2 / "
                      "BlockAllocator / paged_forward (baseline/_ref) with device='cuda', TF32 off, host clock "
                      "per step (each step ends with the reference's own .tolist())"}  # fmt: skip


def run_reference(args, world, rank):
    """``--impl reference``: the reference's own CPU path on the host cores,
    on rank 0 alone, over this build's workload (the whole batch), timed step
    by step (``reference_rate``).  Nothing of this library is imported: the
    reference's ``BlockAllocator``, ``Sequence``, ``GPT2`` and ``paged_forward``
    run as installed in baseline/_ref.  Without that install, the numpy
    restatement (oracle/) is timed instead and labelled ``kind: "port"``."""
    if rank != 0:
        return None
    if args.workload in ("cfg5", "kvwrite"):
        return {"impl": "reference", "unavailable": f"{args.workload}: the CPU reference arm times decode and mixed "
                                                    "steps of the paged forward only"}  # fmt: skip
    threads = os.cpu_count()
    t0 = time.perf_counter()
    common = {"impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
              "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
              "data": "synthetic"}  # fmt: skip
    if args.workload == "cfg3":
        _load_library()
        bs = args.block_size or 16
        rate, sample, threads = cpu_oracle_mixed_rate(bs, max(1, min(args.steps, 3)), replica_seed(3, 0))
        return {**common, "metric": "mixed prefill+decode step rows/s", "value": rate, "unit": "rows/s",
                "config": {"workload": f"BASELINE config 3 mixed step, bs {bs}",
                           "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32"},
                "cpu_baseline": {"value": rate, "unit": "rows/s", "cores": threads, "kind": "port", "sample": sample},
                "e2e": {"value": rate, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "wall_s": time.perf_counter() - t0}  # fmt: skip
    spec = workload_spec(args)
    got = reference_rate(spec, args.steps, max(1, min(args.warmup, 2)), budget_s=150.0, threads=threads)
    if got is None:  # the reference is not installed: its numpy restatement
        _load_library()
        n = min(spec["n_seqs"], 16)
        rate, sample, threads = cpu_oracle_rate(spec, n, args.steps, args.warmup, budget_s=150)
        kind, same = "port", False
    else:
        rate, timed, n, note, threads = got
        kind, same = "reference", not note
        sample = (f"{timed} decode steps x {n} sequences of {spec['desc']}{note}: the reference's own paged_forward "
                  f"(baseline/_ref), float32, {threads} threads")  # fmt: skip
    return {**common, "metric": "decode tok/s", "value": rate, "unit": "tok/s", "ms_per_step": n / rate * 1e3,
            "config": {"workload": spec["desc"], "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32",
                       "same_config": same},
            "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": time.perf_counter() - t0}  # fmt: skip


def run_reference_gpu(args, world, rank, local) -> dict | None:
    """``--impl reference-gpu``: the unmodified reference on the same B200 (the
    "reference on B200" column): its own ``GPT2``, ``BlockAllocator`` and
    ``paged_forward`` with ``device="cuda"`` -- per step Python-built index
    tensors, the advanced-index scatter of the new K/V, the dense gather of
    every sequence's blocks and masked softmax over the padded key axis, torch
    fp32 linears with TF32 off, one step at a time and a ``.tolist()`` per step
    (tokquay/generate.py:63-120).  Same workload as this build's arm; nothing
    of this library is imported.  Each step is timed on the host clock: the
    reference's step ends with its own device-to-host read of the tokens."""
    if reference_package() is None:
        return {"impl": "reference-gpu", "unavailable": "the reference is not installed in baseline/_ref"}
    spec = workload_spec(args)
    device = torch.device("cuda", local)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    barrier(world)
    with ClockSampler(local) as clocks:
        rate, timed, n, note, _ = reference_rate(spec, args.steps, args.warmup, budget_s=120.0, device=device)
    ms = n / rate * 1e3
    ms_max = max_over_ranks(ms, world)
    tokens_all = sum_over_ranks(n, world)
    if rank != 0:
        return None
    return {
        "impl": "reference-gpu",
        "metric": "decode tok/s",
        "value": tokens_all / (ms_max * 1e-3),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": timed,
        "warmup": args.warmup,
        "ms_per_step": ms_max,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": spec["desc"] + note,
                   "model": "GPT-2 124M architecture, random-init N(0,0.02), fp32, TF32 off",
                   "algorithm": "the reference's own code (baseline/_ref) on the GPU: dense gather of every "
                                "sequence's blocks + masked softmax over the padded key axis"},  # fmt: skip
        "clocks": clocks.summary(),
    }


def _emit(res: dict) -> None:
    """The one JSON line, on the process's real stdout (everything else --
    library banners included -- goes to stderr)."""
    os.write(_STDOUT_FD, (json.dumps(res) + "\n").encode())


_STDOUT_FD = 1


def main():
    global _STDOUT_FD
    # Keep stdout for the result line alone: NCCL and other libraries may
    # print banners there during setup.
    sys.stdout.flush()
    _STDOUT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["cfg3", "cfg5", "cfg5-http", "kvwrite"], default="cfg2")
    ap.add_argument("--block-size", type=int, default=0, help="config 3: block size (16 or 32; default 16)")
    ap.add_argument("--trace-requests", type=int, default=400, help="config 5: requests of the trace served")
    ap.add_argument("--rate", default="64", help="config 5: arrival rate in requests/s, or inf for a burst")
    ap.add_argument("--mixed-tokens", type=int, default=0,
                    help="config 5: opt-in chunked-prefill scheduling with this many prompt tokens per step")
    ap.add_argument("--front-ends", type=int, default=1,
                    help="cfg5-http: server processes sharing the port (each over its share of the replicas)")
    ap.add_argument("--http-json", action="store_true",
                    help="cfg5-http: one JSON body per request instead of a server-sent event per token")
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graphs", action="store_true", help="launch every kernel from Python (no CUDA graphs)")
    ap.add_argument("--fused-lm-head", action="store_true",
                    help="opt-in: greedy steps end in the fused ln_f + LM head + argmax kernel "
                         "(tq_lm_head_argmax) instead of torch's fp32 matmul + tq_argmax_rows")
    ap.add_argument("--num-seqs", type=int, default=0, help="override the workload's sequence count (profiling)")
    ap.add_argument("--kernel-table", action="store_true",
                    help="after the run, print per-kernel device times of 10 more decode steps (stderr)")
    ap.add_argument("--pool-gb", type=float, default=0, help="override the KV pool size in GB (profiling)")
    ap.add_argument("--prompt-tile-rows", type=int, default=-1,
                    help="least prompt chunk (rows) run as tensor-core tiles; 0 = every prompt row on warp "
                         "items; default: the library's")
    ap.add_argument("--prompt-tile-pieces", type=int, default=-1,
                    help="most pieces a costly prompt tile is cut into over its keys (merged by a second "
                         "kernel after the attention grid); 1 = never cut; default: the library's")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (timing rule)")
        args.warmup = 3
    if args.workload == "cfg5-http":
        # One process: the front end spawns its own replica processes (--gpus of them).
        if args.impl != "ours" or ReplicaInfo.from_env().world > 1:
            _emit({"impl": args.impl, "unavailable": "cfg5-http runs our front end in one process "
                                                     "(not under torchrun, no reference arm)"})  # fmt: skip
            return
        _emit(run_serving_http(args))
        return
    if args.impl == "reference":
        # The CPU reference arm runs on rank 0 alone; no process group is needed.
        info = ReplicaInfo.from_env()
        world, rank, local = info.world, info.rank, info.local
        res = run_reference(args, world, rank)
        if rank == 0 and res is not None:
            _emit(res)
        return
    info = _replicas.setup()
    world, rank, local = info.world, info.rank, info.local
    if args.impl == "reference-gpu":
        res = run_reference_gpu(args, world, rank, local)
        if rank == 0 and res is not None:
            _emit(res)
        _replicas.teardown(info)
        return
    _load_library()
    if args.prompt_tile_rows >= 0:
        _lib.prompt_tiles(args.prompt_tile_rows)
    if args.prompt_tile_pieces > 0:
        _lib.prompt_tiles(-1, -1, -1, args.prompt_tile_pieces)
    tile_rows = _lib.prompt_tiles()  # (reads the setting)

    def tagged(res):  # the line names the prompt-tile setting it ran with
        if res is not None and isinstance(res.get("config"), dict):
            res["config"]["prompt_tile_min_rows"] = tile_rows
            if args.prompt_tile_pieces > 0:
                res["config"]["prompt_tile_max_pieces"] = args.prompt_tile_pieces
        return res

    if args.workload == "cfg5":
        res = tagged(run_serving(args, world, rank, local))
        if rank == 0 and res is not None:
            _emit(res)
        _replicas.teardown(info)
        return
    if args.workload == "kvwrite":
        res = run_kvwrite(args, world, rank, local)
        if rank == 0 and res is not None:
            _emit(res)
        _replicas.teardown(info)
        return
    if args.workload == "cfg3":
        res = tagged(run_mixed(args, world, rank, local))
        if rank == 0 and world == 1 and not args.no_cpu_baseline and res is not None:
            rate, sample, threads = cpu_oracle_mixed_rate(args.block_size or 16, 1, replica_seed(3, 0))
            res["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": threads, "kind": "port",
                                   "sample": sample}  # fmt: skip
        if rank == 0 and res is not None:
            _emit(res)
        _replicas.teardown(info)
        return
    res = run_ours(args, world, rank, local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(workload_spec(args))
        torch.cuda.empty_cache()
        res["reference_gpu"] = reference_gpu_line(workload_spec(args), args, local)
    if rank == 0 and res is not None:
        _emit(res)
    _replicas.teardown(info)


if __name__ == "__main__":
    main()
