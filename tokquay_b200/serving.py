"""Open-loop serving trace over the engine: BASELINE config 5's workload and metrics.

Restates the reference benchmark's workload and measurements
(bench/workload.py:24-47, bench/harness.py:60-177):

* ``make_workload``: ``n`` requests arriving as a Poisson process of ``rate``
  requests/s (``rate = inf``: a burst at time 0); prompt and output lengths
  uniform; the requests depend only on the seed, the arrival gaps are drawn
  at unit rate and divided by ``rate``, so runs at different rates serve the
  same requests;
* ``run_trace``: an open loop -- requests join when the workload says, whether
  or not the engine has kept up; a token's time is the end of the step that
  produced it (the step ends with its device-to-host read);
* ``summarize``: tokens/s from the first arrival to the last token, TTFT,
  inter-token latency and end-to-end latency percentiles.

``round_robin`` splits a workload over engine replicas the way the reference's
router does (request i to replica i mod N).
"""

from __future__ import annotations

import math
import random
import time
from dataclasses import dataclass, field

import numpy as np

from tokquay_b200._host import ref_sequence

SamplingParams = ref_sequence.SamplingParams

__all__ = ["RequestSpec", "make_workload", "round_robin", "run_trace", "summarize"]

VOCAB_SIZE = 50257  # GPT-2; prompts avoid the last id (<|endoftext|>)


@dataclass(frozen=True)
class RequestSpec:
    arrival: float  # seconds after the start of the run
    prompt_ids: tuple[int, ...]
    output_len: int


def make_workload(rate: float, n: int, seed: int = 0, prompt_len: tuple[int, int] = (16, 256),
                  output_len: tuple[int, int] = (16, 256)) -> list[RequestSpec]:  # fmt: skip
    """``n`` requests of a Poisson process of ``rate`` requests/s (bench/workload.py:24-47)."""
    if rate <= 0 or n < 1:
        raise ValueError("need rate > 0 and n >= 1")
    content, gaps = random.Random(seed), random.Random(seed + 1_000_003)
    t, specs = 0.0, []
    for _ in range(n):
        t += gaps.expovariate(1.0)
        prompt = tuple(content.randrange(VOCAB_SIZE - 1) for _ in range(content.randint(*prompt_len)))
        specs.append(RequestSpec(t / rate if math.isfinite(rate) else 0.0, prompt, content.randint(*output_len)))
    return specs


def round_robin(workload: list[RequestSpec], replicas: int, index: int) -> list[RequestSpec]:
    """The requests replica ``index`` of ``replicas`` serves (request i to replica i mod N)."""
    return workload[index::replicas]


@dataclass
class RequestRecord:
    arrival: float
    prompt_len: int
    output_len: int
    token_times: list[float] = field(default_factory=list)
    token_ids: list[int] = field(default_factory=list)


@dataclass
class StepRecord:
    t_start: float
    t_end: float
    is_prefill: bool
    num_seqs: int
    padded_tokens: int


def run_trace(engine, workload: list[RequestSpec], clock=time.perf_counter, sleep=time.sleep,
              idle_quantum: float = 0.005) -> tuple[list[RequestRecord], list[StepRecord], float]:  # fmt: skip
    """Drive ``engine`` (add_request / step / has_unfinished / last_step) in real time."""
    records: dict[int, RequestRecord] = {}
    steps: list[StepRecord] = []
    i, n = 0, len(workload)
    t0 = clock()
    while i < n or engine.has_unfinished():
        now = clock() - t0
        while i < n and workload[i].arrival <= now:
            spec = workload[i]
            i += 1
            seq = engine.add_request(list(spec.prompt_ids), SamplingParams(max_tokens=spec.output_len, ignore_eos=True))
            records[seq.seq_id] = RequestRecord(spec.arrival, len(spec.prompt_ids), spec.output_len)
        if not engine.has_unfinished():
            sleep(max(0.0, min(workload[i].arrival - now, idle_quantum)))
            continue
        start = clock() - t0
        events = engine.step()
        end = clock() - t0
        info = engine.last_step
        if info is None:
            raise RuntimeError("unfinished requests but nothing the engine can run")
        steps.append(StepRecord(start, end, info.is_prefill, info.num_seqs, info.padded_tokens))
        for ev in events:
            rec = records[ev.seq_id]
            rec.token_times.append(end)
            rec.token_ids.append(ev.token_id)
    return list(records.values()), steps, clock() - t0


def _pct(values) -> dict[str, float]:
    if len(values) == 0:
        return {"p50": float("nan"), "p99": float("nan"), "mean": float("nan")}
    a = np.asarray(values, dtype=float)
    return {"p50": float(np.percentile(a, 50)), "p99": float(np.percentile(a, 99)), "mean": float(a.mean())}


def summarize(records: list[RequestRecord], steps: list[StepRecord]) -> dict:
    """Throughput and latency of one run (bench/harness.py:149-177; times in ms)."""
    done = [r for r in records if r.token_times]
    tokens = sum(len(r.token_times) for r in done)
    first = min(r.arrival for r in records)
    last = max(r.token_times[-1] for r in done)
    gaps = [b - a for r in done for a, b in zip(r.token_times, r.token_times[1:])]
    return {
        "requests": len(records),
        "output_tokens": tokens,
        "duration_s": last - first,
        "throughput_tok_s": tokens / (last - first),
        "ttft_ms": {k: v * 1e3 for k, v in _pct([r.token_times[0] - r.arrival for r in done]).items()},
        "itl_ms": {k: v * 1e3 for k, v in _pct(gaps).items()},
        "latency_ms": {k: v * 1e3 for k, v in _pct([r.token_times[-1] - r.arrival for r in done]).items()},
        "steps": len(steps),
        "prefill_steps": sum(1 for s in steps if s.is_prefill),
        "decode_step_ms": {k: v * 1e3 for k, v in _pct([s.t_end - s.t_start for s in steps if not s.is_prefill]).items()},
    }
