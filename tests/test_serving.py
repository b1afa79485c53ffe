"""The serving workload and metrics (tokquay_b200/serving.py) on the CPU.

The generator must give the reference benchmark's requests (fixture recorded
from bench/workload.py by tests/golden/make_golden.py, case ``workload``), and
the open-loop driver and summary must account tokens and latencies right; a
fake engine with a fixed step time stands in for the GPU.
"""

import math

import pytest

from helpers import load_golden
from tokquay_b200.engine import StepInfo, KVSnapshot, TokenEvent
from tokquay.sequence import Sequence
from tokquay_b200.serving import make_workload, round_robin, run_trace, summarize

GOLDEN = load_golden()


@pytest.mark.parametrize("case", GOLDEN.cases["workload"]["cases"], ids=lambda c: f"rate{c['rate']}-seed{c['seed']}")
def test_workload_matches_the_reference_generator(case):
    rate = math.inf if case["rate"] == "inf" else case["rate"]
    specs = make_workload(rate, case["n"], case["seed"])
    assert [r.arrival for r in specs] == pytest.approx(case["arrivals"], rel=0, abs=0)
    assert [r.output_len for r in specs] == case["output_lens"]
    assert [len(r.prompt_ids) for r in specs] == case["prompt_lens"]
    assert [list(r.prompt_ids[:4]) for r in specs] == case["prompt_heads"]
    assert [sum(r.prompt_ids) for r in specs] == case["prompt_sums"]


def test_round_robin_partitions_the_trace():
    w = make_workload(64.0, 23, 1)
    parts = [round_robin(w, 4, i) for i in range(4)]
    assert sorted((r.arrival for p in parts for r in p)) == [r.arrival for r in w]
    assert [len(p) for p in parts] == [6, 6, 6, 5]


class FakeEngine:
    """Every step takes 10 ms of the fake clock and gives each running request one token."""

    def __init__(self, clock):
        self.clock, self.running, self.next_id, self.last_step = clock, [], 0, None

    def add_request(self, prompt, params):
        s = Sequence(self.next_id, prompt, sampling=params)
        self.next_id += 1
        self.running.append(s)
        return s

    def has_unfinished(self):
        return bool(self.running)

    def step(self):
        self.clock.t += 0.010
        ev = []
        for s in list(self.running):
            s.append_token(1)
            done = len(s.output_token_ids) >= s.sampling.max_tokens
            ev.append(TokenEvent(s.seq_id, 1, "length" if done else None))
            if done:
                self.running.remove(s)
        self.last_step = StepInfo(False, len(ev), len(ev), KVSnapshot(0, 0, len(self.running)))
        return ev


class FakeClock:
    t = 0.0

    def __call__(self):
        return self.t

    def sleep(self, dt):
        self.t += dt


def test_open_loop_driver_and_summary():
    clock = FakeClock()
    w = make_workload(math.inf, 5, 2, prompt_len=(3, 5), output_len=(2, 4))
    records, steps, wall = run_trace(FakeEngine(clock), w, clock=clock, sleep=clock.sleep)
    out = summarize(records, steps)
    assert out["output_tokens"] == sum(r.output_len for r in w)
    assert out["ttft_ms"]["p50"] == pytest.approx(10.0)  # every request's first token after one step
    assert out["itl_ms"]["p99"] == pytest.approx(10.0)
    assert out["throughput_tok_s"] == pytest.approx(out["output_tokens"] / (max(r.output_len for r in w) * 0.010))


def _reference_harness():
    """The reference benchmark's bench/harness.py (installed beside tokquay).
    Its package is named ``bench``, as is this repository's bench.py, so it is
    loaded under that name only for the import."""
    import importlib.util
    import sys
    from pathlib import Path

    import tokquay

    pkg_dir = Path(tokquay.__file__).resolve().parents[1] / "bench"
    saved = {k: sys.modules.pop(k) for k in [m for m in sys.modules if m == "bench" or m.startswith("bench.")]}
    try:
        spec = importlib.util.spec_from_file_location("bench", pkg_dir / "__init__.py",
                                                      submodule_search_locations=[str(pkg_dir)])  # fmt: skip
        pkg = importlib.util.module_from_spec(spec)
        sys.modules["bench"] = pkg
        spec.loader.exec_module(pkg)
        import bench.harness as harness  # noqa: PLC0415

        return harness
    finally:
        for k in [m for m in sys.modules if m == "bench" or m.startswith("bench.")]:
            del sys.modules[k]
        sys.modules.update(saved)


def test_summarize_matches_the_reference_harness():
    """Throughput, TTFT, inter-token latency and end-to-end latency as the
    reference's bench/harness.py:149-177 computes them, on one synthetic run."""
    import random

    from tokquay_b200.serving import RequestRecord, StepRecord

    h = _reference_harness()
    rng = random.Random(3)
    mine, theirs, t = [], [], 0.0
    for i in range(40):
        arrival = rng.uniform(0, 2)
        times = sorted(arrival + rng.uniform(0.001, 3) for _ in range(rng.randint(0 if i == 7 else 1, 30)))
        mine.append(RequestRecord(arrival, 10, len(times), list(times)))
        theirs.append(h.RequestRecord(arrival, 10, len(times), list(times)))
    steps = [StepRecord(0.1 * k, 0.1 * k + 0.05, k % 5 == 0, 4, 16) for k in range(30)]
    ref_steps = [h.StepRecord(s.t_start, s.t_end, s.is_prefill, 4, 16, 64, 40, 4) for s in steps]
    got = summarize(mine, steps)
    want = h.summarize(h.RunResult(theirs, ref_steps, {}, 5.0), 73728)
    for key in ("requests", "output_tokens"):
        assert got[key] == want[key]
    for key in ("duration_s", "throughput_tok_s"):
        assert got[key] == pytest.approx(want[key], rel=1e-12)
    for key in ("ttft_ms", "itl_ms", "latency_ms"):
        for q in ("p50", "p99", "mean"):
            assert got[key][q] == pytest.approx(want[key][q], rel=1e-9), (key, q)
