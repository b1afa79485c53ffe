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
