"""The scheduler (tokquay_b200/scheduler.py) makes the reference's decisions.

Replays the scheduler traces recorded from the unmodified reference scheduler
(tests/golden/make_golden.py, case ``sched_trace``): the same requests arrive
at the same steps, each step advances the sequences as paged_forward and the
engine do (a model-free token function stands in for sampling), and every
step's batch, preemptions, queues, block tables and free list must be equal.
CPU only (the allocator's pool lives on the meta device).
"""

import sys
from pathlib import Path

import pytest

from helpers import load_golden
from tokquay_b200.kv_cache import BlockAllocator
from tokquay_b200.scheduler import RequestRejected, Scheduler, SchedulerConfig
from tokquay_b200.sequence import SamplingParams, Sequence

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_golden  # noqa: E402  (the trace driver the fixtures were recorded with)

GOLDEN = load_golden()
SCENARIOS = GOLDEN.cases["sched_trace"]["scenarios"]


@pytest.mark.parametrize("sc", SCENARIOS, ids=[s["name"] for s in SCENARIOS])
def test_scheduler_matches_the_reference_trace(sc):
    spec = {k: sc[k] for k in ("name", "num_blocks", "block_size", "free_seed", "config", "requests")}
    if "aborts" in sc:
        spec["aborts"] = sc["aborts"]
    got = make_golden.sched_scenario(BlockAllocator, Scheduler, SchedulerConfig, Sequence, SamplingParams, spec)
    assert got["rejected"] == sc["rejected"]
    assert len(got["trace"]) == len(sc["trace"])
    for mine, ref in zip(got["trace"], sc["trace"]):
        assert mine == ref, mine["step"]
    assert got["outputs"] == sc["outputs"]


def test_rejections_and_config_checks():
    alloc = BlockAllocator(make_golden._MiniCfg(), 8, 4, device="meta")
    sched = Scheduler(alloc, SchedulerConfig(max_num_seqs=2, max_num_batched_tokens=40, max_model_len=30))
    with pytest.raises(RequestRejected, match="model supports 30"):
        sched.add_request(Sequence(0, [1] * 20, sampling=SamplingParams(max_tokens=12)))
    with pytest.raises(RequestRejected, match="KV blocks"):
        Scheduler(alloc, SchedulerConfig(max_num_seqs=2, max_num_batched_tokens=200, max_model_len=100)).add_request(
            Sequence(1, [1] * 40, sampling=SamplingParams(max_tokens=5)))
    with pytest.raises(ValueError):
        SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=2)
    assert sched.schedule() is None and not sched.has_unfinished()
