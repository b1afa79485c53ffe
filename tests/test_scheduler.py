"""Scheduling over this package's allocator.

The reference's own scheduler (``tokquay.scheduler.Scheduler``, the default)
over ``tokquay_b200.BlockAllocator`` replays the traces recorded from the
reference scheduler over the reference's allocator (tests/golden/make_golden.py,
case ``sched_trace``): the same requests arrive at the same steps, each step
advances the sequences as paged_forward and the engine do (a model-free token
function stands in for sampling), and every step's batch, preemptions, queues,
block tables and free list must be equal.  The opt-in chunked-prefill policy
(``tokquay_b200.scheduler.Scheduler``) is checked for its invariants.
CPU only (the allocator's pool lives on the meta device).
"""

import sys
from pathlib import Path

import pytest

from helpers import load_golden
from tokquay.scheduler import RequestRejected
from tokquay.scheduler import Scheduler as RefScheduler
from tokquay.sequence import SamplingParams, Sequence
from tokquay_b200.kv_cache import BlockAllocator
from tokquay_b200.scheduler import Scheduler, SchedulerConfig

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_golden  # noqa: E402  (the trace driver the fixtures were recorded with)

GOLDEN = load_golden()
SCENARIOS = GOLDEN.cases["sched_trace"]["scenarios"]


@pytest.mark.parametrize("sc", SCENARIOS, ids=[s["name"] for s in SCENARIOS])
def test_scheduler_matches_the_reference_trace(sc):
    spec = {k: sc[k] for k in ("name", "num_blocks", "block_size", "free_seed", "config", "requests")}
    if "aborts" in sc:
        spec["aborts"] = sc["aborts"]
    got = make_golden.sched_scenario(BlockAllocator, RefScheduler, SchedulerConfig, Sequence, SamplingParams, spec)
    assert got["rejected"] == sc["rejected"]
    assert len(got["trace"]) == len(sc["trace"])
    for mine, ref in zip(got["trace"], sc["trace"]):
        assert mine == ref, mine["step"]
    assert got["outputs"] == sc["outputs"]


@pytest.mark.parametrize("mixed", [0, 16])
def test_rejections_and_config_checks(mixed):
    """The reference's up-front rejections hold for both policies."""
    alloc = BlockAllocator(make_golden._MiniCfg(), 8, 4, device="meta")
    cls = Scheduler if mixed else RefScheduler
    kw = dict(max_num_seqs=2, mixed_prefill_tokens=mixed)
    sched = cls(alloc, SchedulerConfig(max_num_batched_tokens=40, max_model_len=30, **kw))
    with pytest.raises(RequestRejected, match="model supports 30"):
        sched.add_request(Sequence(0, [1] * 20, sampling=SamplingParams(max_tokens=12)))
    with pytest.raises(RequestRejected, match="KV blocks"):
        cls(alloc, SchedulerConfig(max_num_batched_tokens=200, max_model_len=100, **kw)).add_request(
            Sequence(1, [1] * 40, sampling=SamplingParams(max_tokens=5)))
    with pytest.raises(ValueError):
        SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=2)
    with pytest.raises(ValueError):
        SchedulerConfig(mixed_prefill_tokens=-1)
    if not mixed:
        with pytest.raises(ValueError, match="mixed_prefill_tokens must be > 0"):
            Scheduler(alloc, SchedulerConfig())
    assert sched.schedule() is None and not sched.has_unfinished()


def _run_model_free(sched, alloc, requests, arrivals, token_of):
    """Drive a scheduler as the engine does, without a model: each step
    advances every batch sequence by its fed tokens (paged_forward), then each
    sequence at the end of its prompt or decoding gets a token, and finishes
    at max_tokens.  Returns the steps' (seq ids, fed tokens) and the outputs."""
    from tokquay.sequence import SequenceStatus

    seqs, steps = {}, []
    pending = sorted(zip(arrivals, range(len(requests))))
    step = 0
    while pending or sched.has_unfinished():
        while pending and pending[0][0] <= step:
            _, i = pending.pop(0)
            prompt, max_tokens = requests[i]
            seqs[i] = Sequence(i, list(prompt), sampling=SamplingParams(max_tokens=max_tokens, ignore_eos=True))
            sched.add_request(seqs[i])
        batch = sched.schedule()
        step += 1
        if batch is None:
            continue
        lens = getattr(batch, "new_lens", None) or [s.num_uncached_tokens for s in batch.seqs]
        steps.append(([s.seq_id for s in batch.seqs], list(lens), batch.is_prefill))
        for s, n in zip(batch.seqs, lens):
            assert 1 <= n <= s.num_uncached_tokens
            assert len(s.block_table) * alloc.block_size >= s.num_cached_tokens + n  # blocks cover the step
            s.num_cached_tokens += n
        for s in batch.seqs:
            if s.num_uncached_tokens == 0:
                s.append_token(token_of(s))
                if len(s.output_token_ids) >= s.sampling.max_tokens:
                    sched.finish(s, "length")
    assert all(s.status is SequenceStatus.FINISHED for s in seqs.values())
    return steps, {i: s.output_token_ids for i, s in seqs.items()}


@pytest.mark.parametrize("budget", [1, 7, 32, 200])
@pytest.mark.parametrize("tight", [False, True])
def test_mixed_prefill_policy(budget, tight):
    """The opt-in chunked-prefill policy: every decoding sequence runs every
    step, prompt tokens per step stay within the budget, each request gets all
    its tokens, admission is FCFS, preemption under a tight pool recomputes,
    and the pool is whole again at the end.  The token stream of a request
    (a function of its own tokens here) matches the reference policy's."""
    import random

    rng = random.Random(budget * 2 + tight)
    requests = [([rng.randrange(100) for _ in range(rng.randint(1, 40))], rng.randint(1, 12)) for _ in range(25)]
    arrivals = sorted(rng.randint(0, 30) for _ in requests)
    token_of = lambda s: (sum(s.token_ids) * 31 + len(s.token_ids)) % 97  # noqa: E731

    def run(mixed):
        alloc = BlockAllocator(make_golden._MiniCfg(), 20 if tight else 400, 4, device="meta")
        cfg = SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=64, max_model_len=64,
                              mixed_prefill_tokens=budget if mixed else 0)  # fmt: skip
        sched = (Scheduler if mixed else RefScheduler)(alloc, cfg)
        steps, out = _run_model_free(sched, alloc, requests, arrivals, token_of)
        assert alloc.num_free_blocks == alloc.num_blocks and sorted(alloc._free) == list(range(alloc.num_blocks))
        return steps, out, sched

    steps, out, sched = run(True)
    ref_steps, ref_out, _ = run(False)
    assert out == ref_out  # same tokens per request under either policy
    assert all(len(out[i]) == requests[i][1] for i in out)
    admitted = []
    for ids, lens, is_prefill in steps:
        assert not is_prefill
        assert sum(n for n in lens if n > 1) <= max(budget, 1)
        assert len(ids) <= 8
        admitted += [i for i in ids if i not in admitted]
    assert admitted == sorted(admitted)  # first come, first served
    if tight:
        assert sched.num_preemptions > 0
    if budget > 1:  # prompt chunks beside decodes
        assert any(max(lens) > 1 and min(lens) == 1 for _, lens, _ in steps)
