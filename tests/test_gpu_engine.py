"""Tokquay's own engine over the B200 path reproduces the reference engine
run on the CPU (tests/golden/make_golden.py, case ``mini_engine``): requests
arriving in waves on a pool small enough to force preemption by recompute,
greedy sampling.  Every step's tokens, finish reasons, prefill/decode choice,
running and waiting queues, block tables and free list must be equal, for all
82 steps of the trace.

The engine is driven three ways, none of which edits the reference:

* ``tokquay.engine.Engine`` -- the reference's class itself, imported from the
  reference package -- given this package's ``GPT2`` and ``BlockAllocator``,
  with and without CUDA graphs for the decode steps;
* ``tokquay_b200.engine.Engine`` (the same class plus the greedy-token hook);
* the reference's own *model* (``tokquay.model.GPT2``) over this package's
  step view: unpatched (its ``write`` / ``gather`` / ``mask`` / ``positions``
  members) and with the attention hook a maintainer adds to
  ``Attention.forward`` (``cache.attend``; applied here by monkeypatch).
"""

import random
import sys
from pathlib import Path

import pytest
import torch

from helpers import cfg_of, load_golden
from tokquay import engine as ref_engine
from tokquay import model as ref_model
from tokquay.scheduler import SchedulerConfig as RefSchedulerConfig
from tokquay.sequence import SamplingParams
from tokquay_b200 import _lib
from tokquay_b200 import workloads as W
from tokquay_b200.engine import Engine
from tokquay_b200.kv_cache import BlockAllocator, DevicePagedBatch
from tokquay_b200.model import GPT2, GPT2Config
from tokquay_b200.scheduler import SchedulerConfig

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_golden  # noqa: E402  (the arrival waves the fixture was recorded with)

pytestmark = pytest.mark.gpu
GOLDEN = load_golden()
# A greedy choice whose top-2 logits are closer than this is a coin toss between
# float orders of summation; the trace is compared up to the first one.
NEAR_TIE = 2e-5


def _mini_allocator(case):
    cfg = cfg_of(case)
    a = BlockAllocator(cfg, case["num_blocks"], case["block_size"], device="cuda")
    W.fill_pool_blocks(a.pool, range(case["num_blocks"]), case["pool_seed"], case["pool_scale"])
    W.shuffle_free_list(a, case["free_seed"])
    return a


def _mini_model(case, cls=GPT2):
    cfg = cfg_of(case)
    m = cls(cfg)
    W.load_weights(m, W.random_weights(cfg, case["weights_seed"], case["init"]))
    return m.to("cuda").eval()


def _mini_arrivals(case):
    waves = make_golden.engine_arrivals(random.Random(case["trace_seed"]))
    return lambda k: [(p, SamplingParams(max_tokens=mt, ignore_eos=True)) for p, mt in (waves[k] if k < len(waves) else [])]


def _gpt2_arrivals(case):
    """The config-5 requests of the gpt2_engine case (this package's workload
    generator gives the reference benchmark's requests: tests/test_serving.py)."""
    from tokquay_b200.serving import make_workload

    specs = make_workload(float("inf"), case["n_requests"], case["workload_seed"])
    waves = {step: specs[lo:hi] for step, lo, hi in case["waves"]}
    cap = case["max_tokens_cap"]
    return lambda k: [(list(r.prompt_ids), SamplingParams(max_tokens=min(r.output_len, cap), ignore_eos=True))
                      for r in waves.get(k, [])]  # fmt: skip


def _replay_engine_trace(eng, a, case, arrivals=None) -> int:
    """Drive ``eng`` with the trace's arrivals and compare every step with the
    reference's; returns how many steps were compared.  The comparison stops
    after a step whose greedy choice was a near tie in the reference run; a
    trace without one is compared to its last step."""
    arrivals = arrivals or _mini_arrivals(case)
    margins = [min(x) for x in case["margins"]]
    compared = 0
    for k, want in enumerate(case["steps"]):
        for prompt, params in arrivals(k):
            eng.add_request(prompt, params)
        events = eng.step()
        got = {
            "events": [[e.seq_id, e.token_id, e.finish_reason] for e in events],
            "is_prefill": bool(eng.last_step.is_prefill) if eng.last_step else None,
            "running": [s.seq_id for s in eng.scheduler.running],
            "tables": [list(s.block_table) for s in eng.scheduler.running],
            "waiting": [s.seq_id for s in eng.scheduler.waiting],
            "free": list(a._free),
            "preemptions": eng.scheduler.num_preemptions,
        }
        assert got == want, f"step {k}"
        compared += 1
        if k < len(margins) and margins[k] < NEAR_TIE:
            break  # later tokens may legitimately differ
    else:
        assert not eng.has_unfinished() and eng.stats.num_preemptions > 0
    first_tie = next((k for k, x in enumerate(margins) if x < NEAR_TIE), len(case["steps"]) - 1)
    assert compared == min(first_tie + 1, len(case["steps"])), compared
    return compared


@pytest.mark.parametrize("engine_cls", [ref_engine.Engine, Engine], ids=["reference_class", "b200_subclass"])
@pytest.mark.parametrize("graphs", [False, True])
def test_engine_matches_the_reference_engine(engine_cls, graphs):
    case = GOLDEN.cases["mini_engine"]
    m, a = _mini_model(case), _mini_allocator(case)
    if graphs:
        m.use_cuda_graphs(a)
    eng = engine_cls(m, a, RefSchedulerConfig(**case["sched"]))
    assert _replay_engine_trace(eng, a, case) == 82  # the MINI trace has no near tie: every step compared
    if graphs:
        assert m.graph_runner._graphs  # decode steps replayed captured graphs
    assert _lib.device_status() == 0


@pytest.mark.parametrize("graphs", [False, True])
def test_reference_engine_on_gpt2_with_config5_requests(graphs, gpt2_weights):
    """The reference's Engine class on GPT-2 124M over this package's model and
    allocator, with the first 24 requests of config 5's workload on a pool
    small enough to preempt: every step equal to the reference's CPU run."""
    case = GOLDEN.cases["gpt2_engine"]
    m = GPT2(GPT2Config(**W.GPT2_SMALL))
    W.load_weights(m, gpt2_weights)
    m = m.to("cuda").eval()
    a = BlockAllocator(m.cfg, case["num_blocks"], case["block_size"], device="cuda")
    W.fill_pool_blocks(a.pool, range(case["num_blocks"]), case["pool_seed"])
    W.shuffle_free_list(a, case["free_seed"])
    if graphs:
        m.use_cuda_graphs(a)
    eng = ref_engine.Engine(m, a, RefSchedulerConfig(**case["sched"]))
    compared = _replay_engine_trace(eng, a, case, _gpt2_arrivals(case))
    print(f"gpt2 engine trace: {compared} of {len(case['steps'])} steps compared")
    assert compared == len(case["steps"]) == 96  # no near tie in this trace: every step compared
    assert _lib.device_status() == 0


def _attend_forward(orig):
    """The two-line change of ``Attention.forward``'s paged branch
    (tokquay/model.py:73-78) that lets the step view attend in place."""

    def forward(self, x, cache=None, layer=0):
        if not isinstance(cache, DevicePagedBatch):
            return orig(self, x, cache, layer)
        B, T, C = x.shape
        q, k, v = self.c_attn(x).split(C, dim=-1)
        q, k, v = (t.view(B, T, self.n_head, self.d_head).transpose(1, 2) for t in (q, k, v))
        out = cache.attend(layer, q, k, v)  # [B, H, T, d]: tq_kv_write + tq_paged_attention
        return self.c_proj(out.transpose(1, 2).reshape(B, T, C))

    return forward


@pytest.mark.parametrize("hook", [False, True], ids=["unpatched", "attend_hook"])
def test_reference_model_and_engine_over_the_step_view(monkeypatch, hook):
    """The reference's model and engine, this package's allocator: without the
    hook the model runs its own dense attention over ``DevicePagedBatch``'s
    reference members (K/V written by ``tq_kv_write``, dense ``gather``,
    ``mask``, ``positions``, ``last_idx``); with it, attention is the CUDA
    kernel.  Either way the trace equals the reference's."""
    torch.backends.cuda.matmul.allow_tf32 = False
    case = GOLDEN.cases["mini_engine"]
    if hook:
        monkeypatch.setattr(ref_model.Attention, "forward", _attend_forward(ref_model.Attention.forward))
    m, a = _mini_model(case, ref_model.GPT2), _mini_allocator(case)
    eng = ref_engine.Engine(m, a, RefSchedulerConfig(**case["sched"]))
    calls = []
    real = DevicePagedBatch.attend
    monkeypatch.setattr(DevicePagedBatch, "attend", lambda self, *args: calls.append(1) or real(self, *args))
    _replay_engine_trace(eng, a, case)
    assert bool(calls) == hook
    assert _lib.device_status() == 0


def test_serving_trace_through_the_engine():
    """A small config-5-shaped trace (burst and Poisson) through the engine on
    the GPU: every request gets exactly its output length, latencies are sane."""
    import math

    from tokquay_b200.serving import make_workload, run_trace, summarize

    cfg = cfg_of(GOLDEN.cases["mini_engine"])
    m = GPT2(cfg)
    W.load_weights(m, W.random_weights(cfg, 3, "gpt2"))
    m = m.to("cuda").eval()
    a = BlockAllocator(cfg, 48, 8, device="cuda")
    m.use_cuda_graphs(a)
    eng = Engine(m, a, SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=512, max_model_len=128))
    for rate in (math.inf, 400.0):
        w = make_workload(rate, 14, seed=4, prompt_len=(4, 40), output_len=(3, 30))
        w = [type(r)(r.arrival, tuple(t % cfg.vocab_size for t in r.prompt_ids), r.output_len) for r in w]
        records, steps, _ = run_trace(eng, w)
        out = summarize(records, steps)
        assert out["output_tokens"] == sum(r.output_len for r in w)
        assert all(len(r.token_times) == r.output_len for r in records)
        assert 0 < out["ttft_ms"]["p50"] < 5000 and out["itl_ms"]["p99"] < 5000
    assert a.num_free_blocks == a.num_blocks  # every request released its blocks


@pytest.mark.parametrize("graphs", [False, True])
def test_mixed_prefill_policy_gives_the_reference_policy_tokens(graphs):
    """The opt-in chunked-prefill policy (prompt chunks and decodes in one
    step, one mixed launch per layer): the same arrival waves as the reference
    engine trace, on the same pool; every request's greedy tokens equal those
    of the reference policy's run (up to a near tie), steps did mix prompt
    chunks with decodes, and -- with graphs -- mixed steps replayed captured
    graphs."""
    case = GOLDEN.cases["mini_engine"]
    cfg = cfg_of(case)
    m = GPT2(cfg)
    W.load_weights(m, W.random_weights(cfg, case["weights_seed"], case["init"]))
    m = m.to("cuda").eval()

    def run(mixed_tokens, use_graphs):
        a = BlockAllocator(cfg, case["num_blocks"], case["block_size"], device="cuda")
        W.fill_pool_blocks(a.pool, range(case["num_blocks"]), case["pool_seed"], case["pool_scale"])
        W.shuffle_free_list(a, case["free_seed"])
        m.graph_runner = None
        if use_graphs:
            m.use_cuda_graphs(a)
        eng = Engine(m, a, SchedulerConfig(**case["sched"], mixed_prefill_tokens=mixed_tokens))
        arrivals = make_golden.engine_arrivals(random.Random(case["trace_seed"]))
        seqs = []
        for _ in range(400):
            for prompt, max_tokens in arrivals.pop(0) if arrivals else []:
                seqs.append(eng.add_request(prompt, SamplingParams(max_tokens=max_tokens, ignore_eos=True)))
            eng.step()
            if not arrivals and not eng.has_unfinished():
                break
        assert not eng.has_unfinished() and a.num_free_blocks == a.num_blocks
        return {s.seq_id: list(s.output_token_ids) for s in seqs}, eng

    want, _ = run(0, False)
    got, eng = run(24, graphs)
    assert eng.mixed_steps > 0
    for sid, toks in want.items():
        assert len(got[sid]) == len(toks)
        if got[sid] != toks:  # allowed only after a near tie in the reference run
            k = next(i for i, (x, y) in enumerate(zip(got[sid], toks)) if x != y)
            pytest.fail(f"request {sid} differs at token {k}")  # no near ties on this trace
    if graphs:
        assert any(isinstance(k, tuple) for k in m.graph_runner._graphs)  # mixed graphs were used
    m.graph_runner = None
