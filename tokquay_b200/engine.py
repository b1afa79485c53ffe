"""The serving engine: Tokquay's own ``Engine`` over the B200 paged path.

The reference's engine runs as it is.  ``tokquay.engine.Engine(model,
allocator)`` given this package's ``GPT2`` and ``BlockAllocator`` already
drives the CUDA path: its step calls the reference's ``paged_forward``
(tokquay/generate.py:63-87), which asks the allocator for the step view
(``batch_for``: a ``DevicePagedBatch``, or a decode step staged into a
captured CUDA graph) and calls the model, whose fused forward runs the
kernels.  ``Engine`` below is that class with two hooks and nothing else:

* ``_sample`` -- when every row samples greedily and the logits come from a
  replayed decode graph, the graph has already taken the argmax
  (``tq_argmax_rows``), so those tokens are read back instead of running a
  second argmax (tokquay/engine.py:189-194 otherwise, unchanged);
* the opt-in chunked-prefill policy (``SchedulerConfig(mixed_prefill_tokens=P)``,
  ``tokquay_b200.scheduler``): a step feeds each sequence the tokens the
  scheduler gave it, and only sequences whose prompt is complete after the
  step draw a token.  With ``mixed_prefill_tokens`` 0 (the default) the
  scheduler and every step are the reference's.
"""

from __future__ import annotations

import torch

from tokquay_b200._host import ref_engine
from tokquay_b200.generate import paged_forward, paged_greedy_step
from tokquay_b200.scheduler import Scheduler as ChunkedScheduler

__all__ = ["GPT2_EOS_TOKEN_ID", "TokenEvent", "EngineStats", "KVSnapshot", "StepInfo", "Engine",
           "finish_reason_for", "sample_token"]  # fmt: skip

# The reference's records and helpers, re-exported for callers of this module.
GPT2_EOS_TOKEN_ID = ref_engine.GPT2_EOS_TOKEN_ID
TokenEvent = ref_engine.TokenEvent
EngineStats = ref_engine.EngineStats
KVSnapshot = ref_engine.KVSnapshot
StepInfo = ref_engine.StepInfo
finish_reason_for = ref_engine.finish_reason_for
sample_token = ref_engine.sample_token


class Engine(ref_engine.Engine):
    """``tokquay.engine.Engine`` with the greedy-token hook and the opt-in
    chunked-prefill step.  ``mixed_steps`` counts steps that fed prompt chunks
    beside decodes."""

    def __init__(self, model, allocator, config=None, eos_token_id: int = GPT2_EOS_TOKEN_ID):
        super().__init__(model, allocator, config, eos_token_id)
        self.mixed_steps = 0
        if getattr(config, "mixed_prefill_tokens", 0) > 0:
            self.scheduler = ChunkedScheduler(allocator, config)

    @property
    def chunked(self) -> bool:
        return isinstance(self.scheduler, ChunkedScheduler)

    @torch.no_grad()
    def step(self) -> list[TokenEvent]:
        """One iteration (tokquay/engine.py:149-180); the tokens it produced."""
        if not self.chunked:
            return super().step()
        return self._chunked_step()

    def _sample(self, seqs, logits: torch.Tensor) -> list[int]:
        runner = getattr(self.model, "graph_runner", None)
        if runner is not None and all(s.sampling.temperature == 0 for s in seqs):
            tokens = runner.greedy_tokens_for(logits)
            if tokens is not None:
                return tokens.tolist()  # the step's one device-to-host read
        return super()._sample(seqs, logits)

    def _chunked_step(self) -> list[TokenEvent]:
        batch = self.scheduler.schedule()
        if batch is None:
            self.last_step = None
            return []
        seqs, lens, st = batch.seqs, batch.new_lens, self.stats
        # The reference's step accounting (tokquay/engine.py:155-165), counting fed tokens.
        st.steps += 1
        st.decode_steps += 1
        st.max_batch = max(st.max_batch, len(seqs))
        st.peak_used_blocks = max(st.peak_used_blocks, self.allocator.num_used_blocks)
        st.num_preemptions = self.scheduler.num_preemptions
        st.positions_discarded = self.scheduler.num_discarded_positions
        st.positions_computed += sum(lens)
        st.positions_padded += batch.padded_tokens
        self.mixed_steps += max(lens) > 1

        if all(s.sampling.temperature == 0 for s in seqs):
            tokens = paged_greedy_step(self.model, self.allocator, seqs, lens)
        else:
            logits = paged_forward(self.model, self.allocator, seqs, lens)
            ready = [i for i, s in enumerate(seqs) if s.num_uncached_tokens == 0]
            picked = super()._sample([seqs[i] for i in ready], logits[ready]) if ready else []
            tokens = [0] * len(seqs)
            for i, t in zip(ready, picked):
                tokens[i] = t
        self.last_step = StepInfo(False, len(seqs), batch.padded_tokens, self.kv_snapshot())

        events = []
        for seq, tok in zip(seqs, tokens):
            if seq.num_uncached_tokens:  # a prompt chunk short of the prompt's end: no token yet
                continue
            seq.append_token(tok)
            why = self._finish_reason(seq, tok)
            if why:
                self.scheduler.finish(seq, why)
                self._rngs.pop(seq.seq_id, None)
            events.append(TokenEvent(seq.seq_id, tok, why))
        st.tokens_generated += len(events)
        return events
