"""Continuous-batching engine over the B200 paged path (the caller of the hot path).

Restates the reference engine's step loop (tokquay/engine.py:1-13, :98-197):
each ``step()`` asks the scheduler for a batch (which already grew the blocks
for the tokens about to be written), runs one paged forward over it, samples
one token per sequence and applies the stop conditions.  Greedy rows are
sampled with one ``tq_argmax_rows`` kernel; rows with a temperature use
per-request generators exactly as the reference does, so token streams match
it given the same logits.  Synchronous and not thread-safe: one thread drives
an engine (the reference's server does the same, tokquay/async_engine.py:8-11).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from tokquay_b200.generate import paged_forward, paged_greedy_step
from tokquay_b200.kv_cache import BlockAllocator
from tokquay_b200.model import GPT2, argmax_rows
from tokquay_b200.scheduler import Scheduler, SchedulerConfig
from tokquay_b200.sequence import SamplingParams, Sequence

__all__ = ["GPT2_EOS_TOKEN_ID", "TokenEvent", "EngineStats", "KVSnapshot", "StepInfo", "Engine",
           "finish_reason_for", "sample_token"]  # fmt: skip

GPT2_EOS_TOKEN_ID = 50256


@dataclass
class TokenEvent:
    """A new token; ``finish_reason`` ("length" / "stop") on a sequence's last."""

    seq_id: int
    token_id: int
    finish_reason: str | None = None


@dataclass
class EngineStats:
    steps: int = 0
    prefill_steps: int = 0
    decode_steps: int = 0
    tokens_generated: int = 0
    max_batch: int = 0
    peak_used_blocks: int = 0
    num_preemptions: int = 0
    positions_computed: int = 0  # real positions fed to the model (prompts, recomputes, decodes)
    positions_padded: int = 0  # batch x longest row per step, as the reference counts it
    positions_discarded: int = 0  # cached positions thrown away by preemption
    mixed_steps: int = 0  # steps that fed prompt chunks beside decodes (opt-in policy)


@dataclass
class KVSnapshot:
    allocated_tokens: int  # slots of the blocks running sequences hold
    live_tokens: int  # slots holding a cached token
    num_seqs: int


@dataclass
class StepInfo:
    is_prefill: bool
    num_seqs: int
    padded_tokens: int
    kv: KVSnapshot  # after the forward, before finished sequences free their blocks


def finish_reason_for(seq: Sequence, token: int, eos_token_id: int) -> str | None:
    """"stop" on EOS (unless ignored), "length" at max_tokens, else None."""
    if token == eos_token_id and not seq.sampling.ignore_eos:
        return "stop"
    return "length" if len(seq.output_token_ids) >= seq.sampling.max_tokens else None


def sample_token(logits: torch.Tensor, params: SamplingParams, generator: torch.Generator | None) -> int:
    """One token from a row of logits: greedy, or temperature with optional
    top-k (ties at the k-th value kept), drawn with ``generator``."""
    if params.temperature == 0:
        return int(logits.argmax())
    scaled = logits / params.temperature
    if params.top_k > 0:
        kth = torch.topk(scaled, min(params.top_k, scaled.numel())).values[-1]
        scaled = scaled.masked_fill(scaled < kth, float("-inf"))
    return int(torch.multinomial(torch.softmax(scaled, dim=-1), 1, generator=generator))


class Engine:
    """Model + allocator + scheduler (tokquay/engine.py:98-197)."""

    def __init__(self, model: GPT2, allocator: BlockAllocator, config: SchedulerConfig | None = None,
                 eos_token_id: int = GPT2_EOS_TOKEN_ID):  # fmt: skip
        config = config or SchedulerConfig(max_model_len=model.cfg.n_positions)
        if config.max_model_len > model.cfg.n_positions:
            raise ValueError("max_model_len exceeds the model's context window")
        self.model = model
        self.allocator = allocator
        self.scheduler = Scheduler(allocator, config)
        self.eos_token_id = eos_token_id
        self.stats = EngineStats()
        self.last_step: StepInfo | None = None
        self._next_id = 0
        self._rngs: dict[int, torch.Generator] = {}

    # ---- requests --------------------------------------------------------------------
    def add_request(self, prompt_token_ids: list[int], params: SamplingParams | None = None) -> Sequence:
        """Queue a request; ``RequestRejected`` if it can never be served (the
        id is spent only on success)."""
        seq = Sequence(self._next_id, list(prompt_token_ids), sampling=params or SamplingParams())
        self.scheduler.add_request(seq)
        self._next_id += 1
        if seq.sampling.temperature > 0:
            gen = torch.Generator(device=self.allocator.pool.device)
            gen.manual_seed(seq.sampling.seed if seq.sampling.seed is not None else torch.seed() % 2**63)
            self._rngs[seq.seq_id] = gen
        return seq

    def abort_request(self, seq: Sequence) -> None:
        """Cancel a request and free its blocks; call between steps."""
        self.scheduler.abort(seq)
        self._rngs.pop(seq.seq_id, None)

    def has_unfinished(self) -> bool:
        return self.scheduler.has_unfinished()

    def kv_snapshot(self) -> KVSnapshot:
        running = self.scheduler.running
        return KVSnapshot(self.allocator.num_used_blocks * self.allocator.block_size,
                          sum(s.num_cached_tokens for s in running), len(running))  # fmt: skip

    # ---- the loop --------------------------------------------------------------------
    @torch.no_grad()
    def step(self) -> list[TokenEvent]:
        """One iteration; the tokens it produced (none when idle)."""
        batch = self.scheduler.schedule()
        if batch is None:
            self.last_step = None
            return []
        st, sched = self.stats, self.scheduler
        st.steps += 1
        st.prefill_steps += int(batch.is_prefill)
        st.decode_steps += int(not batch.is_prefill)
        st.max_batch = max(st.max_batch, len(batch.seqs))
        st.peak_used_blocks = max(st.peak_used_blocks, self.allocator.num_used_blocks)
        st.num_preemptions = sched.num_preemptions
        st.positions_discarded = sched.num_discarded_positions
        lens = batch.new_lens
        st.positions_computed += sum(lens) if lens else sum(s.num_uncached_tokens for s in batch.seqs)
        st.positions_padded += batch.padded_tokens
        st.mixed_steps += int(bool(lens) and max(lens) > 1)

        if all(s.sampling.temperature <= 0 for s in batch.seqs):  # greedy rows only: tokens straight back
            tokens = paged_greedy_step(self.model, self.allocator, batch.seqs, lens)
        else:
            tokens = self._sample(batch.seqs, paged_forward(self.model, self.allocator, batch.seqs, lens))
        self.last_step = StepInfo(batch.is_prefill, len(batch.seqs), batch.padded_tokens, self.kv_snapshot())
        events = []
        for seq, tok in zip(batch.seqs, tokens):
            if seq.num_uncached_tokens > 0:  # a prompt chunk short of the prompt's end: no token yet
                continue
            seq.append_token(tok)
            why = finish_reason_for(seq, tok, self.eos_token_id)
            if why:
                sched.finish(seq, why)
                self._rngs.pop(seq.seq_id, None)
            events.append(TokenEvent(seq.seq_id, tok, why))
        st.tokens_generated += len(events)
        return events

    def run_until_done(self) -> list[TokenEvent]:
        out: list[TokenEvent] = []
        while self.has_unfinished():
            out += self.step()
        return out

    def _sample(self, seqs: list[Sequence], logits: torch.Tensor) -> list[int]:
        """Greedy rows in one argmax kernel, sampled rows one by one; the
        step's single device-to-host read (tokquay/engine.py:189-194)."""
        tokens = argmax_rows(logits.contiguous())
        for i, s in enumerate(seqs):
            if s.sampling.temperature > 0 and s.num_uncached_tokens == 0:  # mid-prompt rows draw nothing
                tokens[i] = sample_token(logits[i], s.sampling, self._rngs[s.seq_id])
        return tokens.tolist()
