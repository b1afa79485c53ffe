"""CUDA-graph replay of the decode step.

A decode step (one new token per sequence) launches ~75 of this package's
kernels and ~60 torch ops; issued one by one from Python that costs more host
time than the GPU spends on a 64-sequence step.  ``DecodeGraphRunner``
captures the whole step -- paged forward plus the greedy argmax -- once per
batch-size bucket, over a ``PlanWorkspace`` of that bucket's capacities, and
replays it: per step the host only plans (``tq_plan_step``, in C), copies the
plan into the workspace and launches the graph.

A bucket's graph runs any decode batch of up to ``bucket`` sequences: the
kernels read the step's true token, work-item and combine counts from the
device plan, and the GEMMs / argmax run over the bucket's rows (the rows past
the batch hold stale values whose results are never read).  Steps that feed
prompt chunks beside decode rows (the opt-in chunked-prefill scheduler) replay
graphs keyed by (sequence bucket, row capacity) the same way.
"""

from __future__ import annotations

import bisect
import weakref

import torch

from tokquay_b200 import _lib
from tokquay_b200.kv_cache import BatchedKV, BlockAllocator, DevicePagedBatch, PlanWorkspace, _hostpack
from tokquay_b200.model import argmax_rows

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)
# Row capacities of mixed-step graphs: a bucket of b sequences with up to
# b + e rows (decode rows plus prompt chunks), e from this list.
DEFAULT_MIXED_EXTRA = (32, 128, 512)


class DecodeGraphRunner:
    """Captured decode steps for one model and one allocator (pool).

    ``run(seqs)`` = ``paged_forward`` for a batch where every sequence feeds
    exactly one token; returns a fresh ``[B, vocab]`` logits tensor (the
    graph's own output buffer is overwritten by the next replay).
    """

    def __init__(self, model, allocator: BlockAllocator, buckets=DEFAULT_BUCKETS, max_ctx: int | None = None,
                 mixed_extra=DEFAULT_MIXED_EXTRA):  # fmt: skip
        if allocator.pool.device.type != "cuda":
            raise RuntimeError("CUDA graphs need the pool on a CUDA device")
        self.model = model
        self.allocator = allocator
        self.buckets = sorted(set(int(b) for b in buckets))
        self.mixed_extra = sorted(set(int(e) for e in mixed_extra))
        self.max_ctx = max_ctx or model.cfg.n_positions
        # decode bucket (int) or mixed (sequences, rows) capacities -> (graph, workspace,
        # logits, greedy tokens, launches per replay)
        self._graphs: dict[int | tuple[int, int], tuple] = {}
        self._pool = None  # one private memory pool shared by every bucket's graph
        self._staged = 0  # serial number of the last step staged by stage_step()
        self._greedy = None  # (weakref to the last replay's logits, rows, the graph's argmax buffer)

    @property
    def max_batch(self) -> int:
        return self.buckets[-1]

    def bucket_for(self, n: int) -> int | None:
        i = bisect.bisect_left(self.buckets, n)
        return self.buckets[i] if i < len(self.buckets) else None

    def _capture(self, key):
        # int: a decode bucket; (sequences, rows): a mixed step; ("greedy", bucket):
        # a decode bucket that ends in the fused LM head + argmax (no logits).
        greedy = isinstance(key, tuple) and key[0] == "greedy"
        if greedy:
            bucket = rows = key[1]
        else:
            bucket, rows = (key, key) if isinstance(key, int) else key
        ws = PlanWorkspace(self.allocator, bucket, rows, self.max_ctx)
        # A plan whose counts are all zero: every kernel of the step exits at
        # once, so the warm-up run below touches neither the pool nor anything else.
        ws.plan.zero_()
        view = _CaptureView(ws)
        dev = self.allocator.pool.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):  # warm cuBLAS handles and workspaces outside the capture
                if greedy:
                    self.model.forward_paged(view, last_only=True,
                                             greedy_out=torch.empty(bucket, dtype=torch.int64, device=dev))
                else:
                    lg = self.model.forward_paged(view, last_only=True)[:, 0]
                    argmax_rows(lg, d_num_rows=view.count_ptr(3), max_rows=bucket)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        launches = self.model.kernel_launches
        with torch.cuda.graph(graph, pool=self._pool):
            if greedy:
                tokens = torch.empty(bucket, dtype=torch.int64, device=dev)
                self.model.forward_paged(view, last_only=True, greedy_out=tokens)
                logits = None
            else:
                logits = self.model.forward_paged(view, last_only=True)[:, 0]
                tokens = argmax_rows(logits, d_num_rows=view.count_ptr(3), max_rows=bucket)  # greedy sampling
        per_replay = self.model.kernel_launches - launches + (0 if greedy else 1)
        self.model.kernel_launches = launches
        entry = (graph, ws, logits, tokens, per_replay)
        self._graphs[key] = entry
        return entry

    def graph(self, key):
        """The graph of a decode bucket (an int), of a mixed step's (sequences,
        rows) capacities, or of a decode bucket ending in the fused LM head
        (("greedy", bucket)); captured on first use."""
        return self._graphs.get(key) or self._capture(key)

    def mixed_key(self, n_seqs: int, n_rows: int) -> tuple[int, int] | None:
        b = self.bucket_for(n_seqs)
        if b is None:
            return None
        for e in self.mixed_extra:
            if n_rows <= b + e:
                return (b, b + e)
        return None

    def greedy_key(self, bucket: int):
        """The graph key of a decode bucket whose tokens alone are wanted: the
        fused-head variant when the model has it on and the bucket fits it."""
        if self.model.fused_lm_head and bucket <= _lib.LM_HEAD_MAX_ROWS:
            return ("greedy", bucket)
        return bucket

    def _replay_step(self, seqs: list, new_lens: list[int] | None, greedy: bool = False) -> tuple | None:
        B = len(seqs)
        bucket = self.bucket_for(B) if B else None
        if bucket is None:
            return None
        stream = torch.cuda.current_stream(self.allocator.pool.device)
        vocab = self.model.cfg.vocab_size
        entry = None
        if new_lens is None or max(new_lens) == 1:  # a decode step
            entry = self.graph(self.greedy_key(bucket) if greedy else bucket)
            if entry[1].stage_sequences(seqs, new_lens, stream, vocab, decode_max_ctx=self.max_ctx) is None:
                entry = None
        if entry is None and new_lens is not None and self.mixed_extra:  # prompt chunks beside decodes
            key = self.mixed_key(B, sum(new_lens))
            if key is not None:
                entry = self.graph(key)
                if entry[1].stage_sequences(seqs, new_lens, stream, vocab, fit_only=True) is None:
                    entry = None
        if entry is None:
            return None
        graph, ws, _, _, per_replay = entry
        self.model.last_h2d_bytes = ws.last_used_ints * 4
        self._greedy = None  # the argmax buffers change under any earlier replay's logits
        graph.replay()
        self.model.kernel_launches += per_replay
        return entry

    def stage_step(self, seqs, new_lens: list[int] | None = None) -> "GraphStepBatch | None":
        """Plan a decode step into its bucket's workspace and return the step
        view that replays the bucket's graph (``BlockAllocator.batch_for`` with
        graphs on); None, with nothing staged, for any other step."""
        B = len(seqs)
        bucket = self.bucket_for(B) if B else None
        if bucket is None or (new_lens is not None and max(new_lens) != 1):
            return None
        entry = self.graph(bucket)
        stream = torch.cuda.current_stream(self.allocator.pool.device)
        layout = entry[1].stage_sequences(seqs, new_lens, stream, self.model.cfg.vocab_size,
                                          decode_max_ctx=self.max_ctx)  # fmt: skip
        if layout is None:
            return None
        self._staged += 1
        return GraphStepBatch(self, entry, B, int(layout[_lib.PLAN_MAX_CTX]), self._staged)

    def greedy_tokens_for(self, logits: torch.Tensor) -> torch.Tensor | None:
        """The greedy tokens the graph computed with ``logits``, when these are
        (a view of) the logits of the last ``GraphStepBatch`` replay; else None."""
        g = self._greedy
        if g is None or logits.dim() != 2:
            return None
        ref, rows, tokens = g
        base = logits._base if logits._base is not None else logits
        if base is not ref() or logits.shape[0] != rows:
            return None
        return tokens[:rows]

    def try_run(self, seqs: list, new_lens: list[int] | None = None) -> torch.Tensor | None:
        """``run`` for a step that turns out to be a decode step (one new token
        per sequence, context within the graphs' capacity) that fits a
        bucket; None, with nothing planned or launched, for any other step.
        Decides in the native packer, without a Python pass over the sequences."""
        entry = self._replay_step(seqs, new_lens)
        return None if entry is None else entry[2][:len(seqs)].clone()

    def try_run_greedy(self, seqs: list, new_lens: list[int] | None = None) -> torch.Tensor | None:
        """``try_run`` returning the step's greedy tokens instead of its logits:
        the ``[B]`` int64 argmax the graph computed (a copy), so a greedy
        decode loop neither copies the ``[B, vocab]`` logits nor runs a second
        argmax; None, with nothing planned or launched, for any other step."""
        entry = self._replay_step(seqs, new_lens, greedy=True)
        return None if entry is None else entry[3][:len(seqs)].clone()

    def decode_steps(self, seqs: list, n_steps: int) -> list[list[int]] | None:
        """``n_steps`` greedy decode steps of a fixed batch, one step ahead of
        the host: while step k runs, the host already plans step k+1 (the
        sequences' lengths and blocks do not depend on the token values) with a
        placeholder token id, and step k's argmax is copied into step k+1's
        plan on the device; step k's tokens reach the host (and replace the
        placeholders) while step k+1 runs.  After each step every sequence has
        its token appended, and every step but the last is followed by
        ``allocator.append_slot`` -- the state the one-step-at-a-time loop
        leaves.  Returns the tokens per sequence, or None (nothing run) when the
        first step is not a decode step that fits a bucket; a later step that
        does not fit ends the pipeline, and the remaining steps go one at a
        time through ``paged_forward``'s eager path."""
        B = len(seqs)
        bucket = self.bucket_for(B) if B else None
        if bucket is None or n_steps < 1:
            return None
        graph, ws, _, tokens, per_replay = self.graph(self.greedy_key(bucket))
        dev = self.allocator.pool.device
        stream = torch.cuda.current_stream(dev)
        vocab = self.model.cfg.vocab_size
        ids_off = int(ws.layout[_lib.PLAN_OFF_TOKEN_IDS])
        host = torch.empty((n_steps, B), dtype=torch.int64, pin_memory=True)
        ready: list[torch.cuda.Event] = []
        out: list[list[int]] = [[] for _ in seqs]

        self.step_h2d_bytes = []  # host->device plan bytes of each replayed step

        def launch(k: int) -> None:
            self.model.last_h2d_bytes = ws.last_used_ints * 4
            self.step_h2d_bytes.append(ws.last_used_ints * 4)
            if k > 0:  # the previous step's argmax feeds this step, on the device
                ws.plan[ids_off:ids_off + B].copy_(tokens[:B])
            self._greedy = None
            graph.replay()
            self.model.kernel_launches += per_replay
            _advance(seqs)
            host[k].copy_(tokens[:B], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            ready.append(ev)

        def settle(k: int, appended: bool) -> None:
            """Step k's tokens into the sequences (over the placeholders if appended)."""
            ready[k].synchronize()
            toks = host[k].tolist()
            for s, o, t in zip(seqs, out, toks):
                if appended:
                    s.output_token_ids[-1] = t
                else:
                    s.append_token(t)
                o.append(t)

        if ws.stage_sequences(seqs, None, stream, vocab, decode_max_ctx=self.max_ctx) is None:
            return None
        launch(0)
        done = 1
        while done < n_steps:
            n_placed = 0
            try:
                for s in seqs:  # step done-1's token, not known yet: a placeholder
                    s.append_token(0)
                    n_placed += 1
                    self.allocator.append_slot(s)
            except BaseException:  # e.g. OutOfBlocksError: leave the real tokens behind
                ready[done - 1].synchronize()
                for i, (s, o, t) in enumerate(zip(seqs, out, host[done - 1].tolist())):
                    if i < n_placed:
                        s.output_token_ids[-1] = t
                    else:
                        s.append_token(t)
                    o.append(t)
                raise
            if ws.stage_sequences(seqs, None, stream, vocab, decode_max_ctx=self.max_ctx) is None:
                settle(done - 1, True)
                break
            launch(done)
            settle(done - 1, True)
            done += 1
        else:
            settle(n_steps - 1, False)
            return out
        from tokquay_b200.generate import _eager_greedy

        for k in range(done, n_steps):  # the rest one at a time, eagerly
            toks = _eager_greedy(self.model, self.allocator, seqs, None).tolist()
            for s, o, t in zip(seqs, out, toks):
                s.append_token(t)
                o.append(t)
                if k + 1 < n_steps:
                    self.allocator.append_slot(s)
        return out

    def run(self, seqs: list) -> torch.Tensor:
        """``try_run`` for a step known to be a decode step that fits: ``[B, vocab]``
        logits (a copy); ValueError otherwise.  Does not advance the sequences."""
        logits = self.try_run(seqs)
        if logits is None:
            raise ValueError(f"not a decode step of at most {self.max_batch} sequences within "
                             f"{self.max_ctx} positions")
        return logits

    def replay_plan(self, bucket: int, plan: torch.Tensor, ids: torch.Tensor | None = None) -> torch.Tensor:
        """Replay ``bucket``'s graph on a plan already in device memory (built
        with that bucket's workspace capacities and grid, ``PlanWorkspace.caps``
        and ``.n_ctas``),
        optionally overwriting its token ids from a device tensor first.
        Returns the graph's greedy-token buffer (valid until the next replay)."""
        graph, ws, _, tokens, per_replay = self.graph(self.greedy_key(bucket))
        if plan.numel() != ws.total:
            raise ValueError(f"plan of {plan.numel()} int32 does not fit bucket {bucket}'s workspace "
                             f"({ws.total}); plan it with that workspace's caps and n_ctas ({ws.n_ctas})")
        ws.plan.copy_(plan)
        if ids is not None:
            off = int(ws.layout[_lib.PLAN_OFF_TOKEN_IDS])
            ws.plan[off:off + ids.numel()].copy_(ids)
        self._greedy = None
        graph.replay()
        self.model.kernel_launches += per_replay
        return tokens


class GraphStepBatch(BatchedKV):
    """A decode step staged into a captured graph's workspace: the step view
    ``BlockAllocator.batch_for`` returns when CUDA graphs are on.  The model's
    ``forward(input_ids, batch)`` replays the graph with the caller's token ids
    (``replay``).  ``B``, ``T`` (1) and ``max_ctx`` are the reference's
    ``BatchedKV`` members; the dense ``positions`` / ``mask`` / ``gather``
    view is not built for a graph step."""

    def __init__(self, runner: DecodeGraphRunner, entry: tuple, B: int, max_ctx: int, serial: int):
        self.runner, self.entry, self.serial = runner, entry, serial
        self.B, self.T, self.max_ctx = B, 1, max_ctx
        self.allocator = runner.allocator

    def replay(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Run the step: ``input_ids [B, 1]`` (on any device) -> logits ``[B, 1, V]``
        (a copy; the greedy tokens of the same replay stay available through
        ``DecodeGraphRunner.greedy_tokens_for``)."""
        runner = self.runner
        if self.serial != runner._staged:
            raise RuntimeError("another step was staged after this one; build the step view again")
        graph, ws, logits, tokens, per_replay = self.entry
        B = self.B
        off = int(ws.layout[_lib.PLAN_OFF_TOKEN_IDS])
        ws.plan[off:off + B].copy_(input_ids.reshape(-1).to(ws.plan.device, non_blocking=True))
        runner.model.last_h2d_bytes = ws.last_used_ints * 4
        graph.replay()
        runner.model.kernel_launches += per_replay
        runner._staged += 1  # a view replays once
        out = logits[:B].clone()
        runner._greedy = (weakref.ref(out), B, tokens)
        return out.unsqueeze(1)

    @property
    def positions(self):
        raise TypeError("a CUDA-graph decode step has no dense positions/mask view; "
                        "use this package's GPT2, or turn graphs off for the reference model")

    last_idx = mask = positions

    def write(self, layer, k, v):
        raise TypeError("a CUDA-graph decode step runs whole; it has no per-layer write/gather")

    gather = write


def _advance(seqs: list) -> None:
    """num_cached_tokens += 1 for a replayed decode step."""
    if _hostpack is not None and hasattr(_hostpack, "advance_cached"):
        _hostpack.advance_cached(seqs)  # the native packer kept this step's lengths
    else:
        for s in seqs:
            s.num_cached_tokens += 1


class _CaptureView(DevicePagedBatch):
    """A step view over a workspace with no plan of its own: capacities for
    sizing, the workspace's fixed buffers for every pointer.  Used only to
    capture a graph; the plan is filled in before each replay."""

    def __init__(self, ws: PlanWorkspace):  # noqa: D107 -- deliberately skips the planner
        a = ws.allocator
        cfg = a.cfg
        L = ws.layout
        caps = ws.caps
        self.allocator, self.pool, self.block_size = a, a.pool, a.block_size
        self.n_layer, self.n_head, self.d_head = cfg.n_layer, cfg.n_head, cfg.d_head
        self.B = self.N = self.T = 1
        self.max_ctx = 1
        self.layout = L
        self.h2d_bytes = 0
        self.plan = ws.plan
        self.table_stride = int(L[_lib.PLAN_TABLE_STRIDE])
        self.rows_alloc, self.seqs_alloc = int(caps[1]), int(caps[0])
        self.partials_alloc = int(caps[5])
        self.n_ctas = int(L[_lib.PLAN_NUM_CTAS])
        # Replays of a mixed-step capacity may hold prompt tiles: capture the kernel with them.
        self.with_tiles = ws.max_tokens > ws.max_seqs
        self.tile_merges = 0  # plans of fixed capacities never cut a tile
        self.num_items = self.num_combine = self.num_partials = 0
        dev = ws.plan

        def view(k, n):
            o = int(L[k])
            return dev[o:o + int(n)]

        self.counts = view(_lib.PLAN_OFF_COUNTS, 4)
        self.block_tables_i32 = view(_lib.PLAN_OFF_TABLES, int(caps[0]) * self.table_stride)
        self.slot_mapping = view(_lib.PLAN_OFF_SLOTS, int(caps[1]))
        self.row_positions = view(_lib.PLAN_OFF_POSITIONS, int(caps[1]))
        self.token_ids = view(_lib.PLAN_OFF_TOKEN_IDS, int(caps[1]))
        self.last_rows = view(_lib.PLAN_OFF_LAST_ROWS, int(caps[0]))
        self.attn_plan = dev[int(L[_lib.PLAN_OFF_ITEMS]):]
        self.combine_list = view(_lib.PLAN_OFF_COMBINE, 4 * int(caps[4]))
        self._dev_ptr = dev.data_ptr()
        self._off = {k: int(L[k]) * 4 for k in range(_lib.PLAN_OFF_COUNTS, _lib.PLAN_LAYOUT_LEN)}
        self.partial_ml, self.partial_acc = ws.partial_ml, ws.partial_acc
        self.partial_counters = ws.partial_counters
        self._positions = self._last_idx = self._mask = self._flat_bt = None
