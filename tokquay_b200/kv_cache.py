"""Paged KV cache: the block pool, its allocator and the per-step device view.

Pool layout and allocator bookkeeping are the reference's contract
(tokquay/kv_cache.py:1-14, :38-127) and are not restated here:
``BlockAllocator`` subclasses the reference's, so the pool shape

    pool: [num_blocks, n_layer, 2, n_head, block_size, d_head]   (dim 2: 0=K, 1=V)

the LIFO free list, the ref counts and ``OutOfBlocksError`` are the
reference's own code, and its scheduler and engine run on top unchanged.

What changes is the per-step view ``batch_for`` returns.  The reference's
``PagedBatch`` builds padded index tensors with Python loops and, per layer,
gathers every sequence's blocks into a dense copy (kv_cache.py:174-242).
``DevicePagedBatch`` plans the step once on the host in C (``tq_plan_step``),
ships it to the GPU in one copy, and the CUDA kernels scatter new K/V into the
pool and read K/V blocks in place -- no dense copy, no padded query rows.
"""

from __future__ import annotations

import ctypes
import itertools
import math
import threading
from typing import TYPE_CHECKING

import numpy as np
import torch

from tokquay_b200 import _lib
from tokquay_b200._host import ref_kv_cache

try:  # native host-side packing (tokquay_b200/csrc/hostpack.c); same results without it
    from tokquay_b200 import _hostpack
except ImportError:  # pragma: no cover - the Python packer below is used instead
    _hostpack = None

if TYPE_CHECKING:
    from tokquay_b200.model import GPT2Config

# The reference's types, re-exported: the step view is a ``BatchedKV`` for the
# reference model's ``isinstance`` dispatch (tokquay/model.py:73, :155).
BatchedKV = ref_kv_cache.BatchedKV
OutOfBlocksError = ref_kv_cache.OutOfBlocksError
cdiv = ref_kv_cache.cdiv

# Attention work is cut for one CTA per SM; keys of one (row group, head) pair
# are split across CTAs only in pieces of at least this many 32-key chunks
# (cuts between the warps of one CTA have no such floor: they merge in
# shared memory).
MIN_SPLIT_CHUNKS = 8


def attention_chunk_keys() -> int:
    """Keys per attention chunk of the loaded library build (the unit of
    work-item sizes and of the kernel's shared-memory stages)."""
    return _lib.load().tq_attention_chunk_keys()


def attention_warps() -> int:
    """Computing warps per attention CTA of the loaded library build."""
    return _lib.load().tq_attention_warps()


class BlockAllocator(ref_kv_cache.BlockAllocator):
    """The reference's allocator (tokquay/kv_cache.py:38-127), whose step view
    is the device-resident ``DevicePagedBatch``.

    The pool must be float32 (what the kernels read) and ``block_size`` a power
    of two no larger than 256.  A CPU pool is allowed for bookkeeping-only use;
    building a step view needs a CUDA pool.  ``cfg`` is kept (the step view
    reads the model's shape from it).
    """

    def __init__(self, cfg: "GPT2Config", num_blocks: int, block_size: int = 16, device=None,
                 dtype: torch.dtype = torch.float32):  # fmt: skip
        if block_size >= 1 and (block_size & (block_size - 1) or block_size > 256):
            raise ValueError(f"block_size must be a power of two <= 256, got {block_size}")
        if dtype != torch.float32:
            raise ValueError(f"the paged kernels store K/V in float32, got {dtype}")
        super().__init__(cfg, num_blocks, block_size, device, dtype)
        self.cfg = cfg
        self.graph_runner = None  # set by GPT2.use_cuda_graphs(): decode steps then replay a graph

    def batch_for(self, seqs, new_lens: list[int] | None = None) -> "DevicePagedBatch":
        """Step view for ``seqs``: each feeds ``new_lens[i]`` tokens (default: all
        uncached ones) from position ``num_cached_tokens`` (tokquay/kv_cache.py:122-127).
        With CUDA graphs on, a decode step that a captured graph covers is
        staged into that graph's workspace instead (``GraphStepBatch``)."""
        runner = self.graph_runner
        if runner is not None:
            step = runner.stage_step(seqs, new_lens)
            if step is not None:
                return step
        return DevicePagedBatch(self, None, None, None, packed=PackedStep.from_sequences(seqs, new_lens))


# ------------------------------------------------------------------------------ pinned staging
class _PinnedRing:
    """A few grow-only pinned host buffers for the per-step plan copies.  A
    buffer is reused only after the copy that last read it has finished."""

    def __init__(self, n: int = 4):
        self._bufs: list[torch.Tensor | None] = [None] * n
        self._events: list[torch.cuda.Event | None] = [None] * n
        self._i = 0
        self._lock = threading.Lock()

    def take(self, n_ints: int) -> tuple[int, torch.Tensor]:
        with self._lock:
            i = self._i
            self._i = (i + 1) % len(self._bufs)
        ev = self._events[i]
        if ev is not None:
            ev.synchronize()
        buf = self._bufs[i]
        if buf is None or buf.numel() < n_ints:
            size = max(n_ints, 4096, 0 if buf is None else 2 * buf.numel())
            buf = torch.empty(size, dtype=torch.int32, pin_memory=True)
            self._bufs[i] = buf
        return i, buf

    def mark(self, i: int, stream: torch.cuda.Stream) -> None:
        ev = self._events[i]
        if ev is None:
            ev = self._events[i] = torch.cuda.Event()
        ev.record(stream)


_rings: dict[int, _PinnedRing] = {}
_sm_counts: dict[int, int] = {}


def _ring(device: torch.device) -> _PinnedRing:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    r = _rings.get(idx)
    if r is None:
        r = _rings.setdefault(idx, _PinnedRing())
    return r


def sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(idx)
    if n is None:
        n = _sm_counts[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return n


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class PackedStep:
    """One step's host metadata as int32 arrays, the planner's input:
    ``start[B]``, ``lens[B]``, ``offsets[B+1]`` + ``tables`` (block tables,
    CSR), and ``ids`` (the new tokens, in sequence order) or None."""

    __slots__ = ("start", "lens", "offsets", "tables", "ids")

    def __init__(self, start, lens, offsets, tables, ids):
        self.start, self.lens, self.offsets, self.tables, self.ids = start, lens, offsets, tables, ids

    @classmethod
    def from_lists(cls, block_tables, start, new_lens, token_ids=None) -> "PackedStep":
        B = len(block_tables)
        if B == 0 or not (B == len(start) == len(new_lens)):
            raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
        lens = np.fromiter((len(t) for t in block_tables), dtype=np.int64, count=B)
        offs = np.zeros(B + 1, dtype=np.int64)
        np.cumsum(lens, out=offs[1:])
        if offs[-1] > np.iinfo(np.int32).max:
            raise ValueError("block tables too large")
        data = np.fromiter(itertools.chain.from_iterable(block_tables), dtype=np.int32, count=int(offs[-1]))
        ids = None if token_ids is None else np.asarray(token_ids, dtype=np.int32)
        return cls(np.asarray(start, dtype=np.int32), np.asarray(new_lens, dtype=np.int32),
                   offs.astype(np.int32), data, ids)  # fmt: skip

    @classmethod
    def from_sequences(cls, seqs, new_lens: list[int] | None = None) -> "PackedStep":
        """Sequence ``i`` feeds ``new_lens[i]`` tokens (default: all uncached)
        from ``num_cached_tokens``; token ids included.  Uses the native
        ``_hostpack`` helper when it is built (same result, no per-element
        Python work)."""
        if not seqs:
            raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
        if _hostpack is not None:
            st, ln, of, tb, ids = _hostpack.pack_step(seqs, new_lens or None)
            f = np.frombuffer
            return cls(f(st, np.int32), f(ln, np.int32), f(of, np.int32), f(tb, np.int32), f(ids, np.int32))
        starts = [s.num_cached_tokens for s in seqs]
        lens = new_lens or [s.num_uncached_tokens for s in seqs]
        if len(lens) != len(seqs):
            raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
        ids = list(itertools.chain.from_iterable(
            s.token_ids[st:st + n] for s, st, n in zip(seqs, starts, lens) if n > 0 and st >= 0))  # fmt: skip
        return cls.from_lists([s.block_table for s in seqs], starts, lens, ids)


def plan_packed(
    block_size: int,
    num_blocks: int,
    n_head: int,
    packed: PackedStep,
    vocab_size: int = 0,
    n_ctas: int = 148,
    min_split_chunks: int = MIN_SPLIT_CHUNKS,
    out: torch.Tensor | np.ndarray | None = None,
    caps: np.ndarray | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """Run ``tq_plan_step`` on the host: returns ``(plan, layout)`` (int32
    arrays).  ``out`` (an int32 host buffer) is written in place when it is
    large enough; otherwise a new array is returned.  ``caps`` (6 int32:
    max seqs, tokens, table stride, items, combine entries, partials) selects
    the fixed-capacity layout.  Raises ValueError for a batch the reference
    would reject, RuntimeError for one beyond ``caps``."""
    lib = _lib.load()
    B = int(packed.start.size)
    if B == 0 or packed.lens.size != B or packed.offsets.size != B + 1:
        raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
    st, ql, offs, data, ids = (np.ascontiguousarray(a, dtype=np.int32) if a is not None else None
                               for a in (packed.start, packed.lens, packed.offsets, packed.tables, packed.ids))  # fmt: skip
    if ids is not None and ids.size != int(np.maximum(ql, 0).sum()):
        raise ValueError(f"{ids.size} token ids for {int(ql.sum())} new tokens")
    layout = np.zeros(_lib.PLAN_LAYOUT_LEN, dtype=np.int32)
    ids_ptr = _ptr(ids) if ids is not None and ids.size else None
    if ids is not None and ids_ptr is None:
        ids_ptr = _ptr(np.zeros(1, np.int32))
    data_ptr = _ptr(data) if data.size else None
    caps_ptr = None
    if caps is not None:
        caps = np.ascontiguousarray(caps, dtype=np.int32)
        caps_ptr = _ptr(caps)

    def call(buf_ptr, cap):
        return lib.tq_plan_step(B, _ptr(st), _ptr(ql), _ptr(offs), data_ptr, ids_ptr, block_size,
                                num_blocks, n_head, vocab_size, n_ctas, min_split_chunks,
                                caps_ptr, buf_ptr, cap, _ptr(layout))  # fmt: skip

    if out is not None:
        cap = out.numel() if isinstance(out, torch.Tensor) else out.size
        buf_ptr = out.data_ptr() if isinstance(out, torch.Tensor) else _ptr(out)
        status = call(buf_ptr, cap)
        if status == _lib.TQ_OK:
            return out, layout
        if status != _lib.TQ_ERR_CAPACITY or layout[_lib.PLAN_TOTAL_INTS] == 0:
            _lib.check(status, "tq_plan_step")
    status = call(None, 0)
    if status != _lib.TQ_ERR_CAPACITY or layout[_lib.PLAN_TOTAL_INTS] == 0:
        _lib.check(status, "tq_plan_step")
    plan = np.empty(int(layout[_lib.PLAN_TOTAL_INTS]), dtype=np.int32)
    _lib.check(call(_ptr(plan), plan.size), "tq_plan_step")
    return plan, layout


def plan_step_host(
    block_size: int,
    num_blocks: int,
    n_head: int,
    block_tables: list[list[int]],
    start: list[int],
    new_lens: list[int],
    token_ids: list[int] | None = None,
    vocab_size: int = 0,
    n_ctas: int = 148,
    min_split_chunks: int = MIN_SPLIT_CHUNKS,
    out: torch.Tensor | np.ndarray | None = None,
    caps: np.ndarray | None = None,
) -> tuple[np.ndarray, np.ndarray]:
    """``plan_packed`` for Python lists (block tables, starts, lengths, ids)."""
    packed = PackedStep.from_lists(block_tables, start, new_lens, token_ids)
    return plan_packed(block_size, num_blocks, n_head, packed, vocab_size, n_ctas, min_split_chunks,
                       out, caps)  # fmt: skip


_NOT_A_DECODE_STEP = -2  # _hostpack.plan_sequences: the step is not a decode step, nothing planned


class PlanWorkspace:
    """A fixed-capacity home for one step plan on the device.

    Plans written here use the planner's fixed layout, so every device pointer
    a step hands to the kernels -- plan regions, split-K scratch -- is the same
    for every step that fits the capacities.  That is what lets a decode step
    be captured once as a CUDA graph and replayed (``DecodeGraphRunner``).
    One workspace holds one step at a time: planning the next step overwrites
    the device plan (in stream order, after the previous step's kernels).
    """

    def __init__(self, allocator: "BlockAllocator", max_seqs: int, max_tokens: int | None = None,
                 max_ctx: int | None = None):  # fmt: skip
        cfg = allocator.cfg
        bs = allocator.block_size
        max_tokens = max_tokens or max_seqs
        max_ctx = max_ctx or cfg.n_positions
        chunks = cdiv(max_ctx, attention_chunk_keys())
        # Cross-CTA pieces of a pair: at least MIN_SPLIT_CHUNKS long, or as many
        # as the kernel's 64-block item span forces.
        max_piece = max(1, 63 * bs // attention_chunk_keys())
        max_split = max(1, chunks // MIN_SPLIT_CHUNKS, cdiv(chunks, max_piece))
        max_groups = max_tokens  # a query-row group holds at least one token
        self.n_ctas = sm_count(allocator.pool.device)
        self.allocator = allocator
        self.max_seqs, self.max_tokens, self.max_ctx = max_seqs, max_tokens, max_ctx
        max_items = max_groups * cfg.n_head * max_split + self.n_ctas * (attention_warps() - 1)
        self.caps = np.array([max_seqs, max_tokens, cdiv(max_ctx, bs), max_items,
                              max_tokens, max_tokens * cfg.n_head * max_split], dtype=np.int32)  # fmt: skip
        # The layout is fixed by the capacities: get it from a one-token plan.
        _, layout = plan_step_host(bs, allocator.num_blocks, cfg.n_head, [[0]], [0], [1], n_ctas=self.n_ctas,
                                   caps=self.caps)  # fmt: skip
        self.layout = layout
        self.total = int(layout[_lib.PLAN_TOTAL_INTS])
        dev = allocator.pool.device
        self.plan = torch.zeros(self.total, dtype=torch.int32, device=dev)
        n_part = int(self.caps[5])
        self.partial_ml = torch.empty(2 * n_part, dtype=torch.float32, device=dev)
        self.partial_acc = torch.empty(n_part * cfg.d_head, dtype=torch.float32, device=dev)
        self.partial_counters = torch.zeros(n_part, dtype=torch.int32, device=dev)  # kernels leave them 0
        self._pinned = [torch.empty(self.total, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._events: list[torch.cuda.Event | None] = [None, None]
        self._turn = 0
        self._layout = np.zeros(_lib.PLAN_LAYOUT_LEN, dtype=np.int32)
        self._native = _hostpack is not None and hasattr(_hostpack, "plan_sequences")
        self._plan_fn = _lib.function_address("tq_plan_step") if self._native else 0

    def stage(self, packed: PackedStep, stream: torch.cuda.Stream, vocab_size: int = 0) -> np.ndarray:
        """Plan ``packed`` into the next pinned buffer and copy the part of it
        the step uses into the device plan on ``stream``; returns the layout."""
        a = self.allocator
        slot, host = self.pinned_buffer()
        plan, layout = plan_packed(a.block_size, a.num_blocks, a.cfg.n_head, packed, vocab_size, self.n_ctas,
                                   MIN_SPLIT_CHUNKS, out=host, caps=self.caps)  # fmt: skip
        assert plan is host and int(layout[_lib.PLAN_TOTAL_INTS]) == self.total
        used = int(layout[_lib.PLAN_USED_INTS])
        with torch.cuda.stream(stream):
            self.plan[:used].copy_(host[:used], non_blocking=True)
        self.mark_copied(slot, stream)
        self.last_used_ints = used
        return layout

    def stage_sequences(self, seqs, new_lens: list[int] | None, stream: torch.cuda.Stream,
                        vocab_size: int = 0, decode_max_ctx: int = 0,
                        fit_only: bool = False) -> np.ndarray | None:  # fmt: skip
        """``stage`` straight from ``Sequence`` objects: the native packer
        hands its arrays to the planner, so planning a step makes no Python
        objects.  Same plan, same errors as ``stage(PackedStep.from_sequences(...))``.
        With ``decode_max_ctx`` > 0, a step that is not a decode step within
        that context, or does not fit the capacities, returns None (nothing
        staged); with ``fit_only`` any step that does not fit returns None."""
        if not self._native:
            packed = PackedStep.from_sequences(seqs, new_lens)
            if decode_max_ctx > 0 and (packed.lens.max() != 1 or packed.lens.min() != 1
                                       or int(packed.start.max()) + 1 > decode_max_ctx):  # fmt: skip
                return None
            try:
                return self.stage(packed, stream, vocab_size)
            except RuntimeError:
                if decode_max_ctx > 0 or fit_only:
                    return None
                raise
        if not seqs:
            raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
        a = self.allocator
        slot, host = self.pinned_buffer()
        status = _hostpack.plan_sequences(
            self._plan_fn, seqs, new_lens, a.block_size, a.num_blocks, a.cfg.n_head, vocab_size, self.n_ctas,
            MIN_SPLIT_CHUNKS, self.caps.ctypes.data, host.data_ptr(), self.total, self._layout.ctypes.data,
            decode_max_ctx)
        if decode_max_ctx > 0 and status in (_NOT_A_DECODE_STEP, _lib.TQ_ERR_CAPACITY):
            return None
        if fit_only and status == _lib.TQ_ERR_CAPACITY:
            return None
        _lib.check(status, "tq_plan_step")
        used = int(self._layout[_lib.PLAN_USED_INTS])
        with torch.cuda.stream(stream):
            self.plan[:used].copy_(host[:used], non_blocking=True)
        self.mark_copied(slot, stream)
        self.last_used_ints = used
        return self._layout.copy()

    def pinned_buffer(self) -> tuple[int, torch.Tensor]:
        """The next pinned staging buffer, once the copy that last read it is done."""
        i = self._turn
        self._turn ^= 1
        if self._events[i] is not None:
            self._events[i].synchronize()
        return i, self._pinned[i]

    def mark_copied(self, i: int, stream: torch.cuda.Stream) -> None:
        ev = self._events[i]
        if ev is None:
            ev = self._events[i] = torch.cuda.Event()
        ev.record(stream)


class DevicePagedBatch(BatchedKV):
    """One step over paged KV, resident on the GPU.

    Sequence ``b`` feeds ``new_lens[b]`` tokens at positions
    ``start[b] .. start[b]+new_lens[b]-1`` (prefill, decode and a mix of both in
    one batch, as the reference allows).  The step is planned once and reused
    by every layer.  Rows are ragged: row ``n`` of the flattened ``[N, C]``
    activations is the n-th real new token in sequence order.

    With a ``workspace`` the plan goes to the workspace's fixed device buffer
    and split-K scratch; ``graph_sizing`` then makes the model size every
    activation and launch for the workspace's capacities (the shape a CUDA
    graph is captured with), while the kernels read the step's true counts
    from the device plan.

    ``n_ctas`` is the attention grid the plan is cut for (default: the
    device's SM count; a workspace fixes its own).

    ``write`` / ``gather`` / ``positions`` / ``mask`` keep the reference's
    ``BatchedKV`` contract for callers written against it; the model in this
    package uses ``write_rows`` / ``attend_rows`` and never builds the dense
    copies or the mask.
    """

    def __init__(
        self,
        allocator: BlockAllocator,
        block_tables: list[list[int]] | None,
        start: list[int] | None,
        new_lens: list[int] | None,
        token_ids: list[int] | None = None,
        stream: torch.cuda.Stream | None = None,
        workspace: PlanWorkspace | None = None,
        graph_sizing: bool = False,
        packed: PackedStep | None = None,
        n_ctas: int | None = None,
    ):
        pool = allocator.pool
        if pool.device.type != "cuda":
            raise RuntimeError("DevicePagedBatch needs the pool on a CUDA device")
        if packed is None:
            if not block_tables or not (len(block_tables) == len(start) == len(new_lens)):
                raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
            packed = PackedStep.from_lists(block_tables, start, new_lens, token_ids)
        st, ln = packed.start, packed.lens
        if st.size == 0:
            raise ValueError("block_tables, start and new_lens must be non-empty and the same length")
        if int(ln.min()) < 1:
            raise ValueError("every sequence must feed at least one token")
        if graph_sizing and workspace is None:
            raise ValueError("graph_sizing needs a workspace")
        bs = allocator.block_size
        cfg = allocator.cfg
        self.allocator = allocator
        self.pool = pool
        self.block_size = bs
        self.n_layer, self.n_head, self.d_head = cfg.n_layer, cfg.n_head, cfg.d_head
        self.B, self.T = int(st.size), int(ln.max())
        self.N = int(ln.sum())
        self._start = st
        self._new_lens = ln
        ctx = st.astype(np.int64) + ln
        self.max_ctx = int(ctx.max())
        self.num_blocks_gathered = int(-(-ctx.max() // bs))

        device = pool.device
        stream = stream or torch.cuda.current_stream(device)
        vocab = cfg.vocab_size if packed.ids is not None else 0
        if workspace is None:
            ring = _ring(device)
            slot, host = ring.take(0)
            plan, layout = plan_packed(bs, allocator.num_blocks, cfg.n_head, packed, vocab,
                                       n_ctas or sm_count(device), MIN_SPLIT_CHUNKS, out=host)  # fmt: skip
            total = int(layout[_lib.PLAN_USED_INTS])  # the step reads only this prefix
            if plan is not host:  # the plan did not fit: grow the pinned buffer and stage it there
                slot, host = ring.take(total)
                host[:total].copy_(torch.from_numpy(plan[:total]))
            dev = torch.empty(total, dtype=torch.int32, device=device)
            with torch.cuda.stream(stream):
                dev.copy_(host[:total], non_blocking=True)
            ring.mark(slot, stream)
        else:
            if n_ctas is not None and n_ctas != workspace.n_ctas:
                raise ValueError(f"a workspace plans for {workspace.n_ctas} CTAs, not {n_ctas}")
            layout = workspace.stage(packed, stream, vocab)
            total = int(layout[_lib.PLAN_USED_INTS])
            dev = workspace.plan
        self.layout = layout
        self.h2d_bytes = 4 * total  # the one host->device copy this step makes
        self.plan = dev
        L = layout
        self.num_items = int(L[_lib.PLAN_NUM_ITEMS])
        self.num_combine = int(L[_lib.PLAN_NUM_COMBINE])
        self.num_partials = int(L[_lib.PLAN_NUM_PARTIALS])
        self.table_stride = int(L[_lib.PLAN_TABLE_STRIDE])
        self.split_chunks = int(L[_lib.PLAN_SPLIT_CHUNKS])
        self.n_ctas = int(L[_lib.PLAN_NUM_CTAS])
        # The attention kernel that carries the prompt-tile role: for a plan
        # with tile CTAs, and for launches sized for a workspace (captured once,
        # replayed over its steps) whenever a step of its capacity may feed
        # several tokens of one sequence.
        self.with_tiles = int(L[_lib.PLAN_NUM_TILE_CTAS]) > 0 or (
            graph_sizing and workspace.max_tokens > workspace.max_seqs)
        # Rows of tiles cut over their keys (plans without fixed capacities):
        # a merge kernel after the attention grid combines their pieces.
        self.tile_merges = int(L[_lib.PLAN_NUM_TILE_MERGES])
        # What activations and launches are sized for.
        if graph_sizing:
            caps = workspace.caps
            self.rows_alloc, self.seqs_alloc = int(caps[1]), int(caps[0])
            self.partials_alloc = int(caps[5])
        else:
            self.rows_alloc, self.seqs_alloc = self.N, self.B
            self.partials_alloc = self.num_partials
        dims = (workspace.caps if workspace is not None else
                [self.B, self.N, self.table_stride, self.num_items, self.num_combine, self.num_partials])  # fmt: skip

        def view(off_key: int, n: int) -> torch.Tensor:
            o = int(L[off_key])
            return dev[o:o + int(n)]

        self.counts = view(_lib.PLAN_OFF_COUNTS, 4)  # N, items, combine, B
        self.seq_info = view(_lib.PLAN_OFF_SEQ_INFO, 4 * dims[0]).view(-1, 4)
        self.block_tables_i32 = view(_lib.PLAN_OFF_TABLES, dims[0] * self.table_stride)
        self.slot_mapping = view(_lib.PLAN_OFF_SLOTS, dims[1])
        self.row_positions = view(_lib.PLAN_OFF_POSITIONS, dims[1])
        self.token_ids = view(_lib.PLAN_OFF_TOKEN_IDS, dims[1]) if packed.ids is not None else None
        self.last_rows = view(_lib.PLAN_OFF_LAST_ROWS, self.B)
        self.attn_plan = dev[int(L[_lib.PLAN_OFF_ITEMS]):]  # the kernel finds its parts from n_ctas
        self.combine_list = view(_lib.PLAN_OFF_COMBINE, 4 * dims[4])
        self._dev_ptr = dev.data_ptr()
        self._off = {k: int(L[k]) * 4 for k in range(_lib.PLAN_OFF_COUNTS, _lib.PLAN_LAYOUT_LEN)}
        if workspace is not None:
            self.partial_ml, self.partial_acc = workspace.partial_ml, workspace.partial_acc
            self.partial_counters = workspace.partial_counters
        elif self.num_partials:
            self.partial_ml = torch.empty(2 * self.num_partials, dtype=torch.float32, device=device)
            self.partial_acc = torch.empty(self.num_partials * self.d_head, dtype=torch.float32, device=device)
            self.partial_counters = torch.zeros(self.num_partials, dtype=torch.int32, device=device)
        else:
            self.partial_ml = self.partial_acc = self.partial_counters = None
        self._positions = self._last_idx = self._mask = self._flat_bt = None

    # ---- device-resident counts (for the kernels) ------------------------------------
    def count_ptr(self, which: int) -> int:
        """Device address of count ``which`` (0 = N, 1 = items, 2 = combine, 3 = B)."""
        return self._dev_ptr + self._off[_lib.PLAN_OFF_COUNTS] + 4 * which

    # ---- hot path: ragged rows ---------------------------------------------------------
    def write_rows(self, layer: int, qkv: torch.Tensor, k_col: int, v_col: int, stream: int) -> None:
        """Scatter K/V of the ``N`` new rows of ``qkv`` (row-major, K head 0 at
        column ``k_col``, V at ``v_col``) into the pool (tokquay/kv_cache.py:228-232)."""
        lib = _lib.load()
        _lib.check(lib.tq_kv_write(self.pool.data_ptr(), self.allocator.num_blocks, self.n_layer,
                                   self.n_head, self.block_size, self.d_head, layer, qkv.data_ptr(),
                                   qkv.stride(0), k_col, v_col, self.slot_mapping.data_ptr(),
                                   self.count_ptr(0), self.rows_alloc, stream), "tq_kv_write")  # fmt: skip

    def write_qkv_rows(self, layer: int, parts: torch.Tensor, n_parts: int, part_stride: int, bias: torch.Tensor,
                       q_out: torch.Tensor, stream: int) -> None:  # fmt: skip
        """The c_attn epilogue: ``row = sum of the n_parts split-K partial sums
        of c_attn + bias``; q goes to ``q_out`` (``[N, C]`` rows), K and V into
        the pool slots of the ``N`` new tokens (tokquay/model.py:69 +
        tokquay/kv_cache.py:228-232, one kernel)."""
        lib = _lib.load()
        _lib.check(lib.tq_qkv_bias_kv_write(
            q_out.data_ptr(), q_out.stride(0), parts.data_ptr(), n_parts, part_stride, bias.data_ptr(),
            self.pool.data_ptr(), self.allocator.num_blocks, self.n_layer, self.n_head, self.block_size,
            self.d_head, layer, self.slot_mapping.data_ptr(), self.count_ptr(0), self.rows_alloc, stream),
            "tq_qkv_bias_kv_write")  # fmt: skip

    def attend_rows(self, layer: int, q: torch.Tensor, out: torch.Tensor, stream: int) -> None:
        """``out[n, h*d:(h+1)*d] = softmax(q_n,h . K / sqrt(d)) V`` over keys
        0..position(n) of row n's sequence, read in place from the pool
        (replaces tokquay/kv_cache.py:234-242 + tokquay/model.py:94-96).
        ``q`` rows hold head h at columns ``h*d``; row stride is ``q.stride(0)``.
        Keys cut between warps or CTAs are merged in the same launch."""
        lib = _lib.load()
        pm = self.partial_ml.data_ptr() if self.partial_ml is not None else None
        pa = self.partial_acc.data_ptr() if self.partial_acc is not None else None
        pc = self.partial_counters.data_ptr() if self.partial_counters is not None else None
        _lib.check(lib.tq_paged_attention(
            out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), self.pool.data_ptr(),
            self.allocator.num_blocks, self.n_layer, self.n_head, self.block_size, self.d_head, layer,
            self.block_tables_i32.data_ptr(), self.table_stride, self.attn_plan.data_ptr(), self.n_ctas,
            (_lib.ATTN_TILES if self.with_tiles else 0) | (_lib.ATTN_TILE_MERGE if self.tile_merges else 0),
            pm, pa, pc, self.partials_alloc,
            1.0 / math.sqrt(self.d_head), stream), "tq_paged_attention")  # fmt: skip

    # ---- reference BatchedKV contract (not used by this package's model) ---------------
    @property
    def positions(self) -> torch.Tensor:
        if self._positions is None:
            st = torch.from_numpy(self._start.astype(np.int64)).to(self.pool.device)
            self._positions = st[:, None] + torch.arange(self.T, device=self.pool.device)[None, :]
        return self._positions

    @property
    def last_idx(self) -> torch.Tensor:
        if self._last_idx is None:
            self._last_idx = torch.from_numpy(self._new_lens.astype(np.int64) - 1).to(self.pool.device)
        return self._last_idx

    @property
    def mask(self) -> torch.Tensor:
        """``[B, 1, T, nb*bs]`` boolean mask of the reference (kv_cache.py:213-214)."""
        if self._mask is None:
            dev = self.pool.device
            ctx = torch.from_numpy(self._start.astype(np.int64) + self._new_lens).to(dev)
            k_pos = torch.arange(self.num_blocks_gathered * self.block_size, device=dev)[None, None, :]
            self._mask = ((k_pos <= self.positions[:, :, None]) & (k_pos < ctx[:, None, None]))[:, None]
        return self._mask

    def _valid_bt(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self._flat_bt is None:
            b = [i for i, n in enumerate(self._new_lens.tolist()) for _ in range(n)]
            t = [j for n in self._new_lens.tolist() for j in range(n)]
            dev = self.pool.device
            self._flat_bt = (torch.tensor(b, device=dev), torch.tensor(t, device=dev))
        return self._flat_bt

    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Reference-shaped write: ``k``, ``v`` are padded ``[B, H, T, d]``;
        padded slots are never written."""
        b, t = self._valid_bt()
        kv = torch.cat([k[b, :, t].reshape(self.N, -1), v[b, :, t].reshape(self.N, -1)], dim=1)
        kv = kv.to(torch.float32).contiguous()
        C = self.n_head * self.d_head
        self.write_rows(layer, kv, 0, C, torch.cuda.current_stream(self.pool.device).cuda_stream)

    def gather(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense ``[B, H, nb*bs, d]`` copies, for callers of the reference
        contract only; the CUDA attention never builds them."""
        nb = self.num_blocks_gathered
        tbl = self.block_tables_i32.view(self.B, self.table_stride)[:, :nb].long()
        out = []
        for kv in (0, 1):
            g = self.pool[tbl, layer, kv].permute(0, 2, 1, 3, 4)
            out.append(g.reshape(self.B, g.shape[1], -1, g.shape[-1]))
        return out[0], out[1]

    def attend(self, layer: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Drop-in for the reference's paged attention branch (model.py:73-78 +
        :94-96): writes the new K/V, attends with the CUDA kernel, returns
        ``[B, H, T, d]`` (padded query slots are left at zero)."""
        self.write(layer, k, v)
        b, t = self._valid_bt()
        C = self.n_head * self.d_head
        qf = q[b, :, t].reshape(self.N, C).to(torch.float32).contiguous()
        of = torch.empty(self.N, C, dtype=torch.float32, device=q.device)
        self.attend_rows(layer, qf, of, torch.cuda.current_stream(q.device).cuda_stream)
        out = torch.zeros(self.B, self.T, self.n_head, self.d_head, dtype=q.dtype, device=q.device)
        out[b, t] = of.view(self.N, self.n_head, self.d_head).to(q.dtype)
        return out.transpose(1, 2)
