"""Multi-replica serving front end: the reference's HTTP API over N engine
replicas, one process per GPU.

Restates, for several GPUs, the reference's asyncio bridge
(tokquay/async_engine.py:78-205) and server (tokquay/server.py:45-148):

* ``ReplicaRouter`` has the bridge's surface -- ``start`` / ``stop`` /
  ``submit`` / ``stats`` / ``failure`` -- and ``RequestStream`` its per-request
  async iterator with ``abort()``.  The reference drives its one engine from a
  thread of the server process.  Here each replica is a child process
  (spawned, so CUDA starts fresh in it), bound to its own GPU, running the
  same loop (async_engine.py:133-156): idle until a command arrives, apply
  every queued add / abort between steps, one ``Engine.step()``, that step's
  tokens back to the server in one message.  The server process holds no
  CUDA state; it routes and relays.
* Requests go round robin -- request i to replica i mod N -- as the reference
  benchmark splits its workload over replicas.  Replicas that have failed are
  skipped.
* Rejections happen up front, as in the reference (async_engine.py:101-116).
  A request that can never be served raises ``RequestRejected``; an empty
  prompt raises ``ValueError``.  The check runs the replica's own
  ``Scheduler.rejection_reason`` over the limits the replica reported when
  it started.  Token ids must lie in the model's vocabulary.  The reference
  only ever sees ids its tokenizer produced; here clients may send ids.
* A replica whose step raises, or whose process dies, fails every request
  routed to it with ``EngineError`` (async_engine.py:191-202).  The others keep
  serving.  ``/health`` answers 200 "ok" while every replica runs, 200
  "degraded" while some do, and 503 "failed" when none does.

``create_app`` serves ``POST /generate`` (JSON body, or server-sent events
with ``stream: true``) and ``GET /health`` with the reference's request
fields, response bodies and status codes (400 never servable, 422 schema,
503 engine gone, 499 client gone).  It adds one field: ``prompt_token_ids``,
an alternative to ``prompt``.  GPT-2's tokenizer files are not part of this
package, so a server started without a tokenizer answers text prompts with
400 and returns ``text: ""``.
"""

from __future__ import annotations

import asyncio
import itertools
import json
import logging
import multiprocessing as mp
import os
import queue
import threading
import time
from contextlib import asynccontextmanager
from dataclasses import dataclass
from typing import Any, Callable

from fastapi import FastAPI, HTTPException, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse
from pydantic import BaseModel, Field, model_validator

from tokquay_b200._host import ref_scheduler, ref_sequence
from tokquay_b200.scheduler import SchedulerConfig

# The reference's request types and rejection rules (tokquay/scheduler.py:82-104).
RequestRejected, Scheduler = ref_scheduler.RequestRejected, ref_scheduler.Scheduler
SamplingParams, Sequence = ref_sequence.SamplingParams, ref_sequence.Sequence

__all__ = [
    "EngineError",
    "RequestStream",
    "ReplicaRouter",
    "RandomGPT2Engine",
    "IncrementalDetokenizer",
    "GenerateRequest",
    "FrontEnds",
    "create_app",
    "main",
]

log = logging.getLogger(__name__)

_POLL_S = 0.2  # how often the relay thread looks for replicas that died silently


class EngineError(RuntimeError):
    """The replica serving a request is not running (it crashed or was stopped)."""


@dataclass(frozen=True)
class _Token:
    """One generated token as the stream yields it (the engine's TokenEvent)."""

    token_id: int
    finish_reason: str | None = None


class RequestStream:
    """One in-flight request, seen from the event loop (async_engine.py:34-69).

    ``async for event in stream`` yields tokens and ends after the one that
    carries a ``finish_reason``.  If the replica dies first, iteration raises
    ``EngineError``.  Call ``abort()`` when the consumer goes away early."""

    def __init__(self, owner: "ReplicaRouter", req_id: int, replica: int, prompt_token_ids: list[int],
                 params: SamplingParams):  # fmt: skip
        self._owner = owner
        self.req_id = req_id
        self.replica = replica
        self.prompt_token_ids = prompt_token_ids
        self.params = params
        self._queue: asyncio.Queue = asyncio.Queue()
        self._done = False

    def __aiter__(self) -> "RequestStream":
        return self

    async def __anext__(self) -> _Token:
        if self._done:
            raise StopAsyncIteration
        item = await self._queue.get()
        if isinstance(item, BaseException):
            self._done = True
            raise item
        if item.finish_reason is not None:
            self._done = True
        return item

    def abort(self) -> None:
        """Stop generating for this request and free its KV blocks.  Idempotent."""
        if not self._done:
            self._done = True
            self._owner._abort(self)


def _deliver(pairs: list[tuple[RequestStream, Any]]) -> None:
    """Runs on the event loop: hand items to their request's queue."""
    for stream, item in pairs:
        stream._queue.put_nowait(item)


# ---- the replica process ------------------------------------------------------------


def _engine_limits(engine) -> dict:
    a = engine.allocator
    return {
        "config": engine.scheduler.config,
        "num_blocks": a.num_blocks,
        "block_size": a.block_size,
        "vocab_size": engine.model.cfg.vocab_size,
    }


def _engine_stats(engine) -> dict:
    s, a = engine.scheduler, engine.allocator
    return {
        "running": len(s.running),
        "waiting": len(s.waiting),
        "free_blocks": a.num_free_blocks,
        "num_blocks": a.num_blocks,
        "preemptions": s.num_preemptions,
    }


def _replica_main(index: int, device, factory: Callable, inbox, outbox) -> None:
    """A replica's whole life: build the engine on ``device``, then the
    engine loop of async_engine.py:133-156 over ``inbox`` commands
    (``("add", req_id, ids, params)``, ``("abort", req_id)``, ``("stop",)``).
    A replica whose server process has gone (killed, so no "stop" will come
    and nobody drains its outbox) ends itself: within a second when idle,
    before its next step when busy."""
    parent = os.getppid()

    def orphaned() -> bool:
        if os.getppid() == parent:
            return False
        # Nobody reads the outbox any more: its feeder thread may be blocked on a
        # full pipe, and the exit must not wait for it (multiprocessing joins the
        # feeder threads of its queues at exit).
        inbox.cancel_join_thread()
        outbox.cancel_join_thread()
        return True

    try:
        if isinstance(device, int):
            import torch

            torch.cuda.set_device(device)
        engine = factory(device)
        outbox.put(("ready", index, _engine_limits(engine), _engine_stats(engine)))
        seqs: dict[int, Sequence] = {}  # req_id -> its sequence, until it finishes
        req_of: dict[int, int] = {}  # seq_id -> req_id
        while True:
            commands = []
            while not engine.has_unfinished() and not commands:
                try:  # idle: sleep until something arrives
                    commands.append(inbox.get(timeout=_POLL_S * 5))
                except queue.Empty:
                    if orphaned():
                        return
            while True:
                try:
                    commands.append(inbox.get_nowait())
                except queue.Empty:
                    break
            for cmd in commands:
                if cmd[0] == "stop":
                    outbox.put(("stopped", index))
                    return
                if cmd[0] == "add":
                    _, rid, ids, params = cmd
                    try:
                        seq = engine.add_request(ids, params)
                    except ValueError as exc:  # rejected: this request only, the engine is fine
                        outbox.put(("rejected", index, rid, str(exc)))
                        continue
                    seqs[rid] = seq
                    req_of[seq.seq_id] = rid
                elif cmd[0] == "abort":
                    # Commands are FIFO, so an add is always applied before its abort.
                    seq = seqs.pop(cmd[1], None)
                    if seq is not None:
                        req_of.pop(seq.seq_id, None)
                        engine.abort_request(seq)
            if engine.has_unfinished():
                if orphaned():  # busy, but the tokens would go nowhere
                    return
                out = []
                for ev in engine.step():
                    rid = req_of.get(ev.seq_id)
                    if rid is None:
                        continue
                    out.append((rid, ev.token_id, ev.finish_reason))
                    if ev.finish_reason is not None:
                        del req_of[ev.seq_id]
                        seqs.pop(rid, None)
                outbox.put(("tokens", index, out, _engine_stats(engine)))
    except BaseException as exc:  # a failed step leaves the engine inconsistent: no recovery
        outbox.put(("failed", index, repr(exc)))


@dataclass(frozen=True)
class RandomGPT2Engine:
    """Picklable engine factory for a replica: GPT-2 124M with every
    parameter drawn from N(0, 0.02) (no pretrained weights travel with this
    package), its KV pool, CUDA-graph decode steps and a scheduler.  With
    ``warm``, the decode graphs a batch of up to ``max_num_seqs`` can use are
    captured, and a few short requests run, before the replica reports ready,
    so the first requests served pay for neither."""

    num_blocks: int = 1024
    block_size: int = 16
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 2048
    mixed_prefill_tokens: int = 0
    seed: int = 0
    warm: bool = False

    def __call__(self, device):
        import torch

        from tokquay_b200 import GPT2, BlockAllocator, GPT2Config
        from tokquay_b200 import workloads as W
        from tokquay_b200.engine import Engine

        dev = torch.device("cuda", device if isinstance(device, int) else torch.cuda.current_device())
        torch.backends.cuda.matmul.allow_tf32 = False
        cfg = GPT2Config(**W.GPT2_SMALL)
        with torch.device("meta"):
            model = GPT2(cfg)
        model = model.to_empty(device=dev)
        g = torch.Generator(device=dev).manual_seed(self.seed)
        with torch.no_grad():
            for p in model.parameters():
                p.normal_(0.0, 0.02, generator=g)
        model.eval()
        alloc = BlockAllocator(cfg, self.num_blocks, self.block_size, device=dev)
        runner = model.use_cuda_graphs(alloc)
        if self.mixed_prefill_tokens > 0:
            P = self.mixed_prefill_tokens
            runner.mixed_extra = sorted({max(1, P // 4), max(1, P // 2), P})
        sched = SchedulerConfig(max_num_seqs=self.max_num_seqs, max_num_batched_tokens=self.max_num_batched_tokens,
                                max_model_len=cfg.n_positions, mixed_prefill_tokens=self.mixed_prefill_tokens)  # fmt: skip
        if self.warm:
            for b in runner.buckets:
                if b <= self.max_num_seqs:
                    runner.graph(b)
                    for e in runner.mixed_extra if self.mixed_prefill_tokens > 0 else ():
                        runner.graph((b, b + e))
            warm = Engine(model, alloc, sched)
            rng = torch.Generator().manual_seed(99)
            for n in (16, 64, 200, 256):  # the prefill shapes of short and long prompts
                ids = torch.randint(0, cfg.vocab_size - 1, (n,), generator=rng).tolist()
                warm.add_request(ids, SamplingParams(max_tokens=4, ignore_eos=True))
            warm.run_until_done()
            torch.cuda.synchronize(dev)
        return Engine(model, alloc, sched)


class _Limits:
    """The allocator facts ``Scheduler.rejection_reason`` reads, as a replica reported them."""

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks, self.block_size = num_blocks, block_size

    def blocks_needed(self, num_tokens: int) -> int:
        return -(-num_tokens // self.block_size)


@dataclass
class _Replica:
    index: int
    device: Any
    inbox: Any
    process: Any = None
    probe: Scheduler | None = None  # rejection rules over the replica's limits
    vocab_size: int = 0
    alive: bool = False
    failure: str | None = None
    stats: dict | None = None


class ReplicaRouter:
    """N engine replicas behind one ``submit`` (async_engine.py:78-205's surface).

    ``factory(device)`` builds a replica's engine inside its process; it must
    be picklable (a module-level class or function).  ``devices`` has one
    entry per replica: an int is the CUDA device the replica's process binds
    to; any other value labels a replica that uses no GPU (a host-only test
    engine)."""

    def __init__(self, factory: Callable, devices: list, start_timeout_s: float = 600.0,
                 stop_timeout_s: float = 60.0):  # fmt: skip
        if not devices:
            raise ValueError("need at least one replica")
        self._factory = factory
        self._ctx = mp.get_context("spawn")
        self._outbox = self._ctx.Queue()
        self._replicas = [_Replica(i, d, self._ctx.Queue()) for i, d in enumerate(devices)]
        self._start_timeout_s, self._stop_timeout_s = start_timeout_s, stop_timeout_s
        self._streams: dict[int, RequestStream] = {}  # req_id -> stream; relay thread + event loop
        self._lock = threading.RLock()  # guards _streams and the replicas' alive / failure fields
        self._ids = itertools.count()
        self._rr = 0  # next replica in the round robin
        self._loop: asyncio.AbstractEventLoop | None = None
        self._relay: threading.Thread | None = None
        self._started = self._closed = False

    # ---- lifecycle -----------------------------------------------------------------
    async def start(self) -> None:
        """Spawn every replica and wait until each has built its engine."""
        self._loop = asyncio.get_running_loop()
        for r in self._replicas:
            r.process = self._ctx.Process(target=_replica_main, name=f"tokquay-replica-{r.index}",
                                          args=(r.index, r.device, self._factory, r.inbox, self._outbox),
                                          daemon=True)  # fmt: skip
            r.process.start()
        await asyncio.to_thread(self._wait_ready)
        self._relay = threading.Thread(target=self._relay_loop, name="tokquay-relay", daemon=True)
        self._relay.start()
        self._started = True

    def _wait_ready(self) -> None:
        pending = {r.index for r in self._replicas}
        deadline = time.monotonic() + self._start_timeout_s
        while pending:
            left = deadline - time.monotonic()
            if left <= 0:
                self._kill_all()
                raise EngineError(f"replicas {sorted(pending)} did not start within {self._start_timeout_s} s")
            try:
                msg = self._outbox.get(timeout=min(left, _POLL_S))
            except queue.Empty:
                dead = [i for i in pending if not self._replicas[i].process.is_alive()]
                if dead:
                    self._kill_all()
                    raise EngineError(f"replica {dead[0]} exited while starting")
                continue
            r = self._replicas[msg[1]]
            if msg[0] == "failed":
                self._kill_all()
                raise EngineError(f"replica {r.index} failed to start: {msg[2]}")
            if msg[0] == "ready":
                lim = msg[2]
                r.probe = Scheduler(_Limits(lim["num_blocks"], lim["block_size"]), lim["config"])
                r.vocab_size, r.stats, r.alive = lim["vocab_size"], msg[3], True
                pending.discard(r.index)

    async def stop(self) -> None:
        """Stop every replica after its step in flight; open requests get ``EngineError``."""
        if not self._started:
            return
        for r in self._replicas:
            if r.alive:
                r.inbox.put(("stop",))
        await asyncio.to_thread(self._join_all)
        self._closed = True
        if self._relay is not None:
            await asyncio.to_thread(self._relay.join)
        with self._lock:
            pairs = [(s, EngineError("engine stopped")) for s in self._streams.values()]
            self._streams.clear()
        self._send(pairs)

    def _join_all(self) -> None:
        for r in self._replicas:
            r.process.join(self._stop_timeout_s)
            if r.process.is_alive():  # a step that never ended: end the process
                r.process.terminate()
                r.process.join(self._stop_timeout_s)

    def _kill_all(self) -> None:
        for r in self._replicas:
            if r.process is not None and r.process.is_alive():
                r.process.terminate()
                r.process.join(self._stop_timeout_s)

    # ---- requests (event loop side) ------------------------------------------------
    @property
    def failure(self) -> str | None:
        """Why the front end cannot serve: set once no replica is running."""
        with self._lock:
            if any(r.alive for r in self._replicas):
                return None
            return "; ".join(f"replica {r.index}: {r.failure or 'stopped'}" for r in self._replicas)

    def submit(self, prompt_token_ids: list[int], params: SamplingParams) -> RequestStream:
        """Queue a request on the next running replica.  Raises ``ValueError``
        (``RequestRejected`` if it can never be served, plain ``ValueError``
        for an empty prompt or ids outside the vocabulary) or ``EngineError``."""
        if not self._started or self._closed:
            raise EngineError("engine stopped" if self._closed else "engine not started")
        ids = [int(t) for t in prompt_token_ids]
        with self._lock:
            if not any(r.alive for r in self._replicas):
                raise EngineError(self.failure or "engine stopped")
            n = len(self._replicas)
            while not self._replicas[self._rr % n].alive:
                self._rr += 1
            r = self._replicas[self._rr % n]
            self._rr += 1
        probe = Sequence(-1, ids, sampling=params)  # ValueError for an empty prompt
        bad = [t for t in ids if not 0 <= t < r.vocab_size]
        if bad:
            raise ValueError(f"token id {bad[0]} is outside the vocabulary [0, {r.vocab_size})")
        reason = r.probe.rejection_reason(probe)
        if reason:
            raise RequestRejected(reason)
        stream = RequestStream(self, next(self._ids), r.index, ids, params)
        with self._lock:
            if not r.alive:  # the replica failed while we were routing
                raise EngineError(f"replica {r.index} stopped: {r.failure}")
            self._streams[stream.req_id] = stream
        r.inbox.put(("add", stream.req_id, ids, params))
        return stream

    def _abort(self, stream: RequestStream) -> None:
        with self._lock:
            known = self._streams.pop(stream.req_id, None) is not None
            r = self._replicas[stream.replica]
            if known and r.alive:
                r.inbox.put(("abort", stream.req_id))

    def stats(self) -> dict:
        """Sums over running replicas (the reference's /health fields) and one
        entry per replica."""
        with self._lock:
            per = [{"replica": r.index, "device": r.device, "alive": r.alive, **(r.stats or {}),
                    **({"failure": r.failure} if r.failure else {})} for r in self._replicas]  # fmt: skip
        total = {k: sum(p.get(k, 0) for p in per if p["alive"])
                 for k in ("running", "waiting", "free_blocks", "num_blocks", "preemptions")}  # fmt: skip
        return {**total, "replicas": per}

    # ---- the relay thread ------------------------------------------------------------
    def _relay_loop(self) -> None:
        stopped: set[int] = set()
        while len(stopped) < len(self._replicas):
            try:
                msg = self._outbox.get(timeout=_POLL_S)
            except queue.Empty:
                for r in self._replicas:  # a replica that died without a word
                    if r.index not in stopped and not r.process.is_alive():
                        self._replica_down(r, f"process exited with code {r.process.exitcode}")
                        stopped.add(r.index)
                continue
            kind, idx = msg[0], msg[1]
            r = self._replicas[idx]
            if kind == "tokens":
                _, _, out, stats = msg
                pairs = []
                with self._lock:
                    r.stats = stats
                    for rid, token, finish in out:
                        stream = self._streams.get(rid)
                        if stream is None:  # aborted meanwhile
                            continue
                        if finish is not None:
                            del self._streams[rid]
                        pairs.append((stream, _Token(token, finish)))
                self._send(pairs)
            elif kind == "rejected":
                with self._lock:
                    stream = self._streams.pop(msg[2], None)
                if stream is not None:
                    self._send([(stream, RequestRejected(msg[3]))])
            elif kind == "failed":
                log.error("replica %d crashed: %s", idx, msg[2])
                self._replica_down(r, msg[2])
                stopped.add(idx)
            elif kind == "stopped":
                self._replica_down(r, None)
                stopped.add(idx)

    def _replica_down(self, r: _Replica, why: str | None) -> None:
        """No request may be left waiting on a replica that is gone."""
        err = EngineError(f"replica {r.index} stopped" + (f": {why}" if why else ""))
        with self._lock:
            r.alive = False
            r.failure = why
            mine = [rid for rid, s in self._streams.items() if s.replica == r.index]
            pairs = [(self._streams.pop(rid), err) for rid in mine]
        self._send(pairs)

    def _send(self, pairs: list) -> None:
        """One wake-up of the event loop per message, not one per token."""
        if not pairs or self._loop is None:
            return
        try:
            self._loop.call_soon_threadsafe(_deliver, pairs)
        except RuntimeError:  # the loop is already closed: nobody is listening
            pass


# ---- text ---------------------------------------------------------------------------

_REPLACEMENT = "�"


class IncrementalDetokenizer:
    """Token ids to text deltas for byte-level BPE (tokquay/detokenizer.py).

    A character can span several tokens, so the text of a short window of
    recent ids is decoded before and after the newest one and only the
    difference is emitted; a window ending in U+FFFD (an unfinished
    character) emits nothing until more tokens arrive or the stream ends."""

    def __init__(self, tokenizer):
        self._tok = tokenizer
        self._ids: list[int] = []
        self._start = 0  # ids before this are emitted and out of the window
        self._seen = 0  # ids before this have had their text emitted

    def _text(self, ids: list[int]) -> str:
        return self._tok.decode(ids, skip_special_tokens=True, clean_up_tokenization_spaces=False)

    def push(self, token_id: int) -> str:
        self._ids.append(token_id)
        return self._emit(False)

    def flush(self) -> str:
        return self._emit(True)

    def _emit(self, final: bool) -> str:
        old = self._text(self._ids[self._start:self._seen])
        new = self._text(self._ids[self._start:])
        if len(new) <= len(old) or (new.endswith(_REPLACEMENT) and not final):
            return ""
        self._start, self._seen = self._seen, len(self._ids)
        return new[len(old):]


class _NoText:
    """Stand-in detokenizer when the server has no tokenizer: no text."""

    def push(self, token_id: int) -> str:
        return ""

    def flush(self) -> str:
        return ""


# ---- HTTP ---------------------------------------------------------------------------


class GenerateRequest(BaseModel):
    """The reference's request body (tokquay/server.py:45-52), plus
    ``prompt_token_ids`` as an alternative to ``prompt``."""

    prompt: str | None = Field(None, min_length=1)
    prompt_token_ids: list[int] | None = Field(None, min_length=1)
    max_tokens: int = Field(16, ge=1)
    temperature: float = Field(0.0, ge=0)  # 0 = greedy
    top_k: int = Field(0, ge=0)  # 0 = no top-k filtering
    stream: bool = False
    seed: int | None = None  # makes sampled output reproducible
    ignore_eos: bool = False  # keep generating past <|endoftext|> (fixed-length runs)

    @model_validator(mode="after")
    def _one_prompt(self):
        if (self.prompt is None) == (self.prompt_token_ids is None):
            raise ValueError("give exactly one of prompt and prompt_token_ids")
        return self


def create_app(router: ReplicaRouter, tokenizer=None) -> FastAPI:
    """The reference's FastAPI app (tokquay/server.py:104-148) over ``router``."""

    def detok():
        return IncrementalDetokenizer(tokenizer) if tokenizer is not None else _NoText()

    def sse(payload: dict, event: str | None = None) -> str:
        head = f"event: {event}\n" if event else ""
        return f"{head}data: {json.dumps(payload)}\n\n"

    async def stream_events(stream: RequestStream):
        d = detok()
        try:
            async for ev in stream:
                text = d.push(ev.token_id)
                if ev.finish_reason is not None:
                    text += d.flush()
                yield sse({"token_id": ev.token_id, "text": text, "finish_reason": ev.finish_reason})
        except (EngineError, ValueError) as exc:  # the replica died, or rejected the request itself
            yield sse({"error": str(exc)}, event="error")
        finally:
            stream.abort()  # a client that hung up must not keep a GPU busy; no-op if finished

    async def collect(stream: RequestStream, request: Request) -> Response:
        d = detok()
        token_ids: list[int] = []
        pieces: list[str] = []
        finish_reason = None
        try:
            async for ev in stream:
                token_ids.append(ev.token_id)
                pieces.append(d.push(ev.token_id))
                finish_reason = ev.finish_reason
                if finish_reason is None and await request.is_disconnected():
                    return Response(status_code=499)
            pieces.append(d.flush())
        except EngineError as exc:
            raise HTTPException(503, str(exc))
        except ValueError as exc:  # rejected by the replica itself
            raise HTTPException(400, str(exc))
        finally:
            stream.abort()
        return JSONResponse({
            "text": "".join(pieces),
            "token_ids": token_ids,
            "finish_reason": finish_reason,
            "prompt_tokens": len(stream.prompt_token_ids),
            "completion_tokens": len(token_ids),
        })  # fmt: skip

    @asynccontextmanager
    async def lifespan(app):
        await router.start()
        try:
            yield
        finally:
            await router.stop()

    app = FastAPI(title="Tokquay (B200 replicas)", lifespan=lifespan)
    app.state.router = router

    @app.post("/generate")
    async def generate(req: GenerateRequest, request: Request):
        if req.prompt is not None and tokenizer is None:
            raise HTTPException(400, "this server has no tokenizer: send prompt_token_ids")
        ids = tokenizer.encode(req.prompt) if req.prompt is not None else req.prompt_token_ids
        try:
            params = SamplingParams(max_tokens=req.max_tokens, temperature=req.temperature, top_k=req.top_k,
                                    ignore_eos=req.ignore_eos, seed=req.seed)  # fmt: skip
            stream = router.submit(ids, params)
        except EngineError as exc:
            raise HTTPException(503, str(exc))
        except ValueError as exc:  # includes RequestRejected
            raise HTTPException(400, str(exc))
        if req.stream:
            return StreamingResponse(stream_events(stream), media_type="text/event-stream",
                                     headers={"Cache-Control": "no-cache", "X-Accel-Buffering": "no"})  # fmt: skip
        return await collect(stream, request)

    @app.get("/health")
    async def health():
        st = router.stats()
        alive = sum(1 for r in st["replicas"] if r["alive"])
        status = "ok" if alive == len(st["replicas"]) else "degraded" if alive else "failed"
        return JSONResponse({"status": status, **st}, status_code=503 if alive == 0 else 200)

    return app


# ---- several server processes on one port ---------------------------------------------


def _shared_port_socket(host: str, port: int):
    """A TCP socket bound with SO_REUSEPORT: every server process binds its own
    on the same port, and the kernel spreads new connections over them."""
    import socket

    sock = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
    sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
    sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEPORT, 1)
    sock.bind((host, port))
    return sock


def _front_end_main(factory: Callable, devices: list, host: str, port: int, tokenizer_factory, ready) -> None:
    """One server process: uvicorn on the shared port, its own router over
    ``devices``; sets ``ready`` once its replicas have started.  SIGTERM stops
    it gracefully (the router stops its replicas)."""
    import uvicorn

    tokenizer = tokenizer_factory() if tokenizer_factory is not None else None
    app = create_app(ReplicaRouter(factory, devices), tokenizer)
    server = uvicorn.Server(uvicorn.Config(app, log_level="warning", timeout_keep_alive=600))

    async def run():
        task = asyncio.create_task(server.serve(sockets=[_shared_port_socket(host, port)]))
        while not server.started:
            if task.done():
                return
            await asyncio.sleep(0.05)
        ready.set()
        await task

    asyncio.run(run())


class FrontEnds:
    """``n_front_ends`` server processes sharing one port, front end i
    serving replicas ``devices[i::n_front_ends]``.

    One Python server process relays a few tens of thousands of token events
    per second, fewer than two busy replicas produce.  Here the kernel spreads
    connections over the processes (SO_REUSEPORT), so each process relays
    only its own replicas' tokens.  Each request goes to one server process
    and then to its replicas round robin.  ``/health`` answers for the
    replicas of the process that took the connection."""

    def __init__(self, factory: Callable, devices: list, n_front_ends: int, host: str = "127.0.0.1",
                 port: int = 0, tokenizer_factory: Callable | None = None):  # fmt: skip
        if not 1 <= n_front_ends <= len(devices):
            raise ValueError(f"need 1 <= front ends <= replicas, got {n_front_ends} for {len(devices)}")
        self._ctx = mp.get_context("spawn")
        self._groups = [list(devices[i::n_front_ends]) for i in range(n_front_ends)]
        self._factory, self._tokenizer_factory = factory, tokenizer_factory
        self.host = host
        self._hold = _shared_port_socket(host, port)  # keeps the port (not listening: takes no connections)
        self.port = self._hold.getsockname()[1]
        self._procs: list = []

    def start(self, timeout_s: float = 600.0) -> None:
        """Spawn every server process; return once each has its replicas up."""
        events = []
        for i, group in enumerate(self._groups):
            ev = self._ctx.Event()
            p = self._ctx.Process(target=_front_end_main, name=f"tokquay-front-end-{i}",
                                  args=(self._factory, group, self.host, self.port, self._tokenizer_factory, ev))  # fmt: skip
            p.start()
            self._procs.append(p)
            events.append(ev)
        deadline = time.monotonic() + timeout_s
        for i, (p, ev) in enumerate(zip(self._procs, events)):
            while not ev.wait(0.2):
                if not p.is_alive() or time.monotonic() > deadline:
                    self.stop()
                    raise EngineError(f"front end {i} did not start" + ("" if p.is_alive() else
                                      f" (exit code {p.exitcode})"))  # fmt: skip

    def stop(self, timeout_s: float = 60.0) -> None:
        for p in self._procs:
            if p.is_alive():
                p.terminate()  # SIGTERM: uvicorn shuts down and the router stops its replicas
        for p in self._procs:
            p.join(timeout_s)
            if p.is_alive():
                p.kill()
                p.join(timeout_s)
        self._procs = []
        self._hold.close()


def main(argv: list[str] | None = None) -> None:
    """``python -m tokquay_b200.frontend --replicas N [--front-ends K]``: serve
    N random-init GPT-2 replicas, one per GPU (cuda:0 .. cuda:N-1), behind K
    server processes on one port."""
    import argparse

    ap = argparse.ArgumentParser(description="Serve GPT-2 replicas (one per GPU) with a paged KV cache.")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--replicas", type=int, default=1, help="engine replicas, one per GPU")
    ap.add_argument("--num-blocks", type=int, default=1024, help="KV pool size in blocks, per replica")
    ap.add_argument("--block-size", type=int, default=16, help="tokens per KV block")
    ap.add_argument("--max-num-seqs", type=int, default=64)
    ap.add_argument("--max-num-batched-tokens", type=int, default=2048)
    ap.add_argument("--mixed-prefill-tokens", type=int, default=0,
                    help="opt-in chunked prefill: prompt tokens a decode step may carry (0: the reference policy)")
    ap.add_argument("--seed", type=int, default=0, help="seed of the random-init weights")
    ap.add_argument("--front-ends", type=int, default=1,
                    help="server processes sharing the port (each relays the tokens of its share of the replicas)")
    args = ap.parse_args(argv)
    import uvicorn

    factory = RandomGPT2Engine(args.num_blocks, args.block_size, args.max_num_seqs, args.max_num_batched_tokens,
                               args.mixed_prefill_tokens, args.seed, warm=True)  # fmt: skip
    if args.front_ends == 1:
        uvicorn.run(create_app(ReplicaRouter(factory, list(range(args.replicas)))), host=args.host, port=args.port)
        return
    fe = FrontEnds(factory, list(range(args.replicas)), args.front_ends, args.host, args.port)
    fe.start()
    print(f"serving on http://{args.host}:{fe.port} with {args.front_ends} server processes", flush=True)
    try:
        while all(p.is_alive() for p in fe._procs):
            time.sleep(1.0)
    except KeyboardInterrupt:
        pass
    finally:
        fe.stop()


if __name__ == "__main__":
    main()
