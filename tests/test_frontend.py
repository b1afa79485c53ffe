"""The multi-replica serving front end (tokquay_b200/frontend.py) on the host.

Replicas are spawned processes running a host-only stand-in engine
(tests/fake_engine.py) with a fixed token rule, so routing, streaming, abort,
up-front rejection, failure isolation and the HTTP surface are checked without
a GPU.  The cases follow the reference's own serving tests
(tests/test_phase5_server.py, tests/test_phase5_abort.py): JSON and SSE bodies,
400 / 422 / 503 answers, a dead engine failing its open requests, aborted
requests freeing their slots.
"""

import asyncio
import json

import pytest

from fake_engine import EchoFactory, expected_tokens
from tokquay_b200.frontend import EngineError, IncrementalDetokenizer, ReplicaRouter, create_app
from tokquay_b200.scheduler import RequestRejected
from tokquay.sequence import SamplingParams


def run(coro):
    return asyncio.run(asyncio.wait_for(coro, timeout=120))


async def _collect(stream):
    return [(ev.token_id, ev.finish_reason) async for ev in stream]


def test_round_robin_streams_every_token():
    async def main():
        router = ReplicaRouter(EchoFactory(), ["r0", "r1"])
        await router.start()
        try:
            prompts = [[i + 1, 2 * i + 3] for i in range(6)]
            streams = [router.submit(p, SamplingParams(max_tokens=5 + i)) for i, p in enumerate(prompts)]
            assert [s.replica for s in streams] == [0, 1, 0, 1, 0, 1]  # request i to replica i mod 2
            outs = await asyncio.gather(*map(_collect, streams))
            for i, (p, out) in enumerate(zip(prompts, outs)):
                assert [t for t, _ in out] == expected_tokens(p, 5 + i)
                assert [f for _, f in out] == [None] * (4 + i) + ["length"]
            st = router.stats()
            assert st["running"] == 0 and len(st["replicas"]) == 2 and all(r["alive"] for r in st["replicas"])
        finally:
            await router.stop()
        with pytest.raises(EngineError):
            router.submit([1], SamplingParams())

    run(main())


def test_rejections_are_raised_up_front():
    async def main():
        router = ReplicaRouter(EchoFactory(max_model_len=64), ["r0"])
        with pytest.raises(EngineError):  # not started
            router.submit([1], SamplingParams())
        await router.start()
        try:
            with pytest.raises(RequestRejected, match="positions"):
                router.submit(list(range(60)), SamplingParams(max_tokens=10))
            with pytest.raises(ValueError, match="at least one token"):
                router.submit([], SamplingParams())
            with pytest.raises(ValueError, match="vocabulary"):
                router.submit([5, 1000], SamplingParams())
            with pytest.raises(ValueError, match="vocabulary"):
                router.submit([-1], SamplingParams())
            s = router.submit(list(range(50)), SamplingParams(max_tokens=15))  # 64 positions: fits
            assert len(await _collect(s)) == 15
        finally:
            await router.stop()

    run(main())


def test_abort_stops_a_request_and_frees_its_slot():
    async def main():
        router = ReplicaRouter(EchoFactory(step_s=0.005), ["r0"])
        await router.start()
        try:
            long = router.submit([7], SamplingParams(max_tokens=200))
            short = router.submit([9], SamplingParams(max_tokens=20))
            got = []
            async for ev in long:
                got.append(ev.token_id)
                if len(got) == 3:
                    long.abort()
                    long.abort()  # idempotent
            assert got == expected_tokens([7], 3)
            assert [t for t, _ in await _collect(short)] == expected_tokens([9], 20)
            for _ in range(200):  # the replica applies the abort between steps
                if router.stats()["running"] == 0:
                    break
                await asyncio.sleep(0.01)
            assert router.stats()["running"] == 0
        finally:
            await router.stop()

    run(main())


@pytest.mark.parametrize("how", ["raise", "exit"])
def test_a_failed_replica_fails_only_its_requests(how):
    """Replica r1's step raises (or its process exits) after 3 steps: its open
    requests end with EngineError, r0 keeps serving, new requests skip r1."""
    fac = EchoFactory(step_s=0.002, **{"fail" if how == "raise" else "exit": (("r1", 3),)})

    async def main():
        router = ReplicaRouter(fac, ["r0", "r1"])
        await router.start()
        try:
            a = router.submit([1], SamplingParams(max_tokens=50))
            b = router.submit([2], SamplingParams(max_tokens=50))
            assert (a.replica, b.replica) == (0, 1)
            assert len(await _collect(a)) == 50
            with pytest.raises(EngineError, match="replica 1"):
                await _collect(b)
            for _ in range(200):
                if not router.stats()["replicas"][1]["alive"]:
                    break
                await asyncio.sleep(0.01)
            st = router.stats()
            assert not st["replicas"][1]["alive"] and st["replicas"][0]["alive"]
            assert router.failure is None  # r0 still serves
            c, d = (router.submit([3], SamplingParams(max_tokens=4)) for _ in range(2))
            assert c.replica == d.replica == 0
            assert [t for t, _ in await _collect(c)] == expected_tokens([3], 4)
        finally:
            await router.stop()

    run(main())


class ByteTokenizer:
    """Toy byte-level tokenizer: one token per UTF-8 byte, as GPT-2's
    byte-level BPE splits a multi-byte character over tokens (id i stands
    for byte i mod 256, so the stand-in engine's ids all decode)."""

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids, skip_special_tokens=True, clean_up_tokenization_spaces=False) -> str:
        return bytes(i % 256 for i in ids).decode("utf-8", errors="replace")


def test_incremental_detokenizer_holds_back_split_characters():
    tok = ByteTokenizer()
    text = "a€b😀c"
    d = IncrementalDetokenizer(tok)
    pieces = [d.push(t) for t in tok.encode(text)]
    assert "".join(pieces) + d.flush() == text
    assert all("�" not in p for p in pieces)
    assert pieces[1:4] == ["", "", "€"]  # the euro sign's 3 bytes: text only with the last
    d = IncrementalDetokenizer(tok)
    assert d.push(0xE2) == "" and d.flush() == "�"  # end of stream: emit what is held back


def _sse_events(body: str) -> list[dict]:
    return [json.loads(line[6:]) for line in body.splitlines() if line.startswith("data: ")]


def test_http_generate_json_sse_and_errors():
    from fastapi.testclient import TestClient

    with TestClient(create_app(ReplicaRouter(EchoFactory(max_model_len=64), ["r0", "r1"]))) as client:
        r = client.post("/generate", json={"prompt_token_ids": [4, 5, 6], "max_tokens": 6})
        assert r.status_code == 200
        body = r.json()
        assert body["token_ids"] == expected_tokens([4, 5, 6], 6)
        assert body["finish_reason"] == "length" and body["prompt_tokens"] == 3 and body["completion_tokens"] == 6
        assert body["text"] == ""  # no tokenizer
        r = client.post("/generate", json={"prompt_token_ids": [8], "max_tokens": 4, "stream": True})
        assert r.status_code == 200 and r.headers["content-type"].startswith("text/event-stream")
        ev = _sse_events(r.text)
        assert [e["token_id"] for e in ev] == expected_tokens([8], 4)
        assert [e["finish_reason"] for e in ev] == [None, None, None, "length"]
        # 400: never servable / no tokenizer for text; 422: schema violations.
        assert client.post("/generate", json={"prompt_token_ids": list(range(60)), "max_tokens": 10}).status_code == 400
        assert client.post("/generate", json={"prompt_token_ids": [10**6]}).status_code == 400
        assert client.post("/generate", json={"prompt": "hello"}).status_code == 400
        assert client.post("/generate", json={"prompt_token_ids": [1], "max_tokens": 0}).status_code == 422
        assert client.post("/generate", json={}).status_code == 422
        assert client.post("/generate", json={"prompt": "x", "prompt_token_ids": [1]}).status_code == 422
        assert client.post("/generate", json={"prompt_token_ids": []}).status_code == 422
        h = client.get("/health")
        assert h.status_code == 200 and h.json()["status"] == "ok" and h.json()["num_blocks"] == 128


def test_http_text_prompts_with_a_tokenizer():
    from fastapi.testclient import TestClient

    tok = ByteTokenizer()
    with TestClient(create_app(ReplicaRouter(EchoFactory(), ["r0"]), tokenizer=tok)) as client:
        ids = tok.encode("hé")
        r = client.post("/generate", json={"prompt": "hé", "max_tokens": 5})
        assert r.status_code == 200, r.text
        want = expected_tokens(ids, 5)
        assert r.json()["token_ids"] == want and r.json()["prompt_tokens"] == len(ids)
        assert r.json()["text"] == tok.decode(want)


def test_http_health_and_503_once_every_replica_failed():
    from fastapi.testclient import TestClient

    fac = EchoFactory(fail=(("r0", 1),))
    with TestClient(create_app(ReplicaRouter(fac, ["r0"]))) as client:
        r = client.post("/generate", json={"prompt_token_ids": [1], "max_tokens": 5})
        assert r.status_code == 503 and "replica 0" in r.json()["detail"]
        for _ in range(200):
            h = client.get("/health")
            if h.status_code == 503:
                break
        assert h.status_code == 503 and h.json()["status"] == "failed"
        assert client.post("/generate", json={"prompt_token_ids": [1]}).status_code == 503
        r = client.post("/generate", json={"prompt_token_ids": [1], "stream": True})
        assert r.status_code == 503


def test_front_ends_share_one_port():
    """Two server processes on one port (SO_REUSEPORT), one stand-in replica
    each: every request on its own connection gets its tokens, whichever
    process takes it, and stop() ends every process."""
    import httpx

    from tokquay_b200.frontend import FrontEnds

    fe = FrontEnds(EchoFactory(), ["r0", "r1"], 2)
    fe.start(timeout_s=120)
    try:
        url = f"http://{fe.host}:{fe.port}"
        seen = set()
        for i in range(24):
            with httpx.Client(timeout=60) as client:  # a new connection per request
                r = client.post(f"{url}/generate", json={"prompt_token_ids": [i + 1], "max_tokens": 3})
                assert r.status_code == 200 and r.json()["token_ids"] == expected_tokens([i + 1], 3)
                h = client.get(f"{url}/health").json()
                assert h["status"] == "ok" and len(h["replicas"]) == 1  # the process's own replica
                seen.add(h["replicas"][0]["device"])
        assert seen <= {"r0", "r1"}
    finally:
        procs = list(fe._procs)
        fe.stop()
    assert procs and not any(p.is_alive() for p in procs)


def _orphaning_server(out, busy):
    """Runs in a spawned process: starts one replica, reports its pid, then
    exits at once without stopping it (as a killed server process would).
    With ``busy`` the replica is first given long requests, so it is still
    stepping -- and sending a message per step that nobody will read, more
    than a pipe holds -- when the server goes."""
    import multiprocessing as mp
    import os

    from tokquay.sequence import SamplingParams
    from tokquay_b200.frontend import _replica_main

    ctx = mp.get_context("spawn")
    inbox, outbox = ctx.Queue(), ctx.Queue()
    factory = EchoFactory(max_model_len=1024, step_s=0.001 if busy else 0.0)
    p = ctx.Process(target=_replica_main, args=(0, "r0", factory, inbox, outbox), daemon=True)
    p.start()
    assert outbox.get(timeout=120)[0] == "ready"
    if busy:
        for rid in range(8):
            inbox.put(("add", rid, [1, 2, 3, rid], SamplingParams(max_tokens=1000, ignore_eos=True)))
        assert outbox.get(timeout=60)[0] == "tokens"  # stepping now
    out.put(p.pid)
    out.close()
    out.join_thread()  # the pid must leave before the abrupt exit below
    os._exit(0)


def _exited(pid: int) -> bool:
    try:
        with open(f"/proc/{pid}/stat") as f:
            return f.read().rsplit(")", 1)[1].split()[0] in ("Z", "X")  # a zombie has exited
    except FileNotFoundError:
        return True


@pytest.mark.parametrize("busy", [False, True], ids=["idle", "busy"])
def test_an_orphaned_replica_ends_itself(busy):
    import multiprocessing as mp
    import time

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    server = ctx.Process(target=_orphaning_server, args=(q, busy))
    server.start()
    pid = q.get(timeout=180)
    server.join(60)
    deadline = time.monotonic() + 30
    while not _exited(pid) and time.monotonic() < deadline:
        time.sleep(0.2)
    assert _exited(pid)
