"""The serving front end over a real replica: one engine process on cuda:0
behind the HTTP API answers with the tokens the same engine gives in this
process (random-init GPT-2 124M, greedy, requests one at a time)."""

import random

import pytest

from tokquay_b200.frontend import RandomGPT2Engine, ReplicaRouter, create_app
from tokquay.sequence import SamplingParams

pytestmark = pytest.mark.gpu


def test_http_replica_gives_the_engine_tokens():
    from fastapi.testclient import TestClient

    factory = RandomGPT2Engine(num_blocks=256, block_size=16, max_num_seqs=8, seed=3)
    rng = random.Random(0)
    prompts = [[rng.randrange(50256) for _ in range(rng.randint(4, 40))] for _ in range(4)]
    with TestClient(create_app(ReplicaRouter(factory, [0]))) as client:
        got = []
        for p in prompts:
            r = client.post("/generate", json={"prompt_token_ids": p, "max_tokens": 6, "ignore_eos": True})
            assert r.status_code == 200, r.text
            got.append(r.json()["token_ids"])
        r = client.post("/generate", json={"prompt_token_ids": prompts[0], "max_tokens": 6, "ignore_eos": True,
                                           "stream": True})  # fmt: skip
        sse = [line for line in r.text.splitlines() if line.startswith("data: ")]
        assert len(sse) == 6
        h = client.get("/health")
        assert h.status_code == 200 and h.json()["status"] == "ok" and h.json()["free_blocks"] == 256
    eng = factory(0)
    for p, g in zip(prompts, got):
        eng.add_request(p, SamplingParams(max_tokens=6, ignore_eos=True))
        assert g == [ev.token_id for ev in eng.run_until_done()]
