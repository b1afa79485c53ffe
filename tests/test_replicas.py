"""Replica-parallel host logic at world size 2 on CPU (gloo).

N GPUs run N independent decode replicas (tokquay_b200/replicas.py): the only
cross-rank steps are the barrier, the max of the per-rank times and the sum of
the token counts.  These tests run that logic as two gloo ranks, plan each
rank's own decode step with the native planner (no GPU), and check the bench's
reference arm leaves ranks other than 0 idle.
"""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tokquay_b200 import replicas

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))  # fmt: skip
    info = replicas.setup(backend="gloo", timeout_s=60)
    try:
        from tokquay_b200 import BlockAllocator, GPT2Config, Sequence
        from tokquay_b200 import kv_cache as KV
        from tokquay_b200 import workloads as W

        cfg = GPT2Config(**W.MINI)
        a = BlockAllocator(cfg, 256, 16, device="cpu")
        case = W.decode_case(Sequence, a, 4, (8, 64), cfg.vocab_size, seed=replicas.replica_seed(2, info.rank))
        seqs = case.seqs
        starts = [s.num_cached_tokens for s in seqs]
        ids = [s.token_ids[st:st + 1][0] for s, st in zip(seqs, starts)]
        plan, layout = KV.plan_step_host(a.block_size, a.num_blocks, cfg.n_head, [list(s.block_table) for s in seqs],
                                         starts, [1] * len(seqs), ids, cfg.vocab_size, 64, KV.MIN_SPLIT_CHUNKS)  # fmt: skip
        replicas.barrier(info.world)
        tokens = float(len(seqs))
        seconds = 1.0 + info.rank  # rank 1 is the slow one
        total, slowest, rate = replicas.whole_job_rate(tokens, seconds, info.world)
        res = {
            "rank": info.rank,
            "world": info.world,
            "total": total,
            "slowest": slowest,
            "rate": rate,
            "max": replicas.max_over_ranks(10.0 * (info.rank + 1), info.world),
            "sum": replicas.sum_over_ranks(info.rank + 0.5, info.world),
            "ids": ids,
            "plan_words": int(plan.size),
        }
        Path(out_dir, f"rank{info.rank}.json").write_text(json.dumps(res))
    finally:
        replicas.teardown(info)


def test_replica_info_from_env():
    i = replicas.ReplicaInfo.from_env({"WORLD_SIZE": "4", "RANK": "3", "LOCAL_RANK": "3"})
    assert (i.world, i.rank, i.local) == (4, 3, 3)
    assert replicas.ReplicaInfo.from_env({}).world == 1
    with pytest.raises(ValueError):
        replicas.ReplicaInfo(2, 2, 0)


def test_single_rank_reductions_are_identity():
    assert replicas.max_over_ranks(3.5, 1) == 3.5
    assert replicas.sum_over_ranks(3.5, 1) == 3.5
    assert replicas.whole_job_rate(8, 2.0, 1) == (8.0, 2.0, 4.0)


def test_two_gloo_ranks(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(world)]
    for r in res:
        assert r["world"] == 2
        assert r["total"] == 8.0  # 4 sequences per replica
        assert r["slowest"] == 2.0  # max over ranks, not rank 0's own time
        assert r["rate"] == 4.0
        assert r["max"] == 20.0
        assert r["sum"] == 2.0
        assert r["plan_words"] > 0
    # each replica decodes its own sequences
    assert res[0]["ids"] != res[1]["ids"]


def test_reference_arm_other_ranks_exit_idle():
    env = dict(os.environ, WORLD_SIZE="2", RANK="1", LOCAL_RANK="1", MASTER_ADDR="127.0.0.1", MASTER_PORT="1")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)  # fmt: skip
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_seeds_differ_per_rank():
    seeds = {replicas.replica_seed(2, r) for r in range(8)}
    assert len(seeds) == 8
    assert np.all(np.array(sorted(seeds)) >= 2)
