"""Generate the golden fixtures from the unmodified reference implementation.

    python tests/golden/make_golden.py --ref <reference checkout> [--only CASE,...]

Runs the reference Tokquay code (pure Python + torch on the CPU) on seeded
inputs built by ``tokquay_b200.workloads`` and records what it produced:
logits, greedy token streams, block tables, free lists and the K/V rows it
wrote.  The reference is only needed here, once; the fixtures
(``golden.json`` + ``golden.npz``) are committed and every test reads those.
Weights and pool contents are not stored: they are rebuilt from the seeds.

Cases (reference test each one re-hosts, paths inside the Tokquay project):
  mini_decode   prefill 6, decode to 40 across bs=4 block boundaries, f64 + f32,
                plus the full-sequence forward (tests/test_phase3_paged.py:87-106)
  mini_batch8   8 prompts of lengths 1..48 greedy-decoded together, 20 tokens,
                vs each alone on the contiguous cache (tests/test_phase3_paged.py:109-129)
  mini_mixed    one step mixing a decode and a whole-prompt prefill, f64 + f32
                (tests/test_phase3_paged.py:143-164)
  cfg1          BASELINE config 1: GPT-2 124M, 8 decodes, bs 16, 1,024 blocks
  cfg3_bs16/32  BASELINE config 3: 4 prefills + 60 decodes in one step
  cfg2          BASELINE config 2, all 100 greedy steps, 2,048 blocks (every step's
                argmax / top-2 / sparse logit columns; the first 3 steps densely)
  cfg4_sub      BASELINE config 4's shape (bs 32, ctx U[256,1024]) on a 64-sequence
                subset of its 512 (every 8th), 4,096-block pool, 3 greedy steps
  alloc_trace   random allocate / grow / free on a tiny allocator
  sched_trace   three scheduler scenarios (burst with preemption, staggered
                arrivals with aborts, a tight step budget) driven without a model
  mini_engine   the reference Engine on the MINI model, waves of greedy requests
                on a pool small enough to preempt (tokquay/engine.py)
  gpt2_engine   the reference Engine on GPT-2 124M with the first 24 requests of the
                config-5 workload (outputs capped at 24 tokens), 72-block pool
  workload      the reference benchmark's serving workload generator
                (bench/workload.py:24-47) at three rates / seeds
"""

from __future__ import annotations

import argparse
import json
import random
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from tokquay_b200 import workloads as W  # noqa: E402

LOGIT_STRIDE_FULL = 8     # columns kept from GPT-2 124M logits (config 1)
LOGIT_STRIDE_LARGE = 32   # columns kept for the 64-sequence configs
LOGIT_STRIDE_SPARSE = 1024  # columns kept for every step of config 2's 100-step run
DENSE_STEPS = 3           # config-2 steps also kept at LOGIT_STRIDE_LARGE


def summarize_logits(x: torch.Tensor, stride: int) -> dict[str, np.ndarray]:
    x = x.detach().to(torch.float32).cpu()
    top = torch.topk(x, 2, dim=-1)
    return {
        "cols": x[:, ::stride].numpy().copy(),
        "argmax": top.indices[:, 0].numpy().astype(np.int64),
        "top2": top.values.numpy().copy(),
        "absmax": x.abs().amax(-1).numpy().copy(),
    }


# Scheduler scenarios: (name, pool blocks, block size, config, request trace).
# A trace entry is (arrival step, prompt length, max_tokens); "abort" entries
# (step, "abort", request index) drop a request between steps.
SCHED_SCENARIOS = [
    {"name": "burst_preempt", "num_blocks": 40, "block_size": 8, "free_seed": 4,
     "config": {"max_num_seqs": 8, "max_num_batched_tokens": 400, "max_model_len": 160, "watermark_blocks": 1},
     "requests": [[0, 20 + 7 * i % 60, 10 + 13 * i % 50] for i in range(14)]},
    {"name": "staggered", "num_blocks": 64, "block_size": 16, "free_seed": 5,
     "config": {"max_num_seqs": 5, "max_num_batched_tokens": 300, "max_model_len": 256, "watermark_blocks": 2},
     "requests": [[3 * i, 10 + 17 * i % 90, 5 + 11 * i % 70] for i in range(20)], "aborts": [[9, 2], [20, 5], [40, 12]]},
    {"name": "tight_budget", "num_blocks": 24, "block_size": 4, "free_seed": 6,
     "config": {"max_num_seqs": 16, "max_num_batched_tokens": 64, "max_model_len": 64, "watermark_blocks": 0},
     "requests": [[i // 3, 5 + 9 * i % 30, 3 + 5 * i % 25] for i in range(18)]},
]


def fake_token(seq_id: int, n_out: int) -> int:
    """Tokens of the scheduler traces: any deterministic function will do."""
    return (seq_id * 7919 + n_out * 104729) % 50000


def sched_scenario(BlockAllocator, Scheduler, SchedulerConfig, Sequence, SamplingParams, sc) -> dict:
    """Drive a scheduler with a model-free step (what paged_forward and the
    engine do to the sequences' state) and record every decision."""
    alloc = BlockAllocator(_MiniCfg(), sc["num_blocks"], sc["block_size"], device="meta")
    W.shuffle_free_list(alloc, sc["free_seed"])
    sched = Scheduler(alloc, SchedulerConfig(**sc["config"]))
    reqs = [Sequence(i, [(i * 31 + j) % 50000 for j in range(n)], sampling=SamplingParams(max_tokens=mt, ignore_eos=True))
            for i, (_, n, mt) in enumerate(sc["requests"])]  # fmt: skip
    arrivals = {}
    for i, (step, _, _) in enumerate(sc["requests"]):
        arrivals.setdefault(step, []).append(i)
    aborts = {}
    for step, idx in sc.get("aborts", []):
        aborts.setdefault(step, []).append(idx)
    rejected, out = [], []
    k = 0
    while k <= max(arrivals) or sched.has_unfinished():
        for idx in aborts.get(k, []):
            sched.abort(reqs[idx])
        for idx in arrivals.get(k, []):
            try:
                sched.add_request(reqs[idx])
            except ValueError:
                rejected.append(idx)
        batch = sched.schedule()
        rec = {"step": k}
        if batch is not None:
            rec.update(seqs=[s.seq_id for s in batch.seqs], prefill=batch.is_prefill,
                       preempted=[s.seq_id for s in batch.preempted], padded=batch.padded_tokens)  # fmt: skip
            for s in batch.seqs:  # what paged_forward + sampling do to the sequence
                s.num_cached_tokens += s.num_uncached_tokens
                s.append_token(fake_token(s.seq_id, len(s.output_token_ids)))
                if len(s.output_token_ids) >= s.sampling.max_tokens:
                    sched.finish(s, "length")
        rec.update(running=[s.seq_id for s in sched.running], waiting=[s.seq_id for s in sched.waiting],
                   tables=[list(s.block_table) for s in sched.running], free=list(alloc._free),
                   preemptions=sched.num_preemptions, discarded=sched.num_discarded_positions)  # fmt: skip
        out.append(rec)
        k += 1
        if k > 5000:
            raise RuntimeError("scheduler trace did not finish")
    return {**sc, "rejected": rejected, "trace": out, "outputs": [s.output_token_ids for s in reqs]}


class _MiniCfg:  # what BlockAllocator reads from a config
    n_layer, n_head, n_embd = 2, 2, 128
    d_head = 64


# The engine case: MINI model, a small pool (preemption), greedy requests
# arriving in waves.
ENGINE_CASE = {"cfg": W.MINI, "weights_seed": 21, "init": "gpt2", "block_size": 8, "num_blocks": 30,
               "pool_seed": 103, "pool_scale": 50.0, "free_seed": 7, "trace_seed": 5,
               "sched": {"max_num_seqs": 6, "max_num_batched_tokens": 256, "max_model_len": 128,
                         "watermark_blocks": 1}}  # fmt: skip


# The engine on GPT-2 124M with config-5 requests: the first 24 requests of the
# reference benchmark's workload (burst, seed 7) in three waves, output lengths
# capped at 24 tokens (CPU time), on a 72-block pool (preemption by recompute).
GPT2_ENGINE_CASE = {"weights_seed": 0, "init": "normal", "block_size": 16, "num_blocks": 72, "pool_seed": 104,
                    "free_seed": 9, "workload_seed": 7, "n_requests": 24, "max_tokens_cap": 24,
                    "waves": [[0, 0, 8], [4, 8, 16], [10, 16, 24]],
                    "sched": {"max_num_seqs": 64, "max_num_batched_tokens": 2048, "max_model_len": 1024,
                              "watermark_blocks": 1}}  # fmt: skip


def engine_arrivals(rng) -> list[list[tuple[list[int], int]]]:
    """Waves of (prompt, max_tokens): one wave is added before each step."""
    waves = []
    for w in range(8):
        n = [4, 0, 2, 0, 3, 1, 0, 2][w]
        waves.append([([rng.randrange(W.MINI["vocab_size"]) for _ in range(rng.randint(4, 48))],
                       rng.randint(6, 40)) for _ in range(n)])  # fmt: skip
    return waves


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout (or its install)")
    ap.add_argument("--only", default=None, help="comma-separated case names")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from tokquay.generate import greedy_generate, paged_forward  # the reference
    from tokquay.kv_cache import BlockAllocator, OutOfBlocksError
    from tokquay.model import GPT2, GPT2Config
    from tokquay.sequence import Sequence

    torch.set_num_threads(max(1, torch.get_num_threads()))
    only = set(args.only.split(",")) if args.only else None
    meta: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                  "numpy": np.__version__, "cases": {}}  # fmt: skip
    arrays: dict[str, np.ndarray] = {}
    json_path, npz_path = HERE / "golden.json", HERE / "golden.npz"
    if only and json_path.exists():
        meta = json.loads(json_path.read_text())
        with np.load(npz_path) as z:
            arrays = {k: z[k] for k in z.files if k.split("/")[0] not in only}
        for k in list(meta["cases"]):
            if k in only:
                del meta["cases"][k]

    def want(name):
        return only is None or name in only

    def model_for(cfg_kw, seed, init, dtype):
        cfg = GPT2Config(**cfg_kw)
        m = GPT2(cfg)
        W.load_weights(m, W.random_weights(cfg, seed, init), dtype)
        return m.to(dtype).eval()

    def garbage_alloc(cfg, num_blocks, bs, dtype, pool_seed, free_seed, cls=BlockAllocator):
        a = cls(cfg, num_blocks, bs, device="cpu", dtype=dtype)
        W.fill_pool_blocks(a.pool, range(num_blocks), pool_seed, scale=50.0)
        W.shuffle_free_list(a, free_seed)
        return a

    # ---------------------------------------------------------------- mini_decode
    if want("mini_decode"):
        t0 = time.time()
        ids = [random.Random(7).randrange(W.MINI["vocab_size"]) for _ in range(40)]
        case = {"cfg": W.MINI, "weights_seed": 11, "init": "gpt2", "block_size": 4, "num_blocks": 32,
                "pool_seed": 100, "pool_scale": 50.0, "free_seed": 0, "ids": ids, "prefill": 6}  # fmt: skip
        for dt, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
            m = model_for(W.MINI, 11, "gpt2", dt)
            a = garbage_alloc(m.cfg, 32, 4, dt, 100, 0)
            s = Sequence(0, ids[:6])
            a.allocate(s)
            got = [paged_forward(m, a, [s])[0]]
            for t in range(6, len(ids)):
                s.append_token(ids[t])
                a.append_slot(s)
                got.append(paged_forward(m, a, [s])[0])
            arrays[f"mini_decode/logits_{tag}"] = torch.stack(got).numpy()
            if dt == torch.float64:
                with torch.no_grad():
                    arrays["mini_decode/full_f64"] = m(torch.tensor([ids]))[0].numpy()
                case["block_table"] = list(s.block_table)
                case["free_after"] = list(a._free)
        meta["cases"]["mini_decode"] = case
        print(f"mini_decode {time.time() - t0:.1f}s")

    # ---------------------------------------------------------------- mini_batch8
    if want("mini_batch8"):
        t0 = time.time()

        class Recording(BlockAllocator):
            def __init__(self, *a, **kw):
                super().__init__(*a, **kw)
                self.ever_taken: set[int] = set()

            def _take(self, n):
                blocks = super()._take(n)
                self.ever_taken.update(blocks)
                return blocks

        text = [random.Random(8).randrange(W.MINI["vocab_size"]) for _ in range(200)]
        lengths = [1, 3, 7, 12, 16, 17, 33, 48]
        prompts = [text[3 * i:3 * i + n] for i, n in enumerate(lengths)]
        n_new = 20
        m = model_for(W.MINI, 12, "gpt2", torch.float32)
        a = garbage_alloc(m.cfg, 128, 16, torch.float32, 101, 1, cls=Recording)
        before = a.pool.clone()
        seqs = [Sequence(i, list(p)) for i, p in enumerate(prompts)]
        for s in seqs:
            a.allocate(s)
        running, steps, step_logits = seqs, [], []
        while running:
            tables = [list(s.block_table) for s in running]
            logits = paged_forward(m, a, running)
            nxt = logits.argmax(-1).tolist()
            steps.append({"seq_ids": [s.seq_id for s in running], "tables": tables, "next": nxt})
            step_logits.append(logits.numpy())
            still = []
            for s, t in zip(running, nxt):
                s.append_token(t)
                if len(s.output_token_ids) >= n_new:
                    a.free(s)
                else:
                    a.append_slot(s)
                    still.append(s)
            running = still
        alone = [greedy_generate(m, torch.tensor([p]), n_new, use_cache=True) for p in prompts]
        changed = sorted(b for b in range(a.num_blocks) if not torch.equal(a.pool[b], before[b]))
        arrays["mini_batch8/logits"] = np.concatenate(step_logits)
        meta["cases"]["mini_batch8"] = {
            "cfg": W.MINI, "weights_seed": 12, "init": "gpt2", "block_size": 16, "num_blocks": 128,
            "pool_seed": 101, "pool_scale": 50.0, "free_seed": 1, "prompts": prompts, "n_new": n_new,
            "tokens": [s.output_token_ids for s in seqs], "alone": alone, "steps": steps,
            "ever_taken": sorted(a.ever_taken), "changed_blocks": changed, "free_after": list(a._free),
        }  # fmt: skip
        print(f"mini_batch8 {time.time() - t0:.1f}s")

    # ---------------------------------------------------------------- mini_mixed
    if want("mini_mixed"):
        t0 = time.time()
        rng = random.Random(9)
        a_ids = [rng.randrange(W.MINI["vocab_size"]) for _ in range(12)]
        b_ids = [rng.randrange(W.MINI["vocab_size"]) for _ in range(9)]
        case = {"cfg": W.MINI, "weights_seed": 13, "init": "gpt2", "block_size": 4, "num_blocks": 64,
                "pool_seed": 102, "pool_scale": 50.0, "free_seed": 3, "a_ids": a_ids, "b_ids": b_ids}  # fmt: skip
        for dt, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
            m = model_for(W.MINI, 13, "gpt2", dt)
            al = garbage_alloc(m.cfg, 64, 4, dt, 102, 3)
            sa = Sequence(0, a_ids[:-1])
            al.allocate(sa)
            paged_forward(m, al, [sa])
            sa.append_token(a_ids[-1])
            al.append_slot(sa)
            sb = Sequence(1, b_ids)
            al.allocate(sb)
            case[f"tables_{tag}"] = [list(sa.block_table), list(sb.block_table)]
            arrays[f"mini_mixed/logits_{tag}"] = paged_forward(m, al, [sa, sb]).numpy()
            if dt == torch.float64:
                with torch.no_grad():
                    arrays["mini_mixed/full_a_f64"] = m(torch.tensor([a_ids]))[0, -1].numpy()
                    arrays["mini_mixed/full_b_f64"] = m(torch.tensor([b_ids]))[0, -1].numpy()
        meta["cases"]["mini_mixed"] = case
        print(f"mini_mixed {time.time() - t0:.1f}s")

    # ---------------------------------------------------------------- GPT-2 124M configs
    big = None

    def gpt2_model():
        nonlocal big
        if big is None:
            big = model_for(W.GPT2_SMALL, 0, "normal", torch.float32)
        return big

    if want("cfg1"):
        t0 = time.time()
        m = gpt2_model()
        c = W.CONFIGS[1]
        a = BlockAllocator(m.cfg, c["num_blocks"], c["block_size"], device="cpu")
        case = W.decode_case(Sequence, a, c["n_seqs"], c["ctx_range"], m.cfg.vocab_size, seed=0)
        W.fill_pool_blocks(a.pool, W.used_blocks(case), seed=0)
        tables = case.block_tables
        logits = paged_forward(m, a, case.seqs)
        for k, v in summarize_logits(logits, LOGIT_STRIDE_FULL).items():
            arrays[f"cfg1/{k}"] = v
        # The K/V rows this step wrote (the last position of each sequence), layers 0 and 11.
        rows = []
        for s, ctx in zip(case.seqs, case.meta["ctx"]):
            p = ctx - 1
            blk, off = s.block_table[p // c["block_size"]], p % c["block_size"]
            rows.append(a.pool[blk, [0, 11], :, :, off].numpy())  # [2 layers, 2 kv, H, d]
        arrays["cfg1/written_kv"] = np.stack(rows)
        meta["cases"]["cfg1"] = {"seed": 0, "weights_seed": 0, "init": "normal", **{k: c[k] for k in c},
                                 "ctx": case.meta["ctx"], "tables": tables, "free_after": list(a._free),
                                 "logit_stride": LOGIT_STRIDE_FULL}  # fmt: skip
        print(f"cfg1 {time.time() - t0:.1f}s")

    for bs in (16, 32):
        name = f"cfg3_bs{bs}"
        if not want(name):
            continue
        t0 = time.time()
        m = gpt2_model()
        c = W.CONFIGS[3]
        a = BlockAllocator(m.cfg, c["num_blocks"], bs, device="cpu")
        case = W.mixed_case(Sequence, a, c["n_prefill"], c["n_decode"], c["len_range"], m.cfg.vocab_size, seed=3)
        W.fill_pool_blocks(a.pool, W.used_blocks(case), seed=3)
        tables = case.block_tables
        logits = paged_forward(m, a, case.seqs, case.new_lens)
        for k, v in summarize_logits(logits, LOGIT_STRIDE_LARGE).items():
            arrays[f"{name}/{k}"] = v
        meta["cases"][name] = {"seed": 3, "weights_seed": 0, "init": "normal", "block_size": bs,
                               "num_blocks": c["num_blocks"], "n_prefill": c["n_prefill"],
                               "n_decode": c["n_decode"], "len_range": c["len_range"],
                               "kinds": case.meta["kinds"], "lens": case.meta["lens"], "new_lens": case.new_lens,
                               "tables": tables, "logit_stride": LOGIT_STRIDE_LARGE}  # fmt: skip
        print(f"{name} {time.time() - t0:.1f}s")

    if want("cfg2"):
        t0 = time.time()
        m = gpt2_model()
        c = W.CONFIGS[2]
        a = BlockAllocator(m.cfg, c["num_blocks"], c["block_size"], device="cpu")
        case = W.decode_case(Sequence, a, c["n_seqs"], c["ctx_range"], m.cfg.vocab_size, seed=2)
        W.fill_pool_blocks(a.pool, W.used_blocks(case), seed=2)
        steps, sparse, argmax, top2, absmax = [], [], [], [], []
        n_steps = c["steps"]
        # The greedy loop of tokquay/generate.py:109-119 for a batch that runs
        # n_steps more tokens: sample, append, grow the table for the next step.
        for k in range(n_steps):
            tables = [list(s.block_table) for s in case.seqs]
            logits = paged_forward(m, a, case.seqs)
            if k < DENSE_STEPS:
                for key, v in summarize_logits(logits, LOGIT_STRIDE_LARGE).items():
                    arrays[f"cfg2/step{k}_{key}"] = v
                steps.append({"tables": tables})
            summ = summarize_logits(logits, LOGIT_STRIDE_SPARSE)
            sparse.append(summ["cols"])
            argmax.append(summ["argmax"])
            top2.append(summ["top2"])
            absmax.append(summ["absmax"])
            nxt = summ["argmax"].tolist()
            if k < DENSE_STEPS:
                steps[-1]["next"] = nxt
            for s, t in zip(case.seqs, nxt):
                s.append_token(t)
                if k + 1 < n_steps:
                    a.append_slot(s)
            if k % 10 == 9:
                print(f"  cfg2 step {k + 1}/{n_steps} {time.time() - t0:.0f}s", flush=True)
        arrays["cfg2/all_cols"] = np.stack(sparse)        # [steps, B, V / stride]
        arrays["cfg2/all_argmax"] = np.stack(argmax)      # [steps, B]
        arrays["cfg2/all_top2"] = np.stack(top2)          # [steps, B, 2]
        arrays["cfg2/all_absmax"] = np.stack(absmax)      # [steps, B]
        meta["cases"]["cfg2"] = {"seed": 2, "weights_seed": 0, "init": "normal", **{k: c[k] for k in c},
                                 "ctx": case.meta["ctx"], "steps": steps, "n_steps": n_steps,
                                 "dense_steps": DENSE_STEPS, "final_tables": [list(s.block_table) for s in case.seqs],
                                 "free_after": list(a._free), "logit_stride": LOGIT_STRIDE_LARGE,
                                 "sparse_stride": LOGIT_STRIDE_SPARSE}  # fmt: skip
        print(f"cfg2 {time.time() - t0:.1f}s")

    if want("cfg4_sub"):
        t0 = time.time()
        m = gpt2_model()
        c = W.CONFIGS[4]
        sub = W.CFG4_SUBSET
        a = BlockAllocator(m.cfg, sub["num_blocks"], c["block_size"], device="cpu")
        case = W.decode_case(Sequence, a, c["n_seqs"], c["ctx_range"], m.cfg.vocab_size, seed=4,
                             shard=tuple(sub["shard"]))  # fmt: skip
        W.fill_pool_blocks(a.pool, W.used_blocks(case), seed=4)
        first_tables = [list(s.block_table) for s in case.seqs]
        n_steps = sub["steps"]
        for k in range(n_steps):
            logits = paged_forward(m, a, case.seqs)
            summ = summarize_logits(logits, LOGIT_STRIDE_LARGE)
            for key, v in summ.items():
                arrays[f"cfg4_sub/step{k}_{key}"] = v
            for s, t in zip(case.seqs, summ["argmax"].tolist()):
                s.append_token(t)
                if k + 1 < n_steps:
                    a.append_slot(s)
            print(f"  cfg4_sub step {k + 1}/{n_steps} {time.time() - t0:.0f}s", flush=True)
        meta["cases"]["cfg4_sub"] = {"seed": 4, "weights_seed": 0, "init": "normal", "n_seqs": c["n_seqs"],
                                     "ctx_range": c["ctx_range"], "block_size": c["block_size"], **sub,
                                     "ctx": case.meta["ctx"], "tables": first_tables, "n_steps": n_steps,
                                     "tokens": [s.output_token_ids for s in case.seqs],
                                     "final_tables": [list(s.block_table) for s in case.seqs],
                                     "free_after": list(a._free), "logit_stride": LOGIT_STRIDE_LARGE}  # fmt: skip
        del a
        print(f"cfg4_sub {time.time() - t0:.1f}s")

    # ---------------------------------------------------------------- allocator trace
    if want("alloc_trace"):
        tiny = GPT2Config(vocab_size=8, n_positions=64, n_embd=4, n_layer=1, n_head=1)
        a = BlockAllocator(tiny, 24, 4, device="cpu")
        rng = random.Random(5)
        live: dict[int, Sequence] = {}
        ops, nid = [], 0
        for _ in range(400):
            r = rng.random()
            if r < 0.4 or not live:
                n = rng.randint(1, 30)
                s = Sequence(nid, [0] * n)
                nid += 1
                try:
                    a.allocate(s)
                    live[s.seq_id] = s
                    res = "ok"
                except OutOfBlocksError:
                    res = "oob"
                ops.append({"op": "allocate", "id": s.seq_id, "n": n, "res": res})
            elif r < 0.8:
                sid = rng.choice(sorted(live))
                s = live[sid]
                s.append_token(0)
                try:
                    grabbed = a.append_slot(s)
                    res = "grabbed" if grabbed else "same"
                except OutOfBlocksError:
                    s.output_token_ids.pop()
                    res = "oob"
                ops.append({"op": "append", "id": sid, "res": res})
            else:
                sid = rng.choice(sorted(live))
                a.free(live.pop(sid))
                ops.append({"op": "free", "id": sid, "res": "ok"})
            ops[-1]["free"] = list(a._free)
            ops[-1]["tables"] = {str(k): list(v.block_table) for k, v in live.items()}
            ops[-1]["ref_counts"] = list(a.ref_counts)
        meta["cases"]["alloc_trace"] = {"num_blocks": 24, "block_size": 4, "ops": ops}

    # ---------------------------------------------------------------- scheduler traces
    if want("sched_trace"):
        t0 = time.time()
        from tokquay.scheduler import Scheduler, SchedulerConfig
        from tokquay.sequence import SamplingParams

        meta["cases"]["sched_trace"] = {"scenarios": [sched_scenario(BlockAllocator, Scheduler, SchedulerConfig,
                                                                     Sequence, SamplingParams, sc)
                                                      for sc in SCHED_SCENARIOS]}  # fmt: skip
        print(f"sched_trace {time.time() - t0:.1f}s")

    # ---------------------------------------------------------------- engine trace
    if want("mini_engine"):
        t0 = time.time()
        from tokquay.engine import Engine
        from tokquay.scheduler import SchedulerConfig
        from tokquay.sequence import SamplingParams

        case = dict(ENGINE_CASE)
        m = model_for(W.MINI, case["weights_seed"], "gpt2", torch.float32)
        a = garbage_alloc(m.cfg, case["num_blocks"], case["block_size"], torch.float32, case["pool_seed"],
                          case["free_seed"])  # fmt: skip
        eng = Engine(m, a, SchedulerConfig(**case["sched"]))
        orig_sample = eng._sample
        margins: list[list[float]] = []

        def sample_and_record(seqs, logits):
            top = torch.topk(logits.float(), 2, dim=-1).values
            margins.append((top[:, 0] - top[:, 1]).tolist())
            return orig_sample(seqs, logits)

        eng._sample = sample_and_record
        steps = []
        rng = random.Random(case["trace_seed"])
        arrivals = engine_arrivals(rng)
        k = 0
        while arrivals or eng.has_unfinished():
            for prompt, max_tokens in arrivals.pop(0) if arrivals else []:
                eng.add_request(prompt, SamplingParams(max_tokens=max_tokens, ignore_eos=True))
            events = eng.step()
            last = eng.last_step
            steps.append({
                "events": [[e.seq_id, e.token_id, e.finish_reason] for e in events],
                "is_prefill": bool(last.is_prefill) if last else None,
                "running": [s.seq_id for s in eng.scheduler.running],
                "tables": [list(s.block_table) for s in eng.scheduler.running],
                "waiting": [s.seq_id for s in eng.scheduler.waiting],
                "free": list(a._free),
                "preemptions": eng.scheduler.num_preemptions,
            })
            k += 1
        case["steps"] = steps
        case["margins"] = margins
        meta["cases"]["mini_engine"] = case
        print(f"mini_engine {time.time() - t0:.1f}s, {k} steps")

    if want("gpt2_engine"):
        t0 = time.time()
        sys.path.insert(0, args.ref)
        from bench.workload import make_workload  # the reference benchmark's generator
        from tokquay.engine import Engine
        from tokquay.scheduler import SchedulerConfig
        from tokquay.sequence import SamplingParams

        case = dict(GPT2_ENGINE_CASE)
        m = gpt2_model()
        a = BlockAllocator(m.cfg, case["num_blocks"], case["block_size"], device="cpu")
        W.fill_pool_blocks(a.pool, range(case["num_blocks"]), case["pool_seed"])
        W.shuffle_free_list(a, case["free_seed"])
        eng = Engine(m, a, SchedulerConfig(**case["sched"]))
        orig_sample = eng._sample
        margins: list[list[float]] = []

        def sample_and_record(seqs, logits):
            top = torch.topk(logits.float(), 2, dim=-1).values
            margins.append((top[:, 0] - top[:, 1]).tolist())
            return orig_sample(seqs, logits)

        eng._sample = sample_and_record
        specs = make_workload(float("inf"), case["n_requests"], case["workload_seed"])
        waves = {step: specs[lo:hi] for step, lo, hi in case["waves"]}
        steps, k = [], 0
        while k <= max(waves) or eng.has_unfinished():
            for spec in waves.get(k, []):
                eng.add_request(list(spec.prompt_ids), SamplingParams(max_tokens=min(spec.output_len,
                                case["max_tokens_cap"]), ignore_eos=True))  # fmt: skip
            events = eng.step()
            last = eng.last_step
            steps.append({
                "events": [[e.seq_id, e.token_id, e.finish_reason] for e in events],
                "is_prefill": bool(last.is_prefill) if last else None,
                "running": [s.seq_id for s in eng.scheduler.running],
                "tables": [list(s.block_table) for s in eng.scheduler.running],
                "waiting": [s.seq_id for s in eng.scheduler.waiting],
                "free": list(a._free),
                "preemptions": eng.scheduler.num_preemptions,
            })
            k += 1
        case["steps"] = steps
        case["margins"] = margins
        meta["cases"]["gpt2_engine"] = case
        print(f"gpt2_engine {time.time() - t0:.1f}s, {k} steps, {eng.scheduler.num_preemptions} preemptions")

    # ---------------------------------------------------------------- serving workload
    if want("workload"):
        sys.path.insert(0, args.ref)
        from bench.workload import make_workload  # the reference benchmark's generator

        cases = []
        for rate, n, seed in ((64.0, 60, 0), (float("inf"), 25, 3), (7.5, 40, 11)):
            specs = make_workload(rate, n, seed)
            cases.append({"rate": rate if rate != float("inf") else "inf", "n": n, "seed": seed,
                          "arrivals": [r.arrival for r in specs], "output_lens": [r.output_len for r in specs],
                          "prompt_lens": [len(r.prompt_ids) for r in specs],
                          "prompt_heads": [list(r.prompt_ids[:4]) for r in specs],
                          "prompt_sums": [sum(r.prompt_ids) for r in specs]})  # fmt: skip
        meta["cases"]["workload"] = {"cases": cases}
        print("workload done")

    json_path.write_text(json.dumps(meta, separators=(",", ":")))
    np.savez_compressed(npz_path, **arrays)
    print(f"wrote {json_path} ({json_path.stat().st_size} B), {npz_path} ({npz_path.stat().st_size} B)")


if __name__ == "__main__":
    main()
