"""Pin the numpy oracle to the reference: rerun every golden case through
``oracle.paged_forward`` and compare with what the unmodified reference
produced (tests/golden/make_golden.py).  CPU only."""

import numpy as np
import pytest

import oracle
from helpers import (
    F64_ATOL,
    ORACLE_F32_ATOL,
    build_config_case,
    cfg_of,
    numpy_pool,
    weights_of,
)
from tokquay_b200 import workloads as W
from tokquay_b200.kv_cache import BlockAllocator
from tokquay_b200.model import GPT2Config
from tokquay.sequence import Sequence


def _w(case, dtype):
    return {k: v.astype(dtype) for k, v in weights_of(case).items()}


@pytest.mark.parametrize("dtype,tag,atol", [(np.float64, "f64", F64_ATOL), (np.float32, "f32", ORACLE_F32_ATOL)])
def test_mini_decode_across_block_boundaries(golden, dtype, tag, atol):
    """Prefill 6 tokens, then decode one at a time across bs=4 boundaries
    (re-hosts tests/test_phase3_paged.py:87-106)."""
    case = golden.cases["mini_decode"]
    cfg = cfg_of(case)
    w = _w(case, dtype)
    pool = numpy_pool(cfg, case["num_blocks"], case["block_size"], range(case["num_blocks"]),
                      case["pool_seed"], case["pool_scale"], dtype)  # fmt: skip
    ids = case["ids"]
    s = Sequence(0, ids[:case["prefill"]])
    s.block_table = list(case["block_table"])  # the reference allocator's final table (a prefix grows into it)
    got = []
    for t in range(case["prefill"], len(ids) + 1):
        if t > case["prefill"]:
            s.append_token(ids[t - 1])
        got.append(oracle.paged_forward(w, cfg, pool, case["block_size"], [s])[0])
    got = np.stack(got)
    np.testing.assert_allclose(got, golden.arrays[f"mini_decode/logits_{tag}"], atol=atol, rtol=0)
    if dtype == np.float64:  # paged == full-sequence forward (noise-free)
        full = golden.arrays["mini_decode/full_f64"][case["prefill"] - 1:]
        np.testing.assert_allclose(got, full, atol=F64_ATOL, rtol=0)


def test_mini_batch8_every_step(golden):
    """8 prompts of different lengths decoded together: each step's logits and
    greedy tokens (re-hosts tests/test_phase3_paged.py:109-129).  Bookkeeping
    runs on this package's allocator, so its block tables are checked too."""
    case = golden.cases["mini_batch8"]
    cfg = cfg_of(case)
    w = _w(case, np.float32)
    pool = numpy_pool(cfg, case["num_blocks"], case["block_size"], range(case["num_blocks"]),
                      case["pool_seed"], case["pool_scale"])  # fmt: skip
    before = pool.copy()
    alloc = BlockAllocator(cfg, case["num_blocks"], case["block_size"], device="cpu")
    W.shuffle_free_list(alloc, case["free_seed"])
    seqs = [Sequence(i, list(p)) for i, p in enumerate(case["prompts"])]
    for s in seqs:
        alloc.allocate(s)
    ref = golden.arrays["mini_batch8/logits"]
    row = 0
    running = seqs
    for step in case["steps"]:
        assert [s.seq_id for s in running] == step["seq_ids"]
        assert [s.block_table for s in running] == step["tables"]
        logits = oracle.paged_forward(w, cfg, pool, case["block_size"], running)
        np.testing.assert_allclose(logits, ref[row:row + len(running)], atol=ORACLE_F32_ATOL, rtol=0)
        row += len(running)
        nxt = logits.argmax(-1).tolist()
        assert nxt == step["next"]
        still = []
        for s, t in zip(running, nxt):
            s.append_token(t)
            if len(s.output_token_ids) >= case["n_new"]:
                alloc.free(s)
            else:
                alloc.append_slot(s)
                still.append(s)
        running = still
    assert [s.output_token_ids for s in seqs] == case["tokens"] == case["alone"]
    assert alloc._free == case["free_after"]
    changed = {b for b in range(case["num_blocks"]) if not np.array_equal(pool[b], before[b])}
    assert changed == set(case["changed_blocks"])


@pytest.mark.parametrize("dtype,tag,atol", [(np.float64, "f64", F64_ATOL), (np.float32, "f32", ORACLE_F32_ATOL)])
def test_mini_mixed_prefill_and_decode(golden, dtype, tag, atol):
    """A decodes one token while B prefills its prompt, in one step
    (re-hosts tests/test_phase3_paged.py:143-164)."""
    case = golden.cases["mini_mixed"]
    cfg = cfg_of(case)
    w = _w(case, dtype)
    pool = numpy_pool(cfg, case["num_blocks"], case["block_size"], range(case["num_blocks"]),
                      case["pool_seed"], case["pool_scale"], dtype)  # fmt: skip
    ta, tb = case[f"tables_{tag}"]
    a = Sequence(0, case["a_ids"][:-1])
    a.block_table = list(ta)  # its final table; the prefill reads only the prefix it needs
    oracle.paged_forward(w, cfg, pool, case["block_size"], [a])
    a.append_token(case["a_ids"][-1])
    b = Sequence(1, case["b_ids"])
    b.block_table = list(tb)
    logits = oracle.paged_forward(w, cfg, pool, case["block_size"], [a, b])
    np.testing.assert_allclose(logits, golden.arrays[f"mini_mixed/logits_{tag}"], atol=atol, rtol=0)
    if dtype == np.float64:
        np.testing.assert_allclose(logits[0], golden.arrays["mini_mixed/full_a_f64"], atol=F64_ATOL, rtol=0)
        np.testing.assert_allclose(logits[1], golden.arrays["mini_mixed/full_b_f64"], atol=F64_ATOL, rtol=0)


def _cols(golden, key):
    return golden.arrays[key]


@pytest.mark.slow
def test_config1_decode_step(golden, gpt2_weights):
    case = golden.cases["cfg1"]
    cfg = GPT2Config(**W.GPT2_SMALL)
    seqs, _ = build_config_case("cfg1", golden)
    pool = numpy_pool(cfg, case["num_blocks"], case["block_size"], {b for t in case["tables"] for b in t}, case["seed"])
    logits = oracle.paged_forward(gpt2_weights, cfg, pool, case["block_size"], seqs)
    np.testing.assert_allclose(logits[:, ::case["logit_stride"]], _cols(golden, "cfg1/cols"), atol=ORACLE_F32_ATOL, rtol=0)
    assert logits.argmax(-1).tolist() == golden.arrays["cfg1/argmax"].tolist()
    # The K/V rows the step wrote, layers 0 and 11.
    bs = case["block_size"]
    got = []
    for s, c in zip(seqs, case["ctx"]):
        p = c - 1
        got.append(pool[s.block_table[p // bs], [0, 11], :, :, p % bs])
    np.testing.assert_allclose(np.stack(got), golden.arrays["cfg1/written_kv"], atol=ORACLE_F32_ATOL, rtol=0)


@pytest.mark.slow
@pytest.mark.parametrize("bs", [16, 32])
def test_config3_mixed_step(golden, gpt2_weights, bs):
    name = f"cfg3_bs{bs}"
    case = golden.cases[name]
    cfg = GPT2Config(**W.GPT2_SMALL)
    seqs, new_lens = build_config_case(name, golden)
    assert new_lens == case["new_lens"]
    pool = numpy_pool(cfg, case["num_blocks"], bs, {b for t in case["tables"] for b in t}, case["seed"])
    logits = oracle.paged_forward(gpt2_weights, cfg, pool, bs, seqs, new_lens)
    np.testing.assert_allclose(logits[:, ::case["logit_stride"]], _cols(golden, f"{name}/cols"),
                               atol=ORACLE_F32_ATOL, rtol=0)  # fmt: skip
    assert logits.argmax(-1).tolist() == golden.arrays[f"{name}/argmax"].tolist()


@pytest.mark.slow
def test_config2_greedy_steps(golden, gpt2_weights):
    """The oracle on config 2's first steps (the densely recorded ones)."""
    case = golden.cases["cfg2"]
    cfg = GPT2Config(**W.GPT2_SMALL)
    alloc = BlockAllocator(cfg, case["num_blocks"], case["block_size"], device="cpu")
    seqs, _ = build_config_case("cfg2", golden, alloc=alloc)
    used = {b for s in seqs for b in s.block_table}
    pool = numpy_pool(cfg, case["num_blocks"], case["block_size"], used, case["seed"])
    for k, step in enumerate(case["steps"]):
        assert [s.block_table for s in seqs] == step["tables"]
        logits = oracle.paged_forward(gpt2_weights, cfg, pool, case["block_size"], seqs)
        np.testing.assert_allclose(logits[:, ::case["logit_stride"]], _cols(golden, f"cfg2/step{k}_cols"),
                                   atol=ORACLE_F32_ATOL, rtol=0)  # fmt: skip
        nxt = logits.argmax(-1).tolist()
        assert nxt == step["next"] == golden.arrays["cfg2/all_argmax"][k].tolist()
        for s, t in zip(seqs, nxt):
            s.append_token(t)
            alloc.append_slot(s)


def test_config2_allocator_state_over_the_hundred_steps(golden):
    """Config 2's whole greedy run on the allocator alone (the reference's
    tokens fed back): block tables and free list equal the reference's after
    all 100 steps, bit for bit."""
    case = golden.cases["cfg2"]
    alloc = BlockAllocator(GPT2Config(**W.GPT2_SMALL), case["num_blocks"], case["block_size"], device="meta")
    seqs, _ = build_config_case("cfg2", golden, alloc=alloc)
    tokens = golden.arrays["cfg2/all_argmax"]
    for k in range(case["n_steps"]):
        for s, t in zip(seqs, tokens[k].tolist()):
            s.num_cached_tokens += 1
            s.append_token(t)
            if k + 1 < case["n_steps"]:
                alloc.append_slot(s)
    assert [s.block_table for s in seqs] == case["final_tables"]
    assert alloc._free == case["free_after"]


def test_oracle_rejects_what_the_reference_rejects():
    """The batch checks of tokquay/kv_cache.py:182-191 and model.py:157-160."""
    with pytest.raises(ValueError):
        oracle.OracleBatch.build(4, [], [], [])
    with pytest.raises(ValueError):
        oracle.OracleBatch.build(4, [[0]], [0], [0])
    with pytest.raises(ValueError, match="blocks cannot hold"):
        oracle.OracleBatch.build(4, [[0]], [0], [9])
