"""The host step planner (``tq_plan_step``) on the CPU, through the C ABI.

Checks it against the oracle's restatement of PagedBatch.__init__
(tokquay/kv_cache.py:174-226): the same slots, positions and last rows, the
same rejections; and checks that the attention work items cover every query
row's causal key range exactly once, with every bulk copy the kernel would
issue (simulated here, mirroring issue_chunk in paged_attention.cuh) inside
its block and its shared-memory stage.  No GPU needed.
"""

import random

import numpy as np
import pytest

import oracle
from tokquay_b200 import _lib
from tokquay_b200.kv_cache import MIN_SPLIT_CHUNKS, attention_chunk_keys, cdiv, plan_step_host

N_HEAD = 3
KMAX_ROWS = 4
# K (or V) rows one stage holds: the library's chunk size (checked in simulate_copies)


def unpack(plan, layout):
    L = layout
    B, N = int(L[_lib.PLAN_NUM_SEQS]), int(L[_lib.PLAN_NUM_TOKENS])
    ni, nc, stride = int(L[_lib.PLAN_NUM_ITEMS]), int(L[_lib.PLAN_NUM_COMBINE]), int(L[_lib.PLAN_TABLE_STRIDE])

    def v(k, n):
        o = int(L[k])
        return np.asarray(plan[o:o + n])

    return dict(
        B=B, N=N, stride=stride,
        counts=v(_lib.PLAN_OFF_COUNTS, 4),
        seq=v(_lib.PLAN_OFF_SEQ_INFO, 4 * B).reshape(B, 4),
        tables=v(_lib.PLAN_OFF_TABLES, B * stride).reshape(B, stride),
        slots=v(_lib.PLAN_OFF_SLOTS, N), pos=v(_lib.PLAN_OFF_POSITIONS, N), ids=v(_lib.PLAN_OFF_TOKEN_IDS, N),
        last=v(_lib.PLAN_OFF_LAST_ROWS, B), items=v(_lib.PLAN_OFF_ITEMS, 8 * ni).reshape(ni, 8),
        combine=v(_lib.PLAN_OFF_COMBINE, 4 * nc).reshape(nc, 4),
        n_partials=int(L[_lib.PLAN_NUM_PARTIALS]),
    )  # fmt: skip


def random_batch(rng, bs, num_blocks, n_seqs, max_start, max_new):
    free = list(range(num_blocks))
    rng.shuffle(free)
    tables, start, new = [], [], []
    for _ in range(n_seqs):
        s = rng.randint(0, max_start)
        n = rng.randint(1, max_new)
        need = cdiv(s + n, bs)
        extra = rng.randint(0, 2)  # tables may be longer than needed
        tables.append([free.pop() for _ in range(min(need + extra, len(free)))] if len(free) >= need else None)
        start.append(s)
        new.append(n)
        if tables[-1] is None:
            tables.pop(), start.pop(), new.pop()
            break
    return tables, start, new


def simulate_copies(p, bs, num_blocks, n_head):
    """Replay issue_chunk's arithmetic for every (item, head, chunk): every
    copy's source block must be a planned table entry of the sequence and
    every destination inside the stage.  Returns {(row, head): sorted keys}."""
    ATTN_CHUNK = attention_chunk_keys()
    seen: dict[tuple[int, int], list[int]] = {}
    items = p["items"]
    for it in items:
        seq, row0, nrows, pos0, cbeg, cend, part, sn = (int(x) for x in it)
        split, nsplit = sn & 0xFFFF, sn >> 16
        assert 1 <= nrows <= KMAX_ROWS and cbeg < cend
        ctx = int(p["seq"][seq][3])
        need = cdiv(ctx, bs)
        kend = min(pos0 + nrows, cend * ATTN_CHUNK)
        assert kend <= ctx
        # the kernel holds one item's block ids in two registers per lane
        assert (kend - 1) // bs - (cbeg * ATTN_CHUNK) // bs + 1 <= 64
        for c in range(cbeg, cend):
            key0 = c * ATTN_CHUNK
            nkeys = min(ATTN_CHUNK, kend - key0)
            assert nkeys >= 1
            if bs <= ATTN_CHUNK:
                kb = key0 // bs
                while kb * bs < key0 + nkeys:
                    assert kb < need <= p["stride"]
                    blk = int(p["tables"][seq][kb])
                    assert 0 <= blk < num_blocks
                    rows = min(bs, key0 + nkeys - kb * bs)
                    dst = kb * bs - key0
                    assert 0 <= dst and dst + rows <= ATTN_CHUNK
                    kb += 1
            else:
                kb = key0 // bs
                assert kb < need
                off = key0 % bs
                assert off + nkeys <= bs
            for r in range(nrows):
                pos = pos0 + r
                nvalid = min(ATTN_CHUNK, pos + 1 - key0)
                for h in range(n_head):
                    seen.setdefault((row0 + r, h), []).extend(range(key0, key0 + max(0, nvalid)))
        if nsplit > 1:
            assert part >= 0
            for r in range(nrows):
                for h in range(n_head):
                    idx = part + (r * n_head + h) * nsplit + split
                    assert 0 <= idx < p["n_partials"]
        else:
            assert part == -1 and split == 0
    return seen


@pytest.mark.parametrize("bs", [1, 2, 4, 16, 32, 64, 256])
@pytest.mark.parametrize("seed", range(6))
def test_plan_matches_oracle_and_covers_every_key_once(bs, seed):
    rng = random.Random(1000 * bs + seed)
    num_blocks = 12 * cdiv(742, bs) + 50  # room for every sequence of the batch
    tables, start, new = random_batch(rng, bs, num_blocks, rng.randint(1, 12), 700, rng.choice([1, 5, 40]))
    ids = [rng.randrange(1000) for _ in range(sum(new))]
    target = rng.choice([1, 50, 10_000])
    plan, layout = plan_step_host(bs, num_blocks, N_HEAD, tables, start, new, ids, 1000, target, MIN_SPLIT_CHUNKS)
    p = unpack(plan, layout)
    ob = oracle.OracleBatch.build(bs, tables, start, new)
    # Same scatter targets and positions as the reference's index arrays.
    np.testing.assert_array_equal(p["slots"], ob.w_blk * bs + ob.w_off)
    np.testing.assert_array_equal(p["pos"], ob.positions[ob.w_b, ob.w_t])
    np.testing.assert_array_equal(p["ids"], ids)
    assert p["N"] == len(ob.w_b) and layout[_lib.PLAN_MAX_CTX] == ob.max_ctx
    assert p["stride"] == ob.nb
    for b, (st, n) in enumerate(zip(start, new)):  # the entries a sequence can read
        need = cdiv(st + n, bs)
        np.testing.assert_array_equal(p["tables"][b, :need], ob.block_tables[b, :need])
    cu = np.concatenate([[0], np.cumsum(new)])
    np.testing.assert_array_equal(p["last"], cu[1:] - 1)
    np.testing.assert_array_equal(p["counts"], [p["N"], len(p["items"]), len(p["combine"]), p["B"]])
    # Every (row, head) sees keys 0..position exactly once across its items.
    seen = simulate_copies(p, bs, num_blocks, N_HEAD)
    for r in range(p["N"]):
        for h in range(N_HEAD):
            assert seen[(r, h)] == list(range(int(p["pos"][r]) + 1)), (r, h)
    # Rows with split keys have exactly one combine entry each.
    split_rows = {int(it[1]) + k for it in p["items"] if (int(it[7]) >> 16) > 1 for k in range(int(it[2]))}
    assert sorted(int(e[0]) for e in p["combine"]) == sorted(split_rows)


def test_split_policy():
    # 8 decodes of 4096 keys with 12 heads: 96 units < target, so split.
    tables = [list(range(i * 256, (i + 1) * 256)) for i in range(8)]
    plan, layout = plan_step_host(16, 8 * 256, 12, tables, [4095] * 8, [1] * 8, None, 0, 2368, 2)
    p = unpack(plan, layout)
    assert layout[_lib.PLAN_SPLIT_CHUNKS] >= 2 and len(p["combine"]) == 8
    # Enough units already: no split.
    tables = [list(range(i * 2, i * 2 + 2)) for i in range(300)]
    plan, layout = plan_step_host(16, 600, 12, tables, [20] * 300, [1] * 300, None, 0, 2368, 2)
    assert layout[_lib.PLAN_NUM_COMBINE] == 0 and layout[_lib.PLAN_NUM_PARTIALS] == 0


def test_rejections_match_the_reference():
    """tokquay/kv_cache.py:182-191, plus the pool / vocabulary range checks."""
    with pytest.raises(ValueError, match="non-empty"):
        plan_step_host(4, 8, 1, [], [], [])
    with pytest.raises(ValueError, match="at least one token"):
        plan_step_host(4, 8, 1, [[0]], [0], [0])
    with pytest.raises(ValueError, match="1 blocks cannot hold 9 tokens"):
        plan_step_host(4, 8, 1, [[0]], [0], [9])
    with pytest.raises(ValueError, match="outside the pool"):
        plan_step_host(4, 8, 1, [[8]], [0], [1])
    with pytest.raises(ValueError, match="vocabulary"):
        plan_step_host(4, 8, 1, [[0]], [0], [1], token_ids=[50], vocab_size=50)
    with pytest.raises(ValueError, match="token ids"):
        plan_step_host(4, 8, 1, [[0]], [0], [2], token_ids=[1])
    with pytest.raises(RuntimeError, match="power of two"):
        plan_step_host(3, 8, 1, [[0]], [0], [1])


def test_capacity_retry_and_in_place_buffer():
    tables = [[0, 1, 2], [3]]
    small = np.zeros(8, dtype=np.int32)
    plan, layout = plan_step_host(4, 8, 2, tables, [5, 0], [4, 2], None, 0, 10, 1, out=small)
    assert plan is not small and plan.size == layout[_lib.PLAN_TOTAL_INTS]
    big = np.zeros(4096, dtype=np.int32)
    plan2, layout2 = plan_step_host(4, 8, 2, tables, [5, 0], [4, 2], None, 0, 10, 1, out=big)
    assert plan2 is big
    np.testing.assert_array_equal(big[:plan.size], plan)


def test_fixed_capacity_layout_is_step_independent():
    """With caps, every step that fits gets the same offsets and table stride
    (what a captured CUDA graph needs), and the data matches the packed plan."""
    caps = np.array([8, 8, 40, 8 * 16, 8, 8 * 3 * 16], dtype=np.int32)
    rng = random.Random(0)
    layouts = []
    for _ in range(5):
        B = rng.randint(1, 8)
        tables = [list(range(i * 40, i * 40 + rng.randint(1, 40))) for i in range(B)]
        start = [rng.randint(0, len(t) * 16 - 1) for t in tables]
        new = [1] * B
        plan, layout = plan_step_host(16, 8 * 40, 3, tables, start, new, None, 0, 500, 2, caps=caps)
        packed, playout = plan_step_host(16, 8 * 40, 3, tables, start, new, None, 0, 500, 2)
        p, q = unpack(plan, layout), unpack(packed, playout)
        np.testing.assert_array_equal(p["slots"][:q["N"]], q["slots"])
        np.testing.assert_array_equal(p["counts"], q["counts"])
        layouts.append(tuple(int(layout[k]) for k in range(_lib.PLAN_TABLE_STRIDE, _lib.PLAN_LAYOUT_LEN)
                             if k not in (_lib.PLAN_MAX_CTX, _lib.PLAN_SPLIT_CHUNKS)))
    assert len(set(layouts)) == 1
    with pytest.raises(RuntimeError, match="capacities"):
        plan_step_host(16, 8 * 40, 3, [[0]] * 9, [0] * 9, [1] * 9, None, 0, 500, 2, caps=caps)


def test_fixed_capacity_coarsens_the_split_to_fit():
    caps = np.array([4, 4, 64, 4, 4, 4 * 12 * 2], dtype=np.int32)  # room for 1 item per seq
    tables = [list(range(i * 64, (i + 1) * 64)) for i in range(4)]
    plan, layout = plan_step_host(16, 256, 12, tables, [1000] * 4, [1] * 4, None, 0, 10_000, 2, caps=caps)
    assert layout[_lib.PLAN_NUM_ITEMS] <= 4 and layout[_lib.PLAN_NUM_PARTIALS] <= caps[5]
