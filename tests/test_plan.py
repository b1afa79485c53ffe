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
from tokquay_b200.kv_cache import MIN_SPLIT_CHUNKS, attention_chunk_keys, attention_warps, cdiv, plan_step_host

N_HEAD = 3
TILE_FLAG = 8  # a prompt-tile item (or, alone in a first item, the marker of a tile CTA's other warps)
TILE_ROWS = 128
TILE_MAX_ITEMS = 96
FIRST_WORDS = 16  # a warp's first item: 8 item words + the block ids of its first chunk
KMAX_ROWS = 4
# K (or V) rows one stage holds: the library's chunk size (checked in simulate_copies)


def _u32(x) -> int:
    return int(np.uint32(np.int32(x)))


def decode_item(w) -> dict:
    w = [int(x) for x in w]
    return dict(
        seq=w[0], row0=w[1], nrows=w[2] & 0xFF, head=(w[2] >> 8) & 0xFFFF, flags=(_u32(w[2]) >> 24) & 3,
        decode=bool((_u32(w[2]) >> 24) & 4), tile=bool((_u32(w[2]) >> 24) & TILE_FLAG), pos0=w[3],
        cbeg=w[4] & 0xFFFF, cend=_u32(w[4]) >> 16, lsplit=w[5] & 0xFF, lcount=(w[5] >> 8) & 0xFF,
        lslot=_u32(w[5]) >> 16, gbase=w[6], gsplit=w[7] & 0xFFFF, gnsplit=_u32(w[7]) >> 16,
    )  # fmt: skip


def attention_lists(plan, layout) -> list[list[dict]]:
    """Each warp slot's work items (decoded), from the attention region."""
    nw = int(layout[_lib.PLAN_NUM_CTAS]) * attention_warps()
    o = int(layout[_lib.PLAN_OFF_ITEMS])
    first = np.asarray(plan[o:o + FIRST_WORDS * nw]).reshape(nw, FIRST_WORDS)
    offs = np.asarray(plan[o + FIRST_WORDS * nw:o + FIRST_WORDS * nw + nw + 1])
    ro = o + FIRST_WORDS * nw + (nw + 1 + 7) // 8 * 8
    rest = np.asarray(plan[ro:ro + 8 * int(offs[-1])]).reshape(-1, 8)
    W = attention_warps()
    lists = []
    for w in range(nw):
        if _u32(first[w][4]) >> 16:
            it = decode_item(first[w][:8])
            if it["tile"]:  # a tile CTA's list: warp 0 only
                assert w % W == 0
            it["first_blocks"] = [int(x) for x in first[w][8:]]
            lists.append([it] + [decode_item(x) for x in rest[offs[w]:offs[w + 1]]])
            assert all(x["tile"] == it["tile"] for x in lists[-1])
        elif _u32(first[w][2]) >> 24 == TILE_FLAG:  # marker: this warp runs its CTA's tile items
            assert w % W != 0 and lists[w - w % W] and lists[w - w % W][0]["tile"]
            assert not np.delete(first[w], 2).any() and offs[w] == offs[w + 1]
            lists.append([])
        else:
            assert not first[w].any() and offs[w] == offs[w + 1]
            lists.append([])
    return lists


def unpack(plan, layout):
    L = layout
    B, N = int(L[_lib.PLAN_NUM_SEQS]), int(L[_lib.PLAN_NUM_TOKENS])
    nc, stride = int(L[_lib.PLAN_NUM_COMBINE]), int(L[_lib.PLAN_TABLE_STRIDE])

    def v(k, n):
        o = int(L[k])
        return np.asarray(plan[o:o + n])

    warps = attention_lists(plan, layout)
    # The tile-merge trailer after the attention items: [8] (word 0: rows), then [rows][4].
    nw = int(L[_lib.PLAN_NUM_CTAS]) * attention_warps()
    o = int(L[_lib.PLAN_OFF_ITEMS])
    t0 = o + FIRST_WORDS * nw + (nw + 1 + 7) // 8 * 8 + 8 * int(plan[o + FIRST_WORDS * nw + nw])
    n_merges = int(plan[t0])
    assert n_merges == L[_lib.PLAN_NUM_TILE_MERGES] and not np.asarray(plan[t0 + 1:t0 + 8]).any()
    return dict(
        merges=np.asarray(plan[t0 + 8:t0 + 8 + 4 * n_merges]).reshape(n_merges, 4),
        B=B, N=N, stride=stride,
        counts=v(_lib.PLAN_OFF_COUNTS, 4),
        seq=v(_lib.PLAN_OFF_SEQ_INFO, 4 * B).reshape(B, 4),
        tables=v(_lib.PLAN_OFF_TABLES, B * stride).reshape(B, stride),
        slots=v(_lib.PLAN_OFF_SLOTS, N), pos=v(_lib.PLAN_OFF_POSITIONS, N), ids=v(_lib.PLAN_OFF_TOKEN_IDS, N),
        last=v(_lib.PLAN_OFF_LAST_ROWS, B), warps=warps, items=[it for ws in warps for it in ws],
        combine=v(_lib.PLAN_OFF_COMBINE, 4 * nc).reshape(nc, 4),
        n_partials=int(L[_lib.PLAN_NUM_PARTIALS]), n_ctas=int(L[_lib.PLAN_NUM_CTAS]),
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


def simulate_copies(p, bs, num_blocks):
    """Replay the producer's copy arithmetic for every (item, chunk): every
    copy's source block must be a planned table entry of the sequence and
    every destination inside the stage.  Returns {(row, head): sorted keys}."""
    ATTN_CHUNK = attention_chunk_keys()
    seen: dict[tuple[int, int], list[int]] = {}
    for it in p["items"]:
        seq, row0, nrows, pos0, cbeg, cend, h = (it[k] for k in ("seq", "row0", "nrows", "pos0", "cbeg", "cend", "head"))
        if "first_blocks" in it:  # the first chunk's block ids travel with a warp's first item
            key0, key_end = cbeg * ATTN_CHUNK, min(cbeg * ATTN_CHUNK + ATTN_CHUNK, pos0 + nrows)
            kb = list(range(key0 // bs, (key_end - 1) // bs + 1))
            want = [int(p["tables"][seq][b]) for b in kb][:FIRST_WORDS - 8]
            assert it["first_blocks"] == want + [-1] * (FIRST_WORDS - 8 - len(want))
        ctx = int(p["seq"][seq][3])
        need = cdiv(ctx, bs)
        kend = min(pos0 + nrows, cend * ATTN_CHUNK)
        assert kend <= ctx
        if it["tile"]:  # a run of the tile's chunks (all of them, or a piece merged across CTAs)
            assert 1 <= nrows <= TILE_ROWS and cbeg < cend <= cdiv(pos0 + nrows, ATTN_CHUNK)
            assert it["flags"] in (0, 2) and not it["decode"]
            assert it["flags"] == 2 or (cbeg == 0 and cend == cdiv(pos0 + nrows, ATTN_CHUNK))
        else:
            assert 1 <= nrows <= KMAX_ROWS and cbeg < cend
            # the kernel holds one item's block ids in two registers per lane
            assert (kend - 1) // bs - (cbeg * ATTN_CHUNK) // bs + 1 <= 64
        for c in range(cbeg, cend):
            key0 = c * ATTN_CHUNK
            nkeys = min(ATTN_CHUNK, kend - key0)
            assert nkeys >= 1
            if it["tile"]:
                for key in range(key0, key0 + nkeys):
                    assert key // bs < need <= p["stride"]
                    assert 0 <= int(p["tables"][seq][key // bs]) < num_blocks
            elif bs <= ATTN_CHUNK:
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
                seen.setdefault((row0 + r, h), []).extend(range(key0, key0 + max(0, nvalid)))
    return seen


def check_merges(p):
    """Every cut is merged exactly once: shared-memory groups inside one CTA
    (slots in range, disjoint, one merging warp each), split-K groups across
    CTAs (every split index written once, partial indices in range and
    disjoint between groups)."""
    W = attention_warps()
    max_rows = max([it["nrows"] for it in p["items"]] or [1])
    local_slots = 2 * (W - 1) * max_rows
    global_parts: dict[tuple[int, int], dict] = {}
    used_parts: set[int] = set()
    for c in range(p["n_ctas"]):
        groups: dict[int, list[tuple[int, dict]]] = {}
        for w in range(W):
            owned = 0
            for it in p["warps"][c * W + w]:
                if it["flags"] & 1:
                    groups.setdefault(it["lslot"], []).append((w, it))
                    owned += it["lsplit"] == 0
                else:
                    assert it["lcount"] == 0 and it["lsplit"] == 0 and it["lslot"] == 0
            assert owned <= 1  # a warp merges at most one shared-memory group
        slots_used: set[int] = set()
        for base, members in groups.items():
            k = members[0][1]["lcount"]
            assert k >= 2 and sorted(m[1]["lsplit"] for m in members) == list(range(k))
            ws = [m[0] for m in sorted(members, key=lambda m: m[1]["lsplit"])]
            assert ws == sorted(set(ws))  # one piece per warp, in warp order
            first = members[0][1]
            for _, it in members:
                assert all(it[f] == first[f] for f in ("seq", "row0", "nrows", "head", "flags", "gbase", "gsplit"))
            spans = sorted((it["cbeg"], it["cend"]) for _, it in members)
            assert all(spans[i][1] == spans[i + 1][0] for i in range(k - 1))  # contiguous keys
            rng_ = set(range(base, base + k * first["nrows"]))
            assert max(rng_) < local_slots and not (rng_ & slots_used)
            slots_used |= rng_
            if first["flags"] & 2:
                g = global_parts.setdefault((first["row0"], first["head"]), {"splits": [], "item": first})
                g["splits"].append(first["gsplit"])
        for w in range(W):
            for it in p["warps"][c * W + w]:
                if it["flags"] == 2:
                    g = global_parts.setdefault((it["row0"], it["head"]), {"splits": [], "item": it})
                    g["splits"].append(it["gsplit"])
    for (row0, h), g in global_parts.items():
        it = g["item"]
        n = it["gnsplit"]
        assert n >= 2 and sorted(g["splits"]) == list(range(n)), (row0, h, g["splits"])
        idx = {it["gbase"] + r * n + s for r in range(it["nrows"]) for s in range(n)}
        assert max(idx) < p["n_partials"] and min(idx) >= 0 and not (idx & used_parts)
        used_parts |= idx
    # Split tiles are merged after the grid: one trailer entry per row, whose
    # partials (head h at + h * its head stride) are the pieces' of that row.
    merges = {int(e[0]): e for e in p["merges"]}
    assert len(merges) == len(p["merges"])
    tile_rows = set()
    for (row0, h), g in global_parts.items():
        it = g["item"]
        if not it["tile"]:
            continue
        n = it["gnsplit"]
        for r in range(it["nrows"]):
            e = merges[row0 + r]
            tile_rows.add(row0 + r)
            assert e[2] == n and e[3] == it["nrows"] * n and e[1] + h * e[3] == it["gbase"] + r * n, (row0, r, h)
    assert tile_rows == set(merges)


@pytest.mark.parametrize("bs", [1, 2, 4, 16, 32, 64, 256])
@pytest.mark.parametrize("seed", range(6))
def test_plan_matches_oracle_and_covers_every_key_once(bs, seed):
    rng = random.Random(1000 * bs + seed)
    num_blocks = 12 * cdiv(742, bs) + 50  # room for every sequence of the batch
    tables, start, new = random_batch(rng, bs, num_blocks, rng.randint(1, 12), 700, rng.choice([1, 5, 40]))
    ids = [rng.randrange(1000) for _ in range(sum(new))]
    n_ctas = rng.choice([1, 3, 50, 148])
    min_split = rng.choice([1, 2, MIN_SPLIT_CHUNKS])
    plan, layout = plan_step_host(bs, num_blocks, N_HEAD, tables, start, new, ids, 1000, n_ctas, min_split)
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
    assert p["n_ctas"] == n_ctas and len(p["items"]) == layout[_lib.PLAN_NUM_ITEMS]
    # Every (row, head) sees keys 0..position exactly once across its items.
    seen = simulate_copies(p, bs, num_blocks)
    for r in range(p["N"]):
        for h in range(N_HEAD):
            assert sorted(seen[(r, h)]) == list(range(int(p["pos"][r]) + 1)), (r, h)
    check_merges(p)
    # The decode flag (the kernel's licence to read the keys before pos0 ahead
    # of the preceding kernel) marks exactly the items of one-token sequences.
    for it in p["items"]:
        assert it["decode"] == (new[it["seq"]] == 1), it
        assert not it["decode"] or (it["nrows"] == 1 and it["pos0"] == start[it["seq"]])
    # Rows with keys split across CTAs have exactly one combine entry each.
    split_rows = {it["row0"] + k for it in p["items"] if it["flags"] & 2 for k in range(it["nrows"])}
    assert sorted(int(e[0]) for e in p["combine"]) == sorted(split_rows)
    # The used prefix holds everything the step reads.
    o = int(layout[_lib.PLAN_OFF_ITEMS])
    nw = n_ctas * attention_warps()
    n_rest = int(plan[o + FIRST_WORDS * nw + nw])
    trailer = 8 + (4 * len(p["merges"]) + 7) // 8 * 8
    assert layout[_lib.PLAN_USED_INTS] == o + FIRST_WORDS * nw + (nw + 8) // 8 * 8 + 8 * n_rest + trailer
    assert layout[_lib.PLAN_USED_INTS] <= layout[_lib.PLAN_TOTAL_INTS] == plan.size


def test_cuts_balance_the_warps_of_a_cta():
    """Chunks are spread evenly: every warp of a CTA holds within one chunk of
    the CTA's mean, and CTA loads are within one longest piece of each other."""
    rng = random.Random(7)
    tables, start, new = random_batch(rng, 16, 4096, 64, 600, 1)
    plan, layout = plan_step_host(16, 4096, 12, tables, start, new, None, 0, 148, MIN_SPLIT_CHUNKS)
    p = unpack(plan, layout)
    W = attention_warps()
    loads = []
    for c in range(148):
        per = [sum(it["cend"] - it["cbeg"] for it in p["warps"][c * W + w]) for w in range(W)]
        assert max(per) - min(per) <= 1, per
        loads.append(sum(per))
    longest = max(it["cend"] - it["cbeg"] for it in p["items"])
    assert max(loads) - min(loads) <= W * longest


def test_split_policy():
    # 8 decodes of 4096 keys with 12 heads: each pair (128 chunks) is longer
    # than a CTA's share of 148 CTAs, so it is split across CTAs.
    tables = [list(range(i * 256, (i + 1) * 256)) for i in range(8)]
    plan, layout = plan_step_host(16, 8 * 256, 12, tables, [4095] * 8, [1] * 8, None, 0, 148, 2)
    p = unpack(plan, layout)
    assert len(p["combine"]) == 8 and layout[_lib.PLAN_NUM_PARTIALS] > 0
    check_merges(p)
    # Many short sequences: no cross-CTA split, and no global scratch.
    tables = [list(range(i * 2, i * 2 + 2)) for i in range(300)]
    plan, layout = plan_step_host(16, 600, 12, tables, [20] * 300, [1] * 300, None, 0, 148, 2)
    assert layout[_lib.PLAN_NUM_COMBINE] == 0 and layout[_lib.PLAN_NUM_PARTIALS] == 0
    # BASELINE config 2 shapes (64 decodes up to 512 keys): CTA-local cuts only.
    rng = random.Random(3)
    tables, start, new = random_batch(rng, 16, 4096, 64, 511, 1)
    plan, layout = plan_step_host(16, 4096, 12, tables, start, new, None, 0, 148, MIN_SPLIT_CHUNKS)
    p = unpack(plan, layout)
    assert layout[_lib.PLAN_NUM_PARTIALS] == 0 and any(it["flags"] == 1 for it in p["items"])


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
    used = int(layout[_lib.PLAN_USED_INTS])  # past it the buffer is not written
    np.testing.assert_array_equal(big[:used], plan[:used])


def test_fixed_capacity_layout_is_step_independent():
    """With caps, every step that fits gets the same offsets and table stride
    (what a captured CUDA graph needs), and the data matches the packed plan."""
    caps = np.array([8, 8, 40, 8 * 3 * 16 + 500 * (attention_warps() - 1), 8, 8 * 3 * 16], dtype=np.int32)
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
                             if k not in (_lib.PLAN_MAX_CTX, _lib.PLAN_SPLIT_CHUNKS, _lib.PLAN_USED_INTS)))
    assert len(set(layouts)) == 1
    with pytest.raises(RuntimeError, match="capacities"):
        plan_step_host(16, 8 * 40, 3, [[0]] * 9, [0] * 9, [1] * 9, None, 0, 500, 2, caps=caps)


def test_fixed_capacity_coarsens_the_split_to_fit():
    # 4 decodes of 1001 keys, 12 heads, 148 CTAs: unconstrained, every pair is
    # split across CTAs; with room for only 2 cross-CTA pieces per pair the
    # planner coarsens the split until items and partials fit.
    tables = [list(range(i * 64, (i + 1) * 64)) for i in range(4)]
    _, free = plan_step_host(16, 256, 12, tables, [1000] * 4, [1] * 4, None, 0, 148, 2)
    assert free[_lib.PLAN_NUM_PARTIALS] > 4 * 12 * 2
    W = attention_warps()
    caps = np.array([4, 4, 64, 4 * 12 * 2 + 148 * (W - 1), 4, 4 * 12 * 2], dtype=np.int32)
    plan, layout = plan_step_host(16, 256, 12, tables, [1000] * 4, [1] * 4, None, 0, 148, 2, caps=caps)
    assert layout[_lib.PLAN_NUM_ITEMS] <= caps[3] and 0 < layout[_lib.PLAN_NUM_PARTIALS] <= caps[5]
    check_merges(unpack(plan, layout))


@pytest.fixture
def tile_knobs():
    """Restores the planner's process-wide prompt-tile settings after a test."""
    prev = _lib.prompt_tiles()
    yield _lib.prompt_tiles
    _lib.prompt_tiles(prev, 1500, 200, 1)


def test_long_prompt_rows_go_to_tile_ctas_at_the_end_of_the_grid(tile_knobs):
    """Config-3-like mix: 4 prompts of 16..256 rows become (tile, head) items
    on CTAs of their own, the last of the grid; decodes keep the warp path."""
    tile_knobs(16, 600, 200)
    rng = random.Random(11)
    bs, num_blocks = 16, 2048
    free = list(range(num_blocks))
    rng.shuffle(free)
    tables, start, new = [], [], []
    for n in (16, 100, 200, 256):
        tables.append([free.pop() for _ in range(cdiv(n, bs))])
        start.append(0)
        new.append(n)
    for _ in range(60):
        c = rng.randint(16, 256)
        tables.append([free.pop() for _ in range(cdiv(c, bs))])
        start.append(c - 1)
        new.append(1)
    plan, layout = plan_step_host(bs, num_blocks, 12, tables, start, new, None, 0, 148, MIN_SPLIT_CHUNKS)
    p = unpack(plan, layout)
    W = attention_warps()
    tile_ctas = [c for c in range(148) if p["warps"][c * W] and p["warps"][c * W][0]["tile"]]
    assert tile_ctas and tile_ctas == list(range(148 - len(tile_ctas), 148))
    for c in tile_ctas:
        assert len(p["warps"][c * W]) <= TILE_MAX_ITEMS
        assert all(not p["warps"][c * W + w] for w in range(1, W))
    tiles = [it for it in p["items"] if it["tile"]]
    # 16 -> 1 tile, 100 -> 1, 200 -> 2 of 100, 256 -> 2 of 128: 6 tiles x 12 heads,
    # the longest cut into pieces no costlier than a CTA's balanced load
    assert len(tiles) == 6 * 12 and all(it["flags"] == 0 for it in tiles)  # beside decodes: not split
    assert sorted({(it["row0"], it["nrows"]) for it in tiles}) == [
        (0, 16), (16, 100), (116, 100), (216, 100), (316, 128), (444, 128)]
    assert all(it["decode"] for it in p["items"] if not it["tile"])
    seen = simulate_copies(p, bs, num_blocks)
    for r in range(p["N"]):
        for h in range(12):
            assert sorted(seen[(r, h)]) == list(range(int(p["pos"][r]) + 1)), (r, h)
    check_merges(p)


@pytest.mark.parametrize("n_ctas", [1, 2, 5, 148])
def test_tiles_on_any_grid_and_off(tile_knobs, n_ctas):
    """Tiles on any grid (a one-CTA grid beside warp work runs everything on
    the warp path), and with tiles off every row is a warp item."""
    rng = random.Random(n_ctas)
    bs, num_blocks = 4, 4096
    tables, start, new = random_batch(rng, bs, num_blocks, 9, 300, 150)
    for min_rows in (0, 1, 16):
        tile_knobs(min_rows, 600, 200)
        plan, layout = plan_step_host(bs, num_blocks, N_HEAD, tables, start, new, None, 0, n_ctas, 2)
        p = unpack(plan, layout)
        n_tile = sum(it["tile"] for it in p["items"])
        if min_rows == 0:
            assert n_tile == 0
        elif n_ctas > 1:
            assert n_tile > 0
        seen = simulate_copies(p, bs, num_blocks)
        for r in range(p["N"]):
            for h in range(N_HEAD):
                assert sorted(seen[(r, h)]) == list(range(int(p["pos"][r]) + 1)), (min_rows, r, h)
        check_merges(p)
        assert len(p["items"]) == layout[_lib.PLAN_NUM_ITEMS]


def test_prefill_only_steps_split_long_tiles_over_the_grid(tile_knobs):
    """With pieces allowed, a step of prompt rows alone spreads long tiles over the grid: tiles are
    cut over their keys into pieces of at least two chunks, every piece of a
    (tile, head) merged through the split-K scratch."""
    tile_knobs(16, 600, 200, 8)
    tables = [list(range(64))]
    plan, layout = plan_step_host(16, 64, 12, tables, [0], [1024], None, 0, 148, MIN_SPLIT_CHUNKS)
    p = unpack(plan, layout)
    tiles = [it for it in p["items"] if it["tile"]]
    assert len(tiles) > 8 * 12 and any(it["flags"] == 2 for it in tiles)
    assert all(it["cend"] - it["cbeg"] >= 2 for it in tiles)
    assert layout[_lib.PLAN_NUM_PARTIALS] > 0 and len(p["combine"]) > 0 and len(p["merges"]) > 0
    seen = simulate_copies(p, 16, 64)
    for r in range(p["N"]):
        for h in range(12):
            assert sorted(seen[(r, h)]) == list(range(int(p["pos"][r]) + 1)), (r, h)
    check_merges(p)


def test_long_tiles_beside_decodes_split_with_a_merge_after_the_grid(tile_knobs):
    """With pieces allowed, a mixed step cuts its costliest tiles over their
    keys beside the decode items; the trailer lists every row of a cut tile
    once, and plans of fixed capacities never cut a tile."""
    tile_knobs(16, 1500, 200, 4)
    rng = random.Random(3)
    bs, num_blocks = 16, 2048
    free = list(range(num_blocks))
    rng.shuffle(free)
    tables, start, new = [], [], []
    for n in (75, 236, 32, 170):
        tables.append([free.pop() for _ in range(cdiv(n, bs))])
        start.append(0)
        new.append(n)
    for _ in range(60):
        c = rng.randint(16, 256)
        tables.append([free.pop() for _ in range(cdiv(c, bs))])
        start.append(c - 1)
        new.append(1)
    plan, layout = plan_step_host(bs, num_blocks, 12, tables, start, new, None, 0, 148, MIN_SPLIT_CHUNKS)
    p = unpack(plan, layout)
    tiles = [it for it in p["items"] if it["tile"]]
    cut = [it for it in tiles if it["flags"] == 2]
    assert cut and all(it["cend"] - it["cbeg"] >= 2 for it in cut)
    assert max(it["cend"] - it["cbeg"] for it in tiles) < 8  # the 8-chunk tile is cut
    assert len(p["merges"]) == layout[_lib.PLAN_NUM_TILE_MERGES] > 0
    seen = simulate_copies(p, bs, num_blocks)
    for r in range(p["N"]):
        for h in range(12):
            assert sorted(seen[(r, h)]) == list(range(int(p["pos"][r]) + 1)), (r, h)
    check_merges(p)
    # The same step planned for fixed capacities keeps its tiles whole.
    caps = np.array([64, 1024, 64, 20000, 4096, 20000], np.int32)
    plan, layout = plan_step_host(bs, num_blocks, 12, tables, start, new, None, 0, 148, MIN_SPLIT_CHUNKS, caps=caps)
    p = unpack(plan, layout)
    assert layout[_lib.PLAN_NUM_TILE_MERGES] == 0 and not [it for it in p["items"] if it["tile"] and it["flags"]]
    check_merges(p)
