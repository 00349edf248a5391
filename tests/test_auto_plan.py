"""The host plan of the device-side schedule (pkv_build_auto_plan) against a
Python restatement of the schedule the decode kernel derives from seq_lens:
tiles of 32 tokens concatenated in row order, NG equal groups, each group's
first row piece, its slots and the pages of its first boxes."""

import numpy as np
import pytest

from persistentkv_attention_b200 import _native
from persistentkv_attention_b200.scheduler import auto_groups, build_auto_plan, plan_words

HEADER, ENTRY, PAGES = 16, 20, 8


def schedule(lens, table, page, hkv, sms, q_idx=None, o_idx=None, groups=0):
    """The kernel's schedule (auto_init / auto_item) restated: per group the
    entry the plan must hold (``groups`` 0: the maximum group count)."""
    ng = groups or max(1, (2 * sms) // hkv)
    b = len(lens)
    tiles = [(n + 31) // 32 for n in lens]
    prefix = np.concatenate([[0], np.cumsum(tiles)]).astype(np.int64)
    T = int(prefix[-1])

    def group_of(x):
        return ((x + 1) * ng - 1) // T

    gf, gl = [], []
    for r in range(b):
        if T == 0:
            gf.append(0), gl.append(0)
            continue
        P, n = int(prefix[r]), tiles[r]
        first = P if n > 0 else (P if P < T else T - 1)
        last = P + n - 1 if n > 0 else first
        gf.append(group_of(first)), gl.append(group_of(last))
    slots = np.concatenate([[0], np.cumsum([gl[r] - gf[r] + 1 for r in range(b)])])
    box = 16 if page % 16 == 0 else 8
    entries = []
    for g in range(ng):
        rows = [r for r in range(b) if gl[r] >= g]
        if not rows:
            entries.append([-1] * ENTRY)
            continue
        r = rows[0]
        hi = [x for x in range(b) if gf[x] <= g]
        end = hi[-1] + 1 if hi and hi[-1] >= r else r
        e = [r, end, int(prefix[r]), int(slots[r]), lens[r], gf[r], gl[r],
             r if q_idx is None else int(q_idx[r]), r if o_idx is None else int(o_idx[r])]
        pages = [-1] * PAGES
        if tiles[r] > 0:
            s0, s1 = g * T // ng, (g + 1) * T // ng
            P = int(prefix[r])
            tb = max(s0, P) - P
            te = min(P + tiles[r], s1) - P
            t0, t1 = tb * 32, min(te * 32, lens[r])
            for i in range(PAGES):
                tok = t0 + i * box
                if tok >= t1:
                    break
                pages[i] = int(table[r, tok // page])
        entries.append(e + pages + [-1] * (ENTRY - 9 - PAGES))
    return ng, T, entries


CASES = [
    ([4096], 16, 8), ([0, 0, 0], 16, 8), ([1, 7, 33, 1000, 0, 5000], 16, 8),
    ([9000, 33, 4096, 1, 700, 12000, 0, 2500], 32, 4), ([100] * 40, 8, 32),
    ([30000], 16, 8), ([513, 2048, 77, 31, 32, 65], 16, 16),
]


@pytest.mark.parametrize("lens,page,hkv", CASES)
def test_plan_matches_the_device_schedule(lens, page, hkv):
    sms = 148
    rng = np.random.default_rng(len(lens) + page)
    width = max(1, max((n + page - 1) // page for n in lens))
    table = rng.integers(0, 5000, size=(len(lens), width)).astype(np.int32)
    q_idx = rng.permutation(len(lens) + 3)[: len(lens)].astype(np.int32)
    o_idx = rng.permutation(len(lens) + 3)[: len(lens)].astype(np.int32)
    ng, T, entries = schedule(lens, table, page, hkv, sms, q_idx, o_idx)
    assert auto_groups(hkv, sms) == ng
    plan = build_auto_plan(lens, table, width, page, hkv, sms, q_indices=q_idx,
                           out_indices=o_idx)
    assert plan.size == plan_words(hkv, sms) == HEADER + ng * ENTRY
    assert list(plan[:4]) == [0x504B5650, ng, len(lens), T]
    got = plan[HEADER:].reshape(ng, ENTRY)
    assert np.array_equal(got, np.asarray(entries, np.int32))


def test_plan_rejects_lengths_beyond_the_table():
    lib = _native.load()
    with pytest.raises(_native.PkvError):
        build_auto_plan([100, 5000], np.zeros((2, 4), np.int32), 4, 16, 8, 148)
    assert lib.pkv_auto_plan_bytes(0, 148) == 0


@pytest.mark.parametrize("groups", [1, 5, 18, 36])
def test_plan_for_fewer_groups(groups):
    """A router's smaller group count: the header records it and every entry
    follows the schedule cut into that many groups."""
    lens = [9000, 33, 4096, 1, 700, 12000, 0, 2500]
    rng = np.random.default_rng(groups)
    width = max((n + 15) // 16 for n in lens)
    table = rng.integers(0, 5000, size=(len(lens), width)).astype(np.int32)
    ng, T, entries = schedule(lens, table, 16, 8, 148, groups=groups)
    plan = build_auto_plan(lens, table, width, 16, 8, 148, groups=groups)
    assert list(plan[:4]) == [0x504B5650, groups, len(lens), T]
    got = plan[HEADER:HEADER + groups * ENTRY].reshape(groups, ENTRY)
    assert np.array_equal(got, np.asarray(entries, np.int32))
    with pytest.raises(_native.PkvError):
        build_auto_plan(lens, table, width, 16, 8, 148, groups=auto_groups(8, 148) + 1)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_plan_of_a_large_ragged_batch(seed):
    """Hundreds of rows, many of them empty or shorter than a tile, against the
    restated schedule (the builder walks rows and groups in one pass)."""
    rng = np.random.default_rng(seed)
    lens = rng.choice([0, 1, 17, 31, 33, 200, 1500, 7000], size=300).tolist()
    width = max(1, max((n + 15) // 16 for n in lens))
    table = rng.integers(0, 50000, size=(len(lens), width)).astype(np.int32)
    for hkv in (8, 4):
        ng, T, entries = schedule(lens, table, 16, hkv, 148)
        plan = build_auto_plan(lens, table, width, 16, hkv, 148)
        got = plan[HEADER:HEADER + ng * ENTRY].reshape(ng, ENTRY)
        assert np.array_equal(got, np.asarray(entries, np.int32))
