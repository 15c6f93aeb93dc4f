"""Eviction policies: the oracle pinned against the reference's own unit tests, then the
library's victim choice (kcmm_preview_eviction_victims) against the oracle through
random pool histories.  CPU only: pools on the host VMM backend with tiering on (victim
selection needs no device; only the swap itself does)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import policy_oracle as po

# --- the oracle against the reference's unit tests (ref src/kcmm/tiering.rs) ----------


def test_lru_oldest_first_and_untracked_skipped():
    # ref tiering.rs:2170-2224 (test_select_victims_oldest_first, _respects_count,
    # _untracked_blocks_skipped)
    p = po.LruPolicy()
    for h in range(10):
        p.on_allocate(h)
    assert p.select_victims(list(range(10)), 3) == [0, 1, 2]
    assert p.select_victims([], 5) == [] and p.select_victims([0], 0) == []
    q = po.LruPolicy()
    q.on_allocate(0)
    assert q.select_victims([0, 1], 2) == [0]
    q.on_allocate(1)
    q.on_access(0)  # 0 is now the most recent
    assert q.select_victims([0, 1], 2) == [1, 0]
    q.on_evict(1)
    assert q.select_victims([0, 1], 2) == [0]


def test_lfu_least_frequent_first():
    # ref tiering.rs:2283-2335
    p = po.LfuPolicy()
    p.on_access(0)
    for _ in range(3):
        p.on_access(1)
    for _ in range(2):
        p.on_access(2)
    assert p.select_victims([0, 1, 2], 3) == [0, 2, 1]
    q = po.LfuPolicy()
    for i in range(5):
        for _ in range(i + 1):
            q.on_access(i)
    assert q.select_victims(list(range(5)), 2) == [0, 1]
    r = po.LfuPolicy()
    r.on_allocate(0)
    assert r.select_victims([0, 1], 2) == [0]


def test_fifo_ignores_accesses():
    # ref tiering.rs:2372-2420: on_access neither inserts nor reorders
    p = po.FifoPolicy()
    p.on_access(7)
    assert p.select_victims([7], 1) == []
    p.on_allocate(0)
    p.on_allocate(1)
    p.on_access(0)
    assert p.select_victims([0, 1], 2) == [0, 1]


def test_arc_reference_cases():
    # ref tiering.rs:3801-3911
    a = po.ArcPolicy(10)
    a.on_allocate("h")
    assert a.select_victims(["h"], 1) == ["h"]
    a = po.ArcPolicy(10)
    a.on_allocate("h")
    a.on_access("h")
    assert a.select_victims([], 1) == []
    a = po.ArcPolicy(10)
    a.on_allocate("h1")
    a.on_allocate("h2")
    a.on_access("h2")
    a.on_allocate("h3")
    assert a.select_victims(["h1", "h2", "h3"], 1) == ["h1"]
    a = po.ArcPolicy(3)
    a.on_allocate("h1")
    a.on_allocate("h2")
    a.on_access("h2")
    a.on_allocate("h3")
    a.on_evict("h1")
    assert "h1" in a.b1
    a.on_allocate("h1")  # ghost hit in B1: to T2, p grows
    assert "h1" in a.t2 and a.p == 1
    assert len(a.select_victims(["h1"], 1)) == 1
    a = po.ArcPolicy(2)
    a.on_allocate("h1")
    a.on_allocate("h2")
    a.on_allocate("h3")  # over capacity: the LRU of T1 (h1) goes to B1
    v = a.select_victims(["h1", "h2", "h3"], 3)
    assert len(v) == 3 and v[2] == "h1"
    a = po.ArcPolicy(10)
    a.on_allocate("h")
    assert a.select_victims([], 5) == [] and a.select_victims(["h"], 0) == []


def test_sink_window_reference_cases():
    # ref tiering.rs:3913-4027
    s = po.SinkWindowPolicy(2, 2)
    for i in range(6):
        s.register_block(i, 0, i)
    for i in range(6):
        s.on_allocate(i)
    assert s.select_victims(list(range(6)), 6) == [2, 3]
    s = po.SinkWindowPolicy(2, 3)
    for i in range(3):
        s.register_block(i, 0, i)
        s.on_allocate(i)
    assert s.select_victims([0, 1, 2], 3) == []
    s = po.SinkWindowPolicy(1, 1)
    for i in range(4):
        s.register_block(i, 0, i)
        s.on_allocate(i)
    assert s.select_victims([0, 1, 2, 3], 2) == [1, 2]
    s = po.SinkWindowPolicy(1, 4)
    s.register_block(0, 0, 0)
    s.on_allocate(0)
    assert s.select_victims([], 5) == [] and s.select_victims([0], 0) == []


# --- the library against the oracle -----------------------------------------------------


@pytest.mark.parametrize("policy", ["lru", "lfu", "fifo", "arc", "sink_window"])
@pytest.mark.parametrize("seed", [0, 1])
def test_library_picks_the_oracles_victims(policy, seed, kcmm_lib, monkeypatch):
    """Random histories: allocations (some recycled after frees), sequences registered
    and grown, protect / hint accesses.  After every event the library's preview of
    the next victims equals the oracle's choice over the live blocks in id order."""
    from lattice_b200 import kcmm

    monkeypatch.setenv("KCMM_VMM_BACKEND", "host")
    # ARC capacity = 64 blocks x 1 layer x 2 x 4096 B / max_batch_blocks: 128 with 4096,
    # 8 with 65536 (then long histories push entries through B1 / B2)
    cfg = kcmm.make_config(num_layers=1, kv_heads=2, head_dim=64, max_batch=16,
                           max_seq_len=512, tiering=True, max_blocks=64)
    cfg.max_batch_blocks = 4096 if policy != "arc" or seed == 0 else 65536
    pool = kcmm_lib.create_pool(cfg)
    try:
        block_bytes = pool.stats()["block_bytes"]
        arc_cap = 64 * 1 * 2 * block_bytes // cfg.max_batch_blocks
        pool.set_eviction_policy(policy)
        orc = po.make_policy(policy, arc_capacity=arc_cap)
        rng = np.random.default_rng(seed)
        seqs = []
        tables = {}

        def alloc(n):
            ids = pool.alloc_blocks(n)
            for b in ids:
                orc.on_allocate(b)
            return ids

        def compare():
            valid = pool.all_block_valid_flags()
            cand = [i for i, v in enumerate(valid) if v]
            k = int(rng.integers(1, 12))
            assert pool.preview_eviction_victims(k) == orc.select_victims(cand, k)

        for _ in range(120):
            op = int(rng.integers(0, 6))
            if op == 0 or not seqs:
                ids = alloc(int(rng.integers(1, 5)))
                s = pool.register_sequence(ids)
                tables[s] = list(ids)
                for j, b in enumerate(ids):
                    orc.register_block(b, s, j)
                seqs.append(s)
            elif op == 1:
                s = seqs[int(rng.integers(0, len(seqs)))]
                (b,) = alloc(1)
                pool.append_block_to_sequence(s, b)
                tables[s].append(b)
                orc.register_block(b, s, len(tables[s]) - 1)
            elif op == 2:  # protect a few blocks (NEVER_EVICT refreshes them)
                s = seqs[int(rng.integers(0, len(seqs)))]
                pick = [tables[s][int(i)] for i in rng.integers(0, len(tables[s]), 2)]
                arr = (ctypes.c_uint32 * len(pick))(*pick)
                assert pool.lib.kcmm_protect(pool.handle, s, arr, len(pick), 0) == 0
                for b in pick:
                    orc.on_access(b)
            elif op == 3:  # a reuse hint touches every block of the sequence
                s = seqs[int(rng.integers(0, len(seqs)))]
                assert pool.lib.kcmm_hint(pool.handle, s, 1) == 0  # MULTI_TURN
                for b in tables[s]:
                    orc.on_access(b)
            elif op == 4 and len(seqs) > 2:  # a request finishes: its blocks are freed
                s = seqs.pop(int(rng.integers(0, len(seqs))))
                pool.unregister_sequence(s)
                tables.pop(s)
            else:  # stray blocks allocated and freed (their ids are recycled later)
                ids = alloc(int(rng.integers(1, 3)))
                pool.free_blocks(ids)
            compare()
        assert pool.eviction_policy() == policy
    finally:
        pool.destroy()


def test_unknown_policy_names_the_choices(kcmm_lib, monkeypatch):
    from lattice_b200 import kcmm

    monkeypatch.setenv("KCMM_VMM_BACKEND", "host")
    cfg = kcmm.make_config(num_layers=1, kv_heads=2, head_dim=64, max_batch=4,
                           max_seq_len=256, tiering=True, max_blocks=16)
    pool = kcmm_lib.create_pool(cfg)
    try:
        with pytest.raises(kcmm.KcmmError, match="lru, lfu, fifo, arc, or sink_window"):
            pool.set_eviction_policy("mru")
        assert pool.lib.kcmm_start_background_eviction(pool.handle) == -1  # no device
    finally:
        pool.destroy()
