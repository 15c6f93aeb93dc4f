"""Device-resident step tables (`kcmm_step_tables_*`) on the GPU.

The oracle is the reference's per-step host build (src/model/llama_transformer.rs:
288-303: row b = the first max_blocks_per_seq entries of seq_indices[b]'s table, zeros
after; seq_lens[b] = get_seq_len; offsets = get_all_block_offsets_f16), taken here from
the pool's own host queries, whose block arithmetic is pinned against the pool oracle
in test_pool_host.py.  After every sync the device arrays must equal that build bit for
bit, through random pool histories: appends that grow tables, new and dropped
sequences, forks with copy-on-write, frees, and swap out/in that move blocks."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _pool(tiering: bool = False, max_batch: int = 64, max_seq: int = 1024):
    from lattice_b200 import kcmm
    from lattice_b200.workloads import library

    cfg = kcmm.make_config(num_layers=2, kv_heads=2, head_dim=64, max_batch=max_batch,
                           max_seq_len=max_seq, block_size=16, tiering=tiering,
                           max_blocks=4096 if tiering else 0)
    return library().create_pool(cfg)


def _download(tables, batch):
    """The device arrays as numpy: rows [0, batch), lengths, and the offsets array."""
    from lattice_b200.workloads import read_device

    _torch().cuda.synchronize()
    pool = tables.pool
    mbps = pool.lib.kcmm_get_max_blocks_per_seq(pool.handle)
    total = pool.total_blocks()
    bt = read_device(tables.block_tables_ptr, tables.max_batch * mbps * 4).view(np.int32)
    sl = read_device(tables.seq_lens_ptr, tables.max_batch * 4).view(np.int32)
    off = (read_device(tables.block_offsets_ptr, total * 8).view(np.uint64) if total
           else np.zeros(0, np.uint64))
    return bt.reshape(tables.max_batch, mbps)[:batch], sl[:batch], off


def _reference_build(pool, seqs):
    """The reference's host build of the step tables for the ordered batch `seqs`."""
    mbps = pool.lib.kcmm_get_max_blocks_per_seq(pool.handle)
    bt = np.zeros((len(seqs), mbps), np.int32)
    sl = np.zeros(len(seqs), np.int32)
    for b, s in enumerate(seqs):
        t = pool.block_table(s)[:mbps]
        bt[b, :len(t)] = t
        sl[b] = pool.seq_len(s)
    off = np.array(pool.all_block_offsets_f16(), np.uint64)
    return bt, sl, off


def _check(tables, seqs):
    bt, sl, off = _download(tables, len(seqs))
    rbt, rsl, roff = _reference_build(tables.pool, seqs)
    np.testing.assert_array_equal(bt, rbt)
    np.testing.assert_array_equal(sl, rsl)
    np.testing.assert_array_equal(off, roff)


def _grow(pool, s, new_len, bs=16):
    """Advance sequence s to new_len tokens, appending blocks as a scheduler does."""
    need = -(-new_len // bs)
    have = len(pool.block_table(s))
    for _ in range(need - have):
        pool.append_block_to_sequence(s, pool.alloc_blocks(1)[0])
    pool.update_seq_len(s, new_len)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_random_histories_match_the_host_build(seed):
    from lattice_b200.kcmm import StepTables

    _torch()
    rng = np.random.default_rng(seed)
    pool = _pool(tiering=True)
    tables = None
    try:
        live = []
        for _ in range(12):
            L = int(rng.integers(1, 300))
            s = pool.register_sequence(pool.alloc_blocks(-(-L // 16)))
            pool.update_seq_len(s, L)
            live.append(s)
        tables = StepTables(pool, 16)
        for step in range(40):
            op = rng.integers(0, 8)
            if op <= 2:  # decode steps: every live sequence grows by a few tokens
                for s in live:
                    _grow(pool, s, pool.seq_len(s) + int(rng.integers(1, 20)))
            elif op == 3 and len(live) < 20:  # a new request
                L = int(rng.integers(1, 200))
                s = pool.register_sequence(pool.alloc_blocks(-(-L // 16)))
                pool.update_seq_len(s, L)
                live.append(s)
            elif op == 4 and len(live) > 4:  # a finished request
                s = live.pop(int(rng.integers(0, len(live))))
                pool.unregister_sequence(s)
            elif op == 5:  # beam fork, then copy-on-write of the shared tail block
                src = live[int(rng.integers(0, len(live)))]
                f = pool.fork_sequence(src)
                pool.update_seq_len(f, pool.seq_len(src))
                n = len(pool.block_table(f))
                if n:
                    pool.cow_blocks([f], [n - 1])
                live.append(f)
            elif op == 6:  # swap some blocks out and back in (new physical offsets)
                s = live[int(rng.integers(0, len(live)))]
                t = pool.block_table(s)
                pick = [b for b in t[: min(3, len(t))] if pool.refcount(b) == 1]
                if pick:
                    pool.swap_out(pick)
                    pool.swap_in(pick)
            else:  # stray allocations freed again: recycled block ids
                extra = pool.alloc_blocks(int(rng.integers(1, 4)))
                pool.free_blocks(extra)
            k = int(rng.integers(1, min(16, len(live)) + 1))
            order = [live[i] for i in rng.permutation(len(live))[:k]]
            tables.sync(order)
            _check(tables, order)
        st = tables.stats()
        assert st["syncs"] == 40
    finally:
        if tables:
            tables.destroy()
        pool.destroy()


def test_unchanged_batch_uploads_nothing_and_growth_uploads_the_tail():
    from lattice_b200.kcmm import StepTables

    _torch()
    pool = _pool()
    tables = None
    try:
        seqs = []
        for L in (40, 100, 17, 250):
            s = pool.register_sequence(pool.alloc_blocks(-(-L // 16)))
            pool.update_seq_len(s, L)
            seqs.append(s)
        tables = StepTables(pool, 8)
        tables.sync(seqs)
        _check(tables, seqs)
        before = tables.stats()
        tables.sync(seqs)  # nothing changed
        after = tables.stats()
        assert after["bytes"] == before["bytes"] and after["syncs"] == before["syncs"] + 1
        # one token each: lengths only (4 entries)
        for s in seqs:
            pool.update_seq_len(s, pool.seq_len(s) + 1)
        tables.sync(seqs)
        st = tables.stats()
        assert st["table_entries"] - after["table_entries"] == 4
        assert st["offset_entries"] == after["offset_entries"]
        _check(tables, seqs)
        # sequence 0 crosses into a new block: its new table entry, its length, and
        # the new block's offset
        _grow(pool, seqs[0], 49)
        tables.sync(seqs)
        st2 = tables.stats()
        assert st2["table_entries"] - st["table_entries"] == 2
        assert st2["offset_entries"] - st["offset_entries"] == 1
        _check(tables, seqs)
        # a new order: rows move, stale entries past a shorter table become zero
        order = [seqs[3], seqs[2], seqs[0]]
        tables.sync(order)
        _check(tables, order)
    finally:
        if tables:
            tables.destroy()
        pool.destroy()


def test_decode_through_step_tables_equals_decode_through_host_tables():
    """The decode reads the device-resident tables exactly like uploaded host tables."""
    from lattice_b200.kcmm import StepTables
    from lattice_b200.workloads import DecodeWorkload

    torch = _torch()
    wl = DecodeWorkload(batch=12, num_q_heads=8, kv_heads=2, head_dim=128, pool_blocks=1200,
                        min_len=20, max_len=1500, seed=4).build()
    tables = None
    try:
        wl.decode()
        torch.cuda.synchronize()
        ref = wl.out.clone()
        tables = StepTables(wl.pool, wl.batch)
        tables.sync(wl.seq_indices)
        out = torch.zeros_like(wl.q)
        wl.pool.paged_attn_decode(
            0, query_ptr=wl.q.data_ptr(), out_ptr=out.data_ptr(),
            block_tables_ptr=tables.block_tables_ptr, seq_lens_ptr=tables.seq_lens_ptr,
            block_offsets_f16_ptr=tables.block_offsets_ptr, batch=wl.batch,
            num_q_heads=wl.num_q_heads, kv_heads=wl.kv_heads, head_dim=wl.head_dim,
            block_size=wl.block_size, max_blocks_per_seq=wl.max_blocks_per_seq,
            scale=wl.scale, dtype=wl.dtype,
            stream_ptr=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    finally:
        if tables:
            tables.destroy()
        wl.close()
