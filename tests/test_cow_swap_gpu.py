"""Copy-on-write forks and the host swap tier on the GPU: page contents must be
bit-exact (north star), checked against the oracle's block-copy semantics."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def build(tiering=False, layers=2, blocks=64, tmp=None):
    from lattice_b200.workloads import DecodeWorkload

    _torch()
    return DecodeWorkload(batch=4, num_q_heads=8, kv_heads=2, head_dim=128, pool_blocks=blocks,
                          min_len=40, max_len=200, num_layers=layers, tiering=tiering,
                          seed=11).build()


def regions(wl):
    return {(l, k): wl.host_region(l, k).copy() for l in range(wl.num_layers) for k in "kv"}


def test_cow_fork_copies_all_layers():
    torch = _torch()
    wl = build()
    try:
        pool = wl.pool
        s = wl.seq_indices[0]
        table = pool.block_table(s)
        f = pool.fork_sequence(s)
        assert all(pool.refcount(b) == 2 for b in table)
        before = regions(wl)
        last = len(table) - 1
        # both entries are shared (refcount 2): each gets its own fresh copy
        new = pool.cow_blocks([f, s], [last, 0],
                              stream_ptr=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert new[0] not in table and new[1] not in table and new[0] != new[1]
        assert pool.block_table(f)[last] == new[0] and pool.block_table(s)[0] == new[1]
        assert pool.block_table(s)[last] == table[last] and pool.block_table(f)[0] == table[0]
        for b in (table[last], table[0], new[0], new[1]):
            assert pool.refcount(b) == 1
        # a block that is no longer shared is left in place
        assert pool.cow_blocks([f], [last]) == [new[0]]
        bb = pool.stats()["block_bytes"] // 2
        pairs = [(pool.block_va_offset(table[last]) // 2, pool.block_va_offset(new[0]) // 2),
                 (pool.block_va_offset(table[0]) // 2, pool.block_va_offset(new[1]) // 2)]
        after = {(l, k): wl.host_region(l, k) for l in range(wl.num_layers) for k in "kv"}
        for key in before:
            mask = np.ones(len(before[key]), bool)
            for src, dst in pairs:
                assert np.array_equal(after[key][dst:dst + bb], before[key][src:src + bb]), key
                mask[dst:dst + bb] = False
            # every other byte is unchanged
            assert np.array_equal(after[key][mask], before[key][mask])
    finally:
        wl.close()


def test_swap_out_in_roundtrip_bit_exact(tmp_path):
    """ref tests/kcmm_bench_tiering.rs:454-472: data survives evict + restore exactly,
    the block id is kept and its physical slot may move."""
    torch = _torch()
    wl = build(tiering=True)
    try:
        pool = wl.pool
        victims = [int(b) for b in wl.tables[0, :3]]
        before = regions(wl)
        offs_before = {b: pool.block_va_offset(b) for b in victims}
        pool.swap_out(victims)
        assert all(pool.block_location(b) == "cpu" for b in victims)
        # refill the freed slots with other data so a stale restore would be visible
        fresh = pool.alloc_blocks(3)
        assert sorted(pool.block_va_offset(b) for b in fresh) == sorted(offs_before.values())
        from lattice_b200.workloads import memcpy
        junk = torch.full((pool.stats()["block_bytes"] // 2,), 3.0, device="cuda").bfloat16()
        for b in fresh:
            for l in range(wl.num_layers):
                memcpy(pool.va_k(l) + pool.block_va_offset(b), junk.data_ptr(), junk.numel() * 2, "d2d")
        pool.swap_in(victims)
        bb = pool.stats()["block_bytes"] // 2
        after = regions(wl)
        for b in victims:
            assert pool.block_location(b) == "gpu"
            src, dst = offs_before[b] // 2, pool.block_va_offset(b) // 2
            for key in before:
                assert np.array_equal(after[key][dst:dst + bb], before[key][src:src + bb])
        m = pool.metrics()
        assert m["eviction_count"] >= 1 and m["restoration_count"] >= 1
    finally:
        wl.close()


def test_evict_and_restore_reference_api():
    wl = build(tiering=True, blocks=32)
    try:
        pool = wl.pool
        assert pool.eviction_policy() == "lru"
        n = pool.evict_blocks(4)
        assert n == 4
        cpu = [b for b in range(pool.total_blocks()) if pool.is_gpu_resident(b) == 0
               and pool.all_block_valid_flags()[b]]
        assert len(cpu) == 4
        va = pool.restore_evicted_block(cpu[0])
        assert va == pool.block_va_offset(cpu[0]) and pool.is_gpu_resident(cpu[0])
        pool.restore_evicted_blocks(cpu)
        assert all(pool.is_gpu_resident(b) for b in cpu)
        pool.set_eviction_policy("FIFO")
        assert pool.eviction_policy() == "fifo"
    finally:
        wl.close()


def _many_chunks_roundtrip() -> dict:
    """Swap batches that span several halves of the staging buffer, with host slots
    fragmented between batches.  Every block's bytes in every region must come back
    exactly, wherever the block lands.  Returns a summary for the caller to check."""
    import torch

    from lattice_b200.workloads import DecodeWorkload

    # kv_heads 8 x head_dim 128 -> 32 KiB blocks; 2 layers -> 128 KiB host slots, so
    # 256 blocks fill one 32 MiB staging half and 1000 blocks take four chunks
    wl = DecodeWorkload(batch=4, num_q_heads=32, kv_heads=8, head_dim=128, pool_blocks=1200,
                        min_len=40, max_len=200, num_layers=2, tiering=True, seed=12).build()
    try:
        pool = wl.pool
        rng = np.random.default_rng(12)
        ids = [int(b) for b in wl.block_ids]
        bb = pool.stats()["block_bytes"] // 2
        before = regions(wl)
        offs = {b: pool.block_va_offset(b) // 2 for b in ids}
        first = [int(b) for b in rng.choice(ids, 1000, replace=False)]
        pool.swap_out(first)
        back = first[::2]  # frees every other host slot: the next batch's runs are short
        pool.swap_in(back)
        rest = [b for b in ids if b not in set(first)]
        second = [int(b) for b in rng.choice(rest + back, 400, replace=False)]
        pool.swap_out(second)
        cpu = [b for b in ids if pool.block_location(b) == "cpu"]
        pool.swap_in(cpu)
        torch.cuda.synchronize()
        after = regions(wl)
        bad = 0
        for b in ids:
            dst = pool.block_va_offset(b) // 2
            for key in before:
                if not np.array_equal(after[key][dst:dst + bb], before[key][offs[b]:offs[b] + bb]):
                    bad += 1
        return {"bad": bad, "on_cpu": sum(pool.block_location(b) == "cpu" for b in ids),
                "status": pool.kernel_status(), "moved": len(first) + len(second)}
    finally:
        wl.close()


def test_swap_many_chunks_fragmented_slots_bit_exact():
    """The default path (copy engines through the staging buffer)."""
    _torch()
    res = _many_chunks_roundtrip()
    assert res == {"bad": 0, "on_cpu": 0, "status": 0, "moved": 1400}, res


def test_swap_sm_store_path_bit_exact():
    """KCMM_SWAP_IMPL=sm (the swap kernel stores into the mapped host tier); the switch
    is read once per process, so the same round trip runs in a child process."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path

    _torch()
    root = Path(__file__).resolve().parents[1]
    code = ("import json, sys; sys.path.insert(0, %r); sys.path.insert(0, %r); "
            "import test_cow_swap_gpu as t; print(json.dumps(t._many_chunks_roundtrip()))"
            % (str(root), str(root / "tests")))
    env = dict(os.environ, KCMM_SWAP_IMPL="sm")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         env=env, timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert res == {"bad": 0, "on_cpu": 0, "status": 0, "moved": 1400}, res
