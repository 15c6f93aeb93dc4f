"""Policy-driven eviction and the background eviction thread on the GPU, through the
swap kernels: victims equal the policy's preview, only inactive sequences lose blocks
to the background thread, and page contents survive the round trip bit for bit."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _pool(watermark=0.2, interval_ms=100, layers=2):
    from lattice_b200 import kcmm
    from lattice_b200.workloads import library

    cfg = kcmm.make_config(num_layers=layers, kv_heads=2, head_dim=64, max_batch=16,
                           max_seq_len=1024, tiering=True, max_blocks=256)
    cfg.low_watermark_threshold = watermark
    cfg.background_evict_interval_ms = interval_ms
    return library().create_pool(cfg)


def _fill(pool, layers, seed):
    """Random bytes in every layer's K and V region over the used blocks."""
    from lattice_b200.workloads import write_device

    rng = np.random.default_rng(seed)
    used = (max(pool.block_va_offset(b) for b in range(pool.total_blocks())
                if pool.all_block_valid_flags()[b]) + pool.stats()["block_bytes"])
    data = {}
    for l in range(layers):
        for kind, base in (("k", pool.va_k(l)), ("v", pool.va_v(l))):
            d = rng.integers(0, 256, used, dtype=np.uint8)
            write_device(base, d)
            data[(l, kind)] = d
    return data


def _block_bytes(pool, layers, blk, off):
    from lattice_b200.workloads import read_device

    bb = pool.stats()["block_bytes"]
    return {(l, kind): read_device(base + off, bb)
            for l in range(layers)
            for kind, base in (("k", pool.va_k(l)), ("v", pool.va_v(l)))}


@pytest.mark.parametrize("policy", ["lru", "lfu", "fifo", "arc", "sink_window"])
def test_evict_takes_the_policy_victims_and_restores_bit_exact(policy):
    _torch()
    layers = 2
    pool = _pool(layers=layers)
    try:
        pool.set_eviction_policy(policy)
        seqs = []
        for n in (9, 7, 12):
            s = pool.register_sequence(pool.alloc_blocks(n))
            seqs.append(s)
        # some accesses so the orders differ between policies
        for b in pool.block_table(seqs[1])[:4]:
            one = (ctypes.c_uint32 * 1)(b)
            assert pool.lib.kcmm_protect(pool.handle, seqs[1], one, 1, 0) == 0
        data = _fill(pool, layers, seed=5)
        preview = pool.preview_eviction_victims(6)
        assert preview, "the policy offers victims"
        bb = pool.stats()["block_bytes"]
        before = {b: {k: v[pool.block_va_offset(b):pool.block_va_offset(b) + bb].copy()
                      for k, v in data.items()} for b in preview}
        n = pool.evict_blocks(6)
        assert n == len(preview)
        evicted = [b for b in range(pool.total_blocks())
                   if pool.all_block_valid_flags()[b] and pool.block_location(b) == "cpu"]
        assert sorted(evicted) == sorted(preview)
        pool.restore_evicted_blocks(preview)
        # ref src/kcmm/pool.rs:1255-1293: one eviction and one restoration, under the
        # policy that was active
        st = pool.policy_stats(policy)
        assert st["eviction_count"] == 1 and st["evicted_blocks"] == n
        assert st["avg_evict_batch_size"] == pytest.approx(n)
        assert st["restoration_count"] == 1 and st["restored_blocks"] == n
        m = pool.metrics_ext()
        for key in ("eviction_latency", "restoration_latency"):
            h = m[key]
            assert h["count"] == 1 and sum(h["buckets"]) == 1
            assert h["min_us"] == h["max_us"] == h["sum_us"]
        assert m["evicted_blocks_total"] == n and m["restored_blocks_total"] == n
        assert m["background_eviction_count"] == 0
        for b in preview:
            assert pool.block_location(b) == "gpu"
            got = _block_bytes(pool, layers, b, pool.block_va_offset(b))
            for k in got:
                assert np.array_equal(got[k], before[b][k])
    finally:
        pool.destroy()


def test_background_thread_evicts_only_inactive_sequences():
    _torch()
    layers = 1
    # watermark 0.999: the pool's free ratio (one 2 MiB superblock of 4 KiB blocks,
    # a few dozen in use) is always below it, so every round evicts
    pool = _pool(watermark=0.999, interval_ms=5, layers=layers)
    try:
        active = pool.register_sequence(pool.alloc_blocks(10))
        cold = [pool.register_sequence(pool.alloc_blocks(n)) for n in (8, 12)]
        for s in cold:
            pool.cool(s)
        data = _fill(pool, layers, seed=9)
        bb = pool.stats()["block_bytes"]
        cold_blocks = [b for s in cold for b in pool.block_table(s)]
        before = {b: data[(0, "k")][pool.block_va_offset(b):pool.block_va_offset(b) + bb].copy()
                  for b in cold_blocks}
        pool.start_background_eviction()
        pool.start_background_eviction()  # a second start is a no-op
        deadline = time.time() + 10
        while time.time() < deadline:
            if all(pool.block_location(b) == "cpu" for b in cold_blocks):
                break
            time.sleep(0.01)
        pool.stop_background_eviction()
        pool.stop_background_eviction()  # and so is a second stop
        assert all(pool.block_location(b) == "cpu" for b in cold_blocks)
        assert all(pool.block_location(b) == "gpu" for b in pool.block_table(active))
        m = pool.metrics()
        assert m["cpu_blocks"] == len(cold_blocks)
        assert m["eviction_count"] >= 2  # at most 16 blocks per round
        ext = pool.metrics_ext()
        assert ext["background_eviction_count"] == m["eviction_count"]
        assert ext["evicted_blocks_total"] == len(cold_blocks)
        st = pool.policy_stats("lru")
        assert st["avg_evict_batch_size"] == pytest.approx(len(cold_blocks) / st["eviction_count"])
        pool.restore_evicted_blocks(cold_blocks)
        for b in cold_blocks:
            got = _block_bytes(pool, layers, b, pool.block_va_offset(b))[(0, "k")]
            assert np.array_equal(got, before[b])
    finally:
        pool.destroy()


def test_background_thread_idles_above_the_watermark():
    _torch()
    pool = _pool(watermark=0.0, interval_ms=5, layers=1)
    try:
        s = pool.register_sequence(pool.alloc_blocks(6))
        pool.cool(s)
        pool.start_background_eviction()
        time.sleep(0.1)
        pool.stop_background_eviction()
        assert all(pool.block_location(b) == "gpu" for b in pool.block_table(s))
        assert pool.metrics()["cpu_blocks"] == 0
    finally:
        pool.destroy()
