"""Paged decode attention on the GPU through the C ABI, against the CPU oracle.

Tolerance (north star): bf16/f16 outputs within max-abs 2e-3 / max-rel 1e-2 of the
oracle computed in fp64/fp32, i.e. |out - ref| <= 2e-3 + 1e-2 * |ref| elementwise."""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def oracle_out(wl):
    from oracle import native as N

    q = __import__("lattice_b200.workloads", fromlist=["x"]).tensor_bits(wl.q)
    return N.paged_attn(wl.dtype, q, wl.host_region(0, "k"), wl.host_region(0, "v"), wl.tables,
                        wl.seq_lens, wl.offsets, hq=wl.num_q_heads, hkv=wl.kv_heads,
                        d=wl.head_dim, bs=wl.block_size, max_bps=wl.max_blocks_per_seq,
                        scale=wl.scale)


def check(wl, got=None):
    torch = _torch()
    ref = oracle_out(wl)
    got = (wl.out if got is None else got).float().cpu().numpy()
    live = wl.seq_lens > 0
    err = np.abs(got[live] - ref[live])
    bound = ATOL + RTOL * np.abs(ref[live])
    assert (err <= bound).all(), f"max err {err.max()} (worst excess {(err - bound).max()})"
    return ref


def make(**kw):
    from lattice_b200.workloads import DecodeWorkload

    _torch()
    kw.setdefault("pool_blocks", 512)
    kw.setdefault("min_len", 1)
    kw.setdefault("max_len", 700)
    return DecodeWorkload(**kw).build()


SHAPES = [
    # batch, hq, hkv, D, bs
    (4, 4, 4, 64, 16),      # config-1 shape (MHA, D 64)
    (6, 32, 8, 128, 16),    # Llama-3-8B heads (GQA 4)
    (3, 8, 1, 128, 16),     # per-GPU head shard of the 70B config (GQA 8)
    (2, 64, 2, 128, 16),    # GQA 32: two head tiles per kv head
    (3, 12, 4, 80, 32),
    (3, 8, 2, 96, 16),
    (2, 8, 2, 256, 16),
    (2, 6, 3, 72, 16),      # head_dim not a multiple of 16: generic kernel
    (2, 8, 2, 64, 8),       # block_size 8: units span two pages
    (6, 32, 8, 128, 8),     # Llama-3-8B heads on 8-token pages
    (3, 8, 1, 256, 8),
    (2, 8, 2, 64, 4),       # block_size 4: generic kernel
    (3, 10, 4, 64, 16),     # query heads not a multiple of kv heads
]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("shape", SHAPES)
def test_decode_matches_oracle(shape, dtype):
    B, hq, hkv, D, bs = shape
    lens = [1, 15, 16, 17, 255, 700, 333][:B]
    wl = make(batch=B, num_q_heads=hq, kv_heads=hkv, head_dim=D, block_size=bs, dtype=dtype,
              seq_lens_override=lens, seed=hash(shape) % 1000)
    try:
        wl.decode()
        _torch().cuda.synchronize()
        check(wl)
    finally:
        wl.close()


def test_zero_length_rows_untouched():
    torch = _torch()
    wl = make(batch=4, num_q_heads=8, kv_heads=2, head_dim=128, seq_lens_override=[0, 40, -3, 70])
    try:
        wl.out.fill_(7.0)
        wl.decode()
        torch.cuda.synchronize()
        o = wl.out.float().cpu().numpy()
        assert (o[0] == 7.0).all() and (o[2] == 7.0).all()
        check(wl)
    finally:
        wl.close()


@pytest.mark.parametrize("env", [
    {"KCMM_PDL": "0"},                    # split-K, plain stream-ordered launches
    {"KCMM_DECODE_SPLITS": "1"},          # split-K kernel (the default), forced splits
    {"KCMM_DECODE_SPLITS": "3"},
    {"KCMM_DECODE_SPLITS": "7"},
])
def test_work_split_does_not_change_result(env, monkeypatch):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    wl = make(batch=5, num_q_heads=32, kv_heads=8, head_dim=128, min_len=200, max_len=2000,
              pool_blocks=1024, seed=len(env))
    try:
        wl.decode()
        _torch().cuda.synchronize()
        check(wl)
    finally:
        wl.close()


@pytest.mark.parametrize("seed", [0, 2, 9])
def test_short_rows_within_tolerance(seed):
    """64 rows of 1..47 keys: few keys dominate each row, so a P rounded once to 16 bits
    would miss the tolerance; the kernel carries P as a hi + lo pair."""
    lens = list(np.random.default_rng(seed).integers(1, 48, 64))
    wl = make(batch=64, num_q_heads=32, kv_heads=8, head_dim=128, seq_lens_override=lens,
              max_len=64, pool_blocks=512, seed=seed)
    try:
        wl.decode()
        _torch().cuda.synchronize()
        check(wl)
    finally:
        wl.close()


def test_v_row_kat():
    """ref scripts/kcmm/non_default_stream_ffi_smoke.py:172-179: q = 0, seq_len 1,
    k = arange+100, v = arange+1000 -> out equals the V row of the mapped kv head."""
    torch = _torch()
    from lattice_b200.workloads import memcpy

    wl = make(batch=2, num_q_heads=4, kv_heads=2, head_dim=64, dtype="f16",
              seq_lens_override=[1, 1], pool_blocks=8)
    try:
        n = wl.region_used // 2
        k = (torch.arange(n, device="cuda") % 512 + 100).half()
        v = (torch.arange(n, device="cuda") % 512 + 1000).half()
        memcpy(wl.pool.va_k(0), k.data_ptr(), wl.region_used, "d2d")
        memcpy(wl.pool.va_v(0), v.data_ptr(), wl.region_used, "d2d")
        wl.q.zero_()
        for variant in ("sync", "stream", "current"):
            wl.out.zero_()
            kw = dict(query_ptr=wl.q.data_ptr(), out_ptr=wl.out.data_ptr(),
                      block_tables_ptr=wl.d_tables.data_ptr(),
                      seq_lens_ptr=wl.d_seq_lens.data_ptr(),
                      block_offsets_f16_ptr=wl.d_offsets.data_ptr(), batch=2, num_q_heads=4,
                      kv_heads=2, head_dim=64, block_size=16,
                      max_blocks_per_seq=wl.max_blocks_per_seq, scale=1.0, dtype="f16")
            if variant == "sync":
                wl.pool.paged_attn_decode(0, stream_ptr=None, **kw)
            else:
                wl.pool.paged_attn_decode(0, stream_ptr=torch.cuda.current_stream().cuda_stream,
                                          current_context=variant == "current", **kw)
            torch.cuda.synchronize()
            vv = v.cpu().numpy()
            for b in range(2):
                for h in range(4):
                    e = int(wl.offsets[wl.tables[b, 0]]) + (h * 2 // 4) * 64
                    np.testing.assert_array_equal(wl.out[b, h].cpu().numpy(), vv[e:e + 64])
    finally:
        wl.close()


@pytest.mark.parametrize("splits", ["1", "2", "11"])
def test_gqa_head_tiles_with_empty_rows(splits, monkeypatch):
    """Two head tiles per kv head (GQA 32), zero-length rows and forced split counts
    together: empty rows stay untouched, the rest match the oracle."""
    monkeypatch.setenv("KCMM_DECODE_SPLITS", splits)
    wl = make(batch=6, num_q_heads=64, kv_heads=2, head_dim=128,
              seq_lens_override=[0, 33, 700, 1, 0, 257], seed=int(splits))
    try:
        wl.out.fill_(5.0)
        wl.decode()
        _torch().cuda.synchronize()
        o = wl.out.float().cpu().numpy()
        assert (o[0] == 5.0).all() and (o[4] == 5.0).all()
        check(wl)
    finally:
        wl.close()


def test_llama3_8b_config_full_size():
    """BASELINE config 2 at full size: 64 sequences, 512..4096 tokens, 40k-block pool."""
    wl = make(batch=64, num_q_heads=32, kv_heads=8, head_dim=128, min_len=512, max_len=4096,
              pool_blocks=40000, seed=0)
    try:
        wl.decode()
        _torch().cuda.synchronize()
        ref = check(wl)
        # size-independent property: each output is a convex combination of V rows,
        # so it lies inside the per-dim [min, max] of V (checked loosely via the oracle)
        assert np.isfinite(ref).all()
    finally:
        wl.close()


def test_device_diagnostics_clean():
    """A clean run leaves the pool's device diagnostic word at 0 (no bounded wait gave up,
    no bad offset); read through the pool's synchronize path."""
    wl = make(batch=3, num_q_heads=8, kv_heads=2, head_dim=128)
    try:
        wl.decode()
        wl.pool.synchronize()
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


def test_calls_on_two_streams_and_in_a_graph(monkeypatch):
    """Split-K decode (partials in stream-ordered scratch, then the merge launch) run on
    the current stream, on a side stream, and captured in a CUDA graph and replayed,
    interleaved; every result against the oracle."""
    torch = _torch()
    monkeypatch.setenv("KCMM_DECODE_SPLITS", "4")
    wl = make(batch=6, num_q_heads=32, kv_heads=8, head_dim=128, min_len=300, max_len=2000,
              pool_blocks=2048, seed=21)
    graph = None
    try:
        wl.decode()  # loads the modules outside the capture
        torch.cuda.synchronize()
        check(wl)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            wl.decode(stream_ptr=side.cuda_stream)
        for _ in range(2):
            wl.out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            check(wl)
            wl.out.zero_()
            torch.cuda.synchronize()
            with torch.cuda.stream(side):
                wl.decode(stream_ptr=side.cuda_stream)
            torch.cuda.synchronize()
            check(wl)
    finally:
        del graph
        wl.close()


SPLIT_CASES = [
    # batch, hq, hkv, D, lengths (None: random in [min_len, max_len])
    (64, 32, 8, 128, None),                       # the bench shape
    (40, 32, 8, 128, [1, 0, 17, 5, 0, 3] * 6 + [4096, 2048, 1, 0]),  # short and empty rows
    (1, 32, 8, 128, [37]),
    (3, 64, 2, 128, [0, 4000, 33]),               # GQA 32: two head tiles per kv head
    (6, 8, 8, 64, None),                          # MHA, D 64
    (4, 16, 2, 256, None),                        # D 256
    (5, 12, 4, 80, None),
]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("case", SPLIT_CASES)
def test_default_split_matches_oracle_and_forced_splits(case, dtype, monkeypatch):
    """Default plan (split heuristic, merge launched as a programmatic dependent, split
    scratch kept per stream) against the oracle and against two forced splits."""
    torch = _torch()
    B, hq, hkv, D, lens = case
    wl = make(batch=B, num_q_heads=hq, kv_heads=hkv, head_dim=D, dtype=dtype, min_len=1,
              max_len=4096, pool_blocks=max(512, B * 300), seq_lens_override=lens,
              seed=B + hq + D)
    try:
        wl.out.fill_(3.0)
        for _ in range(2):  # the second call reuses the stream's scratch
            wl.decode()
        torch.cuda.synchronize()
        first = wl.out.clone()
        o = first.float().cpu().numpy()
        dead = wl.seq_lens <= 0
        assert (o[dead] == 3.0).all()  # zero-length rows untouched
        check(wl, first)
        monkeypatch.setenv("KCMM_DECODE_SPLITS", "2")
        wl.decode()
        torch.cuda.synchronize()
        check(wl)
        live = ~dead
        a, b = first.float()[live], wl.out.float()[live]
        assert torch.all((a - b).abs() <= 4e-3 + 1e-2 * b.abs())
    finally:
        wl.close()


def test_many_sequences():
    """2,100 short sequences in one call."""
    wl = make(batch=2100, num_q_heads=8, kv_heads=2, head_dim=64, min_len=1, max_len=40,
              pool_blocks=2100 * 3 + 64, seed=77)
    try:
        wl.decode()
        _torch().cuda.synchronize()
        check(wl)
    finally:
        wl.close()


def test_back_to_back_calls_of_growing_size_on_one_stream():
    """Calls with growing split scratch on one stream, launched back to back without a
    host synchronisation: each call's kernels wait for the previous call's merge before
    reusing (or replacing) the stream's scratch."""
    torch = _torch()
    wls = [make(batch=B, num_q_heads=32, kv_heads=8, head_dim=128, min_len=500, max_len=4096,
                pool_blocks=B * 300, seed=90 + B) for B in (4, 16, 48)]
    try:
        outs = []
        for _ in range(3):
            for wl in wls:
                wl.decode()
                outs.append((wl, wl.out.clone()))
        torch.cuda.synchronize()
        for wl, out in outs:
            check(wl, out)
    finally:
        for wl in wls:
            wl.close()
