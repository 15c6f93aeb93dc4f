"""Chunked prefill on the tcgen05 tensor cores, through the C ABI, against the CPU oracle.

Tolerance (north star, fp32 reference): |out - ref| <= 2e-3 + 1e-2 * |ref| elementwise."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def make(**kw):
    from lattice_b200.workloads import PrefillWorkload

    _torch()
    return PrefillWorkload(**kw).build()


def oracle(wl, token_mask=None):
    from lattice_b200.workloads import tensor_bits
    from oracle import native as N

    kv = wl.kv
    q = tensor_bits(wl.q).reshape(wl.q.shape[0], -1)
    return N.paged_prefill(wl.dtype, q, kv.host_region(0, "k"), kv.host_region(0, "v"),
                           kv.tables, wl.q_start, wl.ctx_lens, kv.offsets, hq=wl.num_q_heads,
                           hkv=wl.kv_heads, d=wl.head_dim, bs=wl.block_size,
                           max_bps=kv.max_blocks_per_seq, scale=wl.scale, token_mask=token_mask)


def check(wl, rows=None):
    ref = oracle(wl)
    got = wl.out.float().cpu().numpy()
    total = int(wl.q_start[-1])
    sel = slice(0, total) if rows is None else rows
    err = np.abs(got[sel] - ref[sel])
    bound = ATOL + RTOL * np.abs(ref[sel])
    assert (err <= bound).all(), f"max err {err.max()} (worst excess {(err - bound).max()})"


CASES = [
    # ctx lens, chunk lens, hq, hkv
    ([300, 1000, 777], [100, 256, 777], 8, 1),      # 70B per-GPU shard (GQA 8): full prefill too
    ([129, 513, 64], [1, 200, 64], 32, 8),          # Llama-3-8B heads (GQA 4)
    ([400, 333], [130, 333], 4, 4),                 # MHA: 128 tokens per CTA
    ([600, 90], [77, 90], 32, 2),                   # GQA 16: 8 tokens per CTA
    ([250, 700, 31], [0, 129, 31], 16, 8),          # an empty chunk; GQA 2
    ([300, 517], [300, 200], 12, 3),                # 3 kv heads: blocks not token-aligned in 2 MiB
]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("case", CASES, ids=[f"g{c[2] // c[3]}_{i}" for i, c in enumerate(CASES)])
def test_prefill_matches_oracle(case, dtype):
    ctx, chunks, hq, hkv = case
    wl = make(ctx_lens=ctx, chunk_lens=chunks, num_q_heads=hq, kv_heads=hkv, dtype=dtype,
              seed=sum(ctx) % 97)
    try:
        wl.run()
        _torch().cuda.synchronize()
        check(wl)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


@pytest.mark.parametrize("impl,bs", [("cpasync", 16), ("pair", 32), ("pair", 8), ("ws", 16),
                                     ("ws", 32), ("ws", 8), ("gather", 16), ("cpasync", 8),
                                     ("pair", 4)])
def test_prefill_kernel_paths(impl, bs, monkeypatch):
    """Every kernel path agrees with the oracle: the two-tile kernel (the default) with
    32-token pages (two boxes per page) and with 8-token pages (copy-gather producers, a
    box over two pages); the single-role kernel (forced, and chosen for 4-token pages);
    the one-tile warp-specialised kernel (forced, also on 8-token pages); the
    copy-gather variant (forced) for layouts without tensor maps."""
    if impl != "pair":
        monkeypatch.setenv("KCMM_PREFILL_IMPL", impl)
    wl = make(ctx_lens=[700, 260], chunk_lens=[300, 260], num_q_heads=16, kv_heads=2,
              block_size=bs, seed=bs)
    try:
        wl.run()
        _torch().cuda.synchronize()
        check(wl)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


HEAD_DIMS = [
    # head_dim, dtype, ctx lens, chunk lens, hq, hkv, block size
    (64, "bf16", [300, 1000, 45], [100, 256, 45], 8, 1, 16),
    (64, "f16", [129, 513], [1, 200], 32, 8, 16),
    (80, "bf16", [400, 333], [130, 333], 16, 2, 16),
    (96, "bf16", [600, 90], [77, 90], 32, 2, 8),
    (192, "bf16", [300, 517], [300, 200], 12, 3, 16),
    (256, "bf16", [700, 260, 31], [300, 260, 31], 16, 2, 16),
    (256, "f16", [129, 513], [128, 200], 4, 4, 32),
]


@pytest.mark.parametrize("case", HEAD_DIMS, ids=[f"d{c[0]}_{c[1]}" for c in HEAD_DIMS])
def test_prefill_other_head_dims(case):
    """Head dims other than 128 (vLLM's 64, 80, 96, 192 and 256) run the single-role
    tcgen05 kernel with head_dim padded to a multiple of 64 and 64-key tiles above 128."""
    d, dtype, ctx, chunks, hq, hkv, bs = case
    wl = make(ctx_lens=ctx, chunk_lens=chunks, num_q_heads=hq, kv_heads=hkv, head_dim=d,
              dtype=dtype, block_size=bs, seed=d + len(ctx))
    try:
        wl.run()
        _torch().cuda.synchronize()
        check(wl)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


@pytest.mark.parametrize("hq,hkv,d,bs,impl", [
    (21, 3, 128, 16, None),      # 7 query heads per kv head (Qwen2.5-7B's 28 / 4): rows of 8
    (10, 2, 128, 8, None),       # 5 per kv head on 8-token pages (copy-gather producers)
    (6, 2, 128, 16, "ws"),       # 3 per kv head on the one-tile kernel
    (12, 4, 64, 16, None),       # 3 per kv head, head_dim 64 (single-role kernel)
    (14, 2, 128, 16, "cpasync"), # 7 per kv head on the single-role kernel
])
def test_prefill_group_not_dividing_128(hq, hkv, d, bs, impl, monkeypatch):
    """Query heads per kv head that do not divide a CTA's 128 rows run padded to the next
    power of two; the idle rows are neither read nor stored, so every real head's rows
    must match the oracle (a store from an idle row would land on a real head's row)."""
    if impl:
        monkeypatch.setenv("KCMM_PREFILL_IMPL", impl)
    wl = make(ctx_lens=[300, 517, 64], chunk_lens=[300, 200, 1], num_q_heads=hq, kv_heads=hkv,
              head_dim=d, block_size=bs, seed=hq * 7 + d)
    try:
        wl.run()
        _torch().cuda.synchronize()
        check(wl)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


def test_prefill_last_row_equals_decode():
    """The last row of a chunk is a decode step over the whole context: both kernels agree."""
    torch = _torch()
    wl = make(ctx_lens=[900, 1500], chunk_lens=[300, 64], num_q_heads=32, kv_heads=8, seed=5)
    try:
        wl.run()
        kv = wl.kv
        last = torch.stack([wl.q[int(wl.q_start[b + 1]) - 1] for b in range(2)])
        kv.q.copy_(last)
        kv.decode()
        torch.cuda.synchronize()
        got = torch.stack([wl.out[int(wl.q_start[b + 1]) - 1] for b in range(2)]).float()
        ref = kv.out.float()
        assert torch.allclose(got, ref, atol=ATOL, rtol=RTOL)
    finally:
        wl.close()


def test_prefill_70b_chunk_full_context():
    """Config-5 shape at full context per GPU: a 2048-token chunk at the end of a 32768-token
    sequence (8 q heads on 1 kv head).  Checked on a sample of rows against the oracle."""
    torch = _torch()
    wl = make(ctx_lens=[32768], chunk_lens=[2048], num_q_heads=8, kv_heads=1, seed=11)
    try:
        wl.run()
        torch.cuda.synchronize()
        rng = np.random.default_rng(0)
        toks = np.unique(np.concatenate([[0, 1, 127, 128, 2047], rng.integers(0, 2048, 11)]))
        mask = np.zeros(2048, np.uint8)
        mask[toks] = 1
        ref = oracle(wl, token_mask=mask)
        got = wl.out.float().cpu().numpy()
        err = np.abs(got[toks] - ref[toks])
        assert (err <= ATOL + RTOL * np.abs(ref[toks])).all(), err.max()
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


def test_prefill_rejects_unsupported_shapes():
    from lattice_b200.kcmm import KcmmError

    wl = make(ctx_lens=[40], chunk_lens=[8], num_q_heads=8, kv_heads=1, seed=1)
    try:
        kv = wl.kv
        base = dict(query_ptr=wl.q.data_ptr(), out_ptr=wl.out.data_ptr(),
                    block_tables_ptr=kv.d_tables.data_ptr(),
                    query_start_loc_ptr=wl.d_q_start.data_ptr(),
                    context_lens_ptr=wl.d_ctx.data_ptr(),
                    block_offsets_f16_ptr=kv.d_offsets.data_ptr(), batch=1, max_query_len=8,
                    block_size=16, max_blocks_per_seq=kv.max_blocks_per_seq, scale=0.1)
        with pytest.raises(KcmmError, match="head_dim 100 unsupported"):
            wl.pool.paged_prefill(0, num_q_heads=8, kv_heads=1, head_dim=100, **base)
        with pytest.raises(KcmmError, match="head_dim 264 unsupported"):
            wl.pool.paged_prefill(0, num_q_heads=8, kv_heads=1, head_dim=264, **base)
        with pytest.raises(KcmmError, match="at most 128"):
            wl.pool.paged_prefill(0, num_q_heads=6, kv_heads=4, head_dim=128, **base)
    finally:
        wl.close()


@pytest.mark.parametrize("impl", ["pair", "ws"])
def test_prefill_peaked_rows(impl, monkeypatch):
    """Queries scaled by 6: each row's softmax is dominated by a few keys, so a P rounded
    once to 16 bits is not accurate enough there.  The two-tile kernel must keep the
    P_lo correction on those tiles (its per-row test of sum(P^2) against the running
    sum) and stay within the tolerance."""
    if impl != "pair":
        monkeypatch.setenv("KCMM_PREFILL_IMPL", impl)
    torch = _torch()
    wl = make(ctx_lens=[2600, 900], chunk_lens=[700, 900], num_q_heads=8, kv_heads=1, seed=21)
    try:
        wl.q.mul_(6.0)
        wl.run()
        torch.cuda.synchronize()
        check(wl)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


SPLIT_CASES = [
    # ctx lens, chunk lens, hq, hkv: the two-tile kernel's items (query tiles x kv heads x
    # sequences) against the 148 SMs decide how the tail splits
    ([3000], [960], 8, 1),               # 30 items, all split in 4 parts
    ([1640, 1200], [640, 640], 32, 8),   # 160 items: 148 whole, a tail of 12 in 4 parts
    ([2048], [2048], 8, 1),              # 64 items in 2 parts; full prefill: empty parts
    ([77, 900, 2100], [77, 900, 800], 16, 2),  # ragged: 174 items, the tail in the longest
]


@pytest.mark.parametrize("split", ["1", "0"])
@pytest.mark.parametrize("case", SPLIT_CASES, ids=[f"items{i}" for i in range(len(SPLIT_CASES))])
def test_prefill_tail_split(case, split, monkeypatch):
    """The items past the last whole wave of the two-tile kernel run as 2-4 CTAs over
    consecutive KV ranges whose partial rows a merge kernel combines; every part but the
    last lies below the CTA's first query row (early parts can be empty).  Both the split
    launch and the unsplit one (KCMM_PREFILL_SPLIT=0) match the oracle."""
    monkeypatch.setenv("KCMM_PREFILL_SPLIT", split)
    ctx, chunks, hq, hkv = case
    wl = make(ctx_lens=ctx, chunk_lens=chunks, num_q_heads=hq, kv_heads=hkv, dtype="bf16",
              seed=len(ctx) * 7 + hq)
    try:
        wl.run()
        _torch().cuda.synchronize()
        check(wl)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()
