"""Shared-prefix decode (`kcmm_paged_attn_decode_shared_prefix_{bf16,f16}_on_stream`).

Groups of consecutive sequences get the same block ids in the first table entries (as
kcmm_fork_sequence / kcmm_share_prefix leave beams and shared system prompts).  The
shared-prefix call must give the oracle's result (the fp64 restatement of the
reference kernel, reading every sequence through its own table) within the decode
tolerance, |a - b| <= 2e-3 + 1e-2 |b|, and agree with the plain decode call:
- beams of equal groups;
- ragged groups, including a group larger than max_group_size, a one-member group,
  a prefix length that is not a multiple of 16 or of the block size, a member shorter
  than the prefix, and an empty member;
- 8 query heads per kv head (two members per tile), and f16.
Malformed group arrays only lose the sharing, never the result; a group whose tables
differ inside the promised prefix is reported through bit 2 of the kernel status."""
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


def _oracle(wl):
    from lattice_b200.workloads import tensor_bits
    from oracle import native as N

    return N.paged_attn(wl.dtype, tensor_bits(wl.q), wl.host_region(0, "k"),
                        wl.host_region(0, "v"), wl.tables, wl.seq_lens, wl.offsets,
                        hq=wl.num_q_heads, hkv=wl.kv_heads, d=wl.head_dim, bs=wl.block_size,
                        max_bps=wl.max_blocks_per_seq, scale=wl.scale)


def _build(groups, prefix_blocks, seq_lens, hq=32, hkv=8, dtype="bf16", seed=0):
    """A workload whose groups (sizes in `groups`) share the first prefix_blocks[g]
    table entries of their first member."""
    import torch
    from lattice_b200.workloads import DecodeWorkload

    wl = DecodeWorkload(batch=len(seq_lens), num_q_heads=hq, kv_heads=hkv, head_dim=128,
                        pool_blocks=sum(-(-int(L) // 16) for L in seq_lens) + 64,
                        seq_lens_override=seq_lens,
                        max_len=max(seq_lens) + 16, dtype=dtype, seed=seed, fill="host").build()
    start = 0
    for n, k in zip(groups, prefix_blocks):
        for m in range(start + 1, start + n):
            wl.tables[m, :k] = wl.tables[start, :k]
        start += n
    wl.d_tables = torch.from_numpy(wl.tables).cuda()
    return wl


def _call(wl, starts, prefix_lens, max_group, out):
    import torch

    d_starts = torch.tensor(starts, dtype=torch.int32, device="cuda")
    d_prefix = torch.tensor(prefix_lens, dtype=torch.int32, device="cuda")
    fn = (wl.pool.lib.kcmm_paged_attn_decode_shared_prefix_bf16_on_stream if wl.dtype == "bf16"
          else wl.pool.lib.kcmm_paged_attn_decode_shared_prefix_f16_on_stream)
    rc = fn(wl.pool.handle, 0, wl.q.data_ptr(), out.data_ptr(), wl.d_tables.data_ptr(),
            wl.d_seq_lens.data_ptr(), wl.d_offsets.data_ptr(), wl.batch, wl.num_q_heads,
            wl.kv_heads, wl.head_dim, wl.block_size, wl.max_blocks_per_seq, wl.scale,
            d_starts.data_ptr(), d_prefix.data_ptr(), len(starts) - 1, max_group,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, wl.pool.last_error()
    torch.cuda.synchronize()


def _check(wl, got, ref):
    live = wl.seq_lens > 0
    g = got.float().cpu().numpy()[live]
    err = np.abs(g - ref[live])
    bound = ATOL + RTOL * np.abs(ref[live])
    assert (err <= bound).all(), f"max err {err.max()} (worst excess {(err - bound).max()})"


def _run_case(groups, prefix_blocks, prefix_lens, seq_lens, max_group, **kw):
    torch = _torch()
    wl = _build(groups, prefix_blocks, seq_lens, **kw)
    try:
        ref = _oracle(wl)
        starts = list(np.cumsum([0] + list(groups)))
        sentinel = 3.0
        for _ in range(2):  # the second call reuses the first call's scratch
            out = torch.full_like(wl.q, sentinel)
            _call(wl, starts, prefix_lens, max_group, out)
            _check(wl, out, ref)
            dead = torch.from_numpy(wl.seq_lens <= 0)
            assert bool((out[dead] == sentinel).all()), "empty sequences stay untouched"
        wl.decode()
        torch.cuda.synchronize()
        _check(wl, wl.out, ref)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


def test_beam_groups():
    # 5 requests x 4 beams sharing 40 blocks (640 tokens), tails of 1..300 tokens
    rng = np.random.default_rng(1)
    lens = [640 + int(x) for x in rng.integers(1, 300, 20)]
    _run_case([4] * 5, [40] * 5, [640] * 5, lens, 4)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_ragged_groups(dtype):
    groups = [1, 3, 6, 2, 3]
    prefix_blocks = [10, 13, 20, 8, 12]
    # group 1: 200 tokens (12.5 blocks); group 2: 6 members, max_group 4; group 3 has a
    # member shorter than its prefix; group 4 holds an empty member
    prefix_lens = [160, 200, 320, 128, 192]
    lens = [170,
            230, 201, 420,
            321, 500, 333, 900, 321, 640,
            129, 90,
            300, 0, 250]
    _run_case(groups, prefix_blocks, prefix_lens, lens, 4, dtype=dtype, seed=2)


def test_eight_heads_per_kv_head():
    # G = 8: two members per 16-row tile, so a 5-member group takes 3 tiles
    rng = np.random.default_rng(3)
    lens = [512 + int(x) for x in rng.integers(1, 200, 9)]
    _run_case([5, 4], [32, 32], [512, 500], lens, 5, hq=16, hkv=2, seed=3)


def test_more_sequences_than_prep_threads():
    """1500 sequences in groups of 3 (500 groups): the prep kernel's thread-stride
    loops and a long work list."""
    rng = np.random.default_rng(7)
    lens = [40 + int(x) for x in rng.integers(0, 60, 1500)]
    _run_case([3] * 500, [2] * 500, [32] * 500, lens, 3, hq=8, hkv=2, seed=7)


def test_own_tokens_folded_into_the_prefix_piece_within_its_room():
    """Members a few units past their group's prefix attend those units inside the
    group's last prefix piece while it has room (32 units per warp); the others get
    entries of their own.  40 groups of 4 fill a wave with one 125-unit piece each,
    leaving room for 3 units: per group the members' own units are 1 and 2 (folded),
    then 1 (no room left) and 5 (more than a folded member may bring)."""
    lens = [2000 + 16, 2000 + 32, 2000 + 1, 2000 + 69] * 40
    _run_case([4] * 40, [125] * 40, [2000] * 40, lens, 4, hq=16, hkv=8, seed=8)


@pytest.mark.parametrize("bs,d", [(8, 128), (16, 96)])
def test_shapes_outside_the_shared_kernels_get_the_plain_decode(bs, d):
    """8-token pages and head_dim 96 have no shared-prefix kernel: the call still gives
    the oracle's result (through the plain decode) instead of failing."""
    torch = _torch()
    from lattice_b200.workloads import DecodeWorkload

    lens = [300, 290, 310, 305]
    wl = DecodeWorkload(batch=4, num_q_heads=8, kv_heads=2, head_dim=d, block_size=bs,
                        pool_blocks=sum(-(-L // bs) for L in lens) + 64, seq_lens_override=lens,
                        max_len=max(lens) + 16, seed=9, fill="host").build()
    try:
        k = 256 // bs
        for m in range(1, 4):
            wl.tables[m, :k] = wl.tables[0, :k]
        wl.d_tables = torch.from_numpy(wl.tables).cuda()
        ref = _oracle(wl)
        out = torch.zeros_like(wl.q)
        _call(wl, [0, 4], [256], 4, out)
        _check(wl, out, ref)
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


def test_malformed_groups_keep_the_result():
    torch = _torch()
    wl = _build([4, 4], [20, 20], [400, 380, 330, 390, 350, 341, 399, 333], seed=4)
    try:
        ref = _oracle(wl)
        for starts, lens in (([0, 5, 3, 8], [320, 320, 320]),   # not ascending
                             ([0, 4, 9], [320, 320]),          # end past the batch
                             ([0, 4, 8], [-16, 10000])):       # negative / too long
            out = torch.zeros_like(wl.q)
            _call(wl, starts, lens, 4, out)
            _check(wl, out, ref)
    finally:
        wl.close()


def test_tables_that_differ_inside_the_prefix_are_reported():
    torch = _torch()
    wl = _build([4], [20], [400, 380, 330, 390], seed=5)
    try:
        wl.tables[2, 7] = wl.tables[3, 24]  # member 2 breaks the promise at block 7
        wl.d_tables = torch.from_numpy(wl.tables).cuda()
        out = torch.zeros_like(wl.q)
        _call(wl, [0, 4], [320], 4, out)
        assert wl.pool.kernel_status() & 4
    finally:
        wl.close()


def test_bench_shape_unique_bytes_read_once():
    """BASELINE config 4 attention: 16 requests x 4 beams over a 2048-token shared prefix
    plus 8 own tokens; against the plain decode on the same inputs."""
    torch = _torch()
    lens = [2048 + 8] * 64
    wl = _build([4] * 16, [128] * 16, lens, seed=6)
    try:
        wl.decode()
        out = torch.zeros_like(wl.q)
        _call(wl, list(range(0, 65, 4)), [2048] * 16, 4, out)
        ref = wl.out.float()
        assert bool(((out.float() - ref).abs() <= ATOL + RTOL * ref.abs()).all())
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()
