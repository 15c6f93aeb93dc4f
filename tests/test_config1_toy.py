"""BASELINE config 1, the CPU toy, as its procedure states it: batch 4, 4 q heads = 4 kv
heads, head_dim 64, block_size 16; q/k/v fp32 ~ N(0, 1) from a seed; the physical block
ids of every sequence a seeded permutation of a 128-block pool; 256 tokens pre-filled
per sequence, then one decode step appends one token per sequence and attends over all
257 positions.

* CPU: the library's allocator (host VMM backend) hands out the 128 blocks, and its
  block tables and offsets table equal the allocator oracle's bit for bit.  On the
  resulting fp32 pages the oracle's fp32 attention equals the reference's own
  attention source (kcmm_vllm_paged_attn.cu built over fp32 storage, oracle/_ref)
  within max-abs 1e-5.
* GPU: the same procedure through the C ABI on a device pool (16-bit pages, since
  the kernels store f16/bf16): the pre-fill through kcmm_append_kv_slots, the step's
  token through kcmm_append_kv_step, the attention through kcmm_paged_attn_decode_f16
  (the reference's entry point).  Tables and offsets bit-exact against the allocator
  oracle, the pages bit-exact against the oracle's slot writes, the output within
  max-abs 2e-3 / max-rel 1e-2 of the oracle on the same f16 pages.

Layout note for fp32 pages: the reference kernel indexes elements through its
`__half *`, so with fp32 storage `block_offsets_f16[blk]` is an element index; the
oracle takes offsets in 2-byte units, so it is given twice the table to address the
same bytes."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import native as N
from oracle.pool_oracle import OraclePool

B, HQ, HKV, D, BS = 4, 4, 4, 64, 16
PREFILL, CTX = 256, 257
POOL_BLOCKS = 128
STEP = HKV * D
CFG = dict(num_layers=1, kv_heads=HKV, head_dim=D, max_batch=B, max_seq_len=512, block_size=BS)


def _inputs(seed: int):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(POOL_BLOCKS)
    k_pre = rng.standard_normal((B, PREFILL, STEP)).astype(np.float32)
    v_pre = rng.standard_normal((B, PREFILL, STEP)).astype(np.float32)
    k_new = rng.standard_normal((B, STEP)).astype(np.float32)
    v_new = rng.standard_normal((B, STEP)).astype(np.float32)
    q = rng.standard_normal((B, HQ, D)).astype(np.float32)
    return perm, k_pre, v_pre, k_new, v_new, q


def _allocate(pool, orc, perm):
    """128 blocks from the pool; sequence b takes the ids at perm[17b : 17b + 17]: the
    first 16 hold the pre-fill, the 17th is appended for the step's token."""
    ids = pool.alloc_blocks(POOL_BLOCKS)
    assert ids == orc.alloc_blocks(POOL_BLOCKS)
    per = -(-CTX // BS)
    blocks = [[ids[int(perm[b * per + j])] for j in range(per)] for b in range(B)]
    seqs = []
    for b in range(B):
        s = pool.register_sequence(blocks[b][:-1])
        assert s == orc.register_sequence(blocks[b][:-1])
        pool.update_seq_len(s, PREFILL)
        seqs.append(s)
    return blocks, seqs


def _grow(pool, orc, blocks, seqs):
    for b, s in enumerate(seqs):
        pool.append_block_to_sequence(s, blocks[b][-1])
        orc.append_block_to_sequence(s, blocks[b][-1])
        pool.update_seq_len(s, CTX)


def _check_tables(pool, orc, seqs):
    for s in seqs:
        assert pool.block_table(s) == orc.sequences[s]["table"]
    assert pool.all_block_offsets_f16() == orc.all_block_offsets_f16()


def _tables(blocks):
    t = np.zeros((B, 32), np.int32)
    for b in range(B):
        t[b, :len(blocks[b])] = blocks[b]
    return t


@pytest.mark.skipif(not N.ref_available(), reason="oracle/_ref not built")
def test_config1_cpu_toy_fp32(host_pool_factory):
    perm, k_pre, v_pre, k_new, v_new, q = _inputs(seed=1)
    pool = host_pool_factory(**CFG)
    orc = OraclePool(**CFG)
    blocks, seqs = _allocate(pool, orc, perm)
    _grow(pool, orc, blocks, seqs)
    _check_tables(pool, orc, seqs)
    offs = np.array(pool.all_block_offsets_f16(), np.uint64)
    # fp32 regions; element index of (block, token-in-block, kv head, dim) =
    # offs[block] + token * STEP + kvh * D + dim
    n = int(offs.max()) + BS * STEP
    va_k = np.zeros(n, np.float32)
    va_v = np.zeros(n, np.float32)
    for b in range(B):
        for t in range(CTX):
            blk = blocks[b][t // BS]
            e = int(offs[blk]) + (t % BS) * STEP
            va_k[e:e + STEP] = k_pre[b, t] if t < PREFILL else k_new[b]
            va_v[e:e + STEP] = v_pre[b, t] if t < PREFILL else v_new[b]
    tables = _tables(blocks)
    seq = np.full(B, CTX, np.int32)
    kw = dict(hq=HQ, hkv=HKV, d=D, bs=BS, max_bps=32, scale=D ** -0.5)
    want = N.ref_paged_attn("f32", q, va_k, va_v, tables, seq, offs, **kw)
    got = N.paged_attn("f32", q, va_k, va_v, tables, seq, offs * np.uint64(2), **kw)
    assert np.abs(got - want.reshape(got.shape)).max() <= 1e-5


def test_config1_allocator_matches_oracle(host_pool_factory):
    """The allocation half of the toy, without oracle/_ref: tables and offsets of the
    library's allocator equal the oracle's after the permuted draw and the step's
    block append."""
    perm = _inputs(seed=2)[0]
    pool = host_pool_factory(**CFG)
    orc = OraclePool(**CFG)
    blocks, seqs = _allocate(pool, orc, perm)
    _check_tables(pool, orc, seqs)
    _grow(pool, orc, blocks, seqs)
    _check_tables(pool, orc, seqs)
    assert pool.blocks_in_use() == orc.blocks_in_use()


@pytest.mark.gpu
def test_config1_on_gpu():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from lattice_b200 import kcmm
    from lattice_b200.workloads import library, read_device

    perm, k_pre, v_pre, k_new, v_new, q = _inputs(seed=3)
    pool = library().create_pool(kcmm.make_config(**CFG))
    orc = OraclePool(**CFG)
    try:
        blocks, seqs = _allocate(pool, orc, perm)
        _check_tables(pool, orc, seqs)
        offs = np.array(pool.all_block_offsets_f16(), np.uint64)
        nbytes = (int(offs.max()) + BS * STEP) * 2
        base_k = read_device(pool.va_k(0), nbytes).view(np.uint16).copy()
        base_v = read_device(pool.va_v(0), nbytes).view(np.uint16).copy()
        f16 = N.f32_to_f16_bits
        # pre-fill: every sequence's 256 rows through host-side slots
        slots = np.array([blocks[b][t // BS] * BS + t % BS for b in range(B)
                          for t in range(PREFILL)], np.int64)
        kp = torch.from_numpy(f16(k_pre).view(np.int16).reshape(-1, STEP)).cuda()
        vp = torch.from_numpy(f16(v_pre).view(np.int16).reshape(-1, STEP)).cuda()
        pool.append_kv_slots(0, slots.tolist(), kp.data_ptr(), vp.data_ptr())
        # the decode step: one more block per sequence, its token at position 256
        _grow(pool, orc, blocks, seqs)
        _check_tables(pool, orc, seqs)
        kn = torch.from_numpy(f16(k_new).view(np.int16)).cuda()
        vn = torch.from_numpy(f16(v_new).view(np.int16)).cuda()
        pool.append_kv_step(0, seqs, [PREFILL] * B, kn.data_ptr(), vn.data_ptr())
        torch.cuda.synchronize()
        # pages: the oracle's slot writes on the same starting bytes
        want_k, want_v = base_k.copy(), base_v.copy()
        valid = np.array(orc.all_block_valid(), np.uint8)
        assert N.slot_write(want_k, want_v, slots, offs, valid, f16(k_pre).reshape(-1, STEP),
                            f16(v_pre).reshape(-1, STEP), step=STEP, bs=BS) == 0
        step_slots = np.array([blocks[b][-1] * BS + PREFILL % BS for b in range(B)], np.int64)
        for b, s in enumerate(seqs):
            assert orc.step_destination(s, PREFILL) == \
                int(offs[step_slots[b] // BS]) + (PREFILL % BS) * STEP
        assert N.slot_write(want_k, want_v, step_slots, offs, valid, f16(k_new), f16(v_new),
                            step=STEP, bs=BS) == 0
        got_k = read_device(pool.va_k(0), nbytes).view(np.uint16)
        got_v = read_device(pool.va_v(0), nbytes).view(np.uint16)
        assert np.array_equal(got_k, want_k) and np.array_equal(got_v, want_v)
        # attention over the 257 positions through the reference's entry point
        tables = _tables(blocks)
        dq = torch.from_numpy(f16(q).view(np.int16)).cuda()
        out = torch.zeros_like(dq)
        d_tables = torch.from_numpy(tables).cuda()
        d_seq = torch.full((B,), CTX, dtype=torch.int32, device="cuda")
        d_offs = torch.from_numpy(offs.view(np.int64)).cuda()
        pool.paged_attn_decode(0, query_ptr=dq.data_ptr(), out_ptr=out.data_ptr(),
                               block_tables_ptr=d_tables.data_ptr(),
                               seq_lens_ptr=d_seq.data_ptr(),
                               block_offsets_f16_ptr=d_offs.data_ptr(), batch=B, num_q_heads=HQ,
                               kv_heads=HKV, head_dim=D, block_size=BS, max_blocks_per_seq=32,
                               scale=D ** -0.5, dtype="f16", stream_ptr=None)
        want = N.paged_attn("f16", f16(q), want_k, want_v, tables, np.full(B, CTX, np.int32),
                            offs, hq=HQ, hkv=HKV, d=D, bs=BS, max_bps=32, scale=D ** -0.5)
        got = N.f16_bits_to_f32(out.cpu().numpy().view(np.uint16)).reshape(want.shape)
        assert (np.abs(got - want) <= 2e-3 + 1e-2 * np.abs(want)).all()
        assert pool.kernel_status() == 0
    finally:
        pool.destroy()
