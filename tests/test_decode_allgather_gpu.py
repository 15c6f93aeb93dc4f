"""Decode fused with the KV-head all-gather (`kcmm_paged_attn_decode_{bf16,f16}_allgather_on_stream`).

Two ranks are emulated on one GPU: each has its own pool and its own kv heads, and
each rank's fused call stores its rows into slot `rank` of both ranks' gathered
buffers.  Both ranks' calls finish in stream order before either wait is issued, so
no kernel waits for another one.  After the waits every gathered buffer must equal
the two ranks' regular decode outputs side by side, every rank's own `out` must equal
its slot, and rows of empty sequences stay untouched.  The real two-GPU path (IPC
buffers, stores over NVLink) is in test_peer_allgather_gpu.py.

Tolerance against the regular decode: |a - b| <= 2e-3 + 1e-2 |b| (the merge is the
same arithmetic; the bound only guards against a different contraction order)."""
from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _fused(wl, dst, sig, rank, world, epoch, stream):
    fn = (wl.pool.lib.kcmm_paged_attn_decode_bf16_allgather_on_stream if wl.dtype == "bf16"
          else wl.pool.lib.kcmm_paged_attn_decode_f16_allgather_on_stream)
    return fn(wl.pool.handle, 0, wl.q.data_ptr(), wl.out.data_ptr(), wl.d_tables.data_ptr(),
              wl.d_seq_lens.data_ptr(), wl.d_offsets.data_ptr(), wl.batch, wl.num_q_heads,
              wl.kv_heads, wl.head_dim, wl.block_size, wl.max_blocks_per_seq, wl.scale, dst, sig,
              rank, world, epoch, stream)


CASES = {
    # 70B head-split shard shape, long contexts: every row merges split partials
    "long": dict(batch=4, num_q_heads=16, kv_heads=2, head_dim=128, pool_blocks=4200,
                 min_len=8000, max_len=16000),
    # short and empty rows: one split, rows forwarded from the local output
    "ragged": dict(batch=6, num_q_heads=8, kv_heads=2, head_dim=64, pool_blocks=600,
                   seq_lens_override=[0, 1, 15, 16, 300, 2047], max_len=2048),
}


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("case", list(CASES))
def test_two_ranks_on_one_gpu(case, dtype):
    torch = _torch()
    from lattice_b200.workloads import DecodeWorkload

    world = 2
    wls = [DecodeWorkload(dtype=dtype, seed=70 + r, **CASES[case]).build() for r in range(world)]
    try:
        wl0 = wls[0]
        shape = (2, world) + tuple(wl0.out.shape)  # two halves, by epoch parity
        sentinel = 5.0
        bufs = [torch.full(shape, sentinel, device="cuda").to(wl0.out.dtype)
                for _ in range(world)]
        sigs = [torch.zeros(world * 16, dtype=torch.int64, device="cuda") for _ in range(world)]
        dst = (ctypes.c_uint64 * world)(*[b.data_ptr() for b in bufs])
        sig = (ctypes.c_uint64 * world)(*[s.data_ptr() for s in sigs])
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        sp = torch.cuda.current_stream().cuda_stream
        lib = wl0.pool.lib
        live = torch.from_numpy(wl0.seq_lens > 0).cuda()
        for epoch in range(1, 4):
            for wl in wls:  # new queries every epoch
                wl.q.copy_(torch.randn_like(wl.q.float()).to(wl.q.dtype))
            refs = []
            for wl in wls:
                wl.decode(stream_ptr=sp)
                refs.append(wl.out.clone())
                wl.out.fill_(float("nan"))
            for r, wl in enumerate(wls):
                assert _fused(wl, dst, sig, r, world, epoch, sp) == 0, wl.pool.last_error()
            for r in range(world):
                assert lib.kcmm_peer_wait_on_stream(sigs[r].data_ptr(), world, epoch,
                                                    status.data_ptr(), sp) == 0
            torch.cuda.synchronize()
            assert int(status.item()) == 0
            assert all(int(v) == epoch for s in sigs for v in s.tolist())
            for r, wl in enumerate(wls):
                got, ref = wl.out[live].float(), refs[r][live].float()
                assert bool(((got - ref).abs() <= ATOL + RTOL * ref.abs()).all()), (
                    f"rank {r} epoch {epoch}: max err {(got - ref).abs().max().item()}")
                for b in bufs:
                    half = b[epoch & 1]
                    assert torch.equal(half[r][live], wl.out[live])
                    assert bool((half[r][~live] == sentinel).all())
        for wl in wls:
            assert wl.pool.kernel_status() == 0
    finally:
        for wl in wls:
            wl.close()


def test_one_rank_gathers_into_its_own_buffer():
    """world 1: the gathered buffer is a copy of `out`, the flags carry the epoch."""
    torch = _torch()
    from lattice_b200.workloads import DecodeWorkload

    wl = DecodeWorkload(batch=8, num_q_heads=32, kv_heads=8, head_dim=128, pool_blocks=2200,
                        min_len=100, max_len=4000, seed=77).build()
    try:
        buf = torch.zeros((2, 1) + tuple(wl.out.shape), dtype=wl.out.dtype, device="cuda")
        sg = torch.zeros(16, dtype=torch.int64, device="cuda")
        dst = (ctypes.c_uint64 * 1)(buf.data_ptr())
        sig = (ctypes.c_uint64 * 1)(sg.data_ptr())
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        sp = torch.cuda.current_stream().cuda_stream
        wl.decode(stream_ptr=sp)
        ref = wl.out.clone()
        assert _fused(wl, dst, sig, 0, 1, 7, sp) == 0, wl.pool.last_error()
        assert wl.pool.lib.kcmm_peer_wait_on_stream(sg.data_ptr(), 1, 7, status.data_ptr(),
                                                    sp) == 0
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and all(int(v) == 7 for v in sg.tolist())
        assert torch.equal(buf[7 & 1][0], wl.out)
        assert bool((buf[0] == 0).all())  # epoch 7 writes half 1 only
        assert bool(((wl.out.float() - ref.float()).abs() <= ATOL + RTOL * ref.float().abs())
                    .all())
    finally:
        wl.close()
