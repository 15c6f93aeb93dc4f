"""Strided entry points for views into a fused QKV projection output (the vLLM seam,
which in the reference copies such views to compact tensors first:
scripts/kcmm/kv_read_plan.py:830-838, scripts/kcmm/kv_write_mirror.py:536-537).

The strided calls must give the same bits as the dense calls on compact copies of the
same data: the decode output for every row, and the page bytes of the KV write."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("head_pad", [0, 8])
def test_strided_decode_equals_dense_decode(dtype, head_pad):
    from lattice_b200.workloads import DecodeWorkload

    torch = _torch()
    wl = DecodeWorkload(batch=9, num_q_heads=32, kv_heads=8, head_dim=128, pool_blocks=2000,
                        min_len=1, max_len=3000, dtype=dtype, seed=31).build()
    try:
        B, hq, hkv, D = wl.batch, wl.num_q_heads, wl.kv_heads, wl.head_dim
        wl.decode()
        torch.cuda.synchronize()
        dense = wl.out.clone()
        # q inside a fused [B, hq + 2 hkv, D + pad] projection output
        qkv = torch.randn(B, hq + 2 * hkv, D + head_pad, device="cuda").to(wl.q.dtype)
        qkv[:, :hq, :D] = wl.q
        q_view = qkv[:, :hq, :D]
        # out inside a wider buffer, tables inside a wider int32 array
        out_big = torch.full((B, hq + 3, D + head_pad), 7.0, device="cuda").to(wl.q.dtype)
        out_view = out_big[:, 1:hq + 1, :D]
        tables_big = torch.full((B, wl.max_blocks_per_seq + 5), -9, dtype=torch.int32,
                                device="cuda")
        tables_big[:, :wl.max_blocks_per_seq] = wl.d_tables
        fn = (wl.pool.lib.kcmm_paged_attn_decode_bf16_strided_on_stream if dtype == "bf16"
              else wl.pool.lib.kcmm_paged_attn_decode_f16_strided_on_stream)
        rc = fn(wl.pool.handle, 0, q_view.data_ptr(), q_view.stride(0), q_view.stride(1),
                out_view.data_ptr(), out_view.stride(0), out_view.stride(1),
                tables_big.data_ptr(), tables_big.stride(0), wl.d_seq_lens.data_ptr(),
                wl.d_offsets.data_ptr(), B, hq, hkv, D, wl.block_size, wl.max_blocks_per_seq,
                wl.scale, torch.cuda.current_stream().cuda_stream)
        assert rc == 0, wl.pool.last_error()
        torch.cuda.synchronize()
        assert torch.equal(out_view, dense)
        # nothing outside the view was written
        assert (out_big[:, 0] == 7).all() and (out_big[:, hq + 1:] == 7).all()
        if head_pad:
            assert (out_big[:, :, D:] == 7).all()
    finally:
        wl.close()


def test_strided_slot_write_equals_dense_slot_write():
    from lattice_b200.workloads import DecodeWorkload, read_device

    torch = _torch()
    wl = DecodeWorkload(batch=6, num_q_heads=16, kv_heads=4, head_dim=64, pool_blocks=600,
                        min_len=30, max_len=400, seed=8).build()
    try:
        pool = wl.pool
        B, hq, hkv, D, bs = wl.batch, wl.num_q_heads, wl.kv_heads, wl.head_dim, wl.block_size
        step = hkv * D
        qkv = torch.randn(B, (hq + 2 * hkv) * D, device="cuda").bfloat16()
        k_view = qkv[:, hq * D:(hq + hkv) * D]
        v_view = qkv[:, (hq + hkv) * D:]
        # the last position of every sequence
        slots = torch.tensor([int(wl.tables[b, (int(L) - 1) // bs]) * bs + (int(L) - 1) % bs
                              for b, L in enumerate(wl.seq_lens)], dtype=torch.int64,
                             device="cuda")
        offs = wl.d_offsets
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        sp = torch.cuda.current_stream().cuda_stream
        rc = pool.lib.kcmm_append_kv_device_slots_strided_on_stream(
            pool.handle, 0, slots.data_ptr(), offs.data_ptr(), 0, offs.numel(), B,
            k_view.data_ptr(), k_view.stride(0), v_view.data_ptr(), v_view.stride(0),
            status.data_ptr(), sp)
        assert rc == 0, pool.last_error()
        torch.cuda.synchronize()
        region = wl.region_used
        strided = (read_device(pool.va_k(0), region).copy(), read_device(pool.va_v(0), region).copy())
        # the dense call on compact copies of the same rows writes the same bytes
        k_c, v_c = k_view.contiguous(), v_view.contiguous()
        pool.append_kv_device_slots_on_stream(
            0, slot_mapping_ptr=slots.data_ptr(), block_offsets_f16_ptr=offs.data_ptr(),
            valid_blocks_ptr=0, block_offsets_f16_len=offs.numel(), batch=B,
            k_src_ptr=k_c.data_ptr(), v_src_ptr=v_c.data_ptr(), status_ptr=status.data_ptr(),
            stream_ptr=sp)
        torch.cuda.synchronize()
        dense = (read_device(pool.va_k(0), region), read_device(pool.va_v(0), region))
        assert (strided[0] == dense[0]).all() and (strided[1] == dense[1]).all()
        assert int(status.item()) == 0
        # and the rows really landed: the K row of sequence 0 equals the view's row 0
        b0 = int(slots[0].item())
        off = int(wl.offsets[b0 // bs]) * 2 + (b0 % bs) * step * 2
        row = read_device(pool.va_k(0) + off, step * 2)
        assert (row == k_c[0].cpu().view(torch.int16).numpy().view("uint8")).all()
    finally:
        wl.close()
