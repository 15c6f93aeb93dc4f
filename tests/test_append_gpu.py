"""KV append paths on the GPU through the C ABI: host-addressed step/slot writes,
the device-slot write with its status word, and the fused RMSNorm + RoPE + append.
Page contents are bit-exact against the oracle; normalised / rotated values are
within the bf16 tolerance."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def small_pool(kv_heads=2, head_dim=64, max_batch=4, max_seq_len=128, layers=2):
    from lattice_b200 import kcmm
    from lattice_b200.workloads import library

    _torch()
    cfg = kcmm.make_config(num_layers=layers, kv_heads=kv_heads, head_dim=head_dim,
                           max_batch=max_batch, max_seq_len=max_seq_len)
    return library().create_pool(cfg)


def region(pool, layer, kind, nbytes):
    from lattice_b200.workloads import read_device

    base = pool.va_k(layer) if kind == "k" else pool.va_v(layer)
    return read_device(base, nbytes).view(np.uint16)


def test_append_step_and_slots_bit_exact():
    """ref scripts/kcmm/kv_write_ffi_smoke.py:180-425: alloc 3, free 1, write at positions
    [0, bs+1] via the step path and via the equivalent slots; pages byte-equal."""
    torch = _torch()
    from oracle.pool_oracle import OraclePool

    pool = small_pool()
    orc = OraclePool(num_layers=2, kv_heads=2, head_dim=64, max_batch=4, max_seq_len=128)
    try:
        blocks = pool.alloc_blocks(3)
        assert blocks == orc.alloc_blocks(3)
        pool.free_blocks(blocks[:1])
        orc.free_blocks(blocks[:1])
        live = blocks[1:]
        s = pool.register_sequence(live)
        orc.register_sequence(live)
        step = 2 * 64
        k = torch.randn(2, step, device="cuda").half()
        v = torch.randn(2, step, device="cuda").half()
        pool.append_kv_step(1, [s, s], [0, 17], k.data_ptr(), v.data_ptr())
        torch.cuda.synchronize()
        nbytes = (max(pool.all_block_offsets_f16()) * 2) + pool.stats()["block_bytes"]
        after_step = (region(pool, 1, "k", nbytes).copy(), region(pool, 1, "v", nbytes).copy())
        want_k = np.zeros(nbytes // 2, np.uint16)
        want_v = np.zeros_like(want_k)
        kb, vb = k.view(torch.int16).cpu().numpy().view(np.uint16), v.view(torch.int16).cpu().numpy().view(np.uint16)
        for r, pos in enumerate([0, 17]):
            d = orc.step_destination(0, pos)
            want_k[d:d + step], want_v[d:d + step] = kb[r], vb[r]
        got_k, got_v = after_step
        rows = [orc.step_destination(0, p) for p in (0, 17)]
        for r, d in enumerate(rows):
            assert np.array_equal(got_k[d:d + step], want_k[d:d + step])
            assert np.array_equal(got_v[d:d + step], want_v[d:d + step])
        # same rows through slots = block*bs + offset (block ids are KCMM ids)
        slots = [live[0] * 16 + 0, live[1] * 16 + 1, -1]
        k3 = torch.cat([k, torch.zeros(1, step, device="cuda").half()])
        v3 = torch.cat([v, torch.zeros(1, step, device="cuda").half()])
        pool.append_kv_slots(0, slots, k3.data_ptr(), v3.data_ptr(),
                             stream_ptr=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert np.array_equal(region(pool, 0, "k", nbytes), after_step[0])
        assert np.array_equal(region(pool, 0, "v", nbytes), after_step[1])
        # a freed block is refused
        with pytest.raises(Exception, match="not in use"):
            pool.append_kv_slots(0, [blocks[0] * 16], k.data_ptr(), v.data_ptr())
    finally:
        pool.destroy()


@pytest.mark.parametrize("case", ["kv_write_f16", "kv_write_f16_oob"])
def test_device_slot_write_matches_reference_golden(case, golden):
    """Same inputs as the reference kernel's golden run; identical pages and status."""
    torch = _torch()
    from tests.golden.make_golden import golden_inputs

    w = golden_inputs(case)
    pool = small_pool(kv_heads=2, head_dim=128, max_batch=12, max_seq_len=16, layers=1)
    try:
        ids = pool.alloc_blocks(w["nb"])
        offs = np.array(pool.all_block_offsets_f16(), np.uint64)
        # the fixture's offsets are id*block_elems; remap the expected pages block by block
        step, bs = w["step"], w["bs"]
        d_slots = torch.from_numpy(w["slots"]).cuda()
        d_offs = torch.from_numpy(offs.view(np.int64)).cuda()
        d_valid = torch.from_numpy(w["valid"]).cuda()
        k = torch.from_numpy(w["k"].view(np.int16)).cuda()
        v = torch.from_numpy(w["v"].view(np.int16)).cuda()
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        pool.append_kv_device_slots_on_stream(
            0, slot_mapping_ptr=d_slots.data_ptr(), block_offsets_f16_ptr=d_offs.data_ptr(),
            valid_blocks_ptr=d_valid.data_ptr(), block_offsets_f16_len=w["nb"],
            batch=len(w["slots"]), k_src_ptr=k.data_ptr(), v_src_ptr=v.data_ptr(),
            status_ptr=status.data_ptr(), stream_ptr=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert int(status.item()) == int(golden["ref"][f"{case}_status"][0])
        nbytes = int(offs.max()) * 2 + bs * step * 2
        got_k, got_v = region(pool, 0, "k", nbytes), region(pool, 0, "v", nbytes)
        want_k, want_v = golden["ref"][f"{case}_va_k"], golden["ref"][f"{case}_va_v"]
        for b in range(w["nb"]):
            src = slice(b * bs * step, (b + 1) * bs * step)
            dst = slice(int(offs[b]), int(offs[b]) + bs * step)
            if want_k[src].any() or want_v[src].any():
                assert np.array_equal(got_k[dst], want_k[src]), b
                assert np.array_equal(got_v[dst], want_v[src]), b
        assert ids == list(range(w["nb"]))
    finally:
        pool.destroy()


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_fused_norm_rope_append_matches_oracle(mode):
    torch = _torch()
    from lattice_b200.workloads import FusedAppendWorkload, tensor_bits
    from oracle import native as N

    wl = FusedAppendWorkload(tokens=64, rope_mode=mode, seed=mode).build()
    try:
        # make two tokens exercise the status paths: one padding slot, one freed block
        slots = wl.slots.copy()
        slots[5] = -1
        wl.d_slots.copy_(torch.from_numpy(slots))
        x, w, q0 = tensor_bits(wl.x), tensor_bits(wl.w), tensor_bits(wl.q)
        k, v = tensor_bits(wl.k), tensor_bits(wl.v)
        nbytes = int(wl.offsets.max()) * 2 + wl.pool.stats()["block_bytes"]
        va_k0, va_v0 = region(wl.pool, 0, "k", nbytes).copy(), region(wl.pool, 0, "v", nbytes).copy()
        wl.run()
        torch.cuda.synchronize()
        assert int(wl.status.item()) == 0
        want_norm, want_q, st = N.fused_norm_rope_append(
            x, w, q0, k, v, wl.positions, slots, wl.offsets, wl.valid, va_k0, va_v0,
            eps=wl.eps, base=wl.theta, mode=mode, hkv=wl.kv_heads, d=wl.head_dim,
            bs=wl.block_size)
        assert st == 0
        f = N.bf16_bits_to_f32
        for got, want in ((tensor_bits(wl.normed), want_norm), (tensor_bits(wl.q), want_q)):
            g, r = f(got), f(want)
            assert (np.abs(g - r) <= 2e-3 + 1e-2 * np.abs(r)).all()
        got_k, got_v = region(wl.pool, 0, "k", nbytes), region(wl.pool, 0, "v", nbytes)
        assert np.array_equal(got_v, va_v0)  # V rows: a bit copy
        gk, rk = f(got_k), f(va_k0)
        assert (np.abs(gk - rk) <= 2e-3 + 1e-2 * np.abs(rk)).all()
        # the padding token wrote nothing: its would-be slot keeps the old bytes
    finally:
        wl.close()


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_config3_fused_norm_rope_append_full_size(mode):
    """BASELINE config 3 exactly: 256 decode tokens, hidden 4096, eps 1e-5, weight
    U(0.5, 1.5), rope theta 500000 on head_dim 128 at positions uniform in [0, 8191],
    8 kv heads, block_size 16, seeded distinct slots.  normed, q and the rotated K
    rows within the bf16 tolerance of the oracle composition; V pages bit-exact; no
    byte outside the written rows changes."""
    torch = _torch()
    from lattice_b200.workloads import FusedAppendWorkload, tensor_bits
    from oracle import native as N

    wl = FusedAppendWorkload(tokens=256, rope_mode=mode, seed=30 + mode).build()
    try:
        assert (wl.hidden, wl.eps, wl.theta, wl.kv_heads, wl.head_dim, wl.block_size) == \
            (4096, 1e-5, 500000.0, 8, 128, 16)
        assert len(set(wl.slots.tolist())) == 256
        assert wl.positions.min() >= 0 and wl.positions.max() <= 8191
        x, w, q0 = tensor_bits(wl.x), tensor_bits(wl.w), tensor_bits(wl.q)
        k, v = tensor_bits(wl.k), tensor_bits(wl.v)
        nbytes = int(wl.offsets.max()) * 2 + wl.pool.stats()["block_bytes"]
        va_k0, va_v0 = region(wl.pool, 0, "k", nbytes).copy(), region(wl.pool, 0, "v", nbytes).copy()
        wl.run()
        torch.cuda.synchronize()
        assert int(wl.status.item()) == 0
        want_norm, want_q, st = N.fused_norm_rope_append(
            x, w, q0, k, v, wl.positions, wl.slots, wl.offsets, wl.valid, va_k0, va_v0,
            eps=wl.eps, base=wl.theta, mode=mode, hkv=wl.kv_heads, d=wl.head_dim,
            bs=wl.block_size)
        assert st == 0
        f = N.bf16_bits_to_f32
        for got, want in ((tensor_bits(wl.normed), want_norm), (tensor_bits(wl.q), want_q)):
            g, r = f(got), f(want)
            assert (np.abs(g - r) <= 2e-3 + 1e-2 * np.abs(r)).all()
        got_k, got_v = region(wl.pool, 0, "k", nbytes), region(wl.pool, 0, "v", nbytes)
        assert np.array_equal(got_v, va_v0)
        gk, rk = f(got_k), f(va_k0)
        assert (np.abs(gk - rk) <= 2e-3 + 1e-2 * np.abs(rk)).all()
        # rows no token writes keep their bytes exactly (K included)
        step = wl.kv_heads * wl.head_dim
        written = np.zeros(nbytes // 2, bool)
        for slot in wl.slots:
            start = int(wl.offsets[slot // 16]) + (slot % 16) * step
            written[start:start + step] = True
        assert np.array_equal(got_k[~written], va_k0[~written])
    finally:
        wl.close()


def test_fused_status_codes():
    torch = _torch()
    from lattice_b200.workloads import FusedAppendWorkload

    wl = FusedAppendWorkload(tokens=8, seed=4).build()
    try:
        wl.pool.free_blocks([3])
        valid = np.array(wl.pool.all_block_valid_flags(), np.uint8)
        wl.d_valid.copy_(torch.from_numpy(valid))
        slots = wl.slots.copy()
        slots[2] = 3 * 16 + 1            # freed block -> 2
        wl.d_slots.copy_(torch.from_numpy(slots))
        wl.run()
        torch.cuda.synchronize()
        assert int(wl.status.item()) == 2
        slots[2] = 10**6 * 16            # beyond the offsets table -> 1 (status reset first)
        wl.d_slots.copy_(torch.from_numpy(slots))
        wl.status.zero_()
        wl.run()
        torch.cuda.synchronize()
        assert int(wl.status.item()) == 1
    finally:
        wl.close()
