"""The no-allocation decode entry point (kcmm_paged_attn_decode_bf16_noalloc_on_stream).

Its scratch is a static per-device array, not a stream-ordered allocation.  It
must agree with kcmm_paged_attn_decode_bf16_on_stream on the same inputs, both
on the first call (which resolves the array's address) and on the call after
it (which reuses the scratch the first call left behind).  Named so it is
collected last, and it is also meant to pass when run alone.

Tolerance: max-abs 2e-3 / max-rel 1e-2, |a - b| <= 2e-3 + 1e-2 * |b|."""
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


def _make(**kw):
    from lattice_b200.workloads import DecodeWorkload

    _torch()
    return DecodeWorkload(**kw).build()


def _close(got, ref):
    got = got.float().cpu().numpy()
    ref = ref.float().cpu().numpy()
    err = np.abs(got - ref)
    bound = ATOL + RTOL * np.abs(ref)
    assert (err <= bound).all(), f"max err {err.max()}"


CASES = [
    # Llama-3-8B heads, contexts 512..4096 (several splits per sequence, merged)
    dict(batch=64, pool_blocks=17000, min_len=512, max_len=4096, seed=3),
    # mixed short and empty rows, GQA 8, two head tiles not needed
    dict(batch=5, num_q_heads=8, kv_heads=1, pool_blocks=256,
         seq_lens_override=[0, 1, 17, 700, 1999], max_len=2000, seed=4),
]


@pytest.mark.parametrize("case", CASES, ids=["llama8b_b64", "ragged_gqa8"])
def test_noalloc_matches_regular_twice(case):
    torch = _torch()
    wl = _make(**case)
    try:
        ref = torch.empty_like(wl.q)
        wl.decode(out=ref)
        torch.cuda.synchronize()
        for _ in range(2):
            got = torch.full_like(wl.q, float("nan"))
            wl.decode(out=got, noalloc=True)
            torch.cuda.synchronize()
            live = torch.from_numpy(wl.seq_lens > 0)
            _close(got[live], ref[live])
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()


def test_noalloc_leaves_free_memory_unchanged():
    """After the first call, further calls take no device memory."""
    torch = _torch()
    wl = _make(batch=16, pool_blocks=2400, min_len=200, max_len=2048, seed=6)
    try:
        wl.decode(noalloc=True)
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        for _ in range(3):
            wl.decode(noalloc=True)
        torch.cuda.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0
    finally:
        wl.close()


def test_noalloc_rejects_oversized_scratch(monkeypatch):
    """64 sequences x 64 query heads on one kv head at head_dim 256, split into 10
    pieces (pinned with KCMM_DECODE_SPLITS): 40960 partial rows of 1028 bytes, above
    the 32 MiB array."""
    from lattice_b200.kcmm import KcmmError

    torch = _torch()
    monkeypatch.setenv("KCMM_DECODE_SPLITS", "10")
    wl = _make(batch=64, num_q_heads=64, kv_heads=1, head_dim=256, pool_blocks=128,
               seq_lens_override=[1] * 64, max_len=4096, seed=7)
    try:
        sentinel = torch.full_like(wl.q, 7.0)
        with pytest.raises(KcmmError, match="static limit of 33554432"):
            wl.decode(out=sentinel, noalloc=True)
        torch.cuda.synchronize()
        assert bool((sentinel == 7.0).all()), "a rejected call must launch nothing"
        # the regular entry point still serves the same batch
        monkeypatch.delenv("KCMM_DECODE_SPLITS")
        wl.decode()
        torch.cuda.synchronize()
        assert wl.pool.kernel_status() == 0
    finally:
        wl.close()
