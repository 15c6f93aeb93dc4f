"""Pins the CPU oracle: against the golden outputs of the reference's own kernels
(tests/golden/ref_kernels.npz, made by tests/golden/make_golden.py from oracle/_ref)
and, where oracle/_ref is present, against those kernels directly on fresh inputs."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import native as N
from tests.golden.make_golden import golden_inputs

ref = pytest.mark.skipif(not N.ref_available(), reason="oracle/_ref not built")


def test_attention_matches_reference_golden(golden):
    a = golden_inputs("attn_f16")
    want = N.f16_bits_to_f32(golden["ref"]["attn_f16_out"])
    got = N.paged_attn("f16", a["q"], a["va_k"], a["va_v"], a["tables"], a["seq"],
                       a["offsets"], hq=a["hq"], hkv=a["hkv"], d=a["D"], bs=a["bs"],
                       max_bps=a["max_bps"], scale=a["scale"])
    live = a["seq"] > 0
    # f16 rounding of the reference output: <= half an f16 ulp of |out| < 1
    np.testing.assert_allclose(got[live], want[live], atol=6e-4, rtol=0)
    # seq_len 0 rows are untouched by the reference kernel (zeros here)
    assert not want[~live].any()


def test_rmsnorm_matches_reference_golden(golden):
    r = golden_inputs("rms_f16")
    want = golden["ref"]["rms_f16_out"]
    got = N.rms_norm("f16", r["x"], r["w"], r["eps"])
    diff = np.abs(N.f16_bits_to_f32(got) - N.f16_bits_to_f32(want))
    # identical up to the reduction order of sum(x^2): at most one f16 ulp
    ulp = np.abs(N.f16_bits_to_f32(want)) * 2.0 ** -10 + 2.0 ** -24
    assert (diff <= ulp * 1.01).all()
    assert (got != want).mean() < 0.01


def test_rope_matches_reference_golden(golden):
    ro = golden_inputs("rope_f16")
    n = ro["q"].shape[0]
    q = N.rope("f16", ro["q"], np.full(n, ro["pos"]), 10000.0, 0)
    k = N.rope("f16", ro["k"], np.full(n, ro["pos"]), 10000.0, 0)
    for got, key in ((q, "rope_f16_q"), (k, "rope_f16_k")):
        want = golden["ref"][key]
        diff = np.abs(N.f16_bits_to_f32(got) - N.f16_bits_to_f32(want))
        assert diff.max() <= 2e-3, key
        assert (got != want).mean() < 0.01, key


@pytest.mark.parametrize("case", ["kv_write_f16", "kv_write_f16_oob"])
def test_slot_write_matches_reference_golden(golden, case):
    w = golden_inputs(case)
    va_k = np.zeros(w["nb"] * w["bs"] * w["step"], np.uint16)
    va_v = np.zeros_like(va_k)
    st = N.slot_write(va_k, va_v, w["slots"], w["offsets"], w["valid"], w["k"], w["v"],
                      step=w["step"], bs=w["bs"])
    assert st == int(golden["ref"][f"{case}_status"][0])
    assert np.array_equal(va_k, golden["ref"][f"{case}_va_k"])
    assert np.array_equal(va_v, golden["ref"][f"{case}_va_v"])


def test_decode_v_row_kat(golden):
    """k = arange+100, v = arange+1000, q = 0, seq_len 1, scale 1 -> out == V row."""
    B, hq, hkv, D, bs = 2, 4, 2, 64, 16
    nb = 4
    step = hkv * D
    va_k = N.f32_to_f16_bits((np.arange(nb * bs * step) % 512 + 100).astype(np.float32))
    va_v = N.f32_to_f16_bits((np.arange(nb * bs * step) % 512 + 1000).astype(np.float32))
    offsets = np.arange(nb, dtype=np.uint64) * np.uint64(bs * step)
    tables = np.array([[2, 0], [3, 1]], np.int32)
    seq = np.ones(B, np.int32)
    q = np.zeros(B * hq * D, np.uint16)
    got = N.paged_attn("f16", q, va_k, va_v, tables, seq, offsets, hq=hq, hkv=hkv, d=D, bs=bs,
                       max_bps=2, scale=1.0)
    for b in range(B):
        for h in range(hq):
            kvh = h * hkv // hq
            e = int(offsets[tables[b, 0]]) + kvh * D
            np.testing.assert_array_equal(got[b, h], N.f16_bits_to_f32(va_v[e:e + D]))


@ref
@pytest.mark.parametrize("seed", [0, 1])
@pytest.mark.parametrize("shape", [(3, 4, 4, 64, 16), (2, 8, 2, 128, 16), (2, 6, 3, 96, 32),
                                   (2, 5, 2, 64, 8)])
def test_attention_vs_reference_kernel(seed, shape):
    B, hq, hkv, D, bs = shape
    rng = np.random.default_rng(seed)
    max_bps, nb = 12, 40
    seq = rng.integers(0, max_bps * bs + 1, B).astype(np.int32)
    tables = rng.permutation(nb)[: B * max_bps].reshape(B, max_bps).astype(np.int32)
    step = hkv * D
    offsets = rng.permutation(nb).astype(np.uint64) * np.uint64(bs * step)
    va_k = N.f32_to_f16_bits(rng.standard_normal(nb * bs * step).astype(np.float32))
    va_v = N.f32_to_f16_bits(rng.standard_normal(nb * bs * step).astype(np.float32))
    q = N.f32_to_f16_bits(rng.standard_normal(B * hq * D).astype(np.float32))
    kw = dict(hq=hq, hkv=hkv, d=D, bs=bs, max_bps=max_bps, scale=D ** -0.5)
    want = N.f16_bits_to_f32(N.ref_paged_attn("f16", q, va_k, va_v, tables, seq, offsets, **kw))
    got = N.paged_attn("f16", q, va_k, va_v, tables, seq, offsets, **kw)
    live = seq > 0
    np.testing.assert_allclose(got[live], want.reshape(got.shape)[live], atol=6e-4, rtol=0)


@ref
def test_fused_contract_equals_reference_composition():
    """The fused op's contract = rms_norm -> rope -> slot write of the reference kernels
    (f16, one position, reference rope mode, base 10000), here through the oracle."""
    rng = np.random.default_rng(3)
    T, H, hq, hkv, D, bs = 3, 512, 4, 2, 64, 16
    x = N.f32_to_f16_bits(rng.standard_normal((T, H)).astype(np.float32))
    w = N.f32_to_f16_bits(rng.uniform(0.5, 1.5, H).astype(np.float32))
    q = N.f32_to_f16_bits(rng.standard_normal((T, hq, D)).astype(np.float32))
    k = N.f32_to_f16_bits(rng.standard_normal((T, hkv, D)).astype(np.float32))
    pos = 321
    ref_norm = N.ref_rms_norm(x, w, 1e-5)
    rq, rk = N.ref_rope(q, k, pos)
    on = N.rms_norm("f16", x, w, 1e-5)
    oq = N.rope("f16", q, np.full(T, pos), 10000.0, 0)
    ok = N.rope("f16", k, np.full(T, pos), 10000.0, 0)
    assert np.abs(N.f16_bits_to_f32(on) - N.f16_bits_to_f32(ref_norm)).max() <= 4e-3
    assert np.abs(N.f16_bits_to_f32(oq) - N.f16_bits_to_f32(rq)).max() <= 4e-3
    assert np.abs(N.f16_bits_to_f32(ok) - N.f16_bits_to_f32(rk)).max() <= 4e-3


def test_rope_modes_and_theta():
    """GPT-J / NeoX rotations against a direct numpy statement; base is honoured."""
    rng = np.random.default_rng(11)
    T, H, D = 4, 3, 16
    x = rng.standard_normal((T, H, D)).astype(np.float32)
    pos = np.array([0, 5, 100, 8191], np.int32)
    xb = N.f32_to_bf16_bits(x)
    xf = N.bf16_bits_to_f32(xb).astype(np.float64)
    for mode in (1, 2):
        got = N.bf16_bits_to_f32(N.rope("bf16", xb, pos, 500000.0, mode))
        inv = 1.0 / (500000.0 ** (np.arange(0, D, 2) / D))
        ang = pos[:, None] * inv[None, :]
        c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
        if mode == 1:
            x0, x1 = xf[..., 0::2], xf[..., 1::2]
        else:
            x0, x1 = xf[..., : D // 2], xf[..., D // 2:]
        y0, y1 = x0 * c - x1 * s, x0 * s + x1 * c
        want = np.empty_like(xf)
        if mode == 1:
            want[..., 0::2], want[..., 1::2] = y0, y1
        else:
            want[..., : D // 2], want[..., D // 2:] = y0, y1
        np.testing.assert_allclose(got, want, atol=2e-3, rtol=1e-2)


def test_prefill_oracle_rows_are_decode_steps():
    """Pins the prefill restatement to the decode one (itself pinned to the reference
    kernel): chunk row i equals decode over the first ctx - chunk + i + 1 keys."""
    from oracle import native as N

    rng = np.random.default_rng(3)
    hq, hkv, d, bs = 8, 2, 64, 16
    ctx, chunk = np.array([70, 45], np.int32), np.array([9, 45], np.int32)
    nblk = 8
    tables = np.stack([rng.permutation(nblk)[:5], rng.permutation(nblk)[:5]]).astype(np.int32)
    step = hkv * d
    offsets = np.arange(nblk, dtype=np.uint64) * np.uint64(bs * step)
    va_k = N.f32_to_bf16_bits(rng.standard_normal(nblk * bs * step).astype(np.float32))
    va_v = N.f32_to_bf16_bits(rng.standard_normal(nblk * bs * step).astype(np.float32))
    qs = np.array([0, 9, 54], np.int32)
    q = N.f32_to_bf16_bits(rng.standard_normal((54, hq * d)).astype(np.float32))
    got = N.paged_prefill("bf16", q, va_k, va_v, tables, qs, ctx, offsets, hq=hq, hkv=hkv, d=d,
                          bs=bs, max_bps=5, scale=0.125)
    for b in range(2):
        for i in range(int(chunk[b])):
            tok = qs[b] + i
            L = int(ctx[b] - chunk[b] + i + 1)
            ref = N.paged_attn("bf16", q[tok:tok + 1], va_k, va_v, tables[b:b + 1],
                               np.array([L], np.int32), offsets, hq=hq, hkv=hkv, d=d, bs=bs,
                               max_bps=5, scale=0.125)
            np.testing.assert_allclose(got[tok], ref[0], rtol=1e-6, atol=1e-6)
