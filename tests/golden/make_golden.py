"""Regenerate the golden fixtures in tests/golden/ (run where the reference tree exists).

Two kinds of fixtures:

1. reference_kats.json -- known-answer values transcribed from the
   reference's own unit tests (each entry names the file:line it comes from).
2. ref_kernels.npz -- outputs of the reference's own CUDA kernels (compiled
   for the host from their sources by oracle/Makefile -> oracle/_ref) on small
   seeded inputs.  The inputs are regenerated from the seeds by
   `golden_inputs()` below, so only outputs are stored.

Usage:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import native as N  # noqa: E402

KATS = {
    "superblock_sizing": {
        "source": "src/kcmm/superblock.rs:188-205,244-251,287-301",
        "cases": [
            {"elem_count": 8192, "block_bytes": 16384, "blocks_per_superblock": 128},
            {"elem_count": 4096, "block_bytes": 8192, "blocks_per_superblock": 256},
            {"block_bytes": 65536, "blocks_per_superblock": 32},
            {"block_bytes": 5120, "blocks_per_superblock": 409, "tail_padding": 3072,
             "max_block_index": 408},
        ],
        "rejected_block_bytes": [4194304],
    },
    "lifo_reuse": {
        "source": "src/kcmm/superblock.rs:430-447",
        "block_bytes": 65536,
        "note": "alloc h1,h2; free h1,h2; re-alloc returns h2 then h1",
    },
    "address_formulas": {
        "source": "src/cache/paged_kv.rs:829-867",
        "block_size": 16, "kv_heads": 4, "head_dim": 128,
        "block_bytes": 16384,
        "pos47": {"logical_block": 2, "offset_in_block": 15,
                  "dst_off_phys7": 7 * 16 * 512 + 15 * 512},
        "table": [3, 7, 1],
        "pos25": {"logical_block": 1, "offset_in_block": 9, "phys": 7,
                  "dst_off": 7 * 16 * 512 + 9 * 512},
        "max_blocks": {"max_seq_len": 2048, "max_blocks_per_seq": 128, "max_batch": 8,
                       "max_blocks_total": 1024},
    },
    "capacity": {
        "source": "src/kcmm/pool.rs:2245-2295",
        "num_layers": 2, "kv_heads": 32, "head_dim": 64, "max_batch": 1, "max_seq_len": 16,
        "max_blocks_total": 1, "blocks_per_superblock": 32, "max_physical_blocks_per_layer": 32,
        "error_contains": "physical block capacity exhausted",
    },
    "config_layout": {
        "source": "src/kcmm/ffi.rs:2575-2603, examples/kcmm_c_integration.c:30",
        "size": 376,
        "offsets": {"max_seq_len": 336, "low_watermark_threshold": 344,
                    "background_evict_interval_ms": 352, "attention_sink_blocks": 360,
                    "recent_window_blocks": 368},
    },
    "decode_v_row": {
        "source": "scripts/kcmm/non_default_stream_ffi_smoke.py:172-179,250-345",
        "note": "k = arange + 100, v = arange + 1000, q = 0, seq_len 1, scale 1 "
                "-> out[b,h,:] == V row of kv head h*Hkv/Hq, exactly",
    },
    "cpu_slot_allocator": {
        "source": "src/kcmm/tiering.rs:2578-2745",
        "cases": [
            {"total": 1024, "ops": [["alloc", 1024, 0]], "free_ranges": []},
            {"total": 1024, "ops": [["alloc", 256, 0]], "free_ranges": [[256, 1024]]},
            {"total": 1024, "ops": [["alloc", 0, None]], "free_ranges": [[0, 1024]]},
            {"total": 64, "ops": [["alloc", 64, 0], ["alloc", 1, None]], "free_ranges": []},
            {"total": 640, "initial": [[0, 64], [128, 256], [320, 640]],
             "ops": [["alloc", 48, 0]], "free_ranges": [[48, 64], [128, 256], [320, 640]]},
            {"total": 1024, "ops": [["alloc", 256, 0], ["free", 0, 256]],
             "free_ranges": [[0, 1024]]},
            {"total": 1024, "ops": [["alloc", 256, 0], ["alloc", 256, 256], ["free", 0, 256],
                                    ["free", 256, 256]], "free_ranges": [[0, 1024]]},
            {"total": 1024, "ops": [["alloc", 256, 0], ["alloc", 256, 256], ["alloc", 256, 512],
                                    ["free", 512, 256]], "free_ranges": [[512, 1024]]},
            {"total": 1024, "ops": [["alloc", 256, 0], ["alloc", 256, 256], ["alloc", 256, 512],
                                    ["free", 0, 256], ["free", 512, 256], ["free", 256, 256]],
             "free_ranges": [[0, 1024]]},
            {"total": 1024, "ops": [["free", 100, 0]], "free_ranges": [[0, 1024]]},
            {"total": 1024, "ops": [["alloc", 128, 0], ["alloc", 256, 128], ["alloc", 512, 384]],
             "free_ranges": [[896, 1024]]},
            {"total": 1024, "ops": [["alloc", 512, 0], ["alloc", 512, 512], ["free", 0, 512],
                                    ["alloc", 256, 0]], "free_ranges": [[256, 512]]},
        ],
    },
    "write_then_free": {
        "source": "scripts/kcmm/kv_write_ffi_smoke.py:180-425",
        "note": "alloc 3 blocks, free the first: valid table = [0,1,1]; writes at positions "
                "[0, bs+1] and at the equivalent slots produce identical page bytes",
    },
}


def golden_inputs(case: str):
    """Seeded inputs of each kernel fixture (shared with the tests)."""
    if case == "attn_f16":
        rng = np.random.default_rng(1234)
        B, hq, hkv, D, bs, nb = 4, 8, 2, 64, 16, 96
        max_bps = 20
        seq = np.array([257, 1, 0, 300], np.int32)
        perm = rng.permutation(nb).astype(np.int32)
        tables = perm[: B * max_bps].reshape(B, max_bps)
        step = hkv * D
        offsets = np.arange(nb, dtype=np.uint64) * np.uint64(bs * step)
        va_k = N.f32_to_f16_bits(rng.standard_normal(nb * bs * step).astype(np.float32))
        va_v = N.f32_to_f16_bits(rng.standard_normal(nb * bs * step).astype(np.float32))
        q = N.f32_to_f16_bits(rng.standard_normal(B * hq * D).astype(np.float32))
        return dict(B=B, hq=hq, hkv=hkv, D=D, bs=bs, max_bps=max_bps, seq=seq, tables=tables,
                    offsets=offsets, va_k=va_k, va_v=va_v, q=q, scale=D ** -0.5)
    if case == "rms_f16":
        rng = np.random.default_rng(99)
        x = N.f32_to_f16_bits(rng.standard_normal((6, 4096)).astype(np.float32))
        w = N.f32_to_f16_bits(rng.uniform(0.5, 1.5, 4096).astype(np.float32))
        return dict(x=x, w=w, eps=1e-5)
    if case == "rope_f16":
        rng = np.random.default_rng(7)
        q = N.f32_to_f16_bits(rng.standard_normal((3, 8, 128)).astype(np.float32))
        k = N.f32_to_f16_bits(rng.standard_normal((3, 2, 128)).astype(np.float32))
        return dict(q=q, k=k, pos=777)
    if case in ("kv_write_f16", "kv_write_f16_oob"):
        rng = np.random.default_rng(5)
        nb, bs, step = 12, 16, 256
        offsets = np.arange(nb, dtype=np.uint64) * np.uint64(bs * step)
        valid = np.ones(nb, np.uint8)
        valid[3] = 0
        if case == "kv_write_f16":  # row 3 hits block 3, marked free -> status 2
            slots = np.array([0, 17, -1, 3 * 16 + 4, 5 * 16 + 3, 11 * 16 + 15, 2], np.int64)
        else:  # row 1 hits block 12 >= table length -> status 1
            slots = np.array([0, 12 * 16, 5], np.int64)
        k = N.f32_to_f16_bits(rng.standard_normal((len(slots), step)).astype(np.float32))
        v = N.f32_to_f16_bits(rng.standard_normal((len(slots), step)).astype(np.float32))
        return dict(nb=nb, bs=bs, step=step, offsets=offsets, valid=valid, slots=slots, k=k, v=v)
    raise KeyError(case)


def main() -> None:
    (HERE / "reference_kats.json").write_text(json.dumps(KATS, indent=1) + "\n")
    if not N.ref_available():
        N.build(ref=True)
    out = {}
    a = golden_inputs("attn_f16")
    out["attn_f16_out"] = N.ref_paged_attn(
        "f16", a["q"], a["va_k"], a["va_v"], a["tables"], a["seq"], a["offsets"], hq=a["hq"],
        hkv=a["hkv"], d=a["D"], bs=a["bs"], max_bps=a["max_bps"], scale=a["scale"])
    r = golden_inputs("rms_f16")
    out["rms_f16_out"] = N.ref_rms_norm(r["x"], r["w"], r["eps"])
    ro = golden_inputs("rope_f16")
    out["rope_f16_q"], out["rope_f16_k"] = N.ref_rope(ro["q"], ro["k"], ro["pos"])
    for case in ("kv_write_f16", "kv_write_f16_oob"):
        w = golden_inputs(case)
        va_k = np.zeros(w["nb"] * w["bs"] * w["step"], np.uint16)
        va_v = np.zeros_like(va_k)
        st = N.ref_kv_write_slots(va_k, va_v, w["slots"], w["offsets"], w["valid"], w["k"],
                                  w["v"], step=w["step"], bs=w["bs"])
        out[f"{case}_va_k"], out[f"{case}_va_v"] = va_k, va_v
        out[f"{case}_status"] = np.array([st], np.int32)
    np.savez_compressed(HERE / "ref_kernels.npz", **out)
    print("wrote", HERE / "reference_kats.json", HERE / "ref_kernels.npz")


if __name__ == "__main__":
    main()
