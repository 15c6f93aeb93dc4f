"""TEST INFRASTRUCTURE -- ctypes access to the C oracle and to oracle/_ref.

`liboracle.so` is the C restatement (kcmm_oracle.c).  `libref_kernels.so` is
the reference's own CUDA kernel sources compiled as host C++ (ref_host.cpp);
it exists only where the reference tree was available at build time, and the
tests that need it skip otherwise.  Arrays are numpy; 16-bit float data is
carried as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_kernels.so"
DT = {"f16": 0, "bf16": 1, "f32": 2}


def reference_root() -> Path | None:
    """The reference checkout whose kernel sources oracle/_ref compiles: $REF_ROOT,
    else a checkout named `reference` beside this repository; None when neither
    holds `src/cuda/kernels` (GPU machines carry no reference tree)."""
    env = os.environ.get("REF_ROOT")
    cand = Path(env) if env else HERE.parent.parent / "reference"
    return cand if (cand / "src" / "cuda" / "kernels").is_dir() else None


def build(ref: bool | None = None) -> None:
    """Build liboracle (always) and oracle/_ref (when a reference checkout is found)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    root = reference_root()
    if ref is None:
        ref = root is not None
    if ref:
        if root is None:
            raise RuntimeError("oracle/_ref needs the reference checkout: set REF_ROOT")
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_ROOT={root}"], check=True)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


_oracle = None
_ref = None


def oracle_lib():
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            build(ref=False)
        _oracle = ctypes.CDLL(str(ORACLE_LIB))
        _oracle.oracle_fused_norm_rope_append.restype = ctypes.c_int32
        _oracle.oracle_slot_write.restype = ctypes.c_int32
        _oracle.oracle_f32_to_bf16.restype = ctypes.c_uint16
        _oracle.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
    return _oracle


def ref_available() -> bool:
    return REF_LIB.exists()


def ref_lib():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} not built (needs the reference tree at build time)")
        _ref = ctypes.CDLL(str(REF_LIB))
    return _ref


# --- 16-bit helpers ---------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def bits_to_f32(dtype: str, b: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(b) if dtype == "bf16" else f16_bits_to_f32(b)


def f32_to_bits(dtype: str, x: np.ndarray) -> np.ndarray:
    return f32_to_bf16_bits(x) if dtype == "bf16" else f32_to_f16_bits(x)


# --- oracle entry points ----------------------------------------------------

def paged_attn(dtype: str, q, va_k, va_v, tables, seq_lens, offsets, *, hq, hkv, d, bs,
               max_bps, scale, out=None):
    """Returns the fp32 result [B, hq, d] (rows with seq_len <= 0 hold `out`'s values
    converted, or zeros when out is None)."""
    B = len(seq_lens)
    out_f32 = np.zeros((B, hq, d), np.float32)
    if out is not None:
        out_f32[:] = (bits_to_f32(dtype, out) if dtype != "f32" else out).reshape(B, hq, d)
    lib = oracle_lib()
    lib.oracle_paged_attn(
        ctypes.c_int(DT[dtype]), _ptr(q), None, _ptr(out_f32), _ptr(va_k), _ptr(va_v),
        _ptr(np.ascontiguousarray(tables, np.int32)), _ptr(np.ascontiguousarray(seq_lens, np.int32)),
        _ptr(np.ascontiguousarray(offsets, np.uint64)), ctypes.c_int(B), ctypes.c_int(hq),
        ctypes.c_int(hkv), ctypes.c_int(d), ctypes.c_int(bs), ctypes.c_int(max_bps),
        ctypes.c_float(scale))
    return out_f32


def paged_prefill(dtype: str, q, va_k, va_v, tables, q_start, ctx_lens, offsets, *, hq, hkv,
                  d, bs, max_bps, scale, token_mask=None):
    """Causal chunked-prefill attention; q bits [total_tokens, hq*d].  Returns fp32
    [total_tokens, hq, d]; tokens with token_mask == 0 are left at zero."""
    q_start = np.ascontiguousarray(q_start, np.int32)
    total = int(q_start[-1])
    out_f32 = np.zeros((total, hq, d), np.float32)
    mask = None if token_mask is None else np.ascontiguousarray(token_mask, np.uint8)
    oracle_lib().oracle_paged_prefill(
        ctypes.c_int(DT[dtype]), _ptr(q), _ptr(out_f32), _ptr(va_k), _ptr(va_v),
        _ptr(np.ascontiguousarray(tables, np.int32)), _ptr(q_start),
        _ptr(np.ascontiguousarray(ctx_lens, np.int32)),
        _ptr(np.ascontiguousarray(offsets, np.uint64)), _ptr(mask) if mask is not None else None,
        ctypes.c_int(len(q_start) - 1), ctypes.c_int(hq), ctypes.c_int(hkv), ctypes.c_int(d),
        ctypes.c_int(bs), ctypes.c_int(max_bps), ctypes.c_float(scale))
    return out_f32


def rms_norm(dtype: str, x, w, eps: float):
    rows, cols = x.shape
    y = np.zeros_like(x)
    oracle_lib().oracle_rms_norm(ctypes.c_int(DT[dtype]), _ptr(x), _ptr(w), _ptr(y),
                                 ctypes.c_int(rows), ctypes.c_int(cols), ctypes.c_float(eps))
    return y


def rope(dtype: str, x, positions, base: float, mode: int):
    """x [tokens, heads, d] (copied, rotated copy returned)."""
    x = np.ascontiguousarray(x).copy()
    t, h, d = x.shape
    oracle_lib().oracle_rope(ctypes.c_int(DT[dtype]), _ptr(x), ctypes.c_int(t), ctypes.c_int(h),
                             ctypes.c_int(d), _ptr(np.ascontiguousarray(positions, np.int32)),
                             ctypes.c_float(base), ctypes.c_int(mode))
    return x


def slot_write(va_k, va_v, slots, offsets, valid, k_src, v_src, *, step, bs):
    rows = len(slots)
    return int(oracle_lib().oracle_slot_write(
        _ptr(va_k), _ptr(va_v), _ptr(np.ascontiguousarray(slots, np.int64)),
        _ptr(np.ascontiguousarray(offsets, np.uint64)),
        _ptr(None if valid is None else np.ascontiguousarray(valid, np.uint8)),
        ctypes.c_int(len(offsets)), _ptr(k_src), _ptr(v_src), ctypes.c_int(rows),
        ctypes.c_int(step), ctypes.c_int(bs)))


def fused_norm_rope_append(x, w, q, k, v, positions, slots, offsets, valid, va_k, va_v, *,
                           eps, base, mode, hkv, d, bs):
    """bf16 bit arrays.  Returns (normed, q_rot, status); va_k/va_v updated in place."""
    T, H = x.shape
    hq = q.shape[1]
    normed = np.zeros_like(x)
    q = np.ascontiguousarray(q).copy()
    st = oracle_lib().oracle_fused_norm_rope_append(
        _ptr(x), _ptr(w), _ptr(normed), ctypes.c_int(T), ctypes.c_int(H), ctypes.c_float(eps),
        _ptr(q), ctypes.c_int(hq), _ptr(k), _ptr(v), _ptr(np.ascontiguousarray(positions, np.int32)),
        ctypes.c_float(base), ctypes.c_int(mode), _ptr(np.ascontiguousarray(slots, np.int64)),
        _ptr(np.ascontiguousarray(offsets, np.uint64)),
        _ptr(None if valid is None else np.ascontiguousarray(valid, np.uint8)),
        ctypes.c_int(len(offsets)), ctypes.c_int(hkv), ctypes.c_int(d), ctypes.c_int(bs),
        _ptr(va_k), _ptr(va_v))
    return normed, q, int(st)


# --- the reference's own kernels on the host (oracle/_ref) -------------------

def ref_paged_attn(dtype: str, q, va_k, va_v, tables, seq_lens, offsets, *, hq, hkv, d, bs,
                   max_bps, scale, out=None, workers: int = 1):
    """dtype "f16"/"bf16": 16-bit bit arrays; "f32": float32 arrays, the reference
    source built over fp32 storage, which reads `offsets` as element indices."""
    B = len(seq_lens)
    if out is None:
        out = np.zeros((B, hq, d), np.float32 if dtype == "f32" else np.uint16)
    fn = {"bf16": ref_lib().ref_paged_attn_bf16, "f16": ref_lib().ref_paged_attn_f16,
          "f32": ref_lib().ref_paged_attn_f32}[dtype]
    fn(_ptr(q), _ptr(va_k), _ptr(va_v), _ptr(np.ascontiguousarray(tables, np.int32)),
       _ptr(np.ascontiguousarray(seq_lens, np.int32)), _ptr(np.ascontiguousarray(offsets, np.uint64)),
       _ptr(out), ctypes.c_int(B), ctypes.c_int(hq), ctypes.c_int(hkv), ctypes.c_int(d),
       ctypes.c_int(bs), ctypes.c_int(max_bps), ctypes.c_float(scale), ctypes.c_int(workers))
    return out


def ref_paged_attn_engine(q, va_k, va_v, tables, seq_lens, offsets, *, hq, hkv, d, bs, max_bps,
                          workers: int = 1):
    B = len(seq_lens)
    out = np.zeros((B, hq, d), np.uint16)
    ref_lib().ref_paged_attn_engine_f16(
        _ptr(q), _ptr(va_k), _ptr(va_v), _ptr(np.ascontiguousarray(tables, np.int32)),
        _ptr(np.ascontiguousarray(seq_lens, np.int32)), _ptr(np.ascontiguousarray(offsets, np.uint64)),
        _ptr(out), ctypes.c_int(B), ctypes.c_int(hq), ctypes.c_int(hkv), ctypes.c_int(d),
        ctypes.c_int(bs), ctypes.c_int(max_bps), ctypes.c_int(workers))
    return out


def ref_kv_write_slots(va_k, va_v, slots, offsets, valid, k_src, v_src, *, step, bs):
    status = np.zeros(1, np.int32)
    ref_lib().ref_kv_write_slots_f16(
        _ptr(va_k), _ptr(va_v), _ptr(np.ascontiguousarray(slots, np.int64)),
        _ptr(np.ascontiguousarray(offsets, np.uint64)),
        _ptr(None if valid is None else np.ascontiguousarray(valid, np.uint8)), _ptr(k_src),
        _ptr(v_src), _ptr(status), ctypes.c_int(len(slots)), ctypes.c_int(step), ctypes.c_int(bs),
        ctypes.c_int(len(offsets)))
    return int(status[0])


def ref_rms_norm(x, w, eps: float, workers: int = 1):
    rows, cols = x.shape
    y = np.zeros_like(x)
    ref_lib().ref_rms_norm_f16(_ptr(x), _ptr(w), _ptr(y), ctypes.c_int(rows), ctypes.c_int(cols),
                               ctypes.c_float(eps), ctypes.c_int(workers))
    return y


def ref_rope(q, k, pos: int):
    """q [B, hq, d], k [B, hkv, d] f16 bits; rotated copies (base 10000, one position)."""
    q = np.ascontiguousarray(q).copy()
    k = np.ascontiguousarray(k).copy()
    B, hq, d = q.shape
    ref_lib().ref_rope_f16(_ptr(q), _ptr(k), ctypes.c_int(B), ctypes.c_int(hq),
                           ctypes.c_int(k.shape[1]), ctypes.c_int(d // 2), ctypes.c_int(pos))
    return q, k
