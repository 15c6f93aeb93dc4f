"""ctypes binding of the B200 KCMM library (`libkcmm.so`).

Mirrors the reference's Python seam (ref scripts/kcmm/bindings.py:17-429):
the same class names (`KcmmError`, `KcmmConfig`, `KcmmMetrics`,
`KcmmPoolStats`, `BlockLocation`, `KcmmLibrary`, `KcmmPool`), the same
struct layouts with the same layout assertion, and pool methods with the same
names, argument meaning and error behaviour (a failing call raises
`KcmmError` carrying the pool's last error).  Methods for the B200 additions
(bf16 decode, fused norm/rope/append, refcount/CoW, swap) follow the same
pattern.

There is no fallback: if the native library is missing the import of
`KcmmLibrary()` raises.  Device buffers are passed as integer addresses, so
any framework (torch here, in tests and the bench) can own them.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent


class KcmmError(RuntimeError):
    """A KCMM C API call reported failure."""


class KcmmConfig(ctypes.Structure):
    _fields_ = [
        ("block_size", ctypes.c_size_t),
        ("max_blocks", ctypes.c_size_t),
        ("cpu_cache_path", ctypes.c_char * 256),
        ("tiering", ctypes.c_int32),
        ("eviction_policy", ctypes.c_int32),
        ("prefetch_window", ctypes.c_size_t),
        ("max_batch_blocks", ctypes.c_size_t),
        ("device_ordinal", ctypes.c_size_t),
        ("num_layers", ctypes.c_size_t),
        ("kv_heads", ctypes.c_size_t),
        ("head_dim", ctypes.c_size_t),
        ("max_batch", ctypes.c_size_t),
        ("max_seq_len", ctypes.c_size_t),
        ("low_watermark_threshold", ctypes.c_float),
        ("background_evict_interval_ms", ctypes.c_uint64),
        ("attention_sink_blocks", ctypes.c_size_t),
        ("recent_window_blocks", ctypes.c_size_t),
    ]


class KcmmMetrics(ctypes.Structure):
    _fields_ = [
        ("ifr", ctypes.c_double),
        ("pme", ctypes.c_double),
        ("bu", ctypes.c_double),
        ("rfi", ctypes.c_double),
        ("gpu_blocks", ctypes.c_uint64),
        ("cpu_blocks", ctypes.c_uint64),
        ("nvme_blocks", ctypes.c_uint64),
        ("eviction_count", ctypes.c_uint64),
        ("restoration_count", ctypes.c_uint64),
    ]


class KcmmLatencyHistogram(ctypes.Structure):
    _fields_ = [("count", ctypes.c_uint64), ("sum_us", ctypes.c_uint64),
                ("min_us", ctypes.c_uint64), ("max_us", ctypes.c_uint64),
                ("buckets", ctypes.c_uint64 * 9)]


class KcmmMetricsExt(ctypes.Structure):
    _fields_ = [("base", KcmmMetrics), ("evicted_blocks_total", ctypes.c_uint64),
                ("restored_blocks_total", ctypes.c_uint64),
                ("eviction_failures", ctypes.c_uint64),
                ("restoration_failures", ctypes.c_uint64),
                ("background_eviction_count", ctypes.c_uint64),
                ("eviction_latency", KcmmLatencyHistogram),
                ("restoration_latency", KcmmLatencyHistogram)]


class KcmmPolicyStats(ctypes.Structure):
    _fields_ = [("eviction_count", ctypes.c_uint64), ("restoration_count", ctypes.c_uint64),
                ("evicted_blocks", ctypes.c_uint64), ("restored_blocks", ctypes.c_uint64),
                ("avg_evict_batch_size", ctypes.c_double)]


class KcmmPoolStats(ctypes.Structure):
    _fields_ = [
        ("blocks_in_use", ctypes.c_uint32),
        ("total_blocks", ctypes.c_uint32),
        ("total_physical_blocks", ctypes.c_uint32),
        ("free_physical_blocks", ctypes.c_uint32),
        ("active_sequences", ctypes.c_uint32),
        ("num_layers", ctypes.c_uint32),
        ("blocks_per_superblock", ctypes.c_uint32),
        ("superblock_count", ctypes.c_uint32),
        ("block_size", ctypes.c_uint32),
        ("max_blocks_per_seq", ctypes.c_uint32),
        ("block_bytes", ctypes.c_uint32),
        ("tiering_enabled", ctypes.c_int32),
        ("sharing_enabled", ctypes.c_int32),
        ("physical_idle_ratio", ctypes.c_float),
    ]


class BlockLocation:
    GPU_RESIDENT = 0
    CPU_RESIDENT = 1
    NVME_RESIDENT = 2
    EVICTING = 3
    RESTORING = 4
    _NAMES = {0: "gpu", 1: "cpu", 2: "nvme", 3: "evicting", 4: "restoring"}

    @classmethod
    def name(cls, value: int) -> str:
        return cls._NAMES.get(value, f"unknown({value})")


class RopeMode:
    REFERENCE = 0
    GPTJ = 1
    NEOX = 2


def assert_layout() -> None:
    """The config struct must match the C header byte for byte on LP64."""
    if ctypes.sizeof(ctypes.c_size_t) != 8:
        return
    expected = {
        "max_seq_len": 336,
        "low_watermark_threshold": 344,
        "background_evict_interval_ms": 352,
        "attention_sink_blocks": 360,
        "recent_window_blocks": 368,
    }
    if ctypes.sizeof(KcmmConfig) != 376:
        raise KcmmError(f"kcmm_config_t size {ctypes.sizeof(KcmmConfig)} != 376")
    for name, off in expected.items():
        got = getattr(KcmmConfig, name).offset
        if got != off:
            raise KcmmError(f"kcmm_config_t.{name} at offset {got}, expected {off}")


def library_path() -> Path:
    env = os.environ.get("KCMM_LIB_PATH")
    path = Path(env) if env else _PKG / "libkcmm.so"
    if not path.exists():
        raise KcmmError(
            f"KCMM native library not found at {path}; build it with "
            "`python -m lattice_b200.build` (nvcc, sm_100a)"
        )
    return path


u32, u64, i32, i64, f32 = (ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32, ctypes.c_int64,
                         ctypes.c_float)
P = ctypes.c_void_p
pu32 = ctypes.POINTER(ctypes.c_uint32)
pu64 = ctypes.POINTER(ctypes.c_uint64)
pi64 = ctypes.POINTER(ctypes.c_int64)
pu8 = ctypes.POINTER(ctypes.c_uint8)

# name -> (restype, argtypes); every symbol declared in include/kcmm.h
SIGNATURES: dict[str, tuple] = {
    "kcmm_pool_create": (P, [ctypes.POINTER(KcmmConfig)]),
    "kcmm_pool_destroy": (None, [P]),
    "kcmm_get_last_error": (ctypes.c_size_t, [P, ctypes.c_char_p, ctypes.c_size_t]),
    "kcmm_clear_error": (None, [P]),
    "kcmm_alloc_blocks": (i32, [P, u32, pu32]),
    "kcmm_free_blocks": (i32, [P, pu32, u32]),
    "kcmm_register_sequence": (i32, [P, pu32, u32, pu32]),
    "kcmm_unregister_sequence": (i32, [P, u32]),
    "kcmm_touch": (None, [P, u32]),
    "kcmm_cool": (None, [P, u32]),
    "kcmm_update_seq_len": (None, [P, u32, u32]),
    "kcmm_get_seq_len": (u32, [P, u32]),
    "kcmm_append_block_to_sequence": (i32, [P, u32, u32]),
    "kcmm_get_block_table": (i32, [P, u32, pu32, u32, pu32]),
    "kcmm_get_block_va_offset": (u64, [P, u32]),
    "kcmm_get_all_block_offsets_f16": (i32, [P, pu64, u32, pu32]),
    "kcmm_get_all_block_valid": (i32, [P, pu8, u32, pu32]),
    "kcmm_get_block_location": (i32, [P, u32, ctypes.POINTER(ctypes.c_int)]),
    "kcmm_get_block_table_va_offsets": (i32, [P, u32, pu64, u32, pu32]),
    "kcmm_get_va_k": (u64, [P, u32]),
    "kcmm_get_va_v": (u64, [P, u32]),
    "kcmm_block_state_epoch": (u64, [P]),
    "kcmm_append_kv_step": (i32, [P, u32, pu32, pu32, u32, u64, u64]),
    "kcmm_append_kv_slots": (i32, [P, u32, pi64, u32, u64, u64]),
    "kcmm_append_kv_slots_on_stream": (i32, [P, u32, pi64, u32, u64, u64, u64]),
    "kcmm_append_kv_device_slots_on_stream":
        (i32, [P, u32, u64, u64, u64, u32, u32, u64, u64, u64, u64]),
    "kcmm_precompile_vllm_kv_write_f16": (i32, [P]),
    "kcmm_paged_attn_decode_f16":
        (i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32]),
    "kcmm_paged_attn_decode_f16_on_stream":
        (i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64]),
    "kcmm_paged_attn_decode_f16_on_current_context_stream":
        (i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64]),
    "kcmm_precompile_paged_attn_decode_f16": (i32, [P]),
    "kcmm_evict_blocks": (u32, [P, u32]),
    "kcmm_restore_evicted_block": (u64, [P, u32]),
    "kcmm_restore_evicted_blocks": (i32, [P, pu32, u32]),
    "kcmm_is_gpu_resident": (i32, [P, u32]),
    "kcmm_get_metrics": (i32, [P, ctypes.POINTER(KcmmMetrics)]),
    "kcmm_get_pool_stats": (i32, [P, ctypes.POINTER(KcmmPoolStats)]),
    "kcmm_blocks_in_use": (u32, [P]),
    "kcmm_total_blocks": (u32, [P]),
    "kcmm_free_physical_blocks": (u32, [P]),
    "kcmm_has_free_blocks": (i32, [P]),
    "kcmm_active_sequences": (u32, [P]),
    "kcmm_set_eviction_policy": (i32, [P, ctypes.c_char_p]),
    "kcmm_get_eviction_policy": (u32, [P, ctypes.c_char_p, u32]),
    "kcmm_is_tiering_enabled": (i32, [P]),
    "kcmm_hint": (i32, [P, u32, ctypes.c_int]),
    "kcmm_protect": (i32, [P, u32, pu32, u32, ctypes.c_int]),
    "kcmm_share_prefix": (i32, [P, u32, u32, u32, pu32]),
    "kcmm_below_low_watermark": (i32, [P, f32]),
    "kcmm_synchronize": (i32, [P]),
    "kcmm_get_block_size": (u32, [P]),
    "kcmm_get_max_blocks_per_seq": (u32, [P]),
    "kcmm_get_block_bytes": (u32, [P]),
    "kcmm_get_num_layers": (u32, [P]),
    "kcmm_get_max_batch": (u32, [P]),
    "kcmm_get_max_seq_len": (u32, [P]),
    # --- B200 additions ---
    "kcmm_paged_attn_decode_bf16_on_stream":
        (i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64]),
    "kcmm_paged_attn_decode_bf16_noalloc_on_stream":
        (i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64]),
    "kcmm_paged_prefill_bf16_on_stream":
        (i32, [P, u32, u64, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, f32,
               u64]),
    "kcmm_paged_prefill_f16_on_stream":
        (i32, [P, u32, u64, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, u32, f32,
               u64]),
    "kcmm_append_kv_device_slots_bf16_on_stream":
        (i32, [P, u32, u64, u64, u64, u32, u32, u64, u64, u64, u64]),
    "kcmm_fused_norm_rope_append_bf16_on_stream":
        (i32, [P, u32, u64, u64, u64, u32, f32, u64, u32, u64, u64, u64, f32, u32,
               u64, u64, u64, u32, u32, u64, u64]),
    "kcmm_block_incref": (i32, [P, u32]),
    "kcmm_block_decref": (i32, [P, u32]),
    "kcmm_block_refcount": (u32, [P, u32]),
    "kcmm_fork_sequence": (i32, [P, u32, pu32]),
    "kcmm_cow_blocks_on_stream": (i32, [P, pu32, pu32, u32, pu32, u64]),
    "kcmm_swap_out_blocks_on_stream": (i32, [P, pu32, u32, u64]),
    "kcmm_swap_in_blocks_on_stream": (i32, [P, pu32, u32, u64]),
    "kcmm_get_kernel_status": (i32, [P]),
    "kcmm_paged_attn_decode_bf16_strided_on_stream":
        (i32, [P, u32, u64, i64, i64, u64, i64, i64, u64, i64, u64, u64, u32, u32, u32, u32, u32,
               u32, f32, u64]),
    "kcmm_paged_attn_decode_f16_strided_on_stream":
        (i32, [P, u32, u64, i64, i64, u64, i64, i64, u64, i64, u64, u64, u32, u32, u32, u32, u32,
               u32, f32, u64]),
    "kcmm_append_kv_device_slots_strided_on_stream":
        (i32, [P, u32, u64, u64, u64, u32, u32, u64, i64, u64, i64, u64, u64]),
    "kcmm_peer_signal_words": (u32, [u32]),
    "kcmm_peer_allgather_on_stream": (i32, [u64, u64, pu64, pu64, u32, u32, u64, u64]),
    "kcmm_peer_wait_on_stream": (i32, [u64, u32, u64, u64, u64]),
    "kcmm_paged_attn_decode_shared_prefix_bf16_on_stream": (
        i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64, u64,
              u32, u32, u64]),
    "kcmm_paged_attn_decode_shared_prefix_f16_on_stream": (
        i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, u64, u64,
              u32, u32, u64]),
    "kcmm_paged_attn_decode_bf16_allgather_on_stream": (
        i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, pu64, pu64,
              u32, u32, u64, u64]),
    "kcmm_paged_attn_decode_f16_allgather_on_stream": (
        i32, [P, u32, u64, u64, u64, u64, u64, u32, u32, u32, u32, u32, u32, f32, pu64, pu64,
              u32, u32, u64, u64]),
    "kcmm_get_metrics_ext": (i32, [P, ctypes.c_void_p]),
    "kcmm_get_policy_stats": (i32, [P, ctypes.c_char_p, ctypes.c_void_p]),
    "kcmm_start_background_eviction": (i32, [P]),
    "kcmm_stop_background_eviction": (i32, [P]),
    "kcmm_preview_eviction_victims": (u32, [P, u32, pu32, u32]),
    "kcmm_step_tables_create": (P, [P, u32]),
    "kcmm_step_tables_destroy": (None, [P]),
    "kcmm_step_tables_sync_on_stream": (i32, [P, pu32, u32, u64]),
    "kcmm_step_tables_block_tables": (u64, [P]),
    "kcmm_step_tables_seq_lens": (u64, [P]),
    "kcmm_step_tables_block_offsets": (u64, [P]),
    "kcmm_step_tables_stats": (i32, [P, ctypes.c_void_p]),
    "kcmm_build_info": (ctypes.c_char_p, []),
}


class KcmmStepTablesStats(ctypes.Structure):
    _fields_ = [("syncs", ctypes.c_uint64), ("table_entries", ctypes.c_uint64),
                ("offset_entries", ctypes.c_uint64), ("bytes", ctypes.c_uint64),
                ("full_offsets", ctypes.c_uint64)]


class StepTables:
    """Device-resident block tables / lengths / offsets of one ordered batch
    (`kcmm_step_tables_*`); `sync` uploads only what changed."""

    def __init__(self, pool: "KcmmPool", max_batch: int):
        self.pool = pool
        self.lib = pool.lib
        h = self.lib.kcmm_step_tables_create(pool.handle, max_batch)
        if not h:
            raise KcmmError(f"kcmm_step_tables_create: {pool.last_error()}")
        self.handle = ctypes.c_void_p(h)
        self.max_batch = max_batch

    def sync(self, seq_indices, stream_ptr: int = 0) -> None:
        arr = _u32_array(seq_indices)
        rc = self.lib.kcmm_step_tables_sync_on_stream(self.handle, arr, len(seq_indices),
                                                      stream_ptr)
        if rc != 0:
            raise KcmmError(f"kcmm_step_tables_sync_on_stream: {self.pool.last_error()}")

    @property
    def block_tables_ptr(self) -> int:
        return self.lib.kcmm_step_tables_block_tables(self.handle)

    @property
    def seq_lens_ptr(self) -> int:
        return self.lib.kcmm_step_tables_seq_lens(self.handle)

    @property
    def block_offsets_ptr(self) -> int:
        return self.lib.kcmm_step_tables_block_offsets(self.handle)

    def stats(self) -> dict:
        st = KcmmStepTablesStats()
        if self.lib.kcmm_step_tables_stats(self.handle, ctypes.byref(st)) != 0:
            raise KcmmError("kcmm_step_tables_stats failed")
        return {f: getattr(st, f) for f, _ in st._fields_}

    def destroy(self) -> None:
        if self.handle:
            self.lib.kcmm_step_tables_destroy(self.handle)
            self.handle = None


def _u32_array(values):
    values = [int(v) for v in values]
    return (ctypes.c_uint32 * max(1, len(values)))(*values)


class KcmmLibrary:
    """Loads `libkcmm.so` and binds every exported function."""

    def __init__(self, path: str | Path | None = None):
        assert_layout()
        self.path = Path(path) if path else library_path()
        self.lib = ctypes.CDLL(str(self.path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def create_pool(self, config: KcmmConfig) -> "KcmmPool":
        handle = self.lib.kcmm_pool_create(ctypes.byref(config))
        if not handle:
            raise KcmmError("kcmm_pool_create returned NULL")
        return KcmmPool(self, handle)

    def build_info(self) -> str:
        return self.lib.kcmm_build_info().decode()


def make_config(*, num_layers: int, kv_heads: int, head_dim: int, max_batch: int,
                max_seq_len: int, block_size: int = 16, max_blocks: int = 0,
                tiering: bool = False, eviction_policy: int = 0, device: int = 0,
                cpu_cache_path: str = "") -> KcmmConfig:
    cfg = KcmmConfig()
    cfg.block_size = block_size
    cfg.max_blocks = max_blocks
    cfg.cpu_cache_path = cpu_cache_path.encode()
    cfg.tiering = 1 if tiering else 0
    cfg.eviction_policy = eviction_policy
    cfg.device_ordinal = device
    cfg.num_layers = num_layers
    cfg.kv_heads = kv_heads
    cfg.head_dim = head_dim
    cfg.max_batch = max_batch
    cfg.max_seq_len = max_seq_len
    return cfg


class KcmmPool:
    """One pool handle; every method raises `KcmmError` on a -1 return."""

    def __init__(self, library: KcmmLibrary, handle):
        self.library = library
        self.lib = library.lib
        self.handle = ctypes.c_void_p(handle)
        self._destroyed = False

    def __enter__(self) -> "KcmmPool":
        return self

    def __exit__(self, *_exc) -> None:
        self.destroy()

    # --- errors ---------------------------------------------------------
    def last_error(self) -> str:
        buf = ctypes.create_string_buffer(4096)
        n = self.lib.kcmm_get_last_error(self.handle, buf, ctypes.sizeof(buf))
        return buf.value.decode("utf-8", errors="replace") if n else ""

    def clear_error(self) -> None:
        self.lib.kcmm_clear_error(self.handle)

    def _check(self, rc: int, op: str) -> None:
        if rc != 0:
            raise KcmmError(f"{op} failed: {self.last_error() or 'unknown KCMM error'}")

    def destroy(self) -> None:
        if not self._destroyed:
            self.lib.kcmm_pool_destroy(self.handle)
            self._destroyed = True

    # --- blocks and sequences --------------------------------------------
    def alloc_blocks(self, count: int) -> list[int]:
        if count <= 0:
            raise ValueError("count must be positive")
        out = (ctypes.c_uint32 * count)()
        self._check(self.lib.kcmm_alloc_blocks(self.handle, count, out), "kcmm_alloc_blocks")
        return list(out)

    def free_blocks(self, blocks) -> None:
        if len(blocks) == 0:
            return
        arr = _u32_array(blocks)
        self._check(self.lib.kcmm_free_blocks(self.handle, arr, len(blocks)), "kcmm_free_blocks")

    def register_sequence(self, block_table) -> int:
        arr = _u32_array(block_table)
        out = ctypes.c_uint32()
        self._check(self.lib.kcmm_register_sequence(self.handle, arr, len(block_table),
                                                    ctypes.byref(out)),
                    "kcmm_register_sequence")
        return out.value

    def unregister_sequence(self, seq_idx: int) -> None:
        self._check(self.lib.kcmm_unregister_sequence(self.handle, seq_idx),
                    "kcmm_unregister_sequence")

    def append_block_to_sequence(self, seq_idx: int, block_idx: int) -> None:
        self._check(self.lib.kcmm_append_block_to_sequence(self.handle, seq_idx, block_idx),
                    "kcmm_append_block_to_sequence")

    def touch(self, seq_idx: int) -> None:
        self.lib.kcmm_touch(self.handle, seq_idx)

    def cool(self, seq_idx: int) -> None:
        self.lib.kcmm_cool(self.handle, seq_idx)

    def update_seq_len(self, seq_idx: int, length: int) -> None:
        self.lib.kcmm_update_seq_len(self.handle, seq_idx, length)

    def seq_len(self, seq_idx: int) -> int:
        return self.lib.kcmm_get_seq_len(self.handle, seq_idx)

    def block_table(self, seq_idx: int, max_blocks: int = 1 << 16) -> list[int]:
        out = (ctypes.c_uint32 * max_blocks)()
        count = ctypes.c_uint32()
        self._check(self.lib.kcmm_get_block_table(self.handle, seq_idx, out, max_blocks,
                                                  ctypes.byref(count)),
                    "kcmm_get_block_table")
        return list(out[: count.value])

    def block_table_va_offsets(self, seq_idx: int, max_blocks: int = 1 << 16) -> list[int]:
        out = (ctypes.c_uint64 * max_blocks)()
        count = ctypes.c_uint32()
        self._check(self.lib.kcmm_get_block_table_va_offsets(self.handle, seq_idx, out,
                                                             max_blocks, ctypes.byref(count)),
                    "kcmm_get_block_table_va_offsets")
        return list(out[: count.value])

    def all_block_offsets_f16(self, min_entries: int = 0) -> list[int]:
        n = max(self.total_blocks(), min_entries, 1)
        out = (ctypes.c_uint64 * n)()
        count = ctypes.c_uint32()
        self._check(self.lib.kcmm_get_all_block_offsets_f16(self.handle, out, n,
                                                            ctypes.byref(count)),
                    "kcmm_get_all_block_offsets_f16")
        vals = list(out[: count.value])
        return vals + [0] * (min_entries - len(vals)) if min_entries > len(vals) else vals

    def all_block_valid_flags(self, min_entries: int = 0) -> list[int]:
        n = max(self.total_blocks(), min_entries, 1)
        out = (ctypes.c_uint8 * n)()
        count = ctypes.c_uint32()
        self._check(self.lib.kcmm_get_all_block_valid(self.handle, out, n, ctypes.byref(count)),
                    "kcmm_get_all_block_valid")
        vals = list(out[: count.value])
        return vals + [0] * (min_entries - len(vals)) if min_entries > len(vals) else vals

    def block_va_offset(self, block_idx: int) -> int:
        return self.lib.kcmm_get_block_va_offset(self.handle, block_idx)

    def block_location(self, block_idx: int) -> str:
        loc = ctypes.c_int()
        self._check(self.lib.kcmm_get_block_location(self.handle, block_idx, ctypes.byref(loc)),
                    "kcmm_get_block_location")
        return BlockLocation.name(loc.value)

    def is_gpu_resident(self, block_idx: int) -> bool:
        return bool(self.lib.kcmm_is_gpu_resident(self.handle, block_idx))

    def total_blocks(self) -> int:
        return self.lib.kcmm_total_blocks(self.handle)

    def blocks_in_use(self) -> int:
        return self.lib.kcmm_blocks_in_use(self.handle)

    def free_physical_blocks(self) -> int:
        return self.lib.kcmm_free_physical_blocks(self.handle)

    def active_sequences(self) -> int:
        return self.lib.kcmm_active_sequences(self.handle)

    def block_state_epoch(self) -> int:
        return self.lib.kcmm_block_state_epoch(self.handle)

    def va_k(self, layer: int) -> int:
        va = self.lib.kcmm_get_va_k(self.handle, layer)
        if not va:
            raise KcmmError(f"kcmm_get_va_k: layer {layer} out of bounds")
        return va

    def va_v(self, layer: int) -> int:
        va = self.lib.kcmm_get_va_v(self.handle, layer)
        if not va:
            raise KcmmError(f"kcmm_get_va_v: layer {layer} out of bounds")
        return va

    def stats(self) -> dict:
        s = KcmmPoolStats()
        self._check(self.lib.kcmm_get_pool_stats(self.handle, ctypes.byref(s)),
                    "kcmm_get_pool_stats")
        return {name: getattr(s, name) for name, _ in s._fields_}

    def metrics(self) -> dict:
        m = KcmmMetrics()
        self._check(self.lib.kcmm_get_metrics(self.handle, ctypes.byref(m)), "kcmm_get_metrics")
        return {name: getattr(m, name) for name, _ in m._fields_}

    def kernel_status(self) -> int:
        """Sticky device diagnostics (bit 0 wait timeout, bit 1 bad offset), then cleared."""
        return self.lib.kcmm_get_kernel_status(self.handle)

    def synchronize(self) -> None:
        self._check(self.lib.kcmm_synchronize(self.handle), "kcmm_synchronize")

    # --- KV append --------------------------------------------------------
    def append_kv_step(self, layer: int, seq_indices, positions, k_src_ptr: int,
                       v_src_ptr: int) -> None:
        n = len(seq_indices)
        self._check(self.lib.kcmm_append_kv_step(self.handle, layer, _u32_array(seq_indices),
                                                 _u32_array(positions), n, k_src_ptr, v_src_ptr),
                    "kcmm_append_kv_step")

    def append_kv_slots(self, layer: int, slot_mapping, k_src_ptr: int, v_src_ptr: int,
                        stream_ptr: int | None = None) -> None:
        n = len(slot_mapping)
        arr = (ctypes.c_int64 * max(1, n))(*[int(s) for s in slot_mapping])
        if stream_ptr is None:
            rc = self.lib.kcmm_append_kv_slots(self.handle, layer, arr, n, k_src_ptr, v_src_ptr)
        else:
            rc = self.lib.kcmm_append_kv_slots_on_stream(self.handle, layer, arr, n, k_src_ptr,
                                                         v_src_ptr, stream_ptr)
        self._check(rc, "kcmm_append_kv_slots")

    def append_kv_device_slots_on_stream(self, layer: int, *, slot_mapping_ptr: int,
                                         block_offsets_f16_ptr: int, valid_blocks_ptr: int,
                                         block_offsets_f16_len: int, batch: int,
                                         k_src_ptr: int, v_src_ptr: int, status_ptr: int,
                                         stream_ptr: int) -> None:
        self._check(self.lib.kcmm_append_kv_device_slots_on_stream(
            self.handle, layer, slot_mapping_ptr, block_offsets_f16_ptr, valid_blocks_ptr,
            block_offsets_f16_len, batch, k_src_ptr, v_src_ptr, status_ptr, stream_ptr),
            "kcmm_append_kv_device_slots_on_stream")

    def fused_norm_rope_append_bf16(self, layer: int, *, x_ptr: int, weight_ptr: int,
                                    normed_ptr: int, hidden: int, eps: float, q_ptr: int,
                                    num_q_heads: int, k_ptr: int, v_ptr: int,
                                    positions_ptr: int, rope_theta: float, rope_mode: int,
                                    slot_mapping_ptr: int, block_offsets_f16_ptr: int,
                                    valid_blocks_ptr: int, block_offsets_f16_len: int,
                                    num_tokens: int, status_ptr: int, stream_ptr: int) -> None:
        self._check(self.lib.kcmm_fused_norm_rope_append_bf16_on_stream(
            self.handle, layer, x_ptr, weight_ptr, normed_ptr, hidden, eps, q_ptr, num_q_heads,
            k_ptr, v_ptr, positions_ptr, rope_theta, rope_mode, slot_mapping_ptr,
            block_offsets_f16_ptr, valid_blocks_ptr, block_offsets_f16_len, num_tokens,
            status_ptr, stream_ptr), "kcmm_fused_norm_rope_append_bf16_on_stream")

    # --- decode attention --------------------------------------------------
    def paged_attn_decode(self, layer: int, *, query_ptr: int, out_ptr: int,
                          block_tables_ptr: int, seq_lens_ptr: int,
                          block_offsets_f16_ptr: int, batch: int, num_q_heads: int,
                          kv_heads: int, head_dim: int, block_size: int,
                          max_blocks_per_seq: int, scale: float, dtype: str = "bf16",
                          stream_ptr: int | None = 0, current_context: bool = False,
                          noalloc: bool = False) -> None:
        """`noalloc=True` (bf16 only) calls the entry point whose scratch is a static
        per-device array instead of a stream-ordered allocation."""
        args = (self.handle, layer, query_ptr, out_ptr, block_tables_ptr, seq_lens_ptr,
                block_offsets_f16_ptr, batch, num_q_heads, kv_heads, head_dim, block_size,
                max_blocks_per_seq, scale)
        if noalloc:
            if dtype != "bf16":
                raise ValueError("the no-allocation decode entry point is bf16 only")
            rc = self.lib.kcmm_paged_attn_decode_bf16_noalloc_on_stream(*args, stream_ptr or 0)
            op = "kcmm_paged_attn_decode_bf16_noalloc_on_stream"
        elif dtype == "bf16":
            rc = self.lib.kcmm_paged_attn_decode_bf16_on_stream(*args, stream_ptr or 0)
            op = "kcmm_paged_attn_decode_bf16_on_stream"
        elif stream_ptr is None:
            rc = self.lib.kcmm_paged_attn_decode_f16(*args)
            op = "kcmm_paged_attn_decode_f16"
        elif current_context:
            rc = self.lib.kcmm_paged_attn_decode_f16_on_current_context_stream(*args, stream_ptr)
            op = "kcmm_paged_attn_decode_f16_on_current_context_stream"
        else:
            rc = self.lib.kcmm_paged_attn_decode_f16_on_stream(*args, stream_ptr)
            op = "kcmm_paged_attn_decode_f16_on_stream"
        self._check(rc, op)

    def paged_prefill(self, layer: int, *, query_ptr: int, out_ptr: int, block_tables_ptr: int,
                      query_start_loc_ptr: int, context_lens_ptr: int,
                      block_offsets_f16_ptr: int, batch: int, max_query_len: int,
                      num_q_heads: int, kv_heads: int, head_dim: int, block_size: int,
                      max_blocks_per_seq: int, scale: float, dtype: str = "bf16",
                      stream_ptr: int = 0) -> None:
        op = f"kcmm_paged_prefill_{dtype}_on_stream"
        fn = getattr(self.lib, op)
        self._check(fn(self.handle, layer, query_ptr, out_ptr, block_tables_ptr,
                       query_start_loc_ptr, context_lens_ptr, block_offsets_f16_ptr, batch,
                       max_query_len, num_q_heads, kv_heads, head_dim, block_size,
                       max_blocks_per_seq, scale, stream_ptr), op)

    def precompile_paged_attn_decode_f16(self) -> None:
        self._check(self.lib.kcmm_precompile_paged_attn_decode_f16(self.handle),
                    "kcmm_precompile_paged_attn_decode_f16")

    def precompile_vllm_kv_write_f16(self) -> None:
        self._check(self.lib.kcmm_precompile_vllm_kv_write_f16(self.handle),
                    "kcmm_precompile_vllm_kv_write_f16")

    # --- sharing / copy-on-write ------------------------------------------
    def incref(self, block_idx: int) -> None:
        self._check(self.lib.kcmm_block_incref(self.handle, block_idx), "kcmm_block_incref")

    def decref(self, block_idx: int) -> None:
        self._check(self.lib.kcmm_block_decref(self.handle, block_idx), "kcmm_block_decref")

    def refcount(self, block_idx: int) -> int:
        return self.lib.kcmm_block_refcount(self.handle, block_idx)

    def fork_sequence(self, src_seq: int) -> int:
        out = ctypes.c_uint32()
        self._check(self.lib.kcmm_fork_sequence(self.handle, src_seq, ctypes.byref(out)),
                    "kcmm_fork_sequence")
        return out.value

    def share_prefix(self, src_seq: int, dst_seq: int, num_blocks: int) -> list[int]:
        out = (ctypes.c_uint32 * max(1, num_blocks))()
        self._check(self.lib.kcmm_share_prefix(self.handle, src_seq, dst_seq, num_blocks, out),
                    "kcmm_share_prefix")
        return list(out[:num_blocks])

    def cow_blocks(self, seq_indices, logical_blocks, stream_ptr: int = 0) -> list[int]:
        n = len(seq_indices)
        out = (ctypes.c_uint32 * max(1, n))()
        self._check(self.lib.kcmm_cow_blocks_on_stream(self.handle, _u32_array(seq_indices),
                                                       _u32_array(logical_blocks), n, out,
                                                       stream_ptr),
                    "kcmm_cow_blocks_on_stream")
        return list(out[:n])

    # --- tiering -------------------------------------------------------------
    def evict_blocks(self, count: int) -> int:
        return self.lib.kcmm_evict_blocks(self.handle, count)

    def restore_evicted_block(self, block_idx: int) -> int:
        va = self.lib.kcmm_restore_evicted_block(self.handle, block_idx)
        if va == 0 and self.last_error():
            raise KcmmError(f"kcmm_restore_evicted_block failed: {self.last_error()}")
        return va

    def restore_evicted_blocks(self, blocks) -> None:
        self._check(self.lib.kcmm_restore_evicted_blocks(self.handle, _u32_array(blocks),
                                                         len(blocks)),
                    "kcmm_restore_evicted_blocks")

    def swap_out(self, blocks, stream_ptr: int = 0) -> None:
        self._check(self.lib.kcmm_swap_out_blocks_on_stream(self.handle, _u32_array(blocks),
                                                            len(blocks), stream_ptr),
                    "kcmm_swap_out_blocks_on_stream")

    def swap_in(self, blocks, stream_ptr: int = 0) -> None:
        self._check(self.lib.kcmm_swap_in_blocks_on_stream(self.handle, _u32_array(blocks),
                                                           len(blocks), stream_ptr),
                    "kcmm_swap_in_blocks_on_stream")

    def metrics_ext(self) -> dict:
        m = KcmmMetricsExt()
        self._check(self.lib.kcmm_get_metrics_ext(self.handle, ctypes.byref(m)),
                    "kcmm_get_metrics_ext")

        def hist(h):
            return {"count": h.count, "sum_us": h.sum_us, "min_us": h.min_us,
                    "max_us": h.max_us, "buckets": list(h.buckets)}
        out = {name: getattr(m.base, name) for name, _ in m.base._fields_}
        out.update({name: getattr(m, name) for name, _ in m._fields_[1:6]})
        out["eviction_latency"] = hist(m.eviction_latency)
        out["restoration_latency"] = hist(m.restoration_latency)
        return out

    def policy_stats(self, policy: str) -> dict | None:
        st = KcmmPolicyStats()
        if self.lib.kcmm_get_policy_stats(self.handle, policy.encode(), ctypes.byref(st)) != 0:
            return None
        return {name: getattr(st, name) for name, _ in st._fields_}

    def start_background_eviction(self) -> None:
        self._check(self.lib.kcmm_start_background_eviction(self.handle),
                    "kcmm_start_background_eviction")

    def stop_background_eviction(self) -> None:
        self._check(self.lib.kcmm_stop_background_eviction(self.handle),
                    "kcmm_stop_background_eviction")

    def preview_eviction_victims(self, count: int) -> list[int]:
        buf = (ctypes.c_uint32 * max(1, count))()
        n = self.lib.kcmm_preview_eviction_victims(self.handle, count, buf, max(1, count))
        return list(buf[:n])

    def set_eviction_policy(self, name: str) -> None:
        self._check(self.lib.kcmm_set_eviction_policy(self.handle, name.encode()),
                    "kcmm_set_eviction_policy")

    def eviction_policy(self) -> str:
        buf = ctypes.create_string_buffer(64)
        self.lib.kcmm_get_eviction_policy(self.handle, buf, 64)
        return buf.value.decode()
