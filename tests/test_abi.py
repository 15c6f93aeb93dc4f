"""The drop-in boundary: libkcmm.so loads, exports every symbol include/kcmm.h
declares, and its structs have the reference layout (ref src/kcmm/ffi.rs:2575-2603)."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "kcmm.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kcmm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_reference_surface():
    names = set(declared_functions())
    # every reference export (include/kcmm.h + the ffi.rs-only extras) is present
    reference = {
        "kcmm_pool_create", "kcmm_pool_destroy", "kcmm_get_last_error", "kcmm_clear_error",
        "kcmm_alloc_blocks", "kcmm_free_blocks", "kcmm_register_sequence",
        "kcmm_unregister_sequence", "kcmm_touch", "kcmm_cool", "kcmm_update_seq_len",
        "kcmm_get_seq_len", "kcmm_append_block_to_sequence", "kcmm_get_block_table",
        "kcmm_get_block_va_offset", "kcmm_get_all_block_offsets_f16", "kcmm_get_block_location",
        "kcmm_get_block_table_va_offsets", "kcmm_get_va_k", "kcmm_get_va_v",
        "kcmm_append_kv_step", "kcmm_append_kv_slots", "kcmm_append_kv_slots_on_stream",
        "kcmm_paged_attn_decode_f16", "kcmm_paged_attn_decode_f16_on_stream",
        "kcmm_paged_attn_decode_f16_on_current_context_stream",
        "kcmm_precompile_paged_attn_decode_f16", "kcmm_evict_blocks",
        "kcmm_restore_evicted_block", "kcmm_restore_evicted_blocks", "kcmm_is_gpu_resident",
        "kcmm_get_metrics", "kcmm_get_pool_stats", "kcmm_blocks_in_use", "kcmm_total_blocks",
        "kcmm_free_physical_blocks", "kcmm_has_free_blocks", "kcmm_active_sequences",
        "kcmm_set_eviction_policy", "kcmm_get_eviction_policy", "kcmm_is_tiering_enabled",
        "kcmm_hint", "kcmm_protect", "kcmm_share_prefix", "kcmm_below_low_watermark",
        "kcmm_synchronize", "kcmm_get_block_size", "kcmm_get_max_blocks_per_seq",
        "kcmm_get_block_bytes", "kcmm_get_num_layers", "kcmm_get_max_batch",
        "kcmm_get_max_seq_len",
        # ffi.rs-only exports
        "kcmm_precompile_vllm_kv_write_f16", "kcmm_get_all_block_valid",
        "kcmm_append_kv_device_slots_on_stream", "kcmm_block_state_epoch",
    }
    assert reference <= names, reference - names


def test_library_exports_every_declared_symbol(kcmm_lib):
    lib = ctypes.CDLL(str(kcmm_lib.path))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_alias_library_name(kcmm_lib):
    alias = kcmm_lib.path.parent / "libbaseline_llm_os.so"
    assert alias.exists()
    lib = ctypes.CDLL(str(alias))
    assert lib.kcmm_pool_create


def test_python_binding_covers_header(kcmm_lib):
    from lattice_b200 import kcmm

    assert set(declared_functions()) == set(kcmm.SIGNATURES)


def test_config_layout_python(golden):
    from lattice_b200 import kcmm

    lay = golden["kats"]["config_layout"]
    kcmm.assert_layout()
    assert ctypes.sizeof(kcmm.KcmmConfig) == lay["size"]
    for f, off in lay["offsets"].items():
        assert getattr(kcmm.KcmmConfig, f).offset == off


def test_config_layout_c(tmp_path, golden):
    """The C header itself compiles with the reference's static layout checks."""
    lay = golden["kats"]["config_layout"]
    checks = "\n".join(
        f'_Static_assert(offsetof(kcmm_config_t, {f}) == {o}, "{f}");'
        for f, o in lay["offsets"].items())
    src = tmp_path / "layout.c"
    src.write_text(
        '#include <stddef.h>\n#include "kcmm.h"\n'
        f'_Static_assert(sizeof(kcmm_config_t) == {lay["size"]}, "size");\n{checks}\n'
        "_Static_assert(sizeof(kcmm_metrics_t) == 72, \"metrics\");\n"
        "_Static_assert(sizeof(kcmm_pool_stats_t) == 56, \"stats\");\n"
        "int main(void) { return 0; }\n")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(src),
                    "-o", str(tmp_path / "layout")], check=True)


def test_c_program_links_against_library(tmp_path, kcmm_lib, monkeypatch):
    """A C caller (like ref examples/kcmm_c_integration.c) links and drives the pool."""
    src = tmp_path / "caller.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "kcmm.h"
int main(void) {
  kcmm_config_t cfg; memset(&cfg, 0, sizeof cfg);
  cfg.num_layers = 2; cfg.kv_heads = 4; cfg.head_dim = 64; cfg.max_batch = 2;
  cfg.max_seq_len = 64;
  kcmm_pool_t *p = kcmm_pool_create(&cfg);
  if (!p) return 10;
  uint32_t b[3];
  if (kcmm_alloc_blocks(p, 3, b) != 0) return 11;
  uint32_t seq;
  if (kcmm_register_sequence(p, b, 3, &seq) != 0) return 12;
  kcmm_pool_stats_t st;
  if (kcmm_get_pool_stats(p, &st) != 0 || st.blocks_in_use != 3) return 13;
  if (kcmm_get_block_size(p) != 16 || kcmm_get_block_bytes(p) != 8192) return 14;
  if (kcmm_get_va_k(p, 2) != 0) return 15;   /* out of range -> 0 */
  char msg[256];
  if (kcmm_get_last_error(p, msg, sizeof msg) != 0) return 16;
  if (kcmm_append_block_to_sequence(p, 99, 0) != -1) return 17;
  if (kcmm_get_last_error(p, msg, sizeof msg) == 0) return 18;
  kcmm_clear_error(p);
  if (kcmm_get_last_error(p, msg, sizeof msg) != 0) return 19;
  if (kcmm_unregister_sequence(p, seq) != 0 || kcmm_blocks_in_use(p) != 0) return 20;
  kcmm_pool_destroy(p);
  kcmm_pool_destroy(NULL);
  printf("ok\n");
  return 0;
}
''')
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe),
                    f"-L{kcmm_lib.path.parent}", "-lkcmm", f"-Wl,-rpath,{kcmm_lib.path.parent}"],
                   check=True)
    monkeypatch.setenv("KCMM_VMM_BACKEND", "host")
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.strip() == "ok"


def test_null_pool_conventions(kcmm_lib):
    lib = kcmm_lib.lib
    assert lib.kcmm_alloc_blocks(None, 1, None) == -1
    assert lib.kcmm_free_blocks(None, None, 0) == 0
    assert lib.kcmm_get_va_k(None, 0) == 0
    assert lib.kcmm_blocks_in_use(None) == 0
    assert lib.kcmm_pool_create(None) is None
    assert lib.kcmm_synchronize(None) == -1


def test_kernel_entry_points_refuse_host_pool(host_pool_factory):
    from lattice_b200 import KcmmError

    pool = host_pool_factory(kv_heads=2, head_dim=64, max_batch=1, max_seq_len=32)
    with pytest.raises(KcmmError, match="no device memory"):
        pool.paged_attn_decode(0, query_ptr=1, out_ptr=1, block_tables_ptr=1, seq_lens_ptr=1,
                               block_offsets_f16_ptr=1, batch=1, num_q_heads=2, kv_heads=2,
                               head_dim=64, block_size=16, max_blocks_per_seq=2, scale=0.1)


@pytest.mark.parametrize("kw,msg", [
    (dict(head_dim=100), "head_dim 100 unsupported"),
    (dict(head_dim=264), "head_dim 264 unsupported"),
    (dict(num_q_heads=6, kv_heads=4), "at most 128"),
    (dict(num_q_heads=384, kv_heads=1), "at most 128"),
    (dict(batch=0), "must be positive"),
    (dict(query_ptr=24), "16-byte aligned"),
    (dict(block_tables_ptr=0), "null pointer"),
])
def test_prefill_argument_checks(host_pool_factory, kw, msg):
    """The prefill entry point validates its shapes before it touches the device."""
    from lattice_b200 import KcmmError

    pool = host_pool_factory(kv_heads=2, head_dim=128, max_batch=1, max_seq_len=32)
    args = dict(query_ptr=16, out_ptr=16, block_tables_ptr=16, query_start_loc_ptr=16,
                context_lens_ptr=16, block_offsets_f16_ptr=16, batch=1, max_query_len=4,
                num_q_heads=8, kv_heads=2, head_dim=128, block_size=16, max_blocks_per_seq=2,
                scale=0.1)
    args.update(kw)
    with pytest.raises(KcmmError, match=msg):
        pool.paged_prefill(0, **args)


@pytest.mark.parametrize("hq,hd,bs", [(8, 128, 16), (14, 128, 16), (6, 64, 8), (10, 256, 16),
                                      (256, 96, 32)])
def test_prefill_refuses_host_pool(host_pool_factory, hq, hd, bs):
    """Shapes the prefill accepts (query-head groups of 4, 7, 3, 5 and 128, head dims 64
    to 256, 8- to 32-token pages) pass the argument checks and stop only at the missing
    device memory of a host pool."""
    from lattice_b200 import KcmmError

    pool = host_pool_factory(kv_heads=2, head_dim=hd, max_batch=1, max_seq_len=32,
                             block_size=bs)
    with pytest.raises(KcmmError, match="no device memory"):
        pool.paged_prefill(0, query_ptr=16, out_ptr=16, block_tables_ptr=16,
                           query_start_loc_ptr=16, context_lens_ptr=16,
                           block_offsets_f16_ptr=16, batch=1, max_query_len=4,
                           num_q_heads=hq, kv_heads=2, head_dim=hd, block_size=bs,
                           max_blocks_per_seq=2, scale=0.1)


def test_step_tables_need_a_device_pool(kcmm_lib, host_pool_factory):
    """On the host VMM backend (no device) creation fails with a message; NULL
    handles are refused."""
    from lattice_b200 import kcmm

    lib = kcmm_lib.lib
    pool = host_pool_factory(kv_heads=2, head_dim=64, max_batch=4, max_seq_len=256)
    assert not lib.kcmm_step_tables_create(pool.handle, 8)
    assert "kcmm_step_tables_create" in pool.last_error()
    assert lib.kcmm_step_tables_sync_on_stream(None, None, 0, 0) == -1
    assert lib.kcmm_step_tables_stats(None, None) == -1
    assert lib.kcmm_step_tables_block_tables(None) == 0
    lib.kcmm_step_tables_destroy(None)
    with pytest.raises(kcmm.KcmmError):
        kcmm.StepTables(pool, 8)


def test_strided_entry_points_check_strides(kcmm_lib, host_pool_factory):
    """Head strides below head_dim and table rows shorter than max_blocks_per_seq are
    refused before any device work (host pool: the checks run first)."""
    lib = kcmm_lib.lib
    pool = host_pool_factory(kv_heads=2, head_dim=64, max_batch=4, max_seq_len=256)
    good = dict(qt=8 * 64, qh=64, ot=8 * 64, oh=64, tr=16)

    def call(**kw):
        a = {**good, **kw}
        return lib.kcmm_paged_attn_decode_bf16_strided_on_stream(
            pool.handle, 0, 1, a["qt"], a["qh"], 2, a["ot"], a["oh"], 3, a["tr"], 4, 5,
            2, 8, 2, 64, 16, 16, 0.125, 0)

    assert call(qh=32) == -1 and "strides" in pool.last_error()
    assert call(oh=0) == -1
    assert call(tr=15) == -1
    assert call(qt=-1) == -1
    assert lib.kcmm_append_kv_device_slots_strided_on_stream(
        pool.handle, 0, 1, 2, 0, 4, 2, 3, 100, 4, 0, 0, 0) == -1  # k stride < kv_heads*D
    assert "row strides" in pool.last_error()


def test_extended_metrics_layout_and_host_values(kcmm_lib, host_pool_factory, tmp_path):
    """kcmm_metrics_ext_t / kcmm_policy_stats_t as a C compiler lays them out equal the
    ctypes mirrors; a pool that never swapped reports zeros and no policy stats."""
    from lattice_b200 import kcmm

    src = tmp_path / "layout.c"
    src.write_text(r'''
#include <stdio.h>
#include <stddef.h>
#include "kcmm.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu\n", sizeof(kcmm_metrics_ext_t),
         offsetof(kcmm_metrics_ext_t, background_eviction_count),
         offsetof(kcmm_metrics_ext_t, eviction_latency),
         offsetof(kcmm_metrics_ext_t, restoration_latency), sizeof(kcmm_policy_stats_t));
  return 0;
}
''')
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)],
                   check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    E = kcmm.KcmmMetricsExt
    assert got == [ctypes.sizeof(E), E.background_eviction_count.offset,
                   E.eviction_latency.offset, E.restoration_latency.offset,
                   ctypes.sizeof(kcmm.KcmmPolicyStats)]
    pool = host_pool_factory(kv_heads=2, head_dim=64, max_batch=4, max_seq_len=256,
                             tiering=True, max_blocks=16)
    m = pool.metrics_ext()
    assert m["evicted_blocks_total"] == 0 and m["background_eviction_count"] == 0
    assert m["eviction_latency"]["count"] == 0 and m["restoration_latency"]["count"] == 0
    assert pool.policy_stats("lru") is None
    assert kcmm_lib.lib.kcmm_get_metrics_ext(None, None) == -1


def test_peer_allgather_argument_checks(kcmm_lib):
    """Checked before any device work: NULL pointers, world outside 1..8, a rank outside
    the world, sizes that are not whole 16-byte chunks, epoch 0."""
    lib = kcmm_lib.lib
    assert lib.kcmm_peer_signal_words(2) == 32 and lib.kcmm_peer_signal_words(9) == 0
    ptrs = (ctypes.c_uint64 * 2)(16, 32)
    assert lib.kcmm_peer_allgather_on_stream(0, 16, ptrs, ptrs, 0, 2, 1, 0) == -1
    assert lib.kcmm_peer_allgather_on_stream(16, 16, ptrs, ptrs, 2, 2, 1, 0) == -1
    assert lib.kcmm_peer_allgather_on_stream(16, 24, ptrs, ptrs, 0, 2, 1, 0) == -1
    assert lib.kcmm_peer_allgather_on_stream(16, 16, ptrs, ptrs, 0, 9, 1, 0) == -1
    assert lib.kcmm_peer_allgather_on_stream(16, 16, ptrs, ptrs, 0, 2, 0, 0) == -1
    assert lib.kcmm_peer_wait_on_stream(0, 2, 1, 0, 0) == -1
    assert lib.kcmm_peer_wait_on_stream(8, 0, 1, 0, 0) == -1


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_decode_allgather_argument_checks(kcmm_lib, host_pool_factory, dtype):
    """The decode fused with the peer all-gather checks its peer arguments before any
    device work (host pool: the checks run first): world outside 1..8, a rank outside
    the world, epoch 0, NULL or misaligned buffers."""
    lib = kcmm_lib.lib
    pool = host_pool_factory(kv_heads=2, head_dim=64, max_batch=4, max_seq_len=256)
    fn = getattr(lib, f"kcmm_paged_attn_decode_{dtype}_allgather_on_stream")

    def call(bufs=(256, 512), sigs=(1024, 2048), rank=0, world=2, epoch=1):
        b = (ctypes.c_uint64 * len(bufs))(*bufs)
        s = (ctypes.c_uint64 * len(sigs))(*sigs)
        return fn(pool.handle, 0, 1, 2, 3, 4, 5, 2, 8, 2, 64, 16, 16, 0.125, b, s, rank,
                  world, epoch, 0)

    for kw in (dict(world=0), dict(world=9, bufs=(256,) * 9, sigs=(1024,) * 9),
               dict(rank=2), dict(epoch=0)):
        assert call(**kw) == -1
        assert "allgather" in pool.last_error() and "world" in pool.last_error()
    assert call(bufs=(256, 520)) == -1 and "16-byte aligned" in pool.last_error()
    assert call(sigs=(1024, 0)) == -1 and "signal" in pool.last_error()
    # valid peer arguments get as far as the device check
    assert call() == -1 and "device" in pool.last_error().lower()


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_shared_prefix_decode_argument_checks(kcmm_lib, host_pool_factory, dtype):
    """Group arguments are checked before any device work (host pool): NULL group
    arrays, no groups, more groups than sequences, max_group_size 0, and more than 16
    query heads per kv head."""
    lib = kcmm_lib.lib
    pool = host_pool_factory(kv_heads=2, head_dim=64, max_batch=4, max_seq_len=256)
    fn = getattr(lib, f"kcmm_paged_attn_decode_shared_prefix_{dtype}_on_stream")

    def call(starts=6, lens=7, n=1, mx=2, hq=8, hkv=2):
        return fn(pool.handle, 0, 1, 2, 3, 4, 5, 2, hq, hkv, 64, 16, 16, 0.125, starts, lens,
                  n, mx, 0)

    for kw in (dict(starts=0), dict(lens=0), dict(n=0), dict(n=3), dict(mx=0), dict(mx=3)):
        assert call(**kw) == -1
        assert "shared_prefix" in pool.last_error() and "group" in pool.last_error()
    assert call(hq=34, hkv=2) == -1 and "16 query heads" in pool.last_error()
    assert call() == -1 and "device" in pool.last_error().lower()
