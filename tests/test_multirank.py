"""The N > 1 bench path on CPU: two gloo ranks.

bench.py shards sequences across ranks (weak scaling, no collective on the data
path).  The only cross-rank steps are the barrier around the timed region, the
max-over-ranks of its duration and the gather of per-rank figures; these run here on
gloo exactly as bench.py runs them on NCCL.  Every rank draws the same context
lengths (one shared seed, so every rank moves the same bytes) and owns an independent
pool (host VMM backend)."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import numpy as np
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    os.environ["KCMM_VMM_BACKEND"] = "host"
    import bench
    from lattice_b200 import kcmm

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # every rank owns a pool; the lengths come from the shared seed
        lib = kcmm.KcmmLibrary()
        cfg = kcmm.make_config(num_layers=1, kv_heads=8, head_dim=128, max_batch=64,
                               max_seq_len=4096, block_size=16)
        pool = lib.create_pool(cfg)
        lens = np.random.default_rng(1000).integers(512, 4097, 16)
        tables = []
        for L in lens:
            blocks = pool.alloc_blocks(int(-(-int(L) // 16)))
            s = pool.register_sequence(blocks)
            pool.update_seq_len(s, int(L))
            tables.append(blocks)
        kv_bytes = int(sum(int(L) * 8 * 128 * 2 * 2 for L in lens))
        bench.barrier()
        ms = bench.max_over_ranks(1.0 + rank)  # rank 1 is the slower one
        gbps = bench.whole_job_gbps(kv_bytes, world, ms)
        rows = bench.gather_over_ranks([1.0 + rank, float(kv_bytes)])
        pool.destroy()
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(
            {"ms": ms, "gbps": gbps, "kv_bytes": kv_bytes, "lens": [int(x) for x in lens],
             "first_table": tables[0][:4], "rows": rows}))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_take_the_max(tmp_path, kcmm_lib):
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = json.loads((tmp_path / "rank0.json").read_text())
    r1 = json.loads((tmp_path / "rank1.json").read_text())
    assert r0["ms"] == r1["ms"] == 2.0  # both ranks see the slowest rank's time
    # weak scaling: the job's bytes are world x each rank's own bytes
    assert r0["gbps"] == pytest.approx(r0["kv_bytes"] * 2 / 2e-3 / 1e9)
    assert r0["lens"] == r1["lens"]  # one shared length draw: equal bytes per rank
    assert r0["kv_bytes"] == r1["kv_bytes"]
    for r in (r0, r1):  # every rank sees every rank's figures, indexed by rank
        assert r["rows"] == [[1.0, float(r0["kv_bytes"])], [2.0, float(r1["kv_bytes"])]]
    # each pool is independent: both start from block 0 in the same LIFO order
    assert r0["first_table"] == r1["first_table"]


def test_reference_arm_non_zero_rank_exits_quietly():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True,
                         env=env, timeout=120, cwd=ROOT)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == ""
