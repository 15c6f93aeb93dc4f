"""All-gather over NVLink peer memory (`kcmm_peer_allgather_on_stream` and
`kcmm_peer_wait_on_stream`) with two ranks, one GPU each; skipped with fewer than two
GPUs.  Every rank's gathered buffer must hold every rank's slice after the wait, over
several epochs with changing data (also back to back, with no host barrier and a
slowed reader).  A wait for a rank that never raises its flags
returns after its 1 s bound with status 1, and the GPU stays usable.  The decode fused
with the gather (`kcmm_paged_attn_decode_bf16_allgather_on_stream`) must fill every
rank's buffer with all ranks' outputs the same way."""
from __future__ import annotations

import json
import socket
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    import ctypes
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from lattice_b200.workloads import PeerBuffers, library, read_device

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    lib = library().lib
    result = {"ok": True}
    pb = None
    try:
        slice_bytes = 8 * 32 * 128 * 2  # one rank's [8, 32, 128] bf16 output
        pb = PeerBuffers(slice_bytes, rank, world, rank)
        dst = (ctypes.c_uint64 * world)(*pb.buf_ptrs)
        sig = (ctypes.c_uint64 * world)(*pb.sig_ptrs)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        sp = torch.cuda.current_stream().cuda_stream
        for epoch in range(1, 5):
            src = torch.full((slice_bytes // 2,), float(rank * 10 + epoch), device="cuda")
            src = src.bfloat16()
            assert lib.kcmm_peer_allgather_on_stream(src.data_ptr(), slice_bytes, dst, sig, rank,
                                                     world, epoch, sp) == 0
            assert lib.kcmm_peer_wait_on_stream(pb.signal_ptr, world, epoch, status.data_ptr(),
                                                sp) == 0
            torch.cuda.synchronize()
            got = read_device(pb.half_ptr(epoch), slice_bytes * world).view(np.uint16)
            for r in range(world):
                want = torch.full((1,), float(r * 10 + epoch)).bfloat16().view(torch.int16)
                part = got[r * slice_bytes // 2:(r + 1) * slice_bytes // 2]
                if not (part == np.uint16(want.item() & 0xFFFF)).all():
                    result["ok"] = False
            result[f"status_{epoch}"] = int(status.item())
            dist.barrier()
        # rank 1 skips epoch 5: rank 0's wait runs out and reports it
        if rank == 0:
            assert lib.kcmm_peer_allgather_on_stream(src.data_ptr(), slice_bytes, dst, sig, rank,
                                                     world, 5, sp) == 0
            assert lib.kcmm_peer_wait_on_stream(pb.signal_ptr, world, 5, status.data_ptr(),
                                                sp) == 0
            torch.cuda.synchronize()
            result["timeout_status"] = int(status.item())
            # the context is still usable
            result["after"] = float((torch.ones(4, device="cuda") * 2).sum().item())
        dist.barrier()
        # argument checks
        result["bad_world"] = lib.kcmm_peer_allgather_on_stream(
            src.data_ptr(), slice_bytes, dst, sig, rank, 9, 6, sp)
        result["bad_bytes"] = lib.kcmm_peer_allgather_on_stream(
            src.data_ptr(), 24, dst, sig, rank, world, 6, sp)
    finally:
        if pb is not None:
            dist.barrier()
            pb.close()
        Path(out_dir, f"rank{rank}.json").write_text(json.dumps(result))
        dist.destroy_process_group()


def _fused_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    """Each rank decodes its own kv heads with the fused decode + gather; every
    rank's gathered buffer must hold all ranks' outputs, bit for bit."""
    import ctypes
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from lattice_b200.workloads import DecodeWorkload, PeerBuffers, read_device

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    result = {"ok": True, "close": True}
    pb = wl = None
    try:
        wl = DecodeWorkload(batch=4, num_q_heads=16, kv_heads=2, head_dim=128,
                            pool_blocks=2200, seq_lens_override=[0, 40, 3000, 8000],
                            max_len=8000, seed=90 + rank, device=rank).build()
        slice_bytes = wl.out.numel() * 2
        pb = PeerBuffers(slice_bytes, rank, world, rank)
        dst = (ctypes.c_uint64 * world)(*pb.buf_ptrs)
        sig = (ctypes.c_uint64 * world)(*pb.sig_ptrs)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        sp = torch.cuda.current_stream().cuda_stream
        lib = wl.pool.lib
        live = torch.from_numpy(wl.seq_lens > 0).cuda()
        for epoch in range(1, 4):
            wl.q.copy_(torch.randn_like(wl.q.float()).bfloat16())
            wl.decode(stream_ptr=sp)
            ref = wl.out.clone()
            wl.out.zero_()
            pb.epoch += 1
            assert lib.kcmm_paged_attn_decode_bf16_allgather_on_stream(
                wl.pool.handle, 0, wl.q.data_ptr(), wl.out.data_ptr(), wl.d_tables.data_ptr(),
                wl.d_seq_lens.data_ptr(), wl.d_offsets.data_ptr(), wl.batch, wl.num_q_heads,
                wl.kv_heads, wl.head_dim, wl.block_size, wl.max_blocks_per_seq, wl.scale,
                dst, sig, rank, world, pb.epoch, sp) == 0, wl.pool.last_error()
            assert lib.kcmm_peer_wait_on_stream(pb.signal_ptr, world, pb.epoch,
                                                status.data_ptr(), sp) == 0
            torch.cuda.synchronize()
            err = (wl.out[live].float() - ref[live].float()).abs()
            if not bool((err <= 2e-3 + 1e-2 * ref[live].float().abs()).all()):
                result["close"] = False
            mine = wl.out.view(torch.int16).cpu().numpy().view(np.uint8).reshape(-1)
            everyone = [None] * world
            dist.all_gather_object(everyone, mine)
            got = read_device(pb.half_ptr(pb.epoch), slice_bytes * world)
            if not (got == np.concatenate(everyone)).all() or int(status.item()) != 0:
                result["ok"] = False
            dist.barrier()
    finally:
        if pb is not None:
            dist.barrier()
            pb.close()
        if wl is not None:
            wl.close()
        Path(out_dir, f"fused{rank}.json").write_text(json.dumps(result))
        dist.destroy_process_group()


def _back_to_back_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    """Epochs run back to back with no host barrier between them.  After each wait
    one rank (alternating) is held up by a busy kernel before it snapshots the
    gathered half, while the other rank runs ahead into the next epoch.  Every
    snapshot must still hold exactly that epoch's slices: the next epoch writes the
    other half, and the epoch after it cannot start before the slow rank has
    finished its snapshot and raised its own flags."""
    import ctypes
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist
    from cuda.bindings import runtime as rt

    sys.path.insert(0, str(ROOT))
    from lattice_b200.workloads import PeerBuffers, library

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    lib = library().lib
    result = {"ok": True, "status": 0}
    pb = None
    epochs = 12
    try:
        n = 4096  # bf16 values per slice
        slice_bytes = n * 2
        pb = PeerBuffers(slice_bytes, rank, world, rank)
        dst = (ctypes.c_uint64 * world)(*pb.buf_ptrs)
        sig = (ctypes.c_uint64 * world)(*pb.sig_ptrs)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        stream = torch.cuda.current_stream()
        sp = stream.cuda_stream
        srcs = [torch.full((n,), float(rank * 100 + e), device="cuda").bfloat16()
                for e in range(epochs + 1)]
        snaps = torch.zeros((epochs + 1, world * n), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        dist.barrier()
        for e in range(1, epochs + 1):
            assert lib.kcmm_peer_allgather_on_stream(srcs[e].data_ptr(), slice_bytes, dst, sig,
                                                     rank, world, e, sp) == 0
            assert lib.kcmm_peer_wait_on_stream(pb.signal_ptr, world, e, status.data_ptr(),
                                                sp) == 0
            if e % world == rank:
                torch.cuda._sleep(10_000_000)  # ~5 ms: well inside the 1 s wait bound
            (err,) = rt.cudaMemcpyAsync(snaps[e].data_ptr(), pb.half_ptr(e), world * slice_bytes,
                                        rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, sp)
            assert int(err) == 0
        torch.cuda.synchronize()
        result["status"] = int(status.item())
        got = snaps.float().cpu().numpy()
        for e in range(1, epochs + 1):
            for r in range(world):
                if not (got[e, r * n:(r + 1) * n] == float(r * 100 + e)).all():
                    result["ok"] = False
                    result.setdefault("bad", []).append([e, r])
    finally:
        if pb is not None:
            dist.barrier()
            pb.close()
        Path(out_dir, f"b2b{rank}.json").write_text(json.dumps(result))
        dist.destroy_process_group()


def test_two_rank_back_to_back_epochs_with_a_slow_reader(tmp_path):
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_back_to_back_rank_main, args=(2, port, str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        res = json.loads((tmp_path / f"b2b{r}.json").read_text())
        assert res["ok"] and res["status"] == 0, res


def test_two_rank_decode_fused_with_allgather(tmp_path):
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_fused_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        res = json.loads((tmp_path / f"fused{r}.json").read_text())
        assert res["ok"] and res["close"], res


def test_two_rank_peer_allgather(tmp_path):
    import torch

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = json.loads((tmp_path / "rank0.json").read_text())
    r1 = json.loads((tmp_path / "rank1.json").read_text())
    for r in (r0, r1):
        assert r["ok"]
        assert all(r[f"status_{e}"] == 0 for e in range(1, 5))
        assert r["bad_world"] == -1 and r["bad_bytes"] == -1
    assert r0["timeout_status"] == 1 and r0["after"] == 8.0
