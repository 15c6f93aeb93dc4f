"""KV-cache hot-path benchmark (BASELINE.json metric on its Llama-3-8B decode config).

One step = one decode step of one layer for a batch of 64 sequences:
  1. fused RMSNorm + RoPE + KV append of the 64 new tokens into their pages
     (kcmm_fused_norm_rope_append_bf16_on_stream), and
  2. paged decode attention over every sequence's context
     (kcmm_paged_attn_decode_bf16_on_stream),
both through the C ABI of libkcmm.so.  Context lengths are uniform in
[512, 4096] with block tables drawn without replacement from a 40,000-block
pool.  K/V pages are 1.25 GiB per region, far larger than
the 126 MB L2, so no flush is needed between steps ("inputs larger than L2").

`value` = whole-job KV-path GB/s (all ranks' attention + append bytes per step
/ max-over-ranks step time).  `tokens_per_s` = decode tokens/s of a 32-layer
model's KV path = B_total / (32 * t_step).

On one GPU the line also carries `secondary`: the other BASELINE configurations
(fused append, beam CoW + shared-prefix decode, swap, chunked prefill, step tables)
run after the headline with their own step counts (`--no-secondary` skips them;
`--workload <leg>` runs one alone and prints its own line).

Usage:
  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 launch with torch.distributed.run (one rank per GPU, weak scaling:
each rank owns its own 64 sequences and pool; no collective on the data path).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = ("paged decode attn KV GB/s (% of HBM peak) and decode tokens/s at 1/2/4/8 B200")
CONFIG = {"workload": "llama3-8b decode attention + fused norm/rope/append (BASELINE config 2)",
          "batch_per_gpu": 64, "num_q_heads": 32, "kv_heads": 8, "head_dim": 128,
          "block_size": 16, "context": "uniform [512, 4096]", "pool_blocks": 40000,
          "layers_for_tokens_per_s": 32, "l2": "inputs larger than L2 (2.5 GiB of pages)"}
LAYERS_FOR_TOKENS = 32


_RESULT_FD = [None]  # the process's original stdout once emit_result owns it


def claim_stdout() -> None:
    """Keep stdout for the result line alone: file descriptor 1 is pointed at stderr, so
    that what libraries print there (NCCL prints its version line when a communicator is
    created) cannot come before or between result lines, and emit_result writes to the
    original stdout."""
    if _RESULT_FD[0] is None:
        sys.stdout.flush()
        _RESULT_FD[0] = os.dup(1)
        os.dup2(2, 1)


def emit_result(obj) -> None:
    line = json.dumps(obj) + "\n"
    if _RESULT_FD[0] is None:
        sys.stdout.write(line)
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD[0], line.encode())


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """SM clock and clock-event reasons sampled every ~2 ms by an NVML thread while
    the timed region runs (read-only NVML queries; nothing is set).  Falls back to
    an `nvidia-smi -lms 100` subprocess when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.source = None
        self._thread = None
        self._stop = None
        self._proc = None

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
        return pynvml, h

    def start(self):
        import threading

        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - no NVML: use nvidia-smi
            self._start_smi()
            return
        self.source = "nvml"
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                try:
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((float(mhz), int(rs)))
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(0.002)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        time.sleep(0.01)

    def _start_smi(self):
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.SMI_FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi"
        except (FileNotFoundError, OSError):
            self._proc = None

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
            import pynvml

            reasons = set()
            for _, rs in self.samples:
                for name, const, bit in self.REASONS:
                    if rs & int(getattr(pynvml, const, bit)):
                        reasons.add(name)
            sm = [m for m, _ in self.samples]
        elif self._proc is not None:
            time.sleep(0.25)
            self._proc.terminate()
            try:
                out, _ = self._proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self._proc.kill()
                out, _ = self._proc.communicate()
            sm, reasons = [], set()
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for line in out.strip().splitlines():
                f = [x.strip() for x in line.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm.append(float(f[1]))
                    self.max_mhz = float(f[2])
                except ValueError:
                    continue
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        else:
            return None
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": self.source}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def max_over_ranks(ms: float) -> float:
    """Max of a per-rank duration over all ranks (identity without a process group)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return ms
    dev = (f"cuda:{torch.cuda.current_device()}" if dist.get_backend() == "nccl" else "cpu")
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(values: list[float]) -> list[list[float]]:
    """Every rank's `values`, as a list indexed by rank (the local list alone
    without a process group)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [list(values)]
    dev = (f"cuda:{torch.cuda.current_device()}" if dist.get_backend() == "nccl" else "cpu")
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    rows = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(rows, t)
    return [r.cpu().tolist() for r in rows]


def barrier() -> None:
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def whole_job_gbps(bytes_per_rank_step: int, world: int, ms_step: float) -> float:
    """Weak scaling: every rank processes its own bytes; the job takes the slowest rank."""
    return bytes_per_rank_step * world / (ms_step * 1e-3) / 1e9


def run_ours(args):
    import torch

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    from lattice_b200.workloads import DecodeWorkload, FusedAppendWorkload

    # --profile: same batch, heads and length distribution with the tables drawn
    # from a 12k-block pool, so that an ncu capture saves/restores < 1 GB per pass.
    pool_blocks = 12000 if args.profile else 40000
    # Every rank draws the same context lengths (one shared seed), so each rank moves
    # the same bytes and the 1 -> N curve measures the hardware; pages, tables and
    # queries come from a per-rank seed.
    lens = np.random.default_rng(1000).integers(512, 4097, 64).astype(np.int32).tolist()
    wl = DecodeWorkload(seed=1000 + rank, device=local, pool_blocks=pool_blocks,
                        seq_lens_override=lens).build()
    # the step's new token of sequence b sits at position L_b - 1 of its table
    slots = np.array([int(wl.tables[b, (L - 1) // 16]) * 16 + (L - 1) % 16
                      for b, L in enumerate(wl.seq_lens)], np.int64)
    fa = FusedAppendWorkload(tokens=wl.batch, pool=wl.pool, seed=2000 + rank,
                             device=local).build()
    fa.slots = slots
    fa.d_slots.copy_(torch.from_numpy(slots))
    q_step = wl.q  # the rotated q feeds attention
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step():
        fa.run(stream_ptr=sp, q=q_step)
        wl.decode(stream_ptr=sp)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.start()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    total_ms = max_over_ranks(t0.elapsed_time(t1))
    # per-kernel durations for the roofline: the same K steps again, with an event pair
    # around each of the two calls (kept out of the headline timing above)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        a, b, c = ev[i]
        a.record(stream)
        fa.run(stream_ptr=sp, q=q_step)
        b.record(stream)
        wl.decode(stream_ptr=sp)
        c.record(stream)
    torch.cuda.synchronize()
    attn_ms = [e[1].elapsed_time(e[2]) for e in ev]
    app_ms = [e[0].elapsed_time(e[1]) for e in ev]
    barrier()
    ms_step = total_ms / args.steps
    attn_bytes = wl.kv_bytes()
    app_bytes = fa.bytes_per_launch()
    value = whole_job_gbps(attn_bytes + app_bytes, world, ms_step)
    tokens_per_s = wl.batch * world / (LAYERS_FOR_TOKENS * ms_step * 1e-3)
    attn_avg = statistics.mean(attn_ms)
    achieved = attn_bytes / (attn_avg * 1e-3) / 1e9
    peak, peak_kind = peaks()
    from lattice_b200.kcmm import KcmmError  # noqa: F401  (import check)

    launches_per_step = 1 + 2  # fused append + decode main + split merge
    e2e = run_e2e(args, wl, fa, stream, world) if not args.profile else None
    status = wl.pool.kernel_status()
    per_rank = gather_over_ranks([attn_avg, attn_bytes, float(status)])
    cpu_baseline_sample = (cpu_baseline(wl) if rank == 0 and world == 1 and not args.profile
                           else None)
    wl.close()
    # BASELINE config 5's KV-head split on the same ranks (strong scaling)
    hs = headsplit_measure(args, world, rank, local) if not args.profile else None
    # the other BASELINE configurations, one GPU only
    secondary = (run_secondary_legs(args) if world == 1 and not args.profile
                 and not args.no_secondary else None)

    result = None
    if rank == 0:
        cpu = cpu_baseline_sample if world == 1 and not args.profile else None
        result = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 pages/q/x, uniform context lengths)",
            "config": dict(CONFIG, parallelism=f"replicas x{world} (sequence-sharded, no collective)"),
            "tokens_per_s": round(tokens_per_s, 1),
            "kv_gbs_attention_kernel": round(achieved, 1),
            "hbm_frac_attention": round(achieved / peak, 4),
            "attn_us_per_launch": round(attn_avg * 1e3, 2),
            "append_us_per_launch": round(statistics.mean(app_ms) * 1e3, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic_from_profiles(), "peak_kind": peak_kind,
                         "kernel": "paged decode attention (main + split merge), per launch",
                         "algorithmic_bytes_per_launch": attn_bytes},
            "gpu_launches": launches_per_step * args.steps,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clk,
            "device_status": int(max(r[2] for r in per_rank)),
            "per_rank": {
                "attn_us_min_max": [round(min(r[0] for r in per_rank) * 1e3, 2),
                                    round(max(r[0] for r in per_rank) * 1e3, 2)],
                "roofline_frac_min_max": [
                    round(min(r[1] / (r[0] * 1e-3) / 1e9 for r in per_rank) / peak, 4),
                    round(max(r[1] / (r[0] * 1e-3) / 1e9 for r in per_rank) / peak, 4)],
                "bytes_equal": len({r[1] for r in per_rank}) == 1},
            "headsplit": hs,
            "secondary": secondary,
        }
        emit_result(result)
    if world > 1:
        import torch.distributed as dist

        barrier()
        dist.destroy_process_group()
    return result


def run_e2e(args, wl, fa, stream, world):
    """Same step through the public API with host buffers: every step copies its inputs
    (q, x, k, v) from pinned host memory, makes the two ABI calls and reads the attention
    output back to pinned host memory.  Steps are double-buffered the way a serving loop
    runs them: the copy-in of step i+1 and the copy-out of step i-1 run on their own
    streams while step i computes.  Every rank runs it; the time is the max over ranks."""
    import torch

    dev_sets = [[wl.q, fa.x, fa.k, fa.v]]
    dev_sets.append([torch.empty_like(t) for t in dev_sets[0]])
    outs = [wl.out, torch.empty_like(wl.out)]
    host_in = [[t.detach().cpu().pin_memory() for t in dev_sets[0]] for _ in range(2)]
    host_out = [torch.empty_like(wl.out, device="cpu").pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host_in[0])
    d2h = host_out[0].numel() * host_out[0].element_size()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    sp = stream.cuda_stream
    in_done = [torch.cuda.Event() for _ in range(2)]
    compute_done = [torch.cuda.Event() for _ in range(2)]
    out_done = [torch.cuda.Event() for _ in range(2)]
    for e in compute_done + out_done:
        e.record(stream)

    def step(i):
        b = i & 1
        with torch.cuda.stream(s_in):  # inputs of step i into buffer set b
            s_in.wait_event(compute_done[b])  # step i-2 is done reading it
            for d, h in zip(dev_sets[b], host_in[b]):
                d.copy_(h, non_blocking=True)
            in_done[b].record(s_in)
        stream.wait_event(in_done[b])
        stream.wait_event(out_done[b])  # step i-2's output has been read back
        q, x, k, v = dev_sets[b]
        fa.x, fa.k, fa.v = x, k, v
        fa.run(stream_ptr=sp, q=q)
        wl.q = q
        wl.decode(stream_ptr=sp, out=outs[b])
        compute_done[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(compute_done[b])
            host_out[b].copy_(outs[b], non_blocking=True)
            out_done[b].record(s_out)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    s_in.wait_stream(stream)
    for i in range(args.steps):
        step(i)
    stream.wait_stream(s_out)
    t1.record(stream)
    torch.cuda.synchronize()
    fa.x, fa.k, fa.v = dev_sets[0][1:]
    wl.q = dev_sets[0][0]
    ms = max_over_ranks(t0.elapsed_time(t1)) / args.steps
    byts = wl.kv_bytes() + fa.bytes_per_launch()
    return {"value": round(whole_job_gbps(byts, world, ms), 2), "unit": "GB/s",
            "ms_per_step": round(ms, 5), "h2d_bytes_per_step": int(h2d) * world,
            "d2h_bytes_per_step": int(d2h) * world,
            "tokens_per_s": round(wl.batch * world / (LAYERS_FOR_TOKENS * ms * 1e-3), 1),
            "pipelining": "copy-in / compute / copy-out on three streams, double-buffered"}


def traffic_from_profiles():
    """DRAM bytes per decode launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "decode_attention_llama3_8b.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            return None
    return None


def _ref_attention_sample(wl_like, nseq, workers):
    """Reference kernel on the host for the first `nseq` sequences; returns (seconds, bytes)."""
    from oracle import native as N

    q, va_k, va_v, tables, seq, offsets, meta = wl_like
    t = time.perf_counter()
    if N.ref_available():
        N.ref_paged_attn("bf16", q[:nseq], va_k, va_v, tables[:nseq], seq[:nseq], offsets,
                         workers=workers, **meta)
        kind = "reference"
    else:
        N.paged_attn("bf16", q[:nseq], va_k, va_v, tables[:nseq], seq[:nseq], offsets, **meta)
        kind = "port"
    dt = time.perf_counter() - t
    L = seq[:nseq].astype(np.int64)
    byts = int((L * meta["hkv"] * meta["d"] * 2 * 2).sum() + 4 * np.ceil(L / 16).sum()
               + nseq * meta["hq"] * meta["d"] * 4)
    return dt, byts, kind


def cpu_baseline(wl, nseq: int = 16):
    """The reference's decode attention (its own kernel source compiled for the host,
    oracle/_ref, bf16 storage) on a bounded sample of this workload, all host threads."""
    from lattice_b200.workloads import tensor_bits

    workers = os.cpu_count() or 1
    q = tensor_bits(wl.q).reshape(wl.batch, -1)
    va_k, va_v = wl.host_region(0, "k"), wl.host_region(0, "v")
    meta = dict(hq=wl.num_q_heads, hkv=wl.kv_heads, d=wl.head_dim, bs=wl.block_size,
                max_bps=wl.max_blocks_per_seq, scale=wl.scale)
    dt, byts, kind = _ref_attention_sample(
        (q, va_k, va_v, wl.tables, wl.seq_lens, wl.offsets, meta), nseq, workers)
    return {"value": round(byts / dt / 1e9, 3), "unit": "GB/s", "cores": workers, "kind": kind,
            "sample": f"decode attention of {nseq} of the {wl.batch} sequences "
                      f"({int(wl.seq_lens[:nseq].sum())} tokens x 32 q heads), {dt:.2f} s"}


def run_reference(args):
    """Reference arm: the reference's own decode-attention kernel compiled for the host
    (oracle/_ref; the oracle port when the reference tree was absent at build time),
    on every host thread, over a bounded sample of the same workload per step."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    from oracle import native as N

    rng = np.random.default_rng(1000)
    B, hq, hkv, D, bs, pool = 64, 32, 8, 128, 16, 40000
    seq = rng.integers(512, 4097, B).astype(np.int32)
    max_bps = 256
    need = [-(-int(L) // bs) for L in seq]
    nmax = 4  # at most 4 sequences per step, fewer when K steps would run past ~2 minutes
    used = sum(need[:nmax])
    perm = rng.permutation(used).astype(np.int32)
    tables = np.zeros((B, max_bps), np.int32)
    pos = 0
    for b in range(nmax):
        tables[b, :need[b]] = perm[pos:pos + need[b]]
        pos += need[b]
    step_elems = hkv * D
    offsets = np.arange(used, dtype=np.uint64) * np.uint64(bs * step_elems)
    va_k = N.f32_to_bf16_bits(rng.standard_normal(used * bs * step_elems).astype(np.float32))
    va_v = N.f32_to_bf16_bits(rng.standard_normal(used * bs * step_elems).astype(np.float32))
    q = N.f32_to_bf16_bits(rng.standard_normal((B, hq * D)).astype(np.float32))
    meta = dict(hq=hq, hkv=hkv, d=D, bs=bs, max_bps=max_bps, scale=D ** -0.5)
    workers = os.cpu_count() or 1
    sample = (q, va_k, va_v, tables, seq, offsets, meta)
    t_one = min(_ref_attention_sample(sample, 1, workers)[0]
                for _ in range(max(1, min(args.warmup, 2))))
    nseq = max(1, min(nmax, int(120.0 / (max(args.steps, 1) * max(t_one, 1e-6)))))
    times, byts, kind = [], 0, "reference"
    for _ in range(args.steps):
        dt, byts, kind = _ref_attention_sample(sample, nseq, workers)
        times.append(dt)
    dt = statistics.mean(times)
    value = byts / dt / 1e9
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": dict(CONFIG, parallelism="host cores"),
        "impl": "reference",
        "tokens_per_s": round(nseq / (LAYERS_FOR_TOKENS * dt), 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": workers,
                         "kind": kind if N.ref_available() else "port",
                         "sample": f"decode attention of {nseq} sequences "
                                   f"({int(seq[:nseq].sum())} tokens x 32 q heads) per step"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit_result(line)
    return line


# --- secondary legs (one JSON line each; `--workload` selects one) -----------------


def _gate(torch, cycles: int = 2_000_000):
    """Hold the stream (~1 ms by default) so that the host-side work of the next ABI
    call (allocator bookkeeping, launch) overlaps it and the following event pair
    times only the device work."""
    torch.cuda._sleep(cycles)


_QUIET = [False]  # set while the secondary legs run inside the headline bench


def _line(metric, value, unit, config, roofline, extra=None):
    out = {"metric": metric, "value": round(value, 3), "unit": unit, "n_gpus": 1,
           "higher_is_better": True, "dtype": "bf16", "data": "synthetic", "config": config,
           "roofline": roofline}
    out.update(extra or {})
    if not _QUIET[0]:
        emit_result(out)
    return out


def run_secondary_legs(args) -> dict:
    """The secondary BASELINE configurations, run after the headline on one GPU so that
    their numbers sit in the headline line too: the fused append (config 3), beam
    CoW and shared-prefix decode (config 4), swap and chunked prefill (config 5), and
    the device-resident step tables (config 2).  Each leg is one process-local
    measurement with its own steps; a leg that fails records its error instead."""
    legs = {"append": (run_append_leg, 50, 5), "cow": (run_cow_leg, 20, 3),
            "swap": (run_swap_leg, 5, 2), "prefill": (run_prefill_leg, 3, 2),
            "tables": (run_tables_leg, 64, 3)}
    out = {}
    _QUIET[0] = True
    try:
        for name, (fn, steps, warmup) in legs.items():
            leg_args = argparse.Namespace(**vars(args))
            leg_args.steps, leg_args.warmup = steps, warmup
            t0 = time.perf_counter()
            try:
                res = fn(leg_args)
                res = {k: v for k, v in res.items()
                       if k not in ("n_gpus", "higher_is_better", "dtype", "data")}
            except Exception as e:  # noqa: BLE001 - one leg's failure is reported, not fatal
                res = {"error": f"{type(e).__name__}: {e}"}
            res["leg_wall_s"] = round(time.perf_counter() - t0, 1)
            out[name] = res
    finally:
        _QUIET[0] = False
    return out


def run_append_leg(args):
    """Fused RMSNorm + RoPE + KV append for a 256-token decode batch:
    (i) one launch, L2 flushed between launches; (ii) 32 layers, one launch per layer
    over per-layer buffers (336 MB > L2), replayed as one CUDA graph."""
    import torch

    from lattice_b200 import kcmm
    from lattice_b200.workloads import FusedAppendWorkload, library

    torch.cuda.set_device(0)
    peak, kind = peaks()
    one = FusedAppendWorkload(tokens=256, seed=3).build()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    for _ in range(max(args.warmup, 3)):
        one.run(stream_ptr=sp)
    # One launch after an L2 flush, timed on the device: events around K x (flush,
    # launch) minus events around K x flush.  Both loops are queued ahead of the GPU,
    # so no host launch gap sits inside either (an event pair around one lone launch
    # measures mostly the host's launch latency: ~10 us even for an empty kernel).
    def loop(with_kernel):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(2_000_000)  # the host queues the whole loop meanwhile
        a.record()
        for _ in range(args.steps):
            flush.zero_()
            if with_kernel:
                one.run(stream_ptr=sp)
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    pairs = [(loop(True), loop(False)) for _ in range(5)]
    t1 = statistics.median([(p - f) / args.steps for p, f in pairs])
    st1 = int(one.status.item())
    b1 = one.bytes_per_launch()
    one.close()

    layers = 32
    cfg = kcmm.make_config(num_layers=layers, kv_heads=8, head_dim=128, max_batch=256,
                           max_seq_len=64, block_size=16)
    pool = library().create_pool(cfg)
    pool.alloc_blocks(256)
    legs = [FusedAppendWorkload(tokens=256, seed=100 + l, pool=pool, layer=l).build()
            for l in range(layers)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = None
    with torch.cuda.stream(side):
        for fa in legs:  # warm-up outside capture
            fa.run(stream_ptr=side.cuda_stream)
    torch.cuda.synchronize()
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            cs = torch.cuda.current_stream().cuda_stream
            for fa in legs:
                fa.run(stream_ptr=cs)
        replay = graph.replay
        how = "CUDA graph of 32 launches"
    except Exception as e:  # noqa: BLE001 - report and time the plain launches instead
        graph = None
        how = f"32 plain launches (graph capture failed: {type(e).__name__})"

        def replay():
            for fa in legs:
                fa.run(stream_ptr=torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        replay()
    b.record()
    torch.cuda.synchronize()
    t32 = a.elapsed_time(b) / args.steps
    b32 = sum(fa.bytes_per_launch() for fa in legs)
    st32 = max(int(fa.status.item()) for fa in legs)
    del graph
    for fa in legs:
        fa.close()
    pool.destroy()
    g1 = b1 / (t1 * 1e-3) / 1e9
    g32 = b32 / (t32 * 1e-3) / 1e9
    return _line(
        "fused RMSNorm+RoPE+KV append GB/s (32 layers)", g32, "GB/s",
        {"workload": "BASELINE config 3: 256 tokens, hidden 4096, Hq 32, Hkv 8, D 128, bs 16, "
                     "theta 500000, reference rope mode", "layers": layers, "timing": how},
        {"bound": "hbm", "achieved": round(g32, 1), "peak": peak, "unit": "GB/s",
         "frac": round(g32 / peak, 4), "traffic": None, "peak_kind": kind,
         "algorithmic_bytes_per_launch": b32},
        {"us_32_layers": round(t32 * 1e3, 2),
         "single_launch": {"us": round(t1 * 1e3, 2), "gbs": round(g1, 1),
                           "frac": round(g1 / peak, 4), "bytes": b1,
                           "l2": "flushed (256 MiB written before every launch)",
                           "timing": "events: K x (flush + launch) minus K x flush"},
         "status": max(st1, st32)})


def run_cow_leg(args):
    """Beam-search CoW (BASELINE config 4 shapes, 32 layers): 16 requests x 4 beams share a
    2048-token prefix plus a partly filled tail block; a step forks the 4 beams from their
    request and copies each beam's shared tail (64 whole-block copies across all 64
    regions), then runs decode attention of the 64 beams over the shared pages twice:
    the plain decode (every beam reads the prefix pages) and the shared-prefix decode
    (the 4 beams of a request form a group that reads them once).  Both are reported
    against the unique bytes; the leg checks that they agree."""
    import torch

    from lattice_b200 import kcmm
    from lattice_b200.workloads import library, memcpy

    torch.cuda.set_device(0)
    peak, kind = peaks()
    layers, reqs, beams, prefix_blocks = 32, 16, 4, 128
    cfg = kcmm.make_config(num_layers=layers, kv_heads=8, head_dim=128, max_batch=128,
                           max_seq_len=2048 + 256, block_size=16)
    pool = library().create_pool(cfg)
    parents = []
    for _ in range(reqs):
        blocks = pool.alloc_blocks(prefix_blocks + 1)
        s = pool.register_sequence(blocks)
        pool.update_seq_len(s, 2048 + 8)
        parents.append(s)
    bb = pool.stats()["block_bytes"]
    used = max(pool.block_va_offset(b) for p in parents for b in pool.block_table(p)) + bb
    gen = torch.Generator(device="cuda").manual_seed(4)
    for l in range(layers):
        for base in (pool.va_k(l), pool.va_v(l)):
            t = torch.randn(used // 2, device="cuda", generator=gen).to(torch.bfloat16)
            memcpy(base, t.data_ptr(), used, "d2d")
    del t
    sp = torch.cuda.current_stream().cuda_stream
    copy_ms, attn_ms, shared_ms = [], [], []
    q = torch.randn(reqs * beams, 32, 128, device="cuda", generator=gen).to(torch.bfloat16)
    out = torch.empty_like(q)
    out_shared = torch.empty_like(q)
    # the beams of a request form a group sharing the 2048-token prefix
    g_starts = torch.arange(0, reqs * beams + 1, beams, dtype=torch.int32, device="cuda")
    g_prefix = torch.full((reqs,), 2048, dtype=torch.int32, device="cuda")
    max_diff = 0.0
    copies = 0
    # Both attention calls start from a flushed L2 (256 MiB written first): the shared
    # call would otherwise find much of the 136 MB it reads left in L2 by the plain call.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for it in range(max(args.warmup, 3) + args.steps):
        forks = [pool.fork_sequence(p) for p in parents for _ in range(beams)]
        tails = [prefix_blocks] * len(forks)
        shared = [pool.block_table(f)[prefix_blocks] for f in forks]
        _gate(torch)
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        new = pool.cow_blocks(forks, tails, stream_ptr=sp)
        b.record()
        tables = np.array([pool.block_table(f) for f in forks], np.int32)
        d_tables = torch.from_numpy(tables).cuda()
        d_lens = torch.full((len(forks),), 2048 + 8, dtype=torch.int32, device="cuda")
        d_offs = torch.from_numpy(np.array(pool.all_block_offsets_f16(), np.uint64)
                                  .view(np.int64)).cuda()
        flush.zero_()
        _gate(torch)
        b2 = torch.cuda.Event(enable_timing=True)
        b2.record()
        pool.paged_attn_decode(0, query_ptr=q.data_ptr(), out_ptr=out.data_ptr(),
                               block_tables_ptr=d_tables.data_ptr(),
                               seq_lens_ptr=d_lens.data_ptr(),
                               block_offsets_f16_ptr=d_offs.data_ptr(), batch=len(forks),
                               num_q_heads=32, kv_heads=8, head_dim=128, block_size=16,
                               max_blocks_per_seq=tables.shape[1], scale=128 ** -0.5,
                               stream_ptr=sp)
        c.record()
        flush.zero_()
        _gate(torch)
        c2, d = (torch.cuda.Event(enable_timing=True) for _ in range(2))
        c2.record()
        assert pool.lib.kcmm_paged_attn_decode_shared_prefix_bf16_on_stream(
            pool.handle, 0, q.data_ptr(), out_shared.data_ptr(), d_tables.data_ptr(),
            d_lens.data_ptr(), d_offs.data_ptr(), len(forks), 32, 8, 128, 16, tables.shape[1],
            128 ** -0.5, g_starts.data_ptr(), g_prefix.data_ptr(), reqs, beams, sp) == 0, \
            pool.last_error()
        d.record()
        torch.cuda.synchronize()
        max_diff = max(max_diff, float((out_shared.float() - out.float()).abs().max()))
        if it >= max(args.warmup, 3):
            copy_ms.append(a.elapsed_time(b))
            attn_ms.append(b2.elapsed_time(c))
            shared_ms.append(c2.elapsed_time(d))
        copies = sum(1 for n, o in zip(new, shared) if n != o)
        for f in forks:
            pool.unregister_sequence(f)
    status = pool.kernel_status()
    pool.destroy()
    tc = statistics.median(copy_ms)
    ta = statistics.median(attn_ms)
    ts = statistics.median(shared_ms)
    # unique bytes: each request's 4 beams copy the same parent tail, so a step reads 16
    # distinct source blocks and writes 64 new ones (per region); the 3 repeat reads of a
    # source come from L2 and are not counted as HBM work
    src_unique = min(copies, reqs) * 2 * layers * bb
    cow_bytes = src_unique + copies * 2 * layers * bb
    logical_cow = copies * 2 * layers * bb * 2
    g = cow_bytes / (tc * 1e-3) / 1e9
    ctx = 2048 + 8
    logical = reqs * beams * ctx * 8 * 128 * 2 * 2
    unique = reqs * 2048 * 8 * 128 * 2 * 2 + reqs * beams * 8 * 8 * 128 * 2 * 2
    return _line(
        "CoW block copy GB/s (64 beam tails x 32 layers)", g, "GB/s",
        {"workload": "BASELINE config 4: 16 requests x 4 beams, 2048-token shared prefix, "
                     "Hkv 8, D 128, bs 16, bf16", "layers": layers,
         "timing": "device time of kcmm_cow_blocks_on_stream (host bookkeeping overlapped)",
         "l2": "flushed (256 MiB written) before each attention call"},
        {"bound": "hbm", "achieved": round(g, 1), "peak": peak, "unit": "GB/s",
         "frac": round(g / peak, 4), "traffic": None, "peak_kind": kind,
         "algorithmic_bytes_per_launch": cow_bytes},
        {"copies_per_step": copies, "cow_us": round(tc * 1e3, 2),
         "cow_logical_bytes": logical_cow,
         "cow_logical_gbs": round(logical_cow / (tc * 1e-3) / 1e9, 1),
         "beam_attention": {"us": round(ta * 1e3, 2), "logical_bytes": logical,
                            "unique_bytes": unique,
                            "logical_gbs": round(logical / (ta * 1e-3) / 1e9, 1),
                            "unique_gbs": round(unique / (ta * 1e-3) / 1e9, 1)},
         "beam_attention_shared_prefix": {
             "call": "kcmm_paged_attn_decode_shared_prefix_bf16_on_stream (the 4 beams of a "
                     "request form a group sharing 2048 tokens)",
             "us": round(ts * 1e3, 2),
             "unique_gbs": round(unique / (ts * 1e-3) / 1e9, 1),
             "unique_frac_of_hbm": round(unique / (ts * 1e-3) / 1e9 / peak, 4),
             "logical_gbs": round(logical / (ts * 1e-3) / 1e9, 1),
             "speedup_vs_plain": round(ta / ts, 2),
             "max_abs_diff_vs_plain": round(max_diff, 6)},
         "status": status})


def run_swap_leg(args):
    """Tiering swap (per GPU: 1 kv head, 8 layers -> 64 KiB per block):
    20% of 16,384 blocks swapped to the pinned host tier and back, one launch series each
    way, against the measured pinned host-link copy bandwidth."""
    import torch

    from lattice_b200 import kcmm
    from lattice_b200.workloads import library, memcpy

    torch.cuda.set_device(0)
    layers, seqs, ctx = 8, 8, 32768
    cfg = kcmm.make_config(num_layers=layers, kv_heads=1, head_dim=128, max_batch=seqs,
                           max_seq_len=ctx, block_size=16, tiering=True,
                           max_blocks=seqs * ctx // 16)
    pool = library().create_pool(cfg)
    nblk = seqs * ctx // 16
    blocks = pool.alloc_blocks(nblk)
    for s in range(seqs):
        q = pool.register_sequence(blocks[s * (nblk // seqs):(s + 1) * (nblk // seqs)])
        pool.update_seq_len(q, ctx)
    bb = pool.stats()["block_bytes"]
    used = nblk * bb
    gen = torch.Generator(device="cuda").manual_seed(5)
    for l in range(layers):
        for base in (pool.va_k(l), pool.va_v(l)):
            t = torch.randint(-32768, 32767, (used // 2,), device="cuda", generator=gen,
                              dtype=torch.int16)
            memcpy(base, t.data_ptr(), used, "d2d")
    del t
    rng = np.random.default_rng(5)
    sp = torch.cuda.current_stream().cuda_stream
    nv = nblk // 5
    out_ms, in_ms = [], []
    for it in range(max(2, min(args.warmup, 3)) + min(args.steps, 10)):
        victims = [int(b) for b in rng.choice(blocks, nv, replace=False)]
        _gate(torch, 20_000_000)  # ~10 ms: covers the host bookkeeping of 3276 blocks
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        pool.swap_out(victims, stream_ptr=sp)
        b.record()
        _gate(torch, 20_000_000)  # ~10 ms: covers the host bookkeeping of 3276 blocks
        c, d = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c.record()
        pool.swap_in(victims, stream_ptr=sp)
        d.record()
        torch.cuda.synchronize()
        if it >= max(2, min(args.warmup, 3)):
            out_ms.append(a.elapsed_time(b))
            in_ms.append(c.elapsed_time(d))
    status = pool.kernel_status()
    pool.destroy()
    # pinned host-link reference: one 256 MiB cudaMemcpyAsync each way
    n = 256 << 20
    host = torch.empty(n, dtype=torch.uint8).pin_memory()
    dev = torch.empty(n, dtype=torch.uint8, device="cuda")
    link = {}
    for name, fn in (("h2d", lambda: dev.copy_(host, non_blocking=True)),
                     ("d2h", lambda: host.copy_(dev, non_blocking=True))):
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            fn()
        e1.record()
        torch.cuda.synchronize()
        link[name] = n * 5 / (e0.elapsed_time(e1) * 1e-3) / 1e9
    moved = nv * layers * 2 * bb
    go = moved / (statistics.median(out_ms) * 1e-3) / 1e9
    gi = moved / (statistics.median(in_ms) * 1e-3) / 1e9
    return _line(
        "swap out+in GB/s (20% of blocks, 64 KiB per block)", 2 * moved /
        ((statistics.median(out_ms) + statistics.median(in_ms)) * 1e-3) / 1e9, "GB/s",
        {"workload": "BASELINE config 5 tiering leg per GPU: 8 x 32768 tokens, Hkv 1, D 128, "
                     "bs 16, 8 layers (64 KiB per block across 16 regions), 20% of blocks",
         "timing": "device time of kcmm_swap_{out,in}_blocks_on_stream"},
        {"bound": "host link", "achieved": round(min(go, gi), 2),
         "peak": round(min(link["d2h"], link["h2d"]), 2), "unit": "GB/s",
         "frac": round(min(go / link["d2h"], gi / link["h2d"]), 4), "traffic": None,
         "peak_kind": "measured pinned cudaMemcpyAsync, 256 MiB"},
        {"blocks_per_step": nv, "bytes_each_way": moved,
         "swap_out": {"ms": round(statistics.median(out_ms), 3), "gbs": round(go, 2),
                      "frac_of_d2h": round(go / link["d2h"], 4)},
         "swap_in": {"ms": round(statistics.median(in_ms), 3), "gbs": round(gi, 2),
                     "frac_of_h2d": round(gi / link["h2d"], 4)},
         "pinned_link_gbs": {k: round(v, 2) for k, v in link.items()}, "status": status})


def run_prefill_leg(args):
    """Chunked prefill (per GPU: 8 q heads on 1 kv head, D 128, bf16):
    8 sequences of 32,768 tokens prefilled in 16 chunks of 2048 tokens, one launch per
    chunk for all 8 sequences (one layer).  Tensor-bound: causal FLOPs / time against
    the measured bf16 dense peak.  `--head-dim` runs the same shape at another head_dim
    (128: the two-tile kernel; others: the single-role kernel)."""
    import torch

    from lattice_b200.workloads import PrefillWorkload

    torch.cuda.set_device(0)
    seqs, ctx, chunk, hq, hkv = 8, 32768, 2048, 8, 1
    hd = getattr(args, "head_dim", 128)
    wl = PrefillWorkload(ctx_lens=[ctx] * seqs, chunk_lens=[chunk] * seqs, num_q_heads=hq,
                         kv_heads=hkv, head_dim=hd, seed=5, fill="device").build()
    ctx_by_chunk = [torch.full((seqs,), (c + 1) * chunk, dtype=torch.int32, device="cuda")
                    for c in range(ctx // chunk)]
    sp = torch.cuda.current_stream().cuda_stream

    def chunk_call(c):
        wl.d_ctx = ctx_by_chunk[c]
        wl.run(stream_ptr=sp)

    def flops(c):
        base = c * chunk
        return 4 * hd * hq * seqs * (chunk * base + chunk * (chunk + 1) // 2)

    for _ in range(max(args.warmup, 3)):
        chunk_call(ctx // chunk - 1)
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 5))
    nchunks = ctx // chunk
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(nchunks)] for _ in range(steps)]
    clocks = ClockSampler(0)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for s_ in range(steps):
        for c in range(nchunks):
            ev[s_][c][0].record()
            chunk_call(c)
            ev[s_][c][1].record()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / steps
    total = sum(flops(c) for c in range(nchunks))
    per_chunk = [statistics.median(ev[s_][c][0].elapsed_time(ev[s_][c][1]) for s_ in range(steps))
                 for c in range(nchunks)]
    last_tf = flops(nchunks - 1) / (per_chunk[-1] * 1e-3) / 1e12
    tf = total / (ms * 1e-3) / 1e12
    status = wl.pool.kernel_status()
    wl.close()
    d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(d.get("bf16_tflops", 1590.0))
    kind = "measured (burst)" if d else "fallback"
    return _line(
        "chunked prefill TFLOP/s (causal, 32k context in 2048-token chunks)", tf, "TFLOP/s",
        {"workload": "BASELINE config 5 per GPU: 8 seqs x 32768 tokens, 2048-token chunks, "
                     f"8 q heads / 1 kv head, D {hd}, bf16, one layer", "launches": nchunks},
        {"bound": "tensor", "achieved": round(last_tf, 1), "peak": peak, "unit": "TFLOP/s",
         "frac": round(last_tf / peak, 4), "traffic": None, "peak_kind": kind,
         "kernel": ("prefill_pair_kernel" if hd == 128 else "prefill_kernel (single-role)")
                   + ", last chunk (2048 queries x 32768 keys x 8 seqs)",
         "algorithmic_flops_per_launch": flops(nchunks - 1)},
        {"ms_per_layer": round(ms, 3), "total_flops": total,
         "frac_of_peak_all_chunks": round(tf / peak, 4),
         "sustained_peak": d.get("bf16_tflops_sustained"),
         "us_per_chunk": [round(t * 1e3, 1) for t in per_chunk], "clocks": clk,
         "status": status})


HEADSPLIT = {"num_q_heads": 64, "kv_heads": 8, "seqs": 8, "context": 32768}


def headsplit_measure(args, world: int, rank: int, local: int) -> dict | None:
    """Llama-3-70B decode with KV heads sharded across the N ranks:
    8 sequences of 32,768 tokens, 64 q heads / 8 kv heads, D 128, bf16.  Rank r holds
    kv heads [r*8/N, (r+1)*8/N) and their query heads for every sequence; a step is the
    paged decode of the rank's heads followed by an all-gather of the per-head outputs
    ([8, 64/N, 128] bf16 per rank) so every rank holds the full [8, 64, 128].  The
    all-gather runs three ways: NCCL all_gather_into_tensor after the decode;
    `kcmm_peer_allgather_on_stream` + `kcmm_peer_wait_on_stream` after the decode (stores
    into the peers' buffers over NVLink and per-CTA flags); and
    `kcmm_paged_attn_decode_bf16_allgather_on_stream` + the wait, where the decode's
    merge kernel stores the rows into the peers' buffers itself.  Steps run back to
    back with no host barrier (the gathered buffers alternate halves by epoch).

    Parity, on every rank: the rank's own rows of two sampled sequences against a
    torch fp32 reference of the same pages (max-abs 2e-3 / max-rel 1e-2), and every
    peer-store gather bit-identical to NCCL's; the flags reduced over ranks.
    Strong scaling: the total work is fixed as N grows.  Returns the summary on rank 0
    (None elsewhere); every rank takes the same collective steps."""
    import ctypes

    import torch

    from lattice_b200.workloads import DecodeWorkload, PeerBuffers, library, read_device

    torch.cuda.set_device(local)
    hq, hkv = HEADSPLIT["num_q_heads"], HEADSPLIT["kv_heads"]
    seqs, ctx = HEADSPLIT["seqs"], HEADSPLIT["context"]
    if hkv % world:
        return {"skipped": f"{world} ranks do not divide {hkv} kv heads"} if rank == 0 else None
    hkv_l, hq_l = hkv // world, hq // world
    wl = DecodeWorkload(batch=seqs, num_q_heads=hq_l, kv_heads=hkv_l, head_dim=128,
                        min_len=ctx, max_len=ctx, pool_blocks=seqs * ctx // 16,
                        seed=3000 + rank, device=local).build()
    dev = f"cuda:{local}"
    gathered = torch.empty((world,) + tuple(wl.out.shape), dtype=wl.out.dtype, device=dev)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    import torch.distributed as dist

    lib = library().lib
    slice_bytes = wl.out.numel() * wl.out.element_size()
    pb = PeerBuffers(slice_bytes, rank, world, local) if world > 1 else None
    peer_error = None
    if pb is not None and not pb.ok:  # the same on every rank: NCCL is still measured
        peer_error, pb = pb.error, None
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    if world > 1 and pb is None:
        dst = sig = None
        sig_local = 0
        half = None
    elif pb is not None:
        dst = (ctypes.c_uint64 * world)(*pb.buf_ptrs)
        sig = (ctypes.c_uint64 * world)(*pb.sig_ptrs)
        sig_local = pb.signal_ptr
        half = pb.half_ptr
    else:  # one rank: the fused decode gathers into its own buffer (two halves)
        own = torch.empty((2,) + tuple(gathered.shape), dtype=wl.out.dtype, device=dev)
        own_sig = torch.zeros(lib.kcmm_peer_signal_words(1), dtype=torch.int64, device=dev)
        dst = (ctypes.c_uint64 * 1)(own.data_ptr())
        sig = (ctypes.c_uint64 * 1)(own_sig.data_ptr())
        sig_local = own_sig.data_ptr()
        half = lambda e: own[e & 1].data_ptr()  # noqa: E731
    epoch = [0]

    def step_nccl():
        wl.decode(stream_ptr=sp)
        if world > 1:
            dist.all_gather_into_tensor(gathered, wl.out)
        else:
            gathered[0].copy_(wl.out)

    def step_p2p():
        wl.decode(stream_ptr=sp)
        epoch[0] += 1
        assert lib.kcmm_peer_allgather_on_stream(wl.out.data_ptr(), slice_bytes, dst, sig, rank,
                                                 world, epoch[0], sp) == 0
        assert lib.kcmm_peer_wait_on_stream(sig_local, world, epoch[0], status.data_ptr(),
                                            sp) == 0

    def step_fused():
        # the split merge stores the rows straight into every rank's buffer
        epoch[0] += 1
        assert lib.kcmm_paged_attn_decode_bf16_allgather_on_stream(
            wl.pool.handle, 0, wl.q.data_ptr(), wl.out.data_ptr(), wl.d_tables.data_ptr(),
            wl.d_seq_lens.data_ptr(), wl.d_offsets.data_ptr(), wl.batch, wl.num_q_heads,
            wl.kv_heads, wl.head_dim, wl.block_size, wl.max_blocks_per_seq, wl.scale, dst, sig,
            rank, world, epoch[0], sp) == 0, wl.pool.last_error()
        assert lib.kcmm_peer_wait_on_stream(sig_local, world, epoch[0], status.data_ptr(),
                                            sp) == 0

    def timed(step):
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / args.steps

    ms_nccl = timed(step_nccl)
    ref = gathered.view(torch.int16).cpu().numpy().view(np.uint8).reshape(-1).copy()
    # this rank's rows of two sequences against the torch fp32 reference
    sample = [0, seqs - 1]
    want = wl.torch_reference(sample)
    got = gathered[rank][sample].float()
    err = (got - want).abs()
    close = bool((err <= 2e-3 + 1e-2 * want.abs()).all())
    max_err = float(err.max().item())
    ms_p2p, p2p_same, ms_fused, fused_same = None, True, None, True
    if world > 1 and pb is not None:
        ms_p2p = timed(step_p2p)
        torch.cuda.synchronize()
        p2p_same = bool((read_device(half(epoch[0]), slice_bytes * world) == ref).all())
    if world == 1 or pb is not None:
        ms_fused = timed(step_fused)
        torch.cuda.synchronize()
        fused_same = bool((read_device(half(epoch[0]), slice_bytes * world) == ref).all())
    gather_status = int(status.item())
    # attention alone, for the split of the step
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    a0.record(stream)
    for _ in range(args.steps):
        wl.decode(stream_ptr=sp)
    a1.record(stream)
    torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / args.steps
    kv_rank = wl.kv_bytes()
    dev_status = wl.pool.kernel_status()
    # one row per rank: times, parity flags, status words
    mine = torch.tensor([ms_nccl, ms_p2p if ms_p2p is not None else 0.0,
                         ms_fused if ms_fused is not None else 0.0, attn_ms,
                         float(close and p2p_same and fused_same), float(gather_status),
                         float(dev_status), max_err], dtype=torch.float64, device=dev)
    rows = [torch.zeros_like(mine) for _ in range(world)]
    if world > 1:
        dist.all_gather(rows, mine)
        barrier()
        if pb is not None:
            pb.close()
    else:
        rows = [mine]
    wl.close()
    if rank != 0:
        return None
    r = torch.stack(rows).cpu().numpy()
    ms = {"nccl": float(r[:, 0].max())}
    if ms_fused is not None:
        ms["fused_p2p"] = float(r[:, 2].max())
    if ms_p2p is not None:
        ms["p2p"] = float(r[:, 1].max())
    used = min(ms, key=ms.get)
    attn = r[:, 3]
    peak, kind = peaks()
    kv_total = kv_rank * world  # every rank reads its own heads' pages (equal shards)
    gbs = kv_total / (ms[used] * 1e-3) / 1e9
    per_rank_frac = kv_rank / (attn * 1e-3) / 1e9 / peak
    return {
        "workload": "BASELINE config 5 decode: 8 seqs x 32768 tokens, Hq 64 / Hkv 8, D 128, "
                    "bf16; kv heads sharded over the ranks, outputs all-gathered",
        "scaling": "strong", "ranks": world, "kv_heads_per_rank": hkv_l,
        "value": round(gbs, 1), "unit": "GB/s (whole job, KV bytes / max-over-ranks step)",
        "ms_per_step": round(ms[used], 4), "allgather_used": used,
        "ms_per_step_nccl_allgather": round(ms["nccl"], 4),
        "ms_per_step_p2p_allgather": round(ms["p2p"], 4) if "p2p" in ms else None,
        "ms_per_step_fused_decode_allgather": (round(ms["fused_p2p"], 4)
                                               if "fused_p2p" in ms else None),
        "peer_buffers_error": peer_error,
        "attention_ms": round(float(attn.max()), 4),
        "attention_ms_min_max_over_ranks": [round(float(attn.min()), 4),
                                            round(float(attn.max()), 4)],
        "allgather_ms": {k: round(max(v - float(attn.max()), 0.0), 4) for k, v in ms.items()},
        "roofline_frac_per_rank_min_max": [round(float(per_rank_frac.min()), 4),
                                           round(float(per_rank_frac.max()), 4)],
        "peak_gbs": peak, "peak_kind": kind,
        "tokens_per_s_80_layers": round(seqs / (80 * ms[used] * 1e-3), 1),
        "parity": bool((r[:, 4] == 1.0).all()),
        "parity_check": "every rank: own rows of sequences 0 and 7 vs a torch fp32 reference "
                        "(max-abs 2e-3 / max-rel 1e-2); peer-store and fused gathers "
                        "bit-identical to NCCL's",
        "max_abs_err": float(r[:, 7].max()),
        "status": int(max(r[:, 5].max(), r[:, 6].max())),
    }


def run_headsplit_leg(args):
    """`--workload headsplit`: the KV-head split of config 5 alone, one JSON line."""
    world, rank, local = dist_setup(args)
    hs = headsplit_measure(args, world, rank, local)
    line = None
    if rank == 0:
        roof = None
        if "value" in hs:
            frac = hs["value"] / world / hs["peak_gbs"]
            roof = {"bound": "hbm", "achieved": round(hs["value"] / world, 1),
                    "peak": hs["peak_gbs"], "unit": "GB/s", "frac": round(frac, 4),
                    "traffic": None, "peak_kind": hs["peak_kind"], "per": "GPU"}
        line = _line("70B decode, KV heads sharded: KV GB/s (whole job) and decode tokens/s",
                     hs.get("value", 0.0), "GB/s", {"workload": hs.get("workload"),
                                                    "ranks": world, "scaling": "strong"},
                     roof, {"n_gpus": world, "headsplit": hs})
    if world > 1:
        import torch.distributed as dist

        barrier()
        dist.destroy_process_group()
    return line


def run_tables_leg(args):
    """Block-table maintenance per decode step on the Llama-3-8B decode shape (64
    sequences, contexts U[512, 4096], 32 layers): each step every sequence gains one
    token (a new block every 16 tokens, as the reference scheduler appends them,
    src/batch/continuous_scheduler.rs:692-712).

    * ours: `kcmm_step_tables_sync_on_stream` on the device-resident tables (the
      changed entries in one pinned copy and one scatter kernel), timed from the call
      to the completion of its device work;
    * reference pattern (src/model/llama_transformer.rs:277-303, :338-339): the host
      builds the tables, lengths and offsets table, then copies the offsets once and
      the tables and lengths once per layer from pageable memory.  Its host build runs
      here through the C ABI from Python (ctypes calls; the Rust original makes the
      same queries natively), so the build time is reported on its own and the copies
      on their own.
    Both ways read the same pool; the leg checks that they end with equal tables."""
    import time

    import numpy as np
    import torch

    from lattice_b200.kcmm import StepTables
    from lattice_b200.workloads import DecodeWorkload, read_device, write_device

    torch.cuda.set_device(0)
    steps = min(args.steps, 256)
    rng = np.random.default_rng(1000)
    lens = [int(x) for x in rng.integers(512, 4097, 64)]
    wl = DecodeWorkload(batch=64, num_q_heads=32, kv_heads=8, head_dim=128,
                        pool_blocks=40000, max_len=4096 + 16 * (steps // 16 + 2),
                        seq_lens_override=lens, seed=1000).build()
    pool, seqs = wl.pool, list(wl.seq_indices)
    layers, mbps = 32, wl.max_blocks_per_seq
    # return the blocks no sequence holds, so the steps' appends find free blocks
    used = {int(wl.tables[b, j]) for b, L in enumerate(lens) for j in range(max(1, -(-L // 16)))}
    pool.free_blocks([int(b) for b in wl.block_ids if int(b) not in used][:4096])
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    tables = StepTables(pool, 64)
    d_bt = torch.zeros(64 * mbps, dtype=torch.int32, device="cuda")
    d_sl = torch.zeros(64, dtype=torch.int32, device="cuda")
    d_off = torch.zeros(60000, dtype=torch.int64, device="cuda")

    def advance():
        for b, s in enumerate(seqs):
            if lens[b] % 16 == 0:  # the next token starts a new block
                pool.append_block_to_sequence(s, pool.alloc_blocks(1)[0])
            lens[b] += 1
            pool.update_seq_len(s, lens[b])

    def reference_build():
        bt = np.zeros((64, mbps), np.int32)
        for b, s in enumerate(seqs):
            t = pool.block_table(s)[:mbps]
            bt[b, :len(t)] = t
        sl = np.array([pool.seq_len(s) for s in seqs], np.int32)
        off = np.array(pool.all_block_offsets_f16(), np.uint64)
        return bt, sl, off

    def reference_upload(bt, sl, off):
        write_device(d_off.data_ptr(), off)
        for _ in range(layers):
            write_device(d_bt.data_ptr(), bt)
            write_device(d_sl.data_ptr(), sl)

    for _ in range(max(args.warmup, 3)):
        advance()
        tables.sync(seqs, sp)
        reference_upload(*reference_build())
    torch.cuda.synchronize()
    st0 = tables.stats()
    ours, build, upload, ref_bytes = [], [], [], 0
    for _ in range(steps):
        advance()
        t0 = time.perf_counter()
        tables.sync(seqs, sp)
        stream.synchronize()
        t1 = time.perf_counter()
        bt, sl, off = reference_build()
        t2 = time.perf_counter()
        reference_upload(bt, sl, off)
        t3 = time.perf_counter()
        ours.append(t1 - t0)
        build.append(t2 - t1)
        upload.append(t3 - t2)
        ref_bytes = off.nbytes + layers * (bt.nbytes + sl.nbytes)
    st1 = tables.stats()
    # both ways hold the same tables now
    got_bt = read_device(tables.block_tables_ptr, 64 * mbps * 4).view(np.int32)
    got_sl = read_device(tables.seq_lens_ptr, 64 * 4).view(np.int32)
    got_off = read_device(tables.block_offsets_ptr, off.nbytes).view(np.uint64)
    same = (np.array_equal(got_bt, bt.reshape(-1)) and np.array_equal(got_sl, sl)
            and np.array_equal(got_off, off))
    tables.destroy()
    wl.close()
    med = lambda v: float(np.median(v)) * 1e6  # noqa: E731
    ours_us = med(ours)
    out = _line(
        "block-table maintenance per decode step (us, host + device)", ours_us, "us",
        {"workload": "BASELINE config 2 decode step: 64 seqs, contexts U[512,4096] growing by "
                     "one token per step, 40k-block pool, 32 layers",
         "steps": steps},
        None,
        {"higher_is_better": False,
         "ours": {"us_per_step": round(ours_us, 2),
                  "bytes_per_step": round((st1["bytes"] - st0["bytes"]) / steps, 1),
                  "entries_per_step": round((st1["table_entries"] - st0["table_entries"]
                                             + st1["offset_entries"] - st0["offset_entries"])
                                            / steps, 1)},
         "reference_pattern": {"upload_us_per_step": round(med(upload), 2),
                               "host_build_us_per_step_ctypes": round(med(build), 2),
                               "bytes_per_step": ref_bytes,
                               "copies_per_step": 1 + 2 * layers},
         "tables_equal": bool(same)})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--profile", action="store_true",
                    help="profiling case for ncu: 12k-block pool, no CPU baseline / e2e legs")
    ap.add_argument("--no-secondary", dest="no_secondary", action="store_true",
                    help="skip the secondary configurations after the headline (one GPU)")
    ap.add_argument("--head-dim", dest="head_dim", type=int, default=128,
                    help="head_dim of the prefill leg (BASELINE config 5 uses 128)")
    ap.add_argument("--workload",
                    choices=["step", "append", "cow", "swap", "prefill", "headsplit",
                             "tables"],
                    default="step",
                    help="step = the headline (default); the others print one line for a "
                         "secondary BASELINE config")
    args = ap.parse_args()
    claim_stdout()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "append":
        run_append_leg(args)
    elif args.workload == "cow":
        run_cow_leg(args)
    elif args.workload == "swap":
        run_swap_leg(args)
    elif args.workload == "prefill":
        run_prefill_leg(args)
    elif args.workload == "headsplit":
        run_headsplit_leg(args)
    elif args.workload == "tables":
        run_tables_leg(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
