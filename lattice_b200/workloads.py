"""Seeded synthetic workloads of the benchmark configurations.

Builds a KCMM pool on a GPU, draws block tables from it and fills the K/V
pages, the way the engine would after prefill; shared by bench.py,
__graft_entry__.smoke() and the GPU tests.  torch provides device buffers and
streams only; every KV-path operation goes through the C ABI (`kcmm.py`).

The configurations follow BASELINE.json:
  decode_llama3_8b   Hq 32 / Hkv 8 / D 128, bf16, block 16, batch 64, context
                     lengths uniform in [512, 4096], tables drawn without
                     replacement from a 40,000-block pool, scale 1/sqrt(128)
  fused_append       256 decode tokens, hidden 4096, eps 1e-5, w ~ U(0.5, 1.5),
                     rope theta 500000 on D 128, positions uniform in [0, 8191],
                     8 kv heads, seeded distinct slots
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field

import numpy as np

from . import kcmm


def _torch():
    import torch

    return torch


def _cudart():
    from cuda.bindings import runtime as rt

    return rt


def memcpy(dst: int, src: int, nbytes: int, kind: str) -> None:
    """cudaMemcpy between raw addresses (kind: 'h2d', 'd2h', 'd2d')."""
    rt = _cudart()
    k = {"h2d": rt.cudaMemcpyKind.cudaMemcpyHostToDevice,
         "d2h": rt.cudaMemcpyKind.cudaMemcpyDeviceToHost,
         "d2d": rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice}[kind]
    (err,) = rt.cudaMemcpy(dst, src, nbytes, k)
    if int(err) != 0:
        raise RuntimeError(f"cudaMemcpy {kind} failed: {err}")


def read_device(addr: int, nbytes: int) -> np.ndarray:
    out = np.empty(nbytes, np.uint8)
    memcpy(out.ctypes.data, addr, nbytes, "d2h")
    return out


def write_device(addr: int, data: np.ndarray) -> None:
    data = np.ascontiguousarray(data)
    memcpy(addr, data.ctypes.data, data.nbytes, "h2d")


_LIB = None


def library() -> kcmm.KcmmLibrary:
    global _LIB
    if _LIB is None:
        _LIB = kcmm.KcmmLibrary()
    return _LIB


@dataclass
class DecodeWorkload:
    """A pool with `batch` sequences of paged KV and one query token each."""

    batch: int = 64
    num_q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    block_size: int = 16
    pool_blocks: int = 40000
    min_len: int = 512
    max_len: int = 4096
    dtype: str = "bf16"
    seed: int = 0
    num_layers: int = 1
    device: int = 0
    seq_lens_override: list | None = None
    fill: str = "device"  # "device": torch.randn on the GPU; "host": numpy (readable by the oracle)
    tiering: bool = False
    pool: kcmm.KcmmPool | None = field(default=None, repr=False)

    def build(self) -> "DecodeWorkload":
        torch = _torch()
        torch.cuda.set_device(self.device)
        rng = np.random.default_rng(self.seed)
        bs = self.block_size
        self.max_blocks_per_seq = -(-self.max_len // bs)
        # pool capacity: max_batch * ceil(max_seq_len/bs) >= pool_blocks
        max_batch = max(self.batch, -(-self.pool_blocks // self.max_blocks_per_seq))
        cfg = kcmm.make_config(num_layers=self.num_layers, kv_heads=self.kv_heads,
                               head_dim=self.head_dim, max_batch=max_batch,
                               max_seq_len=self.max_blocks_per_seq * bs, block_size=bs,
                               tiering=self.tiering, device=self.device,
                               max_blocks=self.pool_blocks if self.tiering else 0)
        self.pool = library().create_pool(cfg)
        self.block_ids = np.array(self.pool.alloc_blocks(self.pool_blocks), np.int64)
        if self.seq_lens_override is not None:
            self.seq_lens = np.array(self.seq_lens_override, np.int32)
        else:
            self.seq_lens = rng.integers(self.min_len, self.max_len + 1, self.batch).astype(np.int32)
        need = [max(1, -(-int(L) // bs)) for L in self.seq_lens]
        picks = rng.choice(len(self.block_ids), size=sum(need), replace=False)
        self.tables = np.zeros((self.batch, self.max_blocks_per_seq), np.int32)
        pos = 0
        self.seq_indices = []
        for b, n in enumerate(need):
            ids = self.block_ids[picks[pos:pos + n]]
            pos += n
            self.tables[b, :n] = ids
            self.seq_indices.append(self.pool.register_sequence([int(x) for x in ids]))
            self.pool.update_seq_len(self.seq_indices[-1], int(self.seq_lens[b]))
        self.offsets = np.array(self.pool.all_block_offsets_f16(), np.uint64)
        self.block_bytes = self.pool.stats()["block_bytes"]
        self.region_used = int(self.offsets.max()) * 2 + self.block_bytes
        tdt = torch.bfloat16 if self.dtype == "bf16" else torch.float16
        self.tdtype = tdt
        dev = f"cuda:{self.device}"
        gen = torch.Generator(device=dev).manual_seed(self.seed)
        self.host_regions = {}
        for layer in range(self.num_layers):
            for kind in ("k", "v"):
                base = self.pool.va_k(layer) if kind == "k" else self.pool.va_v(layer)
                n = self.region_used // 2
                if self.fill == "host":
                    vals = rng.standard_normal(n).astype(np.float32)
                    t = torch.from_numpy(vals).to(dev).to(tdt)
                    self.host_regions[(layer, kind)] = t.view(torch.int16).cpu().numpy().view(np.uint16)
                else:
                    t = torch.randn(n, device=dev, dtype=torch.float32, generator=gen).to(tdt)
                memcpy(base, t.data_ptr(), self.region_used, "d2d")
                del t
        self.q = torch.randn(self.batch, self.num_q_heads, self.head_dim, device=dev,
                             generator=gen, dtype=torch.float32).to(tdt)
        self.out = torch.zeros_like(self.q)
        self.d_tables = torch.from_numpy(self.tables).to(dev)
        self.d_seq_lens = torch.from_numpy(self.seq_lens).to(dev)
        self.d_offsets = torch.from_numpy(self.offsets.view(np.int64)).to(dev)
        self.scale = 1.0 / math.sqrt(self.head_dim)
        torch.cuda.synchronize()
        return self

    def decode(self, layer: int = 0, stream_ptr: int | None = None, out=None,
               noalloc: bool = False) -> None:
        torch = _torch()
        if stream_ptr is None:
            stream_ptr = torch.cuda.current_stream().cuda_stream
        out = self.out if out is None else out
        self.pool.paged_attn_decode(
            layer, query_ptr=self.q.data_ptr(), out_ptr=out.data_ptr(),
            block_tables_ptr=self.d_tables.data_ptr(), seq_lens_ptr=self.d_seq_lens.data_ptr(),
            block_offsets_f16_ptr=self.d_offsets.data_ptr(), batch=self.batch,
            num_q_heads=self.num_q_heads, kv_heads=self.kv_heads, head_dim=self.head_dim,
            block_size=self.block_size, max_blocks_per_seq=self.max_blocks_per_seq,
            scale=self.scale, dtype=self.dtype, stream_ptr=stream_ptr, noalloc=noalloc)

    def kv_bytes(self) -> int:
        """Algorithmic bytes of one decode pass (K and V rows, tables, q, out)."""
        e = 2
        L = self.seq_lens.astype(np.int64)
        kv = int((L * self.kv_heads * self.head_dim * e * 2).sum())
        tables = int(4 * np.ceil(L / self.block_size).sum())
        qo = self.batch * self.num_q_heads * self.head_dim * e * 2
        return kv + tables + qo + 4 * self.batch

    def region_tensor(self, layer: int, kind: str):
        """A torch view (16-bit words, no copy) of the used part of a K or V region."""
        torch = _torch()
        base = self.pool.va_k(layer) if kind == "k" else self.pool.va_v(layer)

        class _View:
            __cuda_array_interface__ = {"shape": (self.region_used // 2,), "typestr": "<i2",
                                        "data": (base, False), "version": 3}

        return torch.as_tensor(_View(), device=f"cuda:{self.device}").view(self.tdtype)

    def torch_reference(self, rows: list[int], layer: int = 0):
        """fp32 paged decode attention of sequences `rows` in plain torch on the device
        ([len(rows), Hq, D] float32): every key of the sequence through its block table
        and the offsets table, softmax(scale * q.k) v with kv head h * Hkv // Hq.  An
        independent check of the kernels for callers that cannot run the CPU oracle."""
        torch = _torch()
        dev = f"cuda:{self.device}"
        kr, vr = self.region_tensor(layer, "k"), self.region_tensor(layer, "v")
        step = self.kv_heads * self.head_dim
        outs = []
        for b in rows:
            L = int(self.seq_lens[b])
            if L <= 0:
                outs.append(torch.full((self.num_q_heads, self.head_dim), float("nan"), device=dev))
                continue
            t = torch.arange(L, device=dev)
            blk = torch.from_numpy(self.tables[b].astype(np.int64)).to(dev)[t // self.block_size]
            off = torch.from_numpy(self.offsets.view(np.int64)).to(dev)[blk]
            base = off + (t % self.block_size) * step
            idx = base[:, None] + torch.arange(step, device=dev)[None, :]
            k = kr[idx].float().view(L, self.kv_heads, self.head_dim)
            v = vr[idx].float().view(L, self.kv_heads, self.head_dim)
            q = self.q[b].float()
            kvh = torch.arange(self.num_q_heads, device=dev) * self.kv_heads // self.num_q_heads
            s = torch.einsum("hd,lhd->hl", q, k[:, kvh, :]) * self.scale
            p = torch.softmax(s, dim=-1)
            outs.append(torch.einsum("hl,lhd->hd", p, v[:, kvh, :]))
        return torch.stack(outs)

    def host_region(self, layer: int, kind: str) -> np.ndarray:
        """Current bytes of a region (16-bit words), read back from the device."""
        base = self.pool.va_k(layer) if kind == "k" else self.pool.va_v(layer)
        return read_device(base, self.region_used).view(np.uint16)

    def close(self) -> None:
        if self.pool is not None:
            self.pool.destroy()
            self.pool = None


@dataclass
class FusedAppendWorkload:
    """Inputs of the fused RMSNorm + RoPE + KV append for `tokens` decode tokens."""

    tokens: int = 256
    hidden: int = 4096
    num_q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    block_size: int = 16
    eps: float = 1e-5
    theta: float = 500000.0
    rope_mode: int = kcmm.RopeMode.REFERENCE
    max_pos: int = 8191
    seed: int = 0
    pool: kcmm.KcmmPool | None = None  # reuse a decode pool (same kv shape)
    layer: int = 0
    device: int = 0

    def build(self) -> "FusedAppendWorkload":
        torch = _torch()
        dev = f"cuda:{self.device}"
        rng = np.random.default_rng(self.seed + 1)
        gen = torch.Generator(device=dev).manual_seed(self.seed + 1)
        self.own_pool = self.pool is None
        if self.own_pool:
            cfg = kcmm.make_config(num_layers=1, kv_heads=self.kv_heads, head_dim=self.head_dim,
                                   max_batch=self.tokens, max_seq_len=self.block_size * 4,
                                   block_size=self.block_size, device=self.device)
            self.pool = library().create_pool(cfg)
            self.pool.alloc_blocks(self.tokens)
        nblk = self.pool.total_blocks()
        slots = rng.choice(nblk * self.block_size, size=self.tokens, replace=False)
        self.slots = slots.astype(np.int64)
        self.positions = rng.integers(0, self.max_pos + 1, self.tokens).astype(np.int32)
        bf = torch.bfloat16
        T, H, D = self.tokens, self.hidden, self.head_dim
        self.x = torch.randn(T, H, device=dev, generator=gen).to(bf)
        self.w = (torch.rand(H, device=dev, generator=gen) + 0.5).to(bf)
        self.q = torch.randn(T, self.num_q_heads, D, device=dev, generator=gen).to(bf)
        self.k = torch.randn(T, self.kv_heads, D, device=dev, generator=gen).to(bf)
        self.v = torch.randn(T, self.kv_heads, D, device=dev, generator=gen).to(bf)
        self.normed = torch.empty_like(self.x)
        self.d_pos = torch.from_numpy(self.positions).to(dev)
        self.d_slots = torch.from_numpy(self.slots).to(dev)
        self.offsets = np.array(self.pool.all_block_offsets_f16(), np.uint64)
        self.valid = np.array(self.pool.all_block_valid_flags(), np.uint8)
        self.d_offsets = torch.from_numpy(self.offsets.view(np.int64)).to(dev)
        self.d_valid = torch.from_numpy(self.valid).to(dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        return self

    def run(self, stream_ptr: int | None = None, q=None) -> None:
        torch = _torch()
        if stream_ptr is None:
            stream_ptr = torch.cuda.current_stream().cuda_stream
        q = self.q if q is None else q
        self.pool.fused_norm_rope_append_bf16(
            self.layer, x_ptr=self.x.data_ptr(), weight_ptr=self.w.data_ptr(),
            normed_ptr=self.normed.data_ptr(), hidden=self.hidden, eps=self.eps,
            q_ptr=q.data_ptr(), num_q_heads=self.num_q_heads, k_ptr=self.k.data_ptr(),
            v_ptr=self.v.data_ptr(), positions_ptr=self.d_pos.data_ptr(),
            rope_theta=self.theta, rope_mode=self.rope_mode,
            slot_mapping_ptr=self.d_slots.data_ptr(),
            block_offsets_f16_ptr=self.d_offsets.data_ptr(),
            valid_blocks_ptr=self.d_valid.data_ptr(), block_offsets_f16_len=len(self.offsets),
            num_tokens=self.tokens, status_ptr=self.status.data_ptr(), stream_ptr=stream_ptr)

    def bytes_per_launch(self) -> int:
        """Algorithmic bytes: x, q read+write, k, v read, pos, slot, normed/K/V write, w once."""
        T, H = self.tokens, self.hidden
        qd = self.num_q_heads * self.head_dim
        kd = self.kv_heads * self.head_dim
        per_token = 2 * (H + qd + kd + kd) + 4 + 8 + 2 * (H + qd + kd + kd)
        return T * per_token + 2 * H

    def close(self) -> None:
        if self.own_pool and self.pool is not None:
            self.pool.destroy()
        self.pool = None


@dataclass
class PrefillWorkload:
    """A chunk of new tokens per sequence over paged KV (pages from a DecodeWorkload whose
    seq_lens are the context lengths after the chunk)."""

    ctx_lens: list
    chunk_lens: list
    num_q_heads: int = 8
    kv_heads: int = 1
    head_dim: int = 128
    block_size: int = 16
    pool_blocks: int = 0
    dtype: str = "bf16"
    seed: int = 0
    fill: str = "host"
    device: int = 0

    def build(self) -> "PrefillWorkload":
        torch = _torch()
        assert all(0 <= c <= L for c, L in zip(self.chunk_lens, self.ctx_lens))
        bs = self.block_size
        need = sum(max(1, -(-int(L) // bs)) for L in self.ctx_lens)
        self.kv = DecodeWorkload(
            batch=len(self.ctx_lens), num_q_heads=self.num_q_heads, kv_heads=self.kv_heads,
            head_dim=self.head_dim, block_size=bs, pool_blocks=max(self.pool_blocks, need),
            max_len=max(self.ctx_lens), dtype=self.dtype, seed=self.seed,
            seq_lens_override=list(self.ctx_lens), fill=self.fill, device=self.device).build()
        dev = f"cuda:{self.device}"
        self.q_start = np.concatenate([[0], np.cumsum(self.chunk_lens)]).astype(np.int32)
        total = int(self.q_start[-1])
        gen = torch.Generator(device=dev).manual_seed(self.seed + 7)
        self.q = torch.randn(max(total, 1), self.num_q_heads, self.head_dim, device=dev,
                             generator=gen).to(self.kv.tdtype)
        self.out = torch.zeros_like(self.q)
        self.d_q_start = torch.from_numpy(self.q_start).to(dev)
        self.d_ctx = torch.from_numpy(np.asarray(self.ctx_lens, np.int32)).to(dev)
        self.scale = 1.0 / math.sqrt(self.head_dim)
        self.max_q_len = max(1, max(self.chunk_lens))
        torch.cuda.synchronize()
        return self

    @property
    def pool(self):
        return self.kv.pool

    def run(self, stream_ptr: int | None = None, out=None) -> None:
        torch = _torch()
        if stream_ptr is None:
            stream_ptr = torch.cuda.current_stream().cuda_stream
        out = self.out if out is None else out
        kv = self.kv
        self.pool.paged_prefill(
            0, query_ptr=self.q.data_ptr(), out_ptr=out.data_ptr(),
            block_tables_ptr=kv.d_tables.data_ptr(), query_start_loc_ptr=self.d_q_start.data_ptr(),
            context_lens_ptr=self.d_ctx.data_ptr(), block_offsets_f16_ptr=kv.d_offsets.data_ptr(),
            batch=len(self.ctx_lens), max_query_len=self.max_q_len, num_q_heads=self.num_q_heads,
            kv_heads=self.kv_heads, head_dim=self.head_dim, block_size=self.block_size,
            max_blocks_per_seq=kv.max_blocks_per_seq, scale=self.scale, dtype=self.dtype,
            stream_ptr=stream_ptr)

    def flops(self) -> int:
        """Causal attention FLOPs: 4 * d per (query row, key) pair with key <= position."""
        total = 0
        for L, c in zip(self.ctx_lens, self.chunk_lens):
            base = L - c
            total += c * base + c * (c + 1) // 2
        return 4 * self.head_dim * self.num_q_heads * total

    def close(self) -> None:
        self.kv.close()


def tensor_bits(t) -> np.ndarray:
    """uint16 bit pattern of a bf16/f16 torch tensor (host copy)."""
    torch = _torch()
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def cuda_stream_ptr() -> int:
    return _torch().cuda.current_stream().cuda_stream


_ = ctypes  # keep ctypes imported for users building raw pointers


class PeerBuffers:
    """A gathered-output buffer and a signal array per rank, mapped on every rank
    through CUDA IPC, for `kcmm_peer_allgather_on_stream` / `kcmm_peer_wait_on_stream`.

    Collective over the default process group: every rank allocates its own buffer
    (two halves of world slices of `slice_bytes`; epoch e fills half e & 1) and
    signal array, publishes their IPC handles with `all_gather_object`, and opens
    the peers'.  Pointers are indexed by rank; this rank's entries are its own
    allocations.  Every rank takes part in both exchanges even when its own step
    failed, and `ok` is the same on every rank: False when any rank could not
    allocate or open a mapping (the reason is in `error`), so callers skip the peer
    gathers together instead of one rank leaving the others waiting."""

    def __init__(self, slice_bytes: int, rank: int, world: int, device: int):
        import torch.distributed as dist

        rt = _cudart()
        torch = _torch()
        torch.cuda.set_device(device)
        self.rank, self.world, self.slice_bytes = rank, world, slice_bytes
        self.sig_words = int(library().lib.kcmm_peer_signal_words(world))
        self._own = []
        self._opened = []
        self.error = None
        handles = []
        try:
            for nbytes in (2 * slice_bytes * world, self.sig_words * 8):
                err, ptr = rt.cudaMalloc(nbytes)
                if int(err) != 0:
                    raise RuntimeError(f"cudaMalloc failed: {err}")
                self._own.append(int(ptr))
                (err,) = rt.cudaMemset(ptr, 0, nbytes)
                if int(err) != 0:
                    raise RuntimeError(f"cudaMemset failed: {err}")
                err, h = rt.cudaIpcGetMemHandle(ptr)
                if int(err) != 0:
                    raise RuntimeError(f"cudaIpcGetMemHandle failed: {err}")
                handles.append(bytes(h.reserved))
            rt.cudaDeviceSynchronize()
        except Exception as e:  # noqa: BLE001 - reported to every rank below
            self.error = f"rank {rank}: {e}"
            handles = None
        everyone = [None] * world
        dist.all_gather_object(everyone, handles)
        self.buf_ptrs, self.sig_ptrs = [], []
        failed = [r for r in range(world) if everyone[r] is None]
        if not failed:
            try:
                for r in range(world):
                    if r == rank:
                        self.buf_ptrs.append(self._own[0])
                        self.sig_ptrs.append(self._own[1])
                        continue
                    opened = []
                    for raw in everyone[r]:
                        h = rt.cudaIpcMemHandle_t()
                        h.reserved = raw
                        err, ptr = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                        if int(err) != 0:
                            raise RuntimeError(f"cudaIpcOpenMemHandle of rank {r} failed: {err}")
                        opened.append(int(ptr))
                        self._opened.append(int(ptr))
                    self.buf_ptrs.append(opened[0])
                    self.sig_ptrs.append(opened[1])
            except Exception as e:  # noqa: BLE001 - reported to every rank below
                self.error = f"rank {rank}: {e}"
        errors = [None] * world
        dist.all_gather_object(errors, self.error)
        bad = [e for e in errors if e is not None]
        if failed and not bad:
            bad = [f"rank {r} could not allocate its buffers" for r in failed]
        self.ok = not bad
        if not self.ok:
            self.error = "; ".join(bad)
            self.close()
        self.epoch = 0

    @property
    def gathered_ptr(self) -> int:
        """This rank's whole gathered buffer (both halves)."""
        return self._own[0]

    def half_ptr(self, epoch: int) -> int:
        """The half of this rank's gathered buffer that epoch `epoch` fills."""
        return self._own[0] + (epoch & 1) * self.slice_bytes * self.world

    @property
    def signal_ptr(self) -> int:
        return self._own[1]

    def close(self) -> None:
        rt = _cudart()
        rt.cudaDeviceSynchronize()
        for p in self._opened:
            rt.cudaIpcCloseMemHandle(p)
        for p in self._own:
            rt.cudaFree(p)
        self._opened, self._own = [], []
