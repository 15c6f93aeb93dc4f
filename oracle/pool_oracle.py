"""TEST INFRASTRUCTURE -- restatement of the reference's KCMM block allocator.

Follows the Rust code path by path, keeping its data structures literally:
2*num_layers per-layer allocators advanced in lockstep (with the reference's
lockstep assertions), a `block_info` list, a LIFO list of recycled indices,
append-only sequences and a block-state epoch.

  PhysicalBlockAllocator  ref src/kcmm/superblock.rs:40-142
  ensure_capacity         ref src/kcmm/pool.rs:323-359 (capacity rule 1145-1151)
  alloc_one_block_internal/install_block  ref src/kcmm/pool.rs:364-453
  free_sequence           ref src/kcmm/pool.rs:478-546
  register/unregister     ref src/kcmm/pool.rs:551-572
  offsets/valid tables    ref src/kcmm/pool.rs:724-747
  CpuSlotAllocator        ref src/kcmm/tiering.rs:552-640

Refcounts (the B200 addition) are modelled the way the library defines them:
a block freed while shared only loses one owner.
"""
from __future__ import annotations

SUPERBLOCK_SIZE = 2 * 1024 * 1024


class OracleError(Exception):
    pass


class PhysicalBlockAllocator:
    def __init__(self, block_bytes: int):
        if block_bytes <= 0:
            raise OracleError("block_bytes must be positive")
        self.block_bytes = block_bytes
        self.blocks_per_superblock = SUPERBLOCK_SIZE // block_bytes
        if self.blocks_per_superblock == 0:
            raise OracleError(f"block_bytes ({block_bytes}) too large for superblock")
        self.free_blocks: list[tuple[int, int]] = []
        self.superblock_count = 0

    def try_allocate(self):
        return self.free_blocks.pop() if self.free_blocks else None

    def add_superblock(self) -> None:
        sb = self.superblock_count
        self.superblock_count += 1
        self.free_blocks.extend((sb, i) for i in range(self.blocks_per_superblock))

    def free(self, handle) -> None:
        self.free_blocks.append(handle)

    def free_count(self) -> int:
        return len(self.free_blocks)

    def total_blocks_allocated(self) -> int:
        return self.superblock_count * self.blocks_per_superblock

    def tail_padding_bytes_per_superblock(self) -> int:
        return SUPERBLOCK_SIZE - self.blocks_per_superblock * self.block_bytes


class BlockInfo:
    __slots__ = ("va_offset", "handle", "in_use", "location", "cpu_offset", "refcount")

    def __init__(self, va_offset, handle):
        self.va_offset = va_offset
        self.handle = handle
        self.in_use = True
        self.location = "gpu"
        self.cpu_offset = 0
        self.refcount = 1


class OraclePool:
    def __init__(self, *, num_layers: int, kv_heads: int, head_dim: int, max_batch: int,
                 max_seq_len: int, block_size: int = 16):
        self.block_size = block_size
        self.elem_per_block = kv_heads * block_size * head_dim
        self.block_bytes = self.elem_per_block * 2
        self.step = kv_heads * head_dim
        self.max_blocks_per_seq = (max_seq_len + block_size - 1) // block_size
        self.max_blocks_total = max_batch * self.max_blocks_per_seq
        self.num_layers = num_layers
        self.k_pools = [PhysicalBlockAllocator(self.block_bytes) for _ in range(num_layers)]
        self.v_pools = [PhysicalBlockAllocator(self.block_bytes) for _ in range(num_layers)]
        self.block_info: list[BlockInfo] = []
        self.free_block_indices: list[int] = []
        self.sequences: list[dict] = []
        self.epoch = 0

    # --- capacity -------------------------------------------------------
    def blocks_per_superblock(self) -> int:
        return self.k_pools[0].blocks_per_superblock

    def max_physical_blocks_per_layer(self) -> int:
        bps = self.blocks_per_superblock()
        return -(-self.max_blocks_total // bps) * bps

    def ensure_capacity(self) -> None:
        if self.k_pools[0].free_count() > 0:
            return
        total = self.k_pools[0].total_blocks_allocated()
        max_phys = self.max_physical_blocks_per_layer()
        if total >= max_phys:
            raise OracleError(
                "KCMM physical block capacity exhausted: "
                f"total_physical_blocks={total} max_physical_blocks_per_layer={max_phys} "
                f"max_blocks_total={self.max_blocks_total} "
                f"blocks_per_superblock={self.blocks_per_superblock()}")
        for layer in range(self.num_layers):
            self.k_pools[layer].add_superblock()
            self.v_pools[layer].add_superblock()

    # --- allocation -----------------------------------------------------
    def alloc_block(self) -> int:
        self.ensure_capacity()
        handle = None
        for layer in range(self.num_layers):
            hk = self.k_pools[layer].try_allocate()
            hv = self.v_pools[layer].try_allocate()
            if hk is None or hv is None:
                raise OracleError(f"pool layer {layer}: no free block after ensure_capacity")
            if handle is None:
                handle = hk
            else:
                assert handle == hk == hv, "lockstep violated"
        sb, blk = handle
        va_offset = sb * SUPERBLOCK_SIZE + blk * self.block_bytes
        info = BlockInfo(va_offset, handle)
        if self.free_block_indices:
            idx = self.free_block_indices.pop()
            self.block_info[idx] = info
        else:
            idx = len(self.block_info)
            self.block_info.append(info)
        self.epoch += 1
        return idx

    def alloc_blocks(self, n: int) -> list[int]:
        return [self.alloc_block() for _ in range(n)]

    def free_blocks(self, ids) -> None:
        handles = []
        recycled = []
        for b in ids:
            if b >= len(self.block_info):
                continue
            bi = self.block_info[b]
            if not bi.in_use:
                continue
            if bi.refcount > 1:
                bi.refcount -= 1
                continue
            if bi.location == "gpu":
                bi.in_use = False
                handles.append(bi.handle)
                recycled.append(b)
            elif bi.location in ("cpu", "nvme"):
                bi.in_use = False
                recycled.append(b)
            else:  # evicting / restoring: cleanup skipped
                continue
            bi.refcount = 0
        for h in handles:
            for layer in range(self.num_layers):
                self.k_pools[layer].free(h)
                self.v_pools[layer].free(h)
        if recycled:
            self.epoch += 1
            self.free_block_indices.extend(recycled)

    # --- sequences ------------------------------------------------------
    def register_sequence(self, table) -> int:
        self.sequences.append({"table": list(table), "seq_len": 0})
        return len(self.sequences) - 1

    def unregister_sequence(self, seq: int) -> None:
        if seq >= len(self.sequences):
            return
        table = self.sequences[seq]["table"]
        self.sequences[seq] = {"table": [], "seq_len": 0}
        if table:
            self.free_blocks(table)

    def append_block_to_sequence(self, seq: int, blk: int) -> None:
        if seq >= len(self.sequences):
            raise OracleError(f"seq_idx {seq} out of bounds")
        self.sequences[seq]["table"].append(blk)

    def fork_sequence(self, src: int) -> int:
        t = list(self.sequences[src]["table"])
        for b in t:
            self.block_info[b].refcount += 1
        self.sequences.append({"table": t, "seq_len": self.sequences[src]["seq_len"]})
        return len(self.sequences) - 1

    def cow(self, seq: int, logical: int):
        """Returns (new table entry, (src_off, dst_off) or None)."""
        t = self.sequences[seq]["table"]
        b = t[logical]
        if self.block_info[b].refcount <= 1:
            return b, None
        nb = self.alloc_block()
        self.block_info[b].refcount -= 1
        t[logical] = nb
        return nb, (self.block_info[b].va_offset, self.block_info[nb].va_offset)

    # --- queries ---------------------------------------------------------
    def block_va_offset(self, b: int) -> int:
        if b < len(self.block_info) and self.block_info[b].in_use:
            return self.block_info[b].va_offset
        return 0

    def all_block_offsets_f16(self) -> list[int]:
        return [bi.va_offset // 2 if bi.in_use else 0 for bi in self.block_info]

    def all_block_valid(self) -> list[int]:
        return [1 if bi.in_use else 0 for bi in self.block_info]

    def blocks_in_use(self) -> int:
        return sum(1 for bi in self.block_info if bi.in_use)

    def stats(self) -> dict:
        return {
            "blocks_in_use": self.blocks_in_use(),
            "total_blocks": len(self.block_info),
            "total_physical_blocks": self.k_pools[0].total_blocks_allocated(),
            "free_physical_blocks": self.k_pools[0].free_count(),
            "active_sequences": len(self.sequences),
            "num_layers": self.num_layers,
            "blocks_per_superblock": self.blocks_per_superblock(),
            "superblock_count": self.k_pools[0].superblock_count,
            "block_size": self.block_size,
            "max_blocks_per_seq": self.max_blocks_per_seq,
            "block_bytes": self.block_bytes,
        }

    # --- append addressing (ref src/kcmm/ffi.rs:1138-1186, 1310-1330) ------
    def step_destination(self, seq: int, pos: int) -> int:
        t = self.sequences[seq]["table"]
        lb, off = divmod(pos, self.block_size)
        if lb >= len(t):
            raise OracleError(f"logical_block {lb} >= allocated {len(t)} for seq {seq}")
        bi = self.block_info[t[lb]]
        if not bi.in_use:
            raise OracleError(f"block_idx {t[lb]} not in use")
        return bi.va_offset // 2 + off * self.step

    def slot_destination(self, slot: int):
        if slot < 0:
            return None
        blk, off = divmod(slot, self.block_size)
        if blk >= len(self.block_info) or not self.block_info[blk].in_use:
            raise OracleError(f"block_idx {blk} from slot {slot} not in use")
        return self.block_info[blk].va_offset // 2 + off * self.step


class CpuSlotAllocator:
    """Best-fit byte-range allocator with merge on free (ref src/kcmm/tiering.rs:552-640)."""

    def __init__(self, total: int):
        self.free_ranges = [[0, total]] if total > 0 else []

    def allocate(self, size: int):
        if size == 0 or not self.free_ranges:
            return None
        best, best_len = None, None
        for i, (s, e) in enumerate(self.free_ranges):
            n = e - s
            if n >= size and (best_len is None or n < best_len):
                best, best_len = i, n
        if best is None:
            return None
        off = self.free_ranges[best][0]
        if best_len == size:
            del self.free_ranges[best]
        else:
            self.free_ranges[best][0] += size
        return off

    def free(self, offset: int, size: int) -> None:
        if size == 0:
            return
        end = offset + size
        at = next((i for i, r in enumerate(self.free_ranges) if r[0] > offset),
                  len(self.free_ranges))
        prev = at > 0 and self.free_ranges[at - 1][1] == offset
        nxt = at < len(self.free_ranges) and self.free_ranges[at][0] == end
        if prev and nxt:
            self.free_ranges[at - 1][1] = self.free_ranges[at][1]
            del self.free_ranges[at]
        elif prev:
            self.free_ranges[at - 1][1] = end
        elif nxt:
            self.free_ranges[at][0] = offset
        else:
            self.free_ranges.insert(at, [offset, end])
