"""TEST INFRASTRUCTURE -- restatement of the reference's swap-tier eviction policies.

Follows ref src/kcmm/tiering.rs, trait EvictionPolicy and its implementations,
keeping their data structures literally (dicts for the timestamp / count maps,
Python lists for ARC's T1 / T2 / B1 / B2 with the most recent entry at index 0):

  LruPolicy         ref src/kcmm/tiering.rs:56-99
  LfuPolicy         ref src/kcmm/tiering.rs:103-153
  FifoPolicy        ref src/kcmm/tiering.rs:157-215
  ArcPolicy         ref src/kcmm/tiering.rs:217-446
  SinkWindowPolicy  ref src/kcmm/tiering.rs:448-555
  set_policy        ref src/kcmm/tiering.rs:877-895 (fresh object; ARC capacity =
                    cpu buffer bytes / max_batch_blocks; sink-window (1, 4))

Blocks are opaque hashable keys (the library passes block ids).  A logical clock
replaces Instant::now() (the same order, never equal).  Pinned against the
reference's own unit tests for these policies (tests/test_policy_oracle.py).
"""
from __future__ import annotations

import itertools

_clock = itertools.count(1)


def _by_key(keys: dict, candidates, count):
    """filter_map over the candidates that have a key, stable sort, truncate."""
    if not candidates or count == 0:
        return []
    tracked = [(h, keys[h]) for h in candidates if h in keys]
    tracked.sort(key=lambda x: x[1])  # list.sort is stable, as sort_by_key
    return [h for h, _ in tracked[:count]]


class LruPolicy:
    name = "lru"

    def __init__(self):
        self.access_times = {}

    def on_allocate(self, b):
        self.access_times[b] = next(_clock)

    def select_victims(self, candidates, count):
        return _by_key(self.access_times, candidates, count)

    def on_access(self, b):
        self.access_times[b] = next(_clock)

    def on_evict(self, b):
        self.access_times.pop(b, None)

    def register_block(self, b, seq, pos):
        pass


class LfuPolicy:
    name = "lfu"

    def __init__(self):
        self.access_counts = {}

    def on_allocate(self, b):
        self.access_counts[b] = 1

    def select_victims(self, candidates, count):
        return _by_key(self.access_counts, candidates, count)

    def on_access(self, b):
        self.access_counts[b] = self.access_counts.get(b, 0) + 1

    def on_evict(self, b):
        self.access_counts.pop(b, None)

    def register_block(self, b, seq, pos):
        pass


class FifoPolicy:
    name = "fifo"

    def __init__(self):
        self.alloc_times = {}

    def on_allocate(self, b):
        self.alloc_times[b] = next(_clock)

    def select_victims(self, candidates, count):
        return _by_key(self.alloc_times, candidates, count)

    def on_access(self, b):
        pass

    def on_evict(self, b):
        self.alloc_times.pop(b, None)

    def register_block(self, b, seq, pos):
        pass


class ArcPolicy:
    name = "arc"

    def __init__(self, capacity):
        self.t1, self.t2, self.b1, self.b2 = [], [], [], []
        self.p = 0
        self.capacity = max(capacity, 1)

    def _replace(self):  # ref :268-296
        if self.t1 and (len(self.t1) > self.p or not self.t2):
            v = self.t1.pop()
            self.b1.append(v)
            while len(self.b1) > self.capacity:
                self.b1.pop(0)
            return v
        if self.t2:
            v = self.t2.pop()
            self.b2.append(v)
            while len(self.b2) > self.capacity:
                self.b2.pop(0)
            return v
        return None

    def on_allocate(self, b):  # ref :300-339
        in_b1 = b in self.b1
        if in_b1:
            self.b1.remove(b)
        in_b2 = b in self.b2
        if in_b2:
            self.b2.remove(b)
        if in_b1:
            delta = max(max(len(self.b2), 1) // max(len(self.b1), 1), 1)
            self.p = min(self.p + delta, self.capacity)
            self.t2.insert(0, b)
        elif in_b2:
            delta = max(max(len(self.b1), 1) // max(len(self.b2), 1), 1)
            self.p = max(self.p - delta, 0)
            self.t2.insert(0, b)
        else:
            self.t1.insert(0, b)
        while len(self.t1) + len(self.t2) > self.capacity:
            self._replace()

    def select_victims(self, candidates, count):  # ref :341-392
        if not candidates or count == 0:
            return []

        def pos_from_tail(lst, h):
            for i, x in enumerate(reversed(lst)):
                if x == h:
                    return i
            return None

        scored = []
        for h in candidates:
            p1 = pos_from_tail(self.t1, h)
            p2 = pos_from_tail(self.t2, h)
            if p1 is not None:
                score = p1
            elif p2 is not None:
                score = len(self.t1) + p2
            else:
                score = len(self.t1) + len(self.t2) + 1
            scored.append((h, score))
        scored.sort(key=lambda x: x[1])
        return [h for h, _ in scored[:count]]

    def on_access(self, b):  # ref :394-411
        if b in self.t1:
            self.t1.remove(b)
            self.t2.insert(0, b)
            return
        if b in self.t2:
            self.t2.remove(b)
            self.t2.insert(0, b)

    def on_evict(self, b):  # ref :413-441
        if b in self.t1:
            self.t1.remove(b)
            if b not in self.b1:
                self.b1.append(b)
                while len(self.b1) > self.capacity:
                    self.b1.pop(0)
            return
        if b in self.t2:
            self.t2.remove(b)
            if b not in self.b2:
                self.b2.append(b)
                while len(self.b2) > self.capacity:
                    self.b2.pop(0)

    def register_block(self, b, seq, pos):
        pass


class SinkWindowPolicy:
    name = "sink_window"

    def __init__(self, sink_blocks, window_blocks):
        self.block_positions = {}
        self.access_times = {}
        self.sink_blocks = sink_blocks
        self.window_blocks = window_blocks

    def register_block(self, b, seq, pos):
        self.block_positions[b] = (seq, pos)

    def _is_protected(self, seq_blocks, h):  # ref :474-487
        if h in self.block_positions:
            seq, pos = self.block_positions[h]
            if pos < self.sink_blocks:
                return True
            if seq in seq_blocks and pos >= max(seq_blocks[seq] - self.window_blocks, 0):
                return True
        return False

    def on_allocate(self, b):
        self.access_times[b] = next(_clock)

    def select_victims(self, candidates, count):  # ref :494-523
        if not candidates or count == 0:
            return []
        seq_blocks = {}
        for seq, pos in self.block_positions.values():
            seq_blocks[seq] = max(seq_blocks.get(seq, 0), pos + 1)
        eligible = [h for h in candidates if not self._is_protected(seq_blocks, h)]
        return _by_key(self.access_times, eligible, count)

    def on_access(self, b):
        self.access_times[b] = next(_clock)

    def on_evict(self, b):
        self.access_times.pop(b, None)


def make_policy(name, arc_capacity=1, sink_blocks=1, window_blocks=4):
    """The policy set_policy(name) installs (ref src/kcmm/tiering.rs:877-895)."""
    if name == "lru":
        return LruPolicy()
    if name == "lfu":
        return LfuPolicy()
    if name == "fifo":
        return FifoPolicy()
    if name == "arc":
        return ArcPolicy(arc_capacity)
    if name == "sink_window":
        return SinkWindowPolicy(sink_blocks, window_blocks)
    raise ValueError(f"unknown eviction policy '{name}'")
