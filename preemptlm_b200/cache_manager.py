"""Byte-budget expert cache manager with sampled LFRU / LRU eviction.

Same policy and state machine as ``ExpertCacheManager``
(preempt/engine/expert_io/cache_manager.py:43-310): Redis-style sampling of
``sample_size`` evictable entries with ``np.random.default_rng(seed)``
(``integers(0, n, size=sample_size * 10)`` per decision, full scan below the
sample size or when the sample finds nothing evictable), victim = min of
(freq, last) for LFRU or last for LRU, swap-remove key list, DEMAND admissions
pinned until ``mark_safe_to_evict``.  Keys are plain ints (global expert ids).
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum

import numpy as np

from .bank import ReadPriority


class CacheEvictionPolicy(str, Enum):
    LFRU = "lfru"
    LRU = "lru"


@dataclass
class _Entry:
    num_bytes: int
    freq: int
    last: int
    slot: int
    can_evict: bool


class ExpertCacheManager:
    def __init__(self, *, budget_bytes: int, policy: CacheEvictionPolicy = CacheEvictionPolicy.LFRU,
                 sample_size: int = 5, seed: int = 67):
        if budget_bytes < 1:
            raise ValueError(f"`budget_bytes` must be positive, got `budget_bytes={budget_bytes}`.")
        if sample_size < 1:
            raise ValueError(f"`sample_size` must be positive, got `sample_size={sample_size}`.")
        self._budget_bytes = budget_bytes
        self._policy = CacheEvictionPolicy(policy)
        self._eviction_sample_size = sample_size
        self._rng = np.random.default_rng(seed)
        self._entries: dict[int, _Entry] = {}
        self._expert_idxs: list[int] = []
        self._bytes_size = 0
        self._clock = 0
        self._num_hits = self._num_misses = self._num_evictions = self._num_bytes_read = 0

    def __contains__(self, item) -> bool:
        return item in self._entries

    def __len__(self) -> int:
        return len(self._entries)

    policy = property(lambda self: self._policy)
    budget_bytes = property(lambda self: self._budget_bytes)
    cache_size = property(lambda self: self._bytes_size)
    hits = property(lambda self: self._num_hits)
    misses = property(lambda self: self._num_misses)
    evictions = property(lambda self: self._num_evictions)
    bytes_read = property(lambda self: self._num_bytes_read)

    def touch(self, expert_idx: int) -> bool:
        e = self._entries.get(expert_idx)
        if e is None:
            self._num_misses += 1
            return False
        self._num_hits += 1
        self._clock += 1
        e.freq += 1
        e.last = self._clock
        return True

    def admit(self, expert_idx: int, num_bytes: int, priority: int = ReadPriority.PREFETCH) -> tuple[int, ...]:
        if num_bytes > self._budget_bytes:
            raise ValueError(f"The size of expert {expert_idx} ({num_bytes / 1024**3} GB) exceeds the cache's "
                             f"total memory budget ({self._budget_bytes / 1024**3} GB).")
        if expert_idx in self._entries:
            return tuple()
        self._num_bytes_read += num_bytes
        evicted: list[int] = []
        while self._bytes_size + num_bytes > self._budget_bytes:
            target = self._select_eviction_target()
            self.evict(target)
            evicted.append(target)
            self._num_evictions += 1
        self._clock += 1
        self._entries[expert_idx] = _Entry(num_bytes, 1, self._clock, len(self._expert_idxs),
                                           priority != ReadPriority.DEMAND)
        self._expert_idxs.append(expert_idx)
        self._bytes_size += num_bytes
        return tuple(evicted)

    def mark_safe_to_evict(self, expert_idx: int) -> None:
        if (e := self._entries.get(expert_idx)) is not None:
            e.can_evict = True

    def _select_eviction_target(self) -> int:
        n = len(self._expert_idxs)
        if n <= self._eviction_sample_size:
            targets = [k for k in self._expert_idxs if self._entries[k].can_evict]
        else:
            targets = []
            for i in self._rng.integers(0, n, size=self._eviction_sample_size * 10):
                k = self._expert_idxs[i]
                if self._entries[k].can_evict:
                    targets.append(k)
                    if len(targets) == self._eviction_sample_size:
                        break
            if not targets:
                targets = [k for k in self._expert_idxs if self._entries[k].can_evict]
        if not targets:
            raise RuntimeError("No evictable experts found in the cache: in-flight demand reads exceed the "
                               f"memory budget ({self.budget_bytes / 1024**3} GB).")
        return min(targets, key=self._rank)

    def _rank(self, expert_idx: int) -> tuple[int, int]:
        e = self._entries[expert_idx]
        return (0, e.last) if self._policy is CacheEvictionPolicy.LRU else (e.freq, e.last)

    def evict(self, expert_idx: int) -> None:
        e = self._entries.pop(expert_idx)
        moved = self._expert_idxs.pop()
        if moved != expert_idx:
            self._expert_idxs[e.slot] = moved
            self._entries[moved].slot = e.slot
        self._bytes_size -= e.num_bytes
