"""Expert I/O for slot refills: ``DiskBackedExpertLoader`` with demand reads
that preempt prefetch reads, over a host (pinned) blob cache.

Mirrors preempt/engine/expert_io/loader.py:28-319 -- ``load``, ``load_sync``,
``enqueue_prefetch`` and ``close`` keep their names and results; requests
order by ``ReadPriority`` (DEMAND 0 before PREFETCH 1, requests.py:11-21);
duplicate in-flight reads are merged (loader.py:128-147); cache admission is
serialised (loader.py:100-116); read errors propagate to every waiter and
nothing is cached for them (loader.py:166-171).

The reference runs its reads as asyncio tasks on an event loop; here they run
on worker threads (``os.preadv`` releases the GIL), so ``event_loop`` is
accepted and ignored.  Demand reads (``load_sync``) run immediately on their
own thread pool and, while any is outstanding, prefetch workers hold back
before starting a new read -- a demand refill never queues behind prefetches.
``load_sync`` serves hits from the prefetch cache; the reference's
``load_sync`` bypasses the cache, which is the same result with no reuse.
"""

from __future__ import annotations

import heapq
import itertools
import threading
import time
from collections.abc import Generator, Sequence
from concurrent.futures import Future, ThreadPoolExecutor, as_completed
from dataclasses import dataclass, field

from .bank import ReadPriority, SerializedExpert
from .cache_manager import ExpertCacheManager


@dataclass
class GenerationMetrics:
    """Counters of preempt/engine/metrics.py:28-75 that the loader feeds."""

    cache_hits: int = 0
    cache_misses: int = 0
    demand_stall_s: float = 0.0
    prefetched_bytes: int = 0
    wasted_prefetch_bytes: int = 0
    steps: list = field(default_factory=list)


class HostExpertCache:
    """Blob cache in host memory keyed by global expert id (the role of
    ``MlxExpertCache``, expert_cache.py:99-195, one tier up: blobs stay in
    their pinned read buffers, ready for H2D refills)."""

    def __init__(self, manager: ExpertCacheManager):
        self.manager = manager
        self._entries: dict[int, SerializedExpert] = {}
        self._bytes = 0
        self._prefetched_unused: set[int] = set()

    def __contains__(self, item) -> bool:
        return item in self._entries

    def add(self, expert: SerializedExpert, prefetched: bool = False) -> None:
        prev = self._entries.get(expert.idx)
        if prev is not None:
            self._bytes -= prev.nbytes()
        self._entries[expert.idx] = expert
        self._bytes += expert.nbytes()
        if prefetched:
            self._prefetched_unused.add(expert.idx)

    def get(self, idx: int) -> SerializedExpert:
        try:
            e = self._entries[idx]
        except KeyError:
            raise KeyError(idx) from None
        self._prefetched_unused.discard(idx)
        self.manager.mark_safe_to_evict(idx)
        return e

    def evict(self, idx: int) -> int:
        """Drop ``idx``; returns its bytes if it was prefetched and never used."""
        e = self._entries.pop(idx)
        self._bytes -= e.nbytes()
        if idx in self._prefetched_unused:
            self._prefetched_unused.discard(idx)
            return e.nbytes()
        return 0

    def size(self) -> int:
        return self._bytes


@dataclass(order=True)
class LoadRequest:
    """requests.py:11-21 -- ordered by priority (then arrival)."""

    priority: int
    seq: int
    expert_idx: int = field(compare=False)
    completion_handle: Future = field(compare=False)


class DiskBackedExpertLoader:
    def __init__(self, *, expert_bank, cache: HostExpertCache | None = None,
                 cache_manager: ExpertCacheManager | None = None, event_loop=None, num_worker_threads: int = 8,
                 num_demand_threads: int = 16, max_queue_size: int = 0, metrics: GenerationMetrics | None = None):
        self._expert_bank = expert_bank
        if cache is None:
            if cache_manager is None:
                blob = expert_bank.manifest.expert_num_bytes()
                cache_manager = ExpertCacheManager(budget_bytes=max(blob, 64 * blob))
            cache = HostExpertCache(cache_manager)
        self._cache = cache
        self._cache_manager = cache_manager or cache.manager
        self._metrics = metrics
        self._max_queue_size = max_queue_size
        self._heap: list[LoadRequest] = []
        self._seq = itertools.count()
        self._cv = threading.Condition()
        self._lock = threading.Lock()  # cache admission + in-flight table
        self._inflight: dict[int, Future] = {}
        self._demand_outstanding = 0
        self._closed = False
        self._demand_pool = ThreadPoolExecutor(max_workers=num_demand_threads, thread_name_prefix="sg-demand")
        self._workers = [threading.Thread(target=self._worker_loop, name=f"sg-prefetch-{i}", daemon=True)
                         for i in range(num_worker_threads)]
        for w in self._workers:
            w.start()

    # ------------------------------------------------------------------ internals
    def _bump(self, name: str, value) -> None:
        if self._metrics is not None:
            setattr(self._metrics, name, getattr(self._metrics, name) + value)

    def _admit(self, expert: SerializedExpert, priority: int) -> None:
        with self._lock:
            if expert.idx in self._cache:
                return
            wasted = 0
            for victim in self._cache_manager.admit(expert.idx, expert.nbytes(), priority):
                if victim in self._cache:
                    wasted += self._cache.evict(victim)
            self._cache.add(expert, prefetched=priority == ReadPriority.PREFETCH)
        if wasted:
            self._bump("wasted_prefetch_bytes", wasted)

    def _read(self, idx: int, priority: int) -> SerializedExpert:
        return self._expert_bank.read_sync(idx, priority)

    def _worker_loop(self) -> None:
        while True:
            with self._cv:
                while not self._closed and (not self._heap or (self._heap[0].priority == ReadPriority.PREFETCH
                                                                and self._demand_outstanding > 0)):
                    self._cv.wait(timeout=0.05)
                if self._closed:
                    return
                req = heapq.heappop(self._heap)
                self._cv.notify_all()
            idx = req.expert_idx
            with self._lock:
                if idx in self._cache:
                    req.completion_handle.set_result(None)
                    continue
                first = self._inflight.get(idx)
                if first is None:
                    self._inflight[idx] = req.completion_handle
            if first is not None:
                _chain(first, req.completion_handle)
                continue
            try:
                expert = self._read(idx, req.priority)
                self._admit(expert, req.priority)
                if req.priority == ReadPriority.PREFETCH:
                    self._bump("prefetched_bytes", expert.nbytes())
                req.completion_handle.set_result(None)
            except Exception as exc:  # propagate to every waiter (loader.py:166-171)
                if not req.completion_handle.done():
                    req.completion_handle.set_exception(exc)
            finally:
                with self._lock:
                    self._inflight.pop(idx, None)

    def _enqueue(self, idx: int, priority: int, block: bool) -> Future | None:
        fut: Future = Future()
        with self._cv:
            if self._max_queue_size and len(self._heap) >= self._max_queue_size:
                if not block:
                    return None
                while len(self._heap) >= self._max_queue_size and not self._closed:
                    self._cv.wait(timeout=0.05)
            heapq.heappush(self._heap, LoadRequest(priority, next(self._seq), idx, fut))
            self._cv.notify_all()
        return fut

    # ------------------------------------------------------------------ API
    def load(self, expert_idxs: int | Sequence[int]) -> Generator[int, None, None]:
        """Yield each requested id once it is cached (loader.py:190-240)."""
        start = time.perf_counter()
        idxs = [expert_idxs] if isinstance(expert_idxs, int) else list(expert_idxs)
        hits = misses = 0
        futures: dict[Future, int] = {}
        for idx in dict.fromkeys(idxs):
            count = idxs.count(idx)
            if self._cache_manager.touch(idx):
                hits += count
                yield idx
                continue
            misses += count
            with self._lock:
                existing = self._inflight.get(idx)
            if existing is not None:
                futures[existing] = idx
                continue
            futures[self._enqueue(idx, ReadPriority.DEMAND, block=True)] = idx
        self._bump("cache_hits", hits)
        self._bump("cache_misses", misses)
        if not futures:
            return
        for f in as_completed(futures):
            f.result()
            yield futures[f]
        self._bump("demand_stall_s", time.perf_counter() - start)

    def get(self, idx: int) -> SerializedExpert:
        return self._cache.get(idx)

    def load_sync(self, expert_idxs: Sequence[int]) -> tuple[SerializedExpert, ...]:
        """Blocking demand load of a miss set (loader.py:242-255), in order."""
        start = time.perf_counter()
        idxs = list(expert_idxs)
        out: list[SerializedExpert | None] = [None] * len(idxs)
        waits: list[tuple[int, Future]] = []
        reads: list[tuple[int, Future]] = []
        with self._cv:
            self._demand_outstanding += 1
        try:
            hits = 0
            for i, idx in enumerate(idxs):
                with self._lock:
                    if idx in self._cache:
                        out[i] = self._cache.get(idx)
                        hits += 1
                        continue
                    pending = self._inflight.get(idx)
                if pending is not None:
                    waits.append((i, pending))
                else:
                    reads.append((i, self._demand_pool.submit(self._read, idx, ReadPriority.DEMAND)))
            self._bump("cache_hits", hits)
            self._bump("cache_misses", len(idxs) - hits)
            for i, f in reads:
                out[i] = f.result()
            for i, f in waits:
                f.result()
                with self._lock:
                    out[i] = self._cache.get(idxs[i]) if idxs[i] in self._cache else None
                if out[i] is None:
                    out[i] = self._read(idxs[i], ReadPriority.DEMAND)
        finally:
            with self._cv:
                self._demand_outstanding -= 1
                self._cv.notify_all()
        self._bump("demand_stall_s", time.perf_counter() - start)
        return tuple(out)  # type: ignore[arg-type]

    def enqueue_prefetch(self, expert_idxs: int | Sequence[int], await_free_slot: bool = True) -> list[Future]:
        """Queue speculative reads (loader.py:286-310); ids cached or in flight
        are skipped.  With ``await_free_slot=False`` a full queue drops the id."""
        idxs = [expert_idxs] if isinstance(expert_idxs, int) else list(expert_idxs)
        futures = []
        for idx in dict.fromkeys(idxs):
            with self._lock:
                skip = idx in self._cache or idx in self._inflight
            if skip:
                continue
            f = self._enqueue(idx, ReadPriority.PREFETCH, block=await_free_slot)
            if f is not None:
                futures.append(f)
        return futures

    def close(self) -> None:
        with self._cv:
            self._closed = True
            for req in self._heap:
                if not req.completion_handle.done():
                    req.completion_handle.cancel()
            self._heap.clear()
            self._cv.notify_all()
        for w in self._workers:
            w.join(timeout=2.0)
        self._demand_pool.shutdown(wait=True)
        self._cache._entries.clear()
        if hasattr(self._expert_bank, "close"):
            self._expert_bank.close()

    def __del__(self):
        try:
            if not self._closed:
                self.close()
        except Exception:
            pass


def _chain(first: Future, second: Future) -> None:
    def cb(f: Future) -> None:
        if second.done():
            return
        exc = f.exception()
        if exc is not None:
            second.set_exception(exc)
        else:
            second.set_result(None)

    first.add_done_callback(cb)
