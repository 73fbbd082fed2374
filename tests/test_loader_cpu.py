"""CPU: DiskBackedExpertLoader semantics against a fake expert bank.

Mirrors the reference's loader tests (tests/unit/test_streaming_provider.py:
a miss issues one DEMAND read, a hit none, residency stays within the byte
budget, LFRU and LRU pick different victims, stall time counts demand reads
only, a KeyError / IOError from the bank propagates and nothing is cached,
a failure mid-batch keeps only what was cached before, metrics are optional)
and adds the queue semantics of preempt/engine/expert_io/loader.py:118-171
that those tests leave out: a DEMAND read is served before queued PREFETCH
reads, concurrent requests for one expert share one read, and a failed read
reaches every waiter.  No GPU: blobs are plain bytes.
"""

import threading
import time

import pytest

from preemptlm_b200.bank import ReadPriority, SerializedExpert, TensorSpec
from preemptlm_b200.cache_manager import CacheEvictionPolicy, ExpertCacheManager
from preemptlm_b200.loader import DiskBackedExpertLoader, GenerationMetrics, HostExpertCache

PAYLOAD = 64
SPECS = (TensorSpec("w", "uint8", (PAYLOAD,), PAYLOAD),)


class FakeExpertBank:
    """Records (idx, priority) of every read; ``error`` is raised by reads;
    reads of ids in ``hold`` wait until ``gate`` is set."""

    def __init__(self, error: Exception | None = None):
        self.reads: list[tuple[int, int]] = []
        self.error = error
        self.gate = threading.Event()
        self.gate.set()
        self.hold: set[int] = set()
        self.started = threading.Event()
        self._lock = threading.Lock()

    def read_sync(self, idx: int, priority: int = ReadPriority.DEMAND) -> SerializedExpert:
        with self._lock:
            self.reads.append((idx, priority))
        if idx in self.hold:
            self.started.set()
            assert self.gate.wait(10), "gate never opened"
        if self.error is not None:
            raise self.error
        return SerializedExpert(idx, bytes(PAYLOAD), "mlx-affine-q4-g64-bfloat16", SPECS)


def build(budget_experts=4, bank=None, policy=CacheEvictionPolicy.LFRU, metrics=True, workers=1):
    bank = bank or FakeExpertBank()
    manager = ExpertCacheManager(budget_bytes=budget_experts * PAYLOAD, policy=policy, sample_size=8)
    cache = HostExpertCache(manager)
    m = GenerationMetrics() if metrics else None
    loader = DiskBackedExpertLoader(expert_bank=bank, cache=cache, metrics=m, num_worker_threads=workers)
    return loader, bank, cache, manager, m


def load_batches(loader, batches):
    """What a caller does: load a batch, then take each expert it yielded
    (taking an expert releases the DEMAND pin on it)."""
    for batch in batches:
        for idx in loader.load(batch):
            loader.get(idx)


def test_a_miss_issues_exactly_one_demand_read_and_installs_it():
    loader, bank, cache, manager, m = build()
    try:
        load_batches(loader, [(0,)])
        assert bank.reads == [(0, ReadPriority.DEMAND)]
        assert 0 in cache and 0 in manager
        assert (m.cache_misses, m.cache_hits) == (1, 0)
    finally:
        loader.close()


def test_a_hit_issues_no_read():
    loader, bank, cache, manager, m = build()
    try:
        load_batches(loader, [(0,), (0,)])
        assert len(bank.reads) == 1
        assert (m.cache_hits, m.cache_misses) == (1, 1)
    finally:
        loader.close()


def test_residency_bytes_track_the_cache_and_never_exceed_the_budget():
    loader, bank, cache, manager, m = build(budget_experts=3)
    try:
        load_batches(loader, [(i % 7,) for i in range(30)])
        assert cache.size() == manager.cache_size <= 3 * PAYLOAD
        assert manager.evictions > 0
    finally:
        loader.close()


def test_lru_and_lfru_evict_different_victims_on_the_same_pattern():
    batches = [(0,), (0,), (0,), (1,), (2,), (2,), (1,), (3,)]
    victims = {}
    for policy in (CacheEvictionPolicy.LFRU, CacheEvictionPolicy.LRU):
        loader, bank, cache, manager, m = build(budget_experts=3, policy=policy)
        try:
            load_batches(loader, batches)
            victims[policy] = sorted({0, 1, 2, 3} - set(cache._entries))
        finally:
            loader.close()
    assert victims[CacheEvictionPolicy.LFRU] == [2]
    assert victims[CacheEvictionPolicy.LRU] == [0]


def test_stall_time_accumulates_only_for_demand_reads():
    loader, bank, cache, manager, m = build()
    try:
        load_batches(loader, [(0, 1)])
        after = m.demand_stall_s
        assert after > 0.0
        load_batches(loader, [(0, 1)])
        assert m.demand_stall_s == after
    finally:
        loader.close()


@pytest.mark.parametrize("error", [KeyError("nope"), IOError("short")])
def test_a_failed_read_is_fatal_and_propagates(error):
    loader, bank, cache, manager, m = build(bank=FakeExpertBank(error=error))
    try:
        with pytest.raises(type(error)):
            load_batches(loader, [(0,)])
        assert cache._entries == {}  # nothing silently substituted or skipped
        assert 0 not in manager
        with pytest.raises(type(error)):
            loader.load_sync([1])  # the demand path of the slot refills
        assert 1 not in cache
    finally:
        loader.close()


def test_a_failure_mid_batch_does_not_continue_with_the_experts_it_had():
    loader, bank, cache, manager, m = build(budget_experts=8)
    try:
        load_batches(loader, [(0,)])
        bank.error = KeyError("gone")
        with pytest.raises(KeyError):
            load_batches(loader, [(0, 1, 2)])
        assert set(cache._entries) == {0}
    finally:
        loader.close()


def test_metrics_are_optional():
    loader, bank, cache, manager, m = build(metrics=False)
    try:
        load_batches(loader, [(0,)])
        assert 0 in cache
    finally:
        loader.close()


def test_demand_is_served_before_queued_prefetches():
    """One worker, busy on a prefetch read; more prefetches queue behind it;
    a demand load that arrives later is read next, before them."""
    bank = FakeExpertBank()
    bank.hold, bank.gate = {10}, threading.Event()
    loader, bank, cache, manager, m = build(budget_experts=16, bank=bank)
    try:
        futs = loader.enqueue_prefetch([10, 11, 12])
        assert bank.started.wait(5)
        got = []
        t = threading.Thread(target=lambda: got.extend(loader.load([20])))
        t.start()
        deadline = time.time() + 5
        while not loader._heap or loader._heap[0].priority != ReadPriority.DEMAND:
            assert time.time() < deadline, "demand request never queued"
            time.sleep(0.005)
        bank.gate.set()
        t.join(5)
        for f in futs:
            f.result(5)
        assert got == [20]
        order = [i for i, _ in bank.reads]
        assert order == [10, 20, 11, 12], order
        assert dict(bank.reads)[20] == ReadPriority.DEMAND and dict(bank.reads)[11] == ReadPriority.PREFETCH
        assert m.prefetched_bytes == 3 * PAYLOAD
    finally:
        bank.gate.set()
        loader.close()


def test_load_sync_does_not_queue_behind_prefetches():
    """The slot-refill path (load_sync) reads at once on its own threads while
    the prefetch worker is busy, and prefetches hold back until it is done."""
    bank = FakeExpertBank()
    bank.hold, bank.gate = {10}, threading.Event()
    loader, bank, cache, manager, m = build(budget_experts=16, bank=bank)
    try:
        loader.enqueue_prefetch([10, 11, 12])
        assert bank.started.wait(5)
        blobs = loader.load_sync([30, 31])
        assert [b.idx for b in blobs] == [30, 31]
        order = [i for i, _ in bank.reads]
        assert order[0] == 10 and sorted(order[1:]) == [30, 31], order
        bank.gate.set()
        deadline = time.time() + 5
        while len(bank.reads) < 5:
            assert time.time() < deadline
            time.sleep(0.005)
        assert [i for i, _ in bank.reads][3:] == [11, 12]
    finally:
        bank.gate.set()
        loader.close()


def test_concurrent_requests_for_one_expert_share_one_read():
    bank = FakeExpertBank()
    bank.hold, bank.gate = {5}, threading.Event()
    loader, bank, cache, manager, m = build(budget_experts=16, bank=bank, workers=4)
    try:
        results = []

        def one():
            results.append(list(loader.load([5])))

        threads = [threading.Thread(target=one) for _ in range(3)]
        threads[0].start()
        assert bank.started.wait(5)
        for t in threads[1:]:
            t.start()
        time.sleep(0.05)
        bank.gate.set()
        for t in threads:
            t.join(5)
        assert results == [[5], [5], [5]]
        assert [i for i, _ in bank.reads] == [5]  # one read served all three
    finally:
        bank.gate.set()
        loader.close()


def test_a_failed_read_reaches_every_waiter():
    bank = FakeExpertBank(error=IOError("disk gone"))
    bank.hold, bank.gate = {7}, threading.Event()
    loader, bank, cache, manager, m = build(budget_experts=16, bank=bank, workers=4)
    try:
        errors = []

        def one():
            try:
                list(loader.load([7]))
            except IOError as e:
                errors.append(e)

        threads = [threading.Thread(target=one) for _ in range(3)]
        threads[0].start()
        assert bank.started.wait(5)
        for t in threads[1:]:
            t.start()
        time.sleep(0.05)
        bank.gate.set()
        for t in threads:
            t.join(5)
        assert len(errors) == 3
        assert [i for i, _ in bank.reads] == [7]
        assert 7 not in cache and 7 not in manager
    finally:
        bank.gate.set()
        loader.close()


def test_bank_reads_bypassing_the_page_cache_match_buffered_reads():
    """PreadExpertBank(bypass_page_cache=True): O_DIRECT reads (aligned slice
    of a larger buffer, length rounded up inside the blob's padding) where the
    file system allows them, else buffered reads whose pages are dropped; the
    bytes equal a plain read of every blob of the reference-written bank."""
    from pathlib import Path

    import numpy as np

    from preemptlm_b200.bank import PreadExpertBank

    path = Path(__file__).resolve().parent / "golden" / "bank"
    with PreadExpertBank(path, bypass_page_cache=True, pinned=False) as direct, \
            PreadExpertBank(path, pinned=False) as plain:
        assert not plain.direct_io
        for i in range(len(plain.blob_index)):
            a = direct.read_sync(i)
            b = plain.read_sync(i)
            assert a.nbytes() == b.nbytes() == plain.blob_index[i].length
            assert np.array_equal(a.as_tensor().numpy(), b.as_tensor().numpy())
        with pytest.raises(KeyError):
            direct.read_sync(len(plain.blob_index))
