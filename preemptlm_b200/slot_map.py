"""Per-block slot bookkeeping: eid<->sid tables, LFRU counters and slot choice.

Mirrors ``BaseMoEWrapper`` (preempt/backends/mlx_metal/module_wrappers/
base_moe_wrapper.py:69-172): the same table and counter names, ``_touch`` and
``_choose_slots``.  The host tables stay authoritative (numpy, as in the
reference); a device copy of ``_eid_lookup_table`` feeds the dispatch kernel
and is refreshed after every admission.

Slot policies
-------------
``"reference"`` reproduces ``_choose_slots`` exactly, including its
``np.delete`` index shift (base_moe_wrapper.py:164-172): the positions returned
by argsort index the *shortened* score array, so they can name a slot that the
current step still uses, or repeat a free slot.  The reference then silently
overwrites that slot.  This policy returns the same slot ids whenever they are
safe and raises ``RuntimeError`` where the reference would corrupt a slot.

``"lfru"`` is the intended rule: free slots first (ascending), then the
lowest LFRU score ``freq * (clock + 1) + recency`` among occupied slots not
used by the step, ties to the lower slot id.
"""

from __future__ import annotations

import numpy as np
import torch

EMPTY = -1  # CacheSlotState.EMPTY (preempt/core/enums.py:42-46)
SLOT_POLICIES = ("reference", "lfru")


class SlotCorruptionError(RuntimeError):
    """The reference slot choice would overwrite a slot still in use."""


class SlotTable:
    def __init__(self, num_experts: int, num_slots: int, slot_policy: str = "reference",
                 device: str | torch.device | None = None):
        if slot_policy not in SLOT_POLICIES:
            raise ValueError(f"slot_policy must be one of {SLOT_POLICIES}")
        self.num_experts = int(num_experts)
        self.num_slots = int(num_slots)
        self.slot_policy = slot_policy
        self._eid_lookup_table = np.full(self.num_experts, EMPTY, np.int32)
        self._sid_lookup_table = np.full(self.num_slots, EMPTY, np.int32)
        self._clock = 0
        self._slot_freq = np.zeros(self.num_slots, np.int64)
        self._slot_recency = np.zeros(self.num_slots, np.int64)
        self._device = torch.device(device) if device is not None else None
        self.eid2sid_device = None
        if self._device is not None:
            self.eid2sid_device = torch.full((self.num_experts,), EMPTY, dtype=torch.int32, device=self._device)

    # ------------------------------------------------------------------ tables
    def set_identity(self) -> None:
        """Every expert resident in slot == expert id (the all-resident arena)."""
        if self.num_slots < self.num_experts:
            raise ValueError("identity map needs num_slots >= num_experts")
        self._eid_lookup_table[:] = np.arange(self.num_experts, dtype=np.int32)
        self._sid_lookup_table[:] = EMPTY
        self._sid_lookup_table[: self.num_experts] = np.arange(self.num_experts, dtype=np.int32)
        self.sync_device()

    def assign(self, eids, sids) -> None:
        """Record that expert eids[i] now lives in slot sids[i]."""
        eids = np.asarray(eids, np.int64)
        sids = np.asarray(sids, np.int64)
        old = self._sid_lookup_table[sids]
        self._eid_lookup_table[old[old >= 0]] = EMPTY
        self._eid_lookup_table[eids] = sids
        self._sid_lookup_table[sids] = eids
        self.sync_device()

    def sync_device(self, stream: torch.cuda.Stream | None = None) -> None:
        if self.eid2sid_device is not None:
            src = torch.from_numpy(self._eid_lookup_table)
            if self._device.type == "cuda":
                src = src.pin_memory()
            self.eid2sid_device.copy_(src, non_blocking=True)

    # ------------------------------------------------------------------ LFRU
    def _touch(self, slots: np.ndarray) -> None:
        """base_moe_wrapper.py:152-155."""
        self._clock += 1
        np.add.at(self._slot_freq, slots, 1)
        self._slot_recency[slots] = self._clock

    def _choose_slots(self, n: int, protected: np.ndarray) -> np.ndarray:
        """base_moe_wrapper.py:157-172 under ``slot_policy`` (module docstring)."""
        free = np.nonzero(self._sid_lookup_table < 0)[0]
        if free.size >= n:
            return free[:n]
        prot = self._eid_lookup_table[protected]
        prot = prot[prot >= 0]
        score = self._slot_freq * (self._clock + 1) + self._slot_recency
        if self.slot_policy == "reference":
            shortened = np.delete(score, prot)
            evicted = np.argsort(shortened, kind="stable")[: n - free.size]
            chosen = np.concatenate([free, evicted])
            if np.unique(chosen).size != chosen.size or np.isin(chosen, prot).any():
                raise SlotCorruptionError(
                    f"the reference slot choice {chosen.tolist()} overwrites a slot in use by this step "
                    f"(protected {sorted(prot.tolist())}); use slot_policy='lfru'"
                )
            return chosen
        occupied = self._sid_lookup_table >= 0
        cand = np.nonzero(occupied & ~np.isin(np.arange(self.num_slots), prot))[0]
        need = n - free.size
        if cand.size < need:
            raise RuntimeError(f"only {cand.size} evictable slots for {need} misses")
        order = np.argsort(score[cand], kind="stable")[:need]
        return np.concatenate([free, cand[order]])
