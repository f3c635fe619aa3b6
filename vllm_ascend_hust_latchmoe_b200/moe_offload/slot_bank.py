"""Fixed, address-stable expert slot bank in HBM plus its host-side slot state machine.

Mirrors ``moe_offload/slot_bank.py`` of the reference (``ExpertSlotBank`` :79-336,
``SlotState`` :27-31, ``SlotLease`` :35-40, ``allocate_for`` :211-232, first-EMPTY
:318-322, LRU :324-329). The storage is two device tensors allocated once:

* ``w13_slots [S + P, 2I, H]`` bf16 (rows 0..I-1 gate, I..2I-1 up; K-major rows), and
* ``w2_slots  [S + P, H, I]``  bf16 (K-major rows),

where S dynamic slots form the routed-expert cache and P pinned rows at the end hold
always-resident shared experts. The K-major layout is what the TMA-fed tcgen05 GEMM and
the decode GEMV stream from; captured kernels only ever see these two base addresses.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum

import torch

from .expert_key import ExpertKey


class SlotState(str, Enum):
    EMPTY = "empty"
    LOADING = "loading"
    READY = "ready"
    COMPUTING = "computing"


@dataclass(frozen=True)
class SlotLease:
    """One immutable ownership interval of a slot: (slot, owner, version)."""

    slot_id: int
    expert_key: ExpertKey
    version: int


@dataclass
class ExpertSlot:
    slot_id: int
    state: SlotState = SlotState.EMPTY
    expert_key: ExpertKey | None = None
    version: int = 0
    last_used_step: int = -1

    def lease(self) -> SlotLease:
        if self.expert_key is None:
            raise RuntimeError(f"slot {self.slot_id} has no owner")
        return SlotLease(int(self.slot_id), self.expert_key, int(self.version))

    def matches_lease(self, lease: SlotLease) -> bool:
        return (
            self.slot_id == lease.slot_id
            and self.expert_key == lease.expert_key
            and self.version == lease.version
        )


class ExpertSlotBank:
    def __init__(
        self,
        num_slots: int,
        w13_shape: tuple[int, ...],
        w2_shape: tuple[int, ...],
        *,
        dtype: torch.dtype,
        device: torch.device,
        pinned_logical_ids: tuple[int, ...] = (),
    ) -> None:
        if num_slots <= 0:
            raise ValueError("num_slots must be greater than 0")
        pinned = tuple(int(e) for e in pinned_logical_ids)
        if len(set(pinned)) != len(pinned):
            raise ValueError("pinned logical expert ids must be unique")
        if any(e < 0 for e in pinned):
            raise ValueError("pinned logical expert ids must be non-negative")
        self.num_dynamic_slots = int(num_slots)
        self.pinned_logical_ids = pinned
        self._pinned_slot = {e: self.num_dynamic_slots + i for i, e in enumerate(pinned)}
        rows = self.num_dynamic_slots + len(pinned)
        self.w13_slots = torch.empty((rows, *w13_shape), dtype=dtype, device=device)
        self.w2_slots = torch.empty((rows, *w2_shape), dtype=dtype, device=device)
        self.slots = [ExpertSlot(slot_id=i) for i in range(self.num_dynamic_slots)]
        self._resident: dict[ExpertKey, int] = {}

    # ------------------------------------------------------------------ geometry
    @property
    def physical_expert_count(self) -> int:
        return int(self.w13_slots.shape[0])

    @property
    def pinned_slot_ids(self) -> tuple[int, ...]:
        return tuple(self._pinned_slot[e] for e in self.pinned_logical_ids)

    @property
    def slot_bytes(self) -> int:
        return (self.w13_slots[0].numel() + self.w2_slots[0].numel()) * self.w13_slots.element_size()

    @property
    def dynamic_bytes(self) -> int:
        return self.slot_bytes * self.num_dynamic_slots

    @property
    def pinned_bytes(self) -> int:
        return self.slot_bytes * len(self.pinned_logical_ids)

    @property
    def total_bytes(self) -> int:
        return self.slot_bytes * self.physical_expert_count

    def pinned_slot_for_logical_id(self, logical_id: int) -> int | None:
        return self._pinned_slot.get(int(logical_id))

    # ------------------------------------------------------------------ pinned lane
    def install_pinned_weights(self, w13: torch.Tensor, w2: torch.Tensor) -> None:
        n = len(self.pinned_logical_ids)
        if n == 0:
            if w13.numel() or w2.numel():
                raise ValueError("cannot install pinned weights into a routed-only bank")
            return
        if tuple(w13.shape) != (n, *self.w13_slots.shape[1:]) or tuple(w2.shape) != (
            n, *self.w2_slots.shape[1:]
        ):
            raise ValueError(
                "pinned shared weight layout does not match slot bank: "
                f"w13={tuple(w13.shape)} w2={tuple(w2.shape)}"
            )
        with torch.no_grad():
            self.w13_slots[self.num_dynamic_slots :].copy_(w13)
            self.w2_slots[self.num_dynamic_slots :].copy_(w2)

    def install_pinned_log2phy(self, log2phy: torch.Tensor) -> None:
        for logical_id, slot_id in self._pinned_slot.items():
            if logical_id >= log2phy.numel():
                raise ValueError(
                    f"log2phy does not cover pinned logical expert {logical_id}; "
                    f"size={log2phy.numel()}"
                )
            log2phy[logical_id] = slot_id

    # ------------------------------------------------------------------ allocation
    def allocate_for(self, expert_key: ExpertKey, *, step_id: int) -> ExpertSlot:
        """Resident -> touch. Else first EMPTY slot, else the READY slot with the least
        (last_used_step, slot_id); the new owner starts LOADING with version + 1."""
        sid = self._resident.get(expert_key)
        if sid is not None:
            slot = self.slots[sid]
            slot.last_used_step = int(step_id)
            return slot
        slot = self._first_empty_slot() or self._lru_evictable_slot()
        if slot is None:
            raise RuntimeError(f"no evictable expert slots; states={self.state_counts()}")
        if slot.expert_key is not None:
            self._resident.pop(slot.expert_key, None)
        slot.expert_key = expert_key
        slot.state = SlotState.LOADING
        slot.version += 1
        slot.last_used_step = int(step_id)
        self._resident[expert_key] = slot.slot_id
        return slot

    def assign_transient_slot(self, slot_id: int, expert_key: ExpertKey, *, step_id: int) -> ExpertSlot:
        """Positional wave slot of a stage bank (no resident index is kept)."""
        slot = self.slots[int(slot_id)]
        self._require_reassignable(slot)
        if slot.expert_key is not None:
            self._resident.pop(slot.expert_key, None)
        slot.expert_key = expert_key
        slot.version += 1
        slot.last_used_step = int(step_id)
        slot.state = SlotState.LOADING
        return slot

    def lookup(self, expert_key: ExpertKey) -> ExpertSlot | None:
        sid = self._resident.get(expert_key)
        return None if sid is None else self.slots[sid]

    def mark_ready(self, slot_id: int) -> None:
        self.slots[int(slot_id)].state = SlotState.READY

    def mark_computing(self, slot_id: int) -> None:
        self.slots[int(slot_id)].state = SlotState.COMPUTING

    def clear_slot(self, slot_id: int, *, force: bool = False) -> None:
        slot = self.slots[int(slot_id)]
        if not force and slot.state == SlotState.COMPUTING:
            raise RuntimeError(f"slot {slot.slot_id} is computing and cannot be reassigned")
        if slot.expert_key is not None:
            self._resident.pop(slot.expert_key, None)
        slot.expert_key = None
        slot.state = SlotState.EMPTY

    def ready_slot_ids(self, layer_id: int, experts) -> dict[int, int]:
        out = {}
        for e in experts:
            slot = self.lookup(ExpertKey(int(layer_id), int(e)))
            if slot is not None and slot.state == SlotState.READY:
                out[int(e)] = slot.slot_id
        return out

    def state_counts(self) -> dict[str, int]:
        counts = {s.value: 0 for s in SlotState}
        for slot in self.slots:
            counts[slot.state.value] += 1
        return counts

    def _first_empty_slot(self) -> ExpertSlot | None:
        for slot in self.slots:
            if slot.state == SlotState.EMPTY:
                return slot
        return None

    def _lru_evictable_slot(self) -> ExpertSlot | None:
        ready = [s for s in self.slots if s.state == SlotState.READY]
        return min(ready, key=lambda s: (s.last_used_step, s.slot_id)) if ready else None

    @staticmethod
    def _require_reassignable(slot: ExpertSlot) -> None:
        if slot.state in (SlotState.LOADING, SlotState.COMPUTING):
            raise RuntimeError(f"slot {slot.slot_id} is {slot.state.value} and cannot be reassigned")
