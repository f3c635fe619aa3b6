"""Expert staging on a dedicated copy stream (host store / HBM tier -> slot rows).

Mirrors ``moe_offload/transfer_engine.py`` of the reference (``TransferReadyEvent`` :30-69,
``load_many_async`` :139-187, run batching :246-303). Copies are issued by
``lm_stage_copy`` (one ``cudaMemcpyAsync`` per run of consecutive source rows landing in
consecutive slots) on a stream owned by the engine; an event recorded after the copies is
what the consumer stream waits on. Slots become READY only when a consumer dependency is
installed, after their leases are re-validated, so a mapping can never name a slot whose
copy is not ordered before its reader.

Slot banks placed on the CPU (host-logic tests of the allocation order) are filled with a
synchronous ``copy_``; that is bookkeeping for tests, not a data path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .. import _lib
from .slot_bank import ExpertSlot, SlotLease, SlotState


@dataclass
class TransferReadyEvent:
    """Copy-stream event plus the slot leases it makes consumable."""

    event: torch.cuda.Event | None
    leases: tuple[tuple[ExpertSlot, SlotLease], ...]
    completed: bool = False
    consumer_wait_installed: bool = False
    copies: int = 0
    bytes: int = 0

    def install_consumer_dependency(self, consumer_stream: torch.cuda.Stream | None) -> None:
        """Order the copies before `consumer_stream`, then publish the slots READY."""
        if self.completed:
            return
        self._validate_loading_leases()
        if self.event is not None and consumer_stream is not None:
            consumer_stream.wait_event(self.event)
        self.consumer_wait_installed = True
        self.mark_ready()

    def synchronize(self) -> None:
        if self.event is not None:
            self.event.synchronize()

    def mark_ready(self) -> None:
        if self.completed:
            return
        self._validate_loading_leases()
        for slot, _ in self.leases:
            slot.state = SlotState.READY
        self.completed = True

    def _validate_loading_leases(self) -> None:
        for slot, lease in self.leases:
            if not slot.matches_lease(lease):
                raise RuntimeError(
                    f"stale H2D completion for slot {slot.slot_id}: expected "
                    f"{lease.expert_key} v{lease.version}, found {slot.expert_key} v{slot.version}"
                )
            if slot.state != SlotState.LOADING:
                raise RuntimeError(
                    f"H2D completion for slot {slot.slot_id} requires loading state, "
                    f"found {slot.state.value}"
                )


@dataclass
class TransferStats:
    copies: int = 0
    bytes_h2d: int = 0
    bytes_d2d: int = 0
    calls: int = 0
    history: list[int] = field(default_factory=list)


class TransferEngine:
    def __init__(self, device: torch.device | None = None) -> None:
        self._device = device
        self._stream: torch.cuda.Stream | None = None
        self._pending: list[TransferReadyEvent] = []
        self.stats = TransferStats()

    def stream(self) -> torch.cuda.Stream:
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=self._device)
        return self._stream

    def copy_rows(self, src_w13: torch.Tensor, src_w2: torch.Tensor, src_rows: list[int],
                  dst_w13: torch.Tensor, dst_w2: torch.Tensor, dst_rows: list[int],
                  *, wait_event: torch.cuda.Event | None = None,
                  stream: torch.cuda.Stream | None = None) -> tuple[int, int]:
        """Issue the copies of expert rows on the copy stream; returns (copies, bytes)."""
        if not src_rows:
            return 0, 0
        if not dst_w13.is_cuda:
            with torch.no_grad():
                for s, d in zip(src_rows, dst_rows):
                    dst_w13[d].copy_(src_w13[s])
                    dst_w2[d].copy_(src_w2[s])
            nbytes = (dst_w13[0].numel() + dst_w2[0].numel()) * dst_w13.element_size() * len(src_rows)
            return len(src_rows), nbytes
        st = stream if stream is not None else self.stream()
        if wait_event is not None:
            st.wait_event(wait_event)
        n1 = _lib.stage_copy(dst_w13, src_w13, src_rows, dst_rows, stream=st)
        n2 = _lib.stage_copy(dst_w2, src_w2, src_rows, dst_rows, stream=st)
        nbytes = (dst_w13[0].numel() + dst_w2[0].numel()) * dst_w13.element_size() * len(src_rows)
        self.stats.copies += n1 + n2
        self.stats.calls += 1
        if src_w13.is_cuda:
            self.stats.bytes_d2d += nbytes
        else:
            self.stats.bytes_h2d += nbytes
        return n1 + n2, nbytes

    def load_many_async(self, src_w13: torch.Tensor, src_w2: torch.Tensor, src_rows: list[int],
                        dst_w13: torch.Tensor, dst_w2: torch.Tensor, slots: list[ExpertSlot],
                        *, wait_event: torch.cuda.Event | None = None) -> TransferReadyEvent:
        """Copy ``src[src_rows[i]] -> slot rows`` and return the readiness event.

        Slots must already be LOADING (the allocator's state for a fresh owner).
        """
        leases = tuple((slot, slot.lease()) for slot in slots)
        dst_rows = [slot.slot_id for slot in slots]
        copies, nbytes = self.copy_rows(src_w13, src_w2, list(src_rows), dst_w13, dst_w2,
                                        dst_rows, wait_event=wait_event)
        event = None
        if dst_w13.is_cuda:
            event = torch.cuda.Event()
            event.record(self.stream())
        ready = TransferReadyEvent(event, leases, copies=copies, bytes=nbytes)
        if event is not None:
            self._pending.append(ready)
        return ready

    def record_event(self) -> torch.cuda.Event:
        ev = torch.cuda.Event()
        ev.record(self.stream())
        return ev

    def synchronize(self) -> None:
        """Wait for every queued copy, publishing the slots of completed transfers."""
        if self._stream is not None:
            self._stream.synchronize()
        for ready in self._pending:
            if not ready.completed:
                ready.mark_ready()
        self._pending.clear()
