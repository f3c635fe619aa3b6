"""Offload runtime: owns the slot banks, log2phy tables, stage banks and the staging controller.

Mirrors ``moe_offload/runtime.py`` of the reference (``MoeOffloadRuntime`` :262):
``register_layer_for_fixed_slots`` :591-693, ``stage_fixed_slot_plan`` :2652-2696,
``prepare_fixed_slot_plan_into_log2phy`` :1636-1902, ``begin/end_slot_compute``
:983-1088, ``_drain_slot_bank_inflight_work`` :881-956, ``capture_safe_slot_weights``
:2698-2733 with the address lock :2735-2790, ``prepare_prefill_stage_plan`` :2035-2258,
``stage_full_residency_slot_plan`` :2792-2862, ``get/reset_moe_offload_runtime`` :3025-3034.

B200 specifics: copies run on one copy stream per runtime through ``lm_stage_copy``; the
persistent ``log2phy`` int32 table is rewritten from a pinned host mirror with one small
``cudaMemcpyAsync`` on the consumer stream *after* the consumer has been made to wait for
the copies (a mapping never names a slot whose data is not ordered before its reader).
"""

from __future__ import annotations

import itertools
import threading
from dataclasses import dataclass
from time import perf_counter
from types import SimpleNamespace

import torch

from ..config import MoeOffloadConfig
from ..weight_layout import maybe_tiled
from .expert_key import ExpertKey
from .host_store import HostExpertStore
from .slot_bank import ExpertSlot, ExpertSlotBank, SlotLease, SlotState
from .slot_mapping import ExpertSlotMapping, PreparedSlotWeights
from .transfer_engine import TransferEngine, TransferReadyEvent


@dataclass(frozen=True)
class SlotComputeHandle:
    layer_id: int
    slot_ids: tuple[int, ...]
    leases: tuple[SlotLease, ...]


@dataclass(frozen=True)
class SlotAddressFingerprint:
    w13_ptr: int
    w2_ptr: int
    log2phy_ptr: int
    w13_shape: tuple[int, ...]
    w2_shape: tuple[int, ...]
    device: str
    dtype: str


@dataclass
class StagePool:
    """Double-buffered temporary banks for multi-wave staging, shared by equal layouts."""

    banks: list[ExpertSlotBank]
    release_events: list[torch.cuda.Event | None]


@dataclass(frozen=True)
class MoeOffloadMemoryLedger:
    host_store_bytes: int
    slot_bank_bytes: int
    stage_bank_bytes: int
    log2phy_bytes: int

    def to_jsonable(self) -> dict[str, int]:
        return {
            "host_store_bytes": self.host_store_bytes,
            "slot_bank_bytes": self.slot_bank_bytes,
            "stage_bank_bytes": self.stage_bank_bytes,
            "log2phy_bytes": self.log2phy_bytes,
        }


class _PinnedRing:
    """Ring of pinned host rows for async log2phy uploads (a row is reused only after the
    copy that last read it has completed)."""

    def __init__(self, n: int, depth: int = 4) -> None:
        self.rows = [torch.empty(n, dtype=torch.int32, pin_memory=True) for _ in range(depth)]
        self.events: list[torch.cuda.Event | None] = [None] * depth
        self.cursor = 0

    def upload(self, values: torch.Tensor, dst: torch.Tensor) -> None:
        i = self.cursor
        self.cursor = (i + 1) % len(self.rows)
        if self.events[i] is not None:
            self.events[i].synchronize()
        self.rows[i].copy_(values)
        dst.copy_(self.rows[i], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(dst.device))
        self.events[i] = ev


class MoeOffloadRuntime:
    def __init__(self, config: MoeOffloadConfig | None = None) -> None:
        self.config = config if config is not None else MoeOffloadConfig.from_env()
        self._host_store = HostExpertStore()
        self._transfer_engine = TransferEngine()
        self._slot_banks: dict[int, ExpertSlotBank] = {}
        self._log2phy_buffers: dict[int, torch.Tensor] = {}
        self._log2phy_host: dict[int, torch.Tensor] = {}
        self._log2phy_rings: dict[int, _PinnedRing] = {}
        self._log2phy_slot_by_expert: dict[int, dict[int, int]] = {}
        self._routed_counts: dict[int, int] = {}
        self._total_counts: dict[int, int] = {}
        self._slot_compute_done_events: dict[tuple[int, int, int], object] = {}
        self._graph_slot_address_fingerprints: dict[int, SlotAddressFingerprint] = {}
        self._active_slot_ids_by_layer: dict[int, tuple[int, ...]] = {}
        self._stage_pools: dict[tuple, StagePool] = {}
        self._full_layer_pool: dict[tuple, ExpertSlotBank] = {}
        self._tiled_layout: dict[int, bool] = {}
        self._step_counter = itertools.count()
        self._capturing = False
        self._released_original_weight_layers: set[int] = set()
        self.stage_stats = {"calls": 0, "hits": 0, "misses": 0, "h2d_bytes": 0, "log2phy_updates": 0}
        # Prefill layer calls are recorded (CUDA events, read back on flush) into the profile
        # JSONL that profile-guided residency reads, when a profile path is configured.
        self.prefill_profiler = None
        if self.config.profile_path:
            from .prefill_residency import PrefillProfileRecorder

            self.prefill_profiler = PrefillProfileRecorder(str(self.config.profile_path))

    # ------------------------------------------------------------------ registration
    @property
    def should_use_fixed_slots(self) -> bool:
        return bool(self.config.enabled) and int(self.config.num_slots) > 0

    def is_resident_layer(self, layer_id: int) -> bool:
        return int(layer_id) in self.config.resident_layer_ids

    def is_layer_registered(self, layer_id: int) -> bool:
        return int(layer_id) in self._slot_banks

    def should_use_fixed_slot_plan_for_layer(self, layer_id: int) -> bool:
        return self.should_use_fixed_slots and not self.is_resident_layer(layer_id)

    def register_layer_for_fixed_slots(
        self,
        layer: torch.nn.Module,
        *,
        slot_device: torch.device | None = None,
        store_device: torch.device | None = None,
        num_shared_experts: int = 0,
    ) -> None:
        """Move a layer's experts into the host store and allocate its slot bank + log2phy.

        ``layer`` carries ``layer_id``, ``w13_weight [E, 2I, H]`` and ``w2_weight [E, H, I]``.
        The last ``num_shared_experts`` rows are always-resident shared experts kept in the
        bank's pinned suffix. ``store_device`` places the store in HBM instead of pinned
        host memory (an HBM-resident tier).
        """
        layer_id = int(getattr(layer, "layer_id", -1))
        if layer_id < 0:
            raise ValueError("layer.layer_id is required for fixed-slot registration")
        if layer_id in self._graph_slot_address_fingerprints:
            raise RuntimeError(
                f"layer {layer_id} fixed-slot addresses are already captured; "
                "re-registering would invalidate a CUDA graph replay"
            )
        w13 = layer.w13_weight
        w2 = layer.w2_weight
        if w13.shape[0] != w2.shape[0]:
            raise ValueError("w13_weight and w2_weight must have the same number of experts")
        total = int(w13.shape[0])
        shared = int(num_shared_experts or getattr(layer, "num_fused_shared_experts", 0) or 0)
        routed = total - shared
        if routed <= 0:
            raise ValueError(f"fused shared layout needs a routed expert; total={total}, shared={shared}")
        device = torch.device(slot_device) if slot_device is not None else w13.device
        # Store and banks hold the tile-contiguous layout the kernels stream from.
        w13t, tiled13 = maybe_tiled(w13.detach())
        w2t, tiled2 = maybe_tiled(w2.detach())
        if not (tiled13 and tiled2):
            if device.type == "cuda":
                raise ValueError(
                    "CUDA slot banks need w13 [E, 2I, H] and w2 [E, H, I] with 2I and H multiples "
                    f"of 128 and H and I multiples of 64; got {tuple(w13.shape)}, {tuple(w2.shape)}")
            w13t, w2t = w13.detach(), w2.detach()
        self._tiled_layout[layer_id] = bool(tiled13 and tiled2)
        # A host store holds the routed rows only (the shared suffix lives in the bank). An HBM
        # store also keeps the shared rows, so a resident layer reads routed and shared experts
        # in place in one grouped-MLP launch.
        on_hbm = store_device is not None and torch.device(store_device).type == "cuda"
        self._host_store.register_layer(
            SimpleNamespace(layer_id=layer_id, w13_weight=w13t, w2_weight=w2t),
            pin_memory=self.config.should_pin_host_memory or torch.cuda.is_available(),
            routed_expert_count=total if on_hbm else routed, device=store_device)
        w13, w2 = w13t, w2t
        pinned = tuple(range(routed, total))
        bank = ExpertSlotBank(self.config.num_slots, tuple(w13.shape[1:]), tuple(w2.shape[1:]),
                              dtype=w13.dtype, device=device, pinned_logical_ids=pinned)
        if pinned:
            bank.install_pinned_weights(w13[routed:].to(device), w2[routed:].to(device))
        self._slot_banks[layer_id] = bank
        self._routed_counts[layer_id] = routed
        self._total_counts[layer_id] = total
        log2phy = torch.full((total,), -1, dtype=torch.int32, device=device)
        bank.install_pinned_log2phy(log2phy)
        self._log2phy_buffers[layer_id] = log2phy
        self._log2phy_host[layer_id] = log2phy.to("cpu").clone()
        if device.type == "cuda":
            self._log2phy_rings[layer_id] = _PinnedRing(total)
        self._log2phy_slot_by_expert[layer_id] = {}

    def register_layer_with_store(self, layer_id: int, w13_store: torch.Tensor,
                                  w2_store: torch.Tensor, *, slot_device: torch.device,
                                  num_slots: int | None = None) -> None:
        """Register a routed-only layer whose expert store tensors already exist in the bank
        layout (tile-contiguous), pinned on the host or resident in HBM; no copy is made.
        ``num_slots`` overrides the configured slot count for this layer's bank (an
        HBM-resident layer reads its store in place and needs no real bank)."""
        layer_id = int(layer_id)
        if layer_id in self._graph_slot_address_fingerprints:
            raise RuntimeError(f"layer {layer_id} fixed-slot addresses are already captured; "
                               "re-registering would invalidate a CUDA graph replay")
        self._host_store.adopt_layer(layer_id, w13_store, w2_store)
        E = int(w13_store.shape[0])
        device = torch.device(slot_device)
        self._tiled_layout[layer_id] = True
        self._slot_banks[layer_id] = ExpertSlotBank(
            int(num_slots or self.config.num_slots), tuple(w13_store.shape[1:]),
            tuple(w2_store.shape[1:]), dtype=w13_store.dtype, device=device)
        self._routed_counts[layer_id] = E
        self._total_counts[layer_id] = E
        log2phy = torch.full((E,), -1, dtype=torch.int32, device=device)
        self._log2phy_buffers[layer_id] = log2phy
        self._log2phy_host[layer_id] = torch.full((E,), -1, dtype=torch.int32)
        if device.type == "cuda":
            self._log2phy_rings[layer_id] = _PinnedRing(E)
        self._log2phy_slot_by_expert[layer_id] = {}

    def slot_bank(self, layer_id: int) -> ExpertSlotBank:
        bank = self._slot_banks.get(int(layer_id))
        if bank is None:
            raise RuntimeError(f"layer {layer_id} is not registered for fixed-slot execution")
        return bank

    def host_layer(self, layer_id: int):
        return self._host_store.layer(layer_id)

    @property
    def transfer_engine(self) -> TransferEngine:
        return self._transfer_engine

    def log2phy_buffer(self, layer_id: int) -> torch.Tensor | None:
        return self._log2phy_buffers.get(int(layer_id))

    def routed_expert_count_for_layer(self, *, layer_id: int, fallback: int) -> int:
        return int(self._routed_counts.get(int(layer_id), fallback))

    def total_logical_expert_count_for_layer(self, *, layer_id: int, fallback: int) -> int:
        return int(self._total_counts.get(int(layer_id), fallback))

    def is_static_residency_regime(self, num_logical_experts: int) -> bool:
        """Regime A: every logical expert owns a slot, log2phy is static."""
        return int(self.config.num_slots) >= int(num_logical_experts)

    def should_use_b2_pair_waves(self, *, layer_id: int, active_expert_count: int) -> bool:
        if not self.config.b2_wave_prefill:
            return False
        if not self.should_use_fixed_slot_plan_for_layer(int(layer_id)):
            return False
        return int(active_expert_count) > int(self.config.num_slots)

    def next_step_id(self) -> int:
        return next(self._step_counter)

    # ------------------------------------------------------------------ log2phy
    def _publish_log2phy(self, layer_id: int, experts: tuple[int, ...], slots: tuple[int, ...]) -> int:
        cache = self._log2phy_slot_by_expert[layer_id]
        host = self._log2phy_host[layer_id]
        changed = 0
        for e, s in zip(experts, slots):
            if cache.get(e) != s:
                cache[e] = s
                host[e] = s
                changed += 1
        if changed:
            dst = self._log2phy_buffers[layer_id]
            ring = self._log2phy_rings.get(layer_id)
            if ring is not None:
                ring.upload(host, dst)
            else:
                dst.copy_(host)
        self.stage_stats["log2phy_updates"] += changed
        return changed

    # ------------------------------------------------------------------ decode staging
    def _drain_slot_bank_inflight_work(self, bank: ExpertSlotBank) -> None:
        if any(s.state == SlotState.LOADING for s in bank.slots):
            self._transfer_engine.synchronize()
            loading = [s.slot_id for s in bank.slots if s.state == SlotState.LOADING]
            if loading:
                raise RuntimeError(
                    f"H2D synchronization completed without a matching ready event for slots {loading}")
        computing = [s for s in bank.slots if s.state == SlotState.COMPUTING]
        leases = [s.lease() for s in computing]
        seen: set[int] = set()
        for lease in leases:
            key = (lease.expert_key.layer_id, lease.slot_id, lease.version)
            ev = self._slot_compute_done_events.pop(key, None)
            if ev is None:
                raise RuntimeError(
                    f"computing slot has no completion event: layer={key[0]} slot={key[1]} version={key[2]}")
            if id(ev) not in seen:
                seen.add(id(ev))
                sync = getattr(ev, "synchronize", None)
                if callable(sync):
                    sync()
        for slot, lease in zip(computing, leases):
            if not slot.matches_lease(lease):
                raise RuntimeError(f"slot {lease.slot_id} ownership changed while compute was in flight")
            slot.state = SlotState.READY

    def _allocate_with_drain(self, bank: ExpertSlotBank, key: ExpertKey, step_id: int) -> ExpertSlot:
        try:
            return bank.allocate_for(key, step_id=step_id)
        except RuntimeError:
            if not any(s.state in (SlotState.LOADING, SlotState.COMPUTING) for s in bank.slots):
                raise
            self._drain_slot_bank_inflight_work(bank)
            return bank.allocate_for(key, step_id=step_id)

    def prepare_fixed_slot_plan_into_log2phy(
        self,
        *,
        layer_id: int,
        active_experts: tuple[int, ...],
        num_logical_experts: int,
        log2phy: torch.Tensor | None = None,
        step_id: int | None = None,
        consumer_stream: torch.cuda.Stream | None = None,
    ) -> PreparedSlotWeights:
        """Stage a decode working set (<= num_slots experts) and publish its log2phy entries."""
        if not self.should_use_fixed_slots:
            raise RuntimeError("fixed-slot plan requested while moe offload fixed slots are disabled")
        layer_id = int(layer_id)
        if self.is_resident_layer(layer_id):
            raise RuntimeError(f"fixed-slot plan must not run on resident layer {layer_id}")
        bank = self.slot_bank(layer_id)
        routed = self._routed_counts[layer_id]
        total = self._total_counts[layer_id]
        if int(num_logical_experts) not in (routed, total):
            raise RuntimeError(
                f"fused shared lane logical count mismatch: layer={layer_id} "
                f"requested={num_logical_experts} routed={routed} total={total}")
        active = tuple(dict.fromkeys(int(e) for e in active_experts))
        bad = [e for e in active if e < 0 or e >= routed]
        if bad:
            raise ValueError(f"active experts outside [0, {routed}) for layer {layer_id}: {bad}")
        if len(active) > self.config.num_slots:
            raise RuntimeError(
                f"active expert working set size {len(active)} exceeds num_slots={self.config.num_slots}")
        log2phy = self._log2phy_buffers[layer_id] if log2phy is None else log2phy
        if log2phy.numel() != total:
            raise RuntimeError(f"log2phy buffer for layer {layer_id} has size {log2phy.numel()}, expected {total}")
        if any(s.state in (SlotState.LOADING, SlotState.COMPUTING) for s in bank.slots):
            self._drain_slot_bank_inflight_work(bank)
        step = int(step_id) if step_id is not None and step_id >= 0 else self.next_step_id()
        slot_ids: list[int] = []
        miss_experts: list[int] = []
        miss_slots: list[ExpertSlot] = []
        for e in active:
            key = ExpertKey(layer_id, e)
            slot = bank.lookup(key)
            if slot is not None and slot.state != SlotState.READY:
                self._drain_slot_bank_inflight_work(bank)
                slot = bank.lookup(key)
            if slot is not None and slot.state == SlotState.READY:
                slot.last_used_step = step
            else:
                slot = self._allocate_with_drain(bank, key, step)
                miss_experts.append(e)
                miss_slots.append(slot)
            slot_ids.append(slot.slot_id)
        ready: TransferReadyEvent | None = None
        if miss_slots:
            store = self._host_store.layer(layer_id)
            try:
                ready = self._transfer_engine.load_many_async(
                    store.w13, store.w2, miss_experts, bank.w13_slots, bank.w2_slots, miss_slots)
            except Exception:
                for slot in miss_slots:
                    if slot.state == SlotState.LOADING:
                        bank.clear_slot(slot.slot_id, force=True)
                raise
            consumer = consumer_stream
            if consumer is None and bank.w13_slots.is_cuda:
                consumer = torch.cuda.current_stream(bank.w13_slots.device)
            ready.install_consumer_dependency(consumer)
        self._publish_log2phy(layer_id, active, tuple(slot_ids))
        slot_to_expert: list[int | None] = [None] * bank.physical_expert_count
        for e in bank.pinned_logical_ids:
            slot_to_expert[bank.pinned_slot_for_logical_id(e)] = e
        for e, s in zip(active, slot_ids):
            slot_to_expert[s] = e
        self._active_slot_ids_by_layer[layer_id] = tuple(slot_ids)
        st = self.stage_stats
        st["calls"] += 1
        st["hits"] += len(active) - len(miss_experts)
        st["misses"] += len(miss_experts)
        st["h2d_bytes"] += 0 if ready is None else ready.bytes
        mapping = ExpertSlotMapping(layer_id, active, log2phy, tuple(slot_to_expert), tuple(slot_ids))
        return PreparedSlotWeights(bank.w13_slots, bank.w2_slots, mapping, bank.physical_expert_count)

    def stage_fixed_slot_plan(self, *, layer_id: int, active_experts: tuple[int, ...],
                              num_logical_experts: int, **kw) -> PreparedSlotWeights:
        self._assert_locked_slot_addresses(int(layer_id))
        return self.prepare_fixed_slot_plan_into_log2phy(
            layer_id=layer_id, active_experts=active_experts,
            num_logical_experts=num_logical_experts, **kw)

    def stage_full_residency_slot_plan(self, *, layer_id: int) -> bool:
        """Regime A: stage every routed expert once; log2phy becomes static."""
        layer_id = int(layer_id)
        routed = self._routed_counts[layer_id]
        if not self.is_static_residency_regime(routed):
            return False
        self.prepare_fixed_slot_plan_into_log2phy(layer_id=layer_id,
                                                  active_experts=tuple(range(routed)),
                                                  num_logical_experts=routed)
        return True

    # ------------------------------------------------------------------ compute lifecycle
    def begin_slot_compute(self, prepared: PreparedSlotWeights) -> SlotComputeHandle | None:
        layer_id = int(prepared.mapping.layer_id)
        bank = self._slot_banks.get(layer_id)
        if bank is None or prepared.w1.data_ptr() != bank.w13_slots.data_ptr():
            return None
        slot_ids = tuple(sorted(set(prepared.mapping.active_slot_ids)))
        if not slot_ids:
            return None
        leases = []
        for sid in slot_ids:
            slot = bank.slots[sid]
            expected = prepared.mapping.slot_to_expert[sid]
            expected_key = None if expected is None else ExpertKey(layer_id, int(expected))
            if slot.expert_key != expected_key:
                raise RuntimeError(
                    f"prepared mapping owner mismatch for slot {sid}: expected {expected_key}, found {slot.expert_key}")
            if slot.state != SlotState.READY:
                raise RuntimeError(f"prepared slot {sid} is not ready for compute: {slot.state.value}")
            leases.append(slot.lease())
        for sid in slot_ids:
            bank.mark_computing(sid)
        return SlotComputeHandle(layer_id, slot_ids, tuple(leases))

    def end_slot_compute(self, handle: SlotComputeHandle | None) -> None:
        if handle is None:
            return
        bank = self._slot_banks.get(handle.layer_id)
        if bank is None:
            return
        for lease in handle.leases:
            slot = bank.slots[lease.slot_id]
            if not slot.matches_lease(lease):
                raise RuntimeError(f"slot {lease.slot_id} ownership changed before compute completed")
            if slot.state != SlotState.COMPUTING:
                raise RuntimeError(f"slot {lease.slot_id} is not computing at compute completion: {slot.state.value}")
        event = None
        if bank.w13_slots.is_cuda:
            event = torch.cuda.Event()
            event.record(torch.cuda.current_stream(bank.w13_slots.device))
        for lease in handle.leases:
            if event is None:
                bank.slots[lease.slot_id].state = SlotState.READY
            else:
                self._slot_compute_done_events[(handle.layer_id, lease.slot_id, lease.version)] = event

    # ------------------------------------------------------------------ graph address lock
    def _fingerprint(self, layer_id: int) -> SlotAddressFingerprint:
        bank = self.slot_bank(layer_id)
        l2p = self._log2phy_buffers[layer_id]
        return SlotAddressFingerprint(bank.w13_slots.data_ptr(), bank.w2_slots.data_ptr(),
                                      l2p.data_ptr(), tuple(bank.w13_slots.shape),
                                      tuple(bank.w2_slots.shape), str(bank.w13_slots.device),
                                      str(bank.w13_slots.dtype))

    def capture_safe_slot_weights(self, *, layer_id: int) -> PreparedSlotWeights | None:
        """Fixed (w13_slots, w2_slots, log2phy) for a captured MLP; locks their addresses."""
        layer_id = int(layer_id)
        bank = self._slot_banks.get(layer_id)
        if bank is None:
            return None
        fp = self._fingerprint(layer_id)
        locked = self._graph_slot_address_fingerprints.setdefault(layer_id, fp)
        if locked != fp:
            raise RuntimeError(f"layer {layer_id} slot addresses changed after graph capture")
        mapping = ExpertSlotMapping(layer_id, (), self._log2phy_buffers[layer_id],
                                    tuple([None] * bank.physical_expert_count),
                                    self._active_slot_ids_by_layer.get(layer_id, ()))
        return PreparedSlotWeights(bank.w13_slots, bank.w2_slots, mapping, bank.physical_expert_count)

    def _assert_locked_slot_addresses(self, layer_id: int) -> None:
        locked = self._graph_slot_address_fingerprints.get(layer_id)
        if locked is not None and locked != self._fingerprint(layer_id):
            raise RuntimeError(f"layer {layer_id} slot addresses changed after graph capture")

    # ------------------------------------------------------------------ prefill stage banks
    def _stage_pool(self, layer_id: int) -> StagePool:
        bank = self.slot_bank(layer_id)
        key = (tuple(bank.w13_slots.shape[1:]), tuple(bank.w2_slots.shape[1:]),
               bank.w13_slots.dtype, str(bank.w13_slots.device))
        pool = self._stage_pools.get(key)
        n = self.config.effective_prefill_buffer_count
        if pool is None or len(pool.banks) < n:
            pool = StagePool(
                [ExpertSlotBank(self.config.num_slots, tuple(bank.w13_slots.shape[1:]),
                                tuple(bank.w2_slots.shape[1:]), dtype=bank.w13_slots.dtype,
                                device=bank.w13_slots.device) for _ in range(n)],
                [None] * n)
            self._stage_pools[key] = pool
        return pool

    def prefill_stage_bank(self, layer_id: int, buffer_index: int) -> ExpertSlotBank:
        pool = self._stage_pool(layer_id)
        if not 0 <= int(buffer_index) < len(pool.banks):
            raise ValueError(f"prefill buffer index {buffer_index} out of range [0, {len(pool.banks)})")
        return pool.banks[int(buffer_index)]

    def prefill_stage_buffer_release_event(self, layer_id: int, buffer_index: int):
        return self._stage_pool(layer_id).release_events[int(buffer_index)]

    def remember_prefill_stage_buffer_release(self, layer_id: int, buffer_index: int, event) -> None:
        self._stage_pool(layer_id).release_events[int(buffer_index)] = event

    def prepare_prefill_stage_plan(
        self,
        *,
        layer_id: int,
        active_experts: tuple[int, ...],
        buffer_index: int,
        wait_event=None,
        step_id: int | None = None,
    ) -> tuple[ExpertSlotBank, TransferReadyEvent]:
        """Stage one wave into stage buffer ``buffer_index`` at positional slots 0..n-1.

        Main-bank READY experts are copied device-to-device, the rest come from the store.
        Copies wait for ``wait_event`` (the buffer's previous consumer) on the copy stream.
        """
        layer_id = int(layer_id)
        wave = tuple(int(e) for e in active_experts)
        if len(wave) > self.config.num_slots:
            raise RuntimeError(f"wave of {len(wave)} experts exceeds num_slots={self.config.num_slots}")
        stage = self.prefill_stage_bank(layer_id, buffer_index)
        main = self.slot_bank(layer_id)
        store = self._host_store.layer(layer_id)
        step = int(step_id) if step_id is not None else self.next_step_id()
        slots = [stage.assign_transient_slot(i, ExpertKey(layer_id, e), step_id=step)
                 for i, e in enumerate(wave)]
        ready_main = main.ready_slot_ids(layer_id, wave)
        d2d = [(ready_main[e], i) for i, e in enumerate(wave) if e in ready_main]
        miss = [(e, i) for i, e in enumerate(wave) if e not in ready_main]
        eng = self._transfer_engine
        if stage.w13_slots.is_cuda and wait_event is not None:
            eng.stream().wait_event(wait_event)
        if d2d:
            eng.copy_rows(main.w13_slots, main.w2_slots, [s for s, _ in d2d],
                          stage.w13_slots, stage.w2_slots, [i for _, i in d2d])
        if miss:
            eng.copy_rows(store.w13, store.w2, [e for e, _ in miss],
                          stage.w13_slots, stage.w2_slots, [i for _, i in miss])
        event = eng.record_event() if stage.w13_slots.is_cuda else None
        nbytes = stage.slot_bytes * len(wave)
        return stage, TransferReadyEvent(event, tuple((s, s.lease()) for s in slots), bytes=nbytes)

    def prepare_full_layer_prefill_plan(self, *, layer_id: int, step_id: int | None = None
                                        ) -> tuple[ExpertSlotBank, TransferReadyEvent, dict]:
        """Stage every routed expert of a layer into a full-layer bank (row e = expert e).

        Recoverable fallback of the multi-wave executor (reference
        ``runtime.py:2260-2370``, ``patch_fused_moe.py:3472-3650``): one bank per weight
        layout and expert count, reused by every layer of that layout, so only one complete
        layer is resident at a time. The copies are ordered on the copy stream (the consumer
        waits on the returned event) instead of blocking the host.
        """
        layer_id = int(layer_id)
        if self.is_resident_layer(layer_id):
            raise RuntimeError(f"full-layer prefill plan must not run on resident layer {layer_id}")
        template = self._slot_banks.get(layer_id)
        if template is None:
            raise RuntimeError(f"layer {layer_id} is not registered for fixed-slot execution")
        store = self._host_store.layer(layer_id)
        E = int(self._routed_counts.get(layer_id, store.w13.shape[0]))
        key = (tuple(template.w13_slots.shape[1:]), tuple(template.w2_slots.shape[1:]),
               template.w13_slots.dtype, str(template.w13_slots.device), E)
        reused = key in self._full_layer_pool
        if not reused:
            self._full_layer_pool[key] = ExpertSlotBank(
                E, tuple(template.w13_slots.shape[1:]), tuple(template.w2_slots.shape[1:]),
                dtype=template.w13_slots.dtype, device=template.w13_slots.device)
        bank = self._full_layer_pool[key]
        step = int(step_id) if step_id is not None and int(step_id) >= 0 else self.next_step_id()
        slots = [bank.assign_transient_slot(e, ExpertKey(layer_id, e), step_id=step)
                 for e in range(E)]
        t0 = perf_counter()
        eng = self._transfer_engine
        eng.copy_rows(store.w13, store.w2, list(range(E)), bank.w13_slots, bank.w2_slots,
                      list(range(E)))
        event = eng.record_event() if bank.w13_slots.is_cuda else None
        payload = {
            "execution_mode": "reference_full_layer",
            "routed_expert_count": E,
            "physical_expert_count": int(bank.physical_expert_count),
            "h2d_bytes": int(bank.slot_bytes * E),
            "stage_issue_ms": round((perf_counter() - t0) * 1000.0, 3),
            "pool_reused": bool(reused),
        }
        return bank, TransferReadyEvent(event, tuple((sl, sl.lease()) for sl in slots),
                                        bytes=bank.slot_bytes * E), payload

    def wait_prefill_stage_plan(self, ready: TransferReadyEvent,
                                consumer_stream: torch.cuda.Stream | None = None) -> None:
        if consumer_stream is None and ready.event is not None:
            consumer_stream = torch.cuda.current_stream()
        ready.install_consumer_dependency(consumer_stream)

    # ------------------------------------------------------------------ ledger
    @property
    def released_original_weight_layers(self) -> tuple[int, ...]:
        """Layers whose original expert tensors were released, ascending."""
        return tuple(sorted(self._released_original_weight_layers))

    def release_original_expert_weights_if_ready(self, layer: torch.nn.Module
                                                 ) -> tuple[bool, tuple[str, ...]]:
        """Opt-in release of a non-resident layer's original expert tensors once its host
        store holds a copy (``moe_offload/runtime.py:1400-1453``). ``w13_weight`` and
        ``w2_weight`` keep their per-expert shape but hold zero experts, so their device memory
        returns to the allocator while the module stays intact. Returns (released, blockers)."""
        if not self.config.release_original_expert_weights:
            return False, ("release_original_expert_weights_disabled",)
        if not self.should_use_fixed_slots:
            return False, ("fixed_slots_disabled",)
        layer_id = int(getattr(layer, "layer_id", -1))
        if layer_id < 0:
            return False, ("invalid_layer_id",)
        if self.is_resident_layer(layer_id):
            return False, (f"resident_layer:{layer_id}",)
        if layer_id in self._released_original_weight_layers:
            return True, ()
        if layer_id not in self._slot_banks or self._host_store.layer(layer_id).on_device:
            return False, (f"host_store_missing:{layer_id}",)
        for name in ("w13_weight", "w2_weight"):
            param = getattr(layer, name)
            param.data = param.data.new_empty((0, *param.shape[1:]))
        self._released_original_weight_layers.add(layer_id)
        return True, ()

    def memory_ledger(self) -> MoeOffloadMemoryLedger:
        stage = sum(b.total_bytes for p in self._stage_pools.values() for b in p.banks)
        return MoeOffloadMemoryLedger(
            host_store_bytes=self._host_store.total_bytes,
            slot_bank_bytes=sum(b.total_bytes for b in self._slot_banks.values()),
            stage_bank_bytes=stage + sum(b.total_bytes for b in self._full_layer_pool.values()),
            log2phy_bytes=sum(t.numel() * 4 for t in self._log2phy_buffers.values()),
        )


_runtime: MoeOffloadRuntime | None = None
_runtime_lock = threading.Lock()


def get_moe_offload_runtime() -> MoeOffloadRuntime:
    global _runtime
    with _runtime_lock:
        if _runtime is None:
            _runtime = MoeOffloadRuntime()
        return _runtime


def reset_moe_offload_runtime() -> None:
    global _runtime
    with _runtime_lock:
        _runtime = None
