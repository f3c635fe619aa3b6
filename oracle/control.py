"""Integer control-plane oracle (pinned against the reference's own control plane).

Each function restates one reference algorithm; golden vectors produced by running the
reference itself (tests/golden/make_golden.py) and the vectors in its unit tests pin them.
"""

from __future__ import annotations

import numpy as np

EMPTY, LOADING, READY, COMPUTING = "empty", "loading", "ready", "computing"


class SlotAllocator:
    """Slot-bank allocation of the decode stage, in one stage call per ``stage()``.

    Restates ``moe_offload/slot_bank.py:211-232`` (allocate_for: resident -> touch; else
    first EMPTY slot, else the READY slot with the least ``(last_used_step, slot_id)``;
    version += 1, state LOADING) driven by the loop of
    ``moe_offload/runtime.py:1636-1902`` (prepare_fixed_slot_plan_into_log2phy): in-flight
    slots are drained to READY first; active experts are visited in the caller's order
    (the stage seam passes them sorted, ``ops/fused_moe/moe_offload_stage_op.py:304``); a
    READY hit only bumps ``last_used_step``; misses allocate. Loads complete (READY) at the
    next drain, and only changed log2phy entries are rewritten (``runtime.py:1904-1925``).
    """

    def __init__(self, num_slots: int, num_experts: int):
        self.num_slots = int(num_slots)
        self.state = [EMPTY] * self.num_slots
        self.owner = [-1] * self.num_slots
        self.version = [0] * self.num_slots
        self.last_used = [-1] * self.num_slots
        self.resident: dict[int, int] = {}
        self.log2phy = np.full(int(num_experts), -1, dtype=np.int32)
        self._cached: dict[int, int] = {}
        self.step = 0

    def _allocate(self, expert: int, step: int) -> int:
        if expert in self.resident:
            s = self.resident[expert]
            self.last_used[s] = step
            return s
        slot = next((s for s in range(self.num_slots) if self.state[s] == EMPTY), None)
        if slot is None:
            ready = [s for s in range(self.num_slots) if self.state[s] == READY]
            if not ready:
                raise RuntimeError("no evictable expert slots")
            slot = min(ready, key=lambda s: (self.last_used[s], s))
        if self.owner[slot] >= 0:
            self.resident.pop(self.owner[slot], None)
        self.owner[slot] = expert
        self.state[slot] = LOADING
        self.version[slot] += 1
        self.last_used[slot] = step
        self.resident[expert] = slot
        return slot

    def stage(self, active: tuple[int, ...]) -> dict[str, object]:
        active = tuple(dict.fromkeys(int(e) for e in active))
        if len(active) > self.num_slots:
            raise RuntimeError("active expert working set exceeds num_slots")
        for s in range(self.num_slots):
            if self.state[s] in (LOADING, COMPUTING):
                self.state[s] = READY
        step = self.step
        self.step += 1
        slots, misses = [], []
        for e in active:
            s = self.resident.get(e)
            if s is not None and self.state[s] == READY:
                self.last_used[s] = step
            else:
                s = self._allocate(e, step)
                misses.append(e)
            slots.append(s)
        changed = [(e, s) for e, s in zip(active, slots) if self._cached.get(e) != s]
        for e, s in changed:
            self.log2phy[e] = s
            self._cached[e] = s
        return {
            "active_slot_ids": tuple(slots),
            "misses": tuple(misses),
            "log2phy_updates": tuple(changed),
            "log2phy": self.log2phy.copy(),
        }


def plan_balanced_waves(token_counts: dict[int, int], num_slots: int) -> tuple[tuple[int, ...], ...]:
    """Canonical capacity-bounded waves (``moe_offload/phase_split.py:495-555``).

    Experts sorted by (-count, id); ceil(U/S) bins to start; each expert goes to the
    least-loaded bin that still has room (first such bin on a load tie); a new bin only
    when all are full; members sorted inside each wave. Readiness never changes the plan.
    """
    if num_slots <= 0:
        raise ValueError("num_slots must be greater than 0")
    active = {int(e): int(c) for e, c in token_counts.items() if int(c) > 0}
    if not active:
        return ()
    order = sorted(active, key=lambda e: (-active[e], e))
    nb = (len(order) + num_slots - 1) // num_slots
    bins: list[list[int]] = [[] for _ in range(nb)]
    loads = [0] * nb
    for e in order:
        best = None
        for i, b in enumerate(bins):
            if len(b) >= num_slots:
                continue
            if best is None or loads[i] < loads[best]:
                best = i
        if best is None:
            bins.append([e])
            loads.append(active[e])
        else:
            bins[best].append(e)
            loads[best] += active[e]
    return tuple(tuple(sorted(b)) for b in bins)


def async_schedule(waves, readiness: dict[int, bool] | None = None, prefetch_depth: int = 1,
                   buffer_count: int = 2, h2d_bytes_by_wave=None, compute_cost_by_wave=None,
                   transfer_aware: bool = False) -> dict[str, object]:
    """Stage/compute order of the multi-wave executor (``phase_split.py:557-640``)."""
    readiness = readiness or {}
    hit, staged = [], []
    for i, wave in enumerate(waves):
        (hit if all(readiness.get(int(e), False) for e in wave) else staged).append(i)
    depth = max(0, int(prefetch_depth))
    bufs = max(1, int(buffer_count))
    n = len(waves)

    def norm(est, cast):
        if est is None:
            return tuple(cast(0) for _ in range(n))
        if isinstance(est, dict):
            return tuple(max(cast(0), cast(est.get(i, 0))) for i in range(n))
        vals = tuple(cast(v) for v in est)
        return tuple(max(cast(0), vals[i]) if i < len(vals) else cast(0) for i in range(n))

    h2d = norm(h2d_bytes_by_wave, int)
    cost = norm(compute_cost_by_wave, float)
    aware = bool(transfer_aware) and n > 0 and depth > 0 and bufs > 1
    if aware:
        hit_order = tuple(sorted(hit, key=lambda i: (-cost[i], i)))
        issue = tuple(sorted(staged, key=lambda i: (-h2d[i], -cost[i], i)))
        compute = hit_order + issue
    else:
        issue = tuple(staged)
        compute = tuple(range(n))
    return {
        "compute_order": compute,
        "hit_wave_indices": tuple(hit),
        "staged_wave_indices": tuple(staged),
        "staged_issue_order": issue,
        "prefetch_depth": depth,
        "buffer_count": bufs,
        "initial_stage_count": min(depth, bufs, len(staged)),
        "transfer_aware": aware,
    }


def simulate_issue_log(schedule: dict[str, object], prefetch_depth: int | None = None,
                       buffer_count: int | None = None) -> tuple[tuple[str, int], ...]:
    """Issue/compute event order of the executor loop (``phase_split.py:681-766``)."""
    log: list[tuple[str, int]] = []
    order = list(schedule["staged_issue_order"])
    cursor = 0
    issued: set[int] = set()
    depth = int(schedule["prefetch_depth"] if prefetch_depth is None else prefetch_depth)
    bufs = int(schedule["buffer_count"] if buffer_count is None else buffer_count)
    initial = min(max(depth, 0), max(bufs, 1), len(order))
    records: dict[int, int] = {}

    def free_buffer(current=None):
        busy = set(records.values())
        if current is not None:
            busy.add(int(current))
        for b in range(max(bufs, 1)):
            if b not in busy:
                return b
        return None

    def issue_next(current=None) -> bool:
        nonlocal cursor
        if cursor >= len(order):
            return False
        b = free_buffer(current)
        if b is None:
            return False
        w = int(order[cursor])
        cursor += 1
        issued.add(w)
        records[w] = b
        log.append(("issue_stage", w))
        return True

    while cursor < initial:
        if not issue_next():
            break

    def prefetch(current=None):
        if depth <= 0:
            return
        target = min(max(depth, 0), max(bufs, 1) - (1 if current is not None else 0))
        while len(records) < target:
            if not issue_next(current):
                break

    staged = set(int(i) for i in schedule["staged_wave_indices"])
    for w in schedule["compute_order"]:
        w = int(w)
        if w not in issued:
            if w in staged:
                if not issue_next():
                    raise RuntimeError(f"unable to issue staged wave {w}")
            else:
                issued.add(w)
                log.append(("issue_hit", w))
        current = records.pop(w, None)
        prefetch(current)
        log.append(("compute", w))
        prefetch()
    return tuple(log)


def group_pairs(topk_ids: np.ndarray, expert_to_group: np.ndarray, num_groups: int):
    """Stable counting sort of routed pairs by group (the device pair grouping).

    Returns ``(group_offsets[G+1], pair_to_row[P], row_to_pair[R])``: rows of group g are
    contiguous and keep the original flat pair order (``phase_split.py:1224-1385`` compacts
    each wave's pairs with ``nonzero`` in ascending flat order; ``slot_mapping.py:116-141``
    maps logical ids through ``log2phy``). Unmapped pairs get ``pair_to_row = -1``.
    """
    flat = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    e2g = np.asarray(expert_to_group, dtype=np.int64)
    valid = (flat >= 0) & (flat < e2g.size)
    g = np.full(flat.shape, -1, dtype=np.int64)
    g[valid] = e2g[flat[valid]]
    g[(g < 0) | (g >= num_groups)] = -1
    counts = np.bincount(g[g >= 0], minlength=num_groups)[:num_groups]
    offsets = np.zeros(num_groups + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    mapped = np.nonzero(g >= 0)[0]
    order = mapped[np.argsort(g[mapped], kind="stable")]
    pair_to_row = np.full(flat.shape, -1, dtype=np.int32)
    pair_to_row[order] = np.arange(order.size, dtype=np.int32)
    return offsets, pair_to_row, order.astype(np.int32)


def wave_pair_plans(topk_ids: np.ndarray, waves, ready_slots: dict[int, int] | None = None):
    """Per-wave pair compaction (``phase_split.py:1224-1385``).

    For every wave: flat pair offsets of its experts in ascending order, their token
    indices (offset // k) and physical slots: the position inside the wave, or the
    main-bank slot when every member of the wave is a READY hit (pure-hit wave).
    """
    flat = np.asarray(topk_ids).reshape(-1)
    k = np.asarray(topk_ids).shape[1] if np.asarray(topk_ids).ndim > 1 else 1
    ready = ready_slots or {}
    plans = []
    for wave in waves:
        pure_hit = bool(ready) and all(int(e) in ready for e in wave)
        slot_of = {int(e): (int(ready[int(e)]) if pure_hit else i) for i, e in enumerate(wave)}
        offs = np.nonzero(np.isin(flat, np.asarray(wave)))[0]
        plans.append({
            "flat_pair_offsets": offs.astype(np.int64),
            "token_indices": (offs // k).astype(np.int64),
            "physical_slot_ids": np.asarray([slot_of[int(flat[o])] for o in offs], dtype=np.int64),
        })
    return plans


def native_combine_index(wave_pair_offsets, wave_local_unpermute, total_pairs: int):
    """Global unpermute index in original pair order over concatenated wave outputs
    (``phase_split.py:1765-1856``): ``index[pair_offsets[w][i]] = local[w][i] + rows_before(w)``.
    Fails closed when the waves do not cover every pair exactly once."""
    index = np.full(int(total_pairs), -1, dtype=np.int64)
    base = 0
    covered = 0
    for offs, local in zip(wave_pair_offsets, wave_local_unpermute):
        offs = np.asarray(offs, dtype=np.int64)
        local = np.asarray(local, dtype=np.int64)
        if offs.size != local.size:
            raise ValueError("wave unpermute index does not match its pair count")
        index[offs] = local + base
        base += offs.size
        covered += offs.size
    if covered != total_pairs or (index < 0).any():
        raise ValueError("waves must cover every original top-k pair exactly once")
    return index
