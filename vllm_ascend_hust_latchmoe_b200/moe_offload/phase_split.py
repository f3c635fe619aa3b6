"""Capacity-bounded multi-wave planning (host side) for the slot-bank MoE layer.

Mirrors the planning API of the reference's ``moe_offload/phase_split.py``:
``plan_balanced_b2_waves`` (:495-555), ``plan_b2_prefill_async_schedule`` (:557-640),
``simulate_b2_prefill_issue_log`` (:681-766), ``count_routed_tokens_by_expert`` (:479-492)
and the recoverable ``B2WaveFallback`` (:292). The per-pair work the reference does with
tensor ops (pair compaction, physical slot ids, the global combine index) runs on the GPU
in ``lm_build_groups``; the host only authors the tiny expert -> (group, bank row) table.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

import torch


class B2WaveFallback(RuntimeError):
    """Recoverable multi-wave qualification failure detected before any result is
    published; the caller may rerun the layer on the blocking full-layer path."""


@dataclass(frozen=True)
class B2WavePlan:
    waves: tuple[tuple[int, ...], ...]
    token_counts_by_expert: dict[int, int]

    @property
    def active_expert_count(self) -> int:
        return len(self.token_counts_by_expert)

    @property
    def total_pairs(self) -> int:
        return sum(self.token_counts_by_expert.values())

    def wave_tokens(self, wave: tuple[int, ...]) -> int:
        return sum(self.token_counts_by_expert.get(int(e), 0) for e in wave)

    def to_jsonable(self) -> dict[str, object]:
        return {
            "n_active": self.active_expert_count,
            "n_pairs": self.total_pairs,
            "n_waves": len(self.waves),
            "waves": [{"experts": list(w), "tokens": self.wave_tokens(w)} for w in self.waves],
        }


@dataclass(frozen=True)
class B2PrefillAsyncSchedule:
    compute_order: tuple[int, ...]
    hit_wave_indices: tuple[int, ...]
    staged_wave_indices: tuple[int, ...]
    staged_issue_order: tuple[int, ...]
    prefetch_depth: int
    buffer_count: int
    initial_stage_count: int
    transfer_aware: bool
    estimated_h2d_bytes_by_wave: tuple[int, ...] = ()
    estimated_compute_cost_by_wave: tuple[float, ...] = ()

    def to_jsonable(self) -> dict[str, object]:
        return {
            "compute_order": list(self.compute_order),
            "hit_wave_indices": list(self.hit_wave_indices),
            "staged_wave_indices": list(self.staged_wave_indices),
            "staged_issue_order": list(self.staged_issue_order),
            "prefetch_depth": self.prefetch_depth,
            "buffer_count": self.buffer_count,
            "initial_stage_count": self.initial_stage_count,
            "transfer_aware": self.transfer_aware,
            "estimated_h2d_bytes_by_wave": list(self.estimated_h2d_bytes_by_wave),
            "estimated_compute_cost_by_wave": list(self.estimated_compute_cost_by_wave),
        }


def count_routed_tokens_by_expert(topk_ids: torch.Tensor) -> dict[int, int]:
    """Routed (token, top-k) pairs per logical expert (host tensors only)."""
    if topk_ids.numel() == 0:
        return {}
    counts = torch.bincount(topk_ids.detach().reshape(-1).to("cpu", torch.int64).clamp_min(-1) + 1)
    return {e - 1: int(c) for e, c in enumerate(counts.tolist()) if e > 0 and c > 0}


def counts_from_histogram(counts: list[int] | torch.Tensor) -> dict[int, int]:
    values = counts.tolist() if isinstance(counts, torch.Tensor) else list(counts)
    return {e: int(c) for e, c in enumerate(values) if int(c) > 0}


def plan_balanced_b2_waves(
    token_counts_by_expert: dict[int, int],
    num_slots: int,
    *,
    slot_readiness: dict[int, bool] | None = None,
    fold_partial_hits_into_miss: bool = True,
) -> B2WavePlan:
    """Canonical waves: experts by (-count, id) into the least-loaded non-full wave.

    Starts with ceil(U / S) waves, opens a new one only when all are full, and sorts the
    members of each wave. Slot readiness is accepted for API compatibility and never
    changes membership, so equal routings always produce the same GEMM groups.
    """
    if num_slots <= 0:
        raise ValueError(f"num_slots must be greater than 0, got {num_slots}")
    del slot_readiness, fold_partial_hits_into_miss
    active = {int(e): int(c) for e, c in token_counts_by_expert.items() if int(c) > 0}
    if not active:
        return B2WavePlan((), {})
    order = sorted(active, key=lambda e: (-active[e], e))
    n0 = -(-len(order) // num_slots)
    waves: list[list[int]] = [[] for _ in range(n0)]
    heap = [(0, i) for i in range(n0)]  # (load, wave index) of waves with free capacity
    for e in order:
        if heap:
            load, i = heapq.heappop(heap)
            waves[i].append(e)
            if len(waves[i]) < num_slots:
                heapq.heappush(heap, (load + active[e], i))
        else:
            waves.append([e])
            if num_slots > 1:
                heapq.heappush(heap, (active[e], len(waves) - 1))
    return B2WavePlan(tuple(tuple(sorted(w)) for w in waves), active)


def _per_wave(estimates, n: int, cast) -> tuple:
    if estimates is None:
        return tuple(cast(0) for _ in range(n))
    if isinstance(estimates, dict):
        return tuple(max(cast(0), cast(estimates.get(i, 0))) for i in range(n))
    vals = [cast(v) for v in estimates]
    return tuple(max(cast(0), vals[i]) if i < len(vals) else cast(0) for i in range(n))


def plan_b2_prefill_async_schedule(
    waves: tuple[tuple[int, ...], ...],
    *,
    slot_readiness: dict[int, bool] | None = None,
    prefetch_depth: int = 1,
    buffer_count: int = 2,
    h2d_bytes_by_wave=None,
    compute_cost_by_wave=None,
    transfer_aware: bool = False,
) -> B2PrefillAsyncSchedule:
    """Stage-issue and compute order of the waves. Pure-hit waves read the main bank and
    need no stage buffer; the others are staged, primed up to the prefetch depth. With
    ``transfer_aware`` the longest transfers are staged first and the most expensive hit
    waves computed first to cover them."""
    ready = slot_readiness or {}
    hit = [i for i, w in enumerate(waves) if all(ready.get(int(e), False) for e in w)]
    staged = [i for i, w in enumerate(waves) if not all(ready.get(int(e), False) for e in w)]
    depth = max(0, int(prefetch_depth))
    bufs = max(1, int(buffer_count))
    n = len(waves)
    h2d = _per_wave(h2d_bytes_by_wave, n, int)
    cost = _per_wave(compute_cost_by_wave, n, float)
    aware = bool(transfer_aware) and n > 0 and depth > 0 and bufs > 1
    if aware:
        issue = tuple(sorted(staged, key=lambda i: (-h2d[i], -cost[i], i)))
        compute = tuple(sorted(hit, key=lambda i: (-cost[i], i))) + issue
    else:
        issue = tuple(staged)
        compute = tuple(range(n))
    return B2PrefillAsyncSchedule(
        compute_order=compute,
        hit_wave_indices=tuple(hit),
        staged_wave_indices=tuple(staged),
        staged_issue_order=issue,
        prefetch_depth=depth,
        buffer_count=bufs,
        initial_stage_count=min(depth, bufs, len(staged)),
        transfer_aware=aware,
        estimated_h2d_bytes_by_wave=h2d,
        estimated_compute_cost_by_wave=cost,
    )


class WaveIssuer:
    """Drives stage buffers through the schedule: yields ("issue_stage", wave, buffer),
    ("issue_hit", wave, None) and ("compute", wave, buffer) events in executor order."""

    def __init__(self, schedule: B2PrefillAsyncSchedule, prefetch_depth: int | None = None,
                 buffer_count: int | None = None) -> None:
        self.schedule = schedule
        self.depth = schedule.prefetch_depth if prefetch_depth is None else int(prefetch_depth)
        self.bufs = schedule.buffer_count if buffer_count is None else int(buffer_count)

    def events(self):
        order = list(self.schedule.staged_issue_order)
        cursor = 0
        issued: set[int] = set()
        held: dict[int, int] = {}  # wave -> stage buffer holding it
        staged = set(self.schedule.staged_wave_indices)
        out: list[tuple[str, int, int | None]] = []

        def issue(current: int | None = None) -> bool:
            nonlocal cursor
            if cursor >= len(order):
                return False
            busy = set(held.values()) | ({current} if current is not None else set())
            free = next((b for b in range(max(self.bufs, 1)) if b not in busy), None)
            if free is None:
                return False
            w = order[cursor]
            cursor += 1
            issued.add(w)
            held[w] = free
            out.append(("issue_stage", w, free))
            return True

        def prefetch(current: int | None = None) -> None:
            if self.depth <= 0:
                return
            target = min(self.depth, max(self.bufs, 1) - (1 if current is not None else 0))
            while len(held) < target and issue(current):
                pass

        initial = min(max(self.depth, 0), max(self.bufs, 1), len(order))
        while cursor < initial and issue():
            pass
        for w in self.schedule.compute_order:
            if w not in issued:
                if w in staged:
                    if not issue():
                        raise RuntimeError(f"unable to issue staged wave {w}; no buffer available")
                else:
                    issued.add(w)
                    out.append(("issue_hit", w, None))
            current = held.pop(w, None)
            prefetch(current)
            out.append(("compute", w, current))
            prefetch()
        return out


def simulate_b2_prefill_issue_log(schedule: B2PrefillAsyncSchedule, *, prefetch_depth=None,
                                  buffer_count=None) -> tuple[tuple[str, int], ...]:
    """The (event, wave) sequence of the executor loop, without tensors or streams."""
    return tuple((kind, w) for kind, w, _ in
                 WaveIssuer(schedule, prefetch_depth, buffer_count).events())
