"""Profile-guided prefill residency: which layers keep their experts in HBM.

Prefill cost differs a lot between the two tiers. A resident layer reads its experts in place
(one grouped-MLP pass); an offloaded layer runs the capacity-bounded wave executor and stages
its experts. With a fixed offload budget the better use of it is to keep the layers whose
prefill is most expensive resident and offload cheaper ones instead. This module follows the
reference's planner (``moe_offload/prefill_residency.py:223``, applied by
``moe_offload/autoconfig.py:585-640``): it reads per-layer prefill cost records from JSONL
profiles and swaps the costliest default-offloaded layers with the cheapest default-resident
layers while the swap lowers the cost; layers without profile evidence keep the default plan.

The profile schema is the reference's (event names ``b2_work_conserving_prefill`` for an
offloaded layer's call and ``prefill_resident_native`` for a resident layer's), so profiles
cross between the two implementations. On B200 the records come from
:class:`PrefillProfileRecorder`: each layer call is bracketed by CUDA events on its stream,
and the events are read back only when the recorder flushes, never inside the forward.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Iterable

B2_EVENT = "b2_work_conserving_prefill"
RESIDENT_EVENT = "prefill_resident_native"


def _as_float(value: Any, default: float = 0.0) -> float:
    try:
        return float(default) if value is None else float(value)
    except (TypeError, ValueError):
        return float(default)


def _as_int(value: Any, default: int = 0) -> int:
    try:
        return int(default) if value is None else int(float(value))
    except (TypeError, ValueError):
        return int(default)


@dataclass
class PrefillLayerCost:
    """Accumulated prefill profile evidence of one layer."""

    layer_id: int
    calls: int = 0
    end_to_end_ms: float = 0.0
    loop_ms: float = 0.0
    scatter_ms: float = 0.0
    gmm_ms: float = 0.0
    stage_wait_ms: float = 0.0
    h2d_bytes: int = 0
    pairs: int = 0
    waves: int = 0
    active_experts: int = 0
    b2_calls: int = 0
    resident_native_calls: int = 0

    @property
    def score_ms(self) -> float:
        """Total sampled time: a layer seen more often in the profiled workload weighs more."""
        return float(self.end_to_end_ms)

    def add_event(self, record: dict[str, Any]) -> None:
        payload = record.get("payload") or {}
        control = payload.get("control_ms") or {}
        name = str(record.get("name") or "")
        seconds_ms = _as_float(record.get("seconds")) * 1000.0
        self.calls += 1
        per_wave = payload.get("waves") or ()
        if name == B2_EVENT:
            self.b2_calls += 1
            self.end_to_end_ms += _as_float(control.get("end_to_end"), seconds_ms)
            self.pairs += _as_int(payload.get("n_pairs"))
            self.waves += _as_int(payload.get("n_waves"))
            self.active_experts += _as_int(payload.get("n_active"))
            self.loop_ms += _as_float(control.get("loop"))
            summary = payload.get("wave_summary")
            if isinstance(summary, dict):
                # a summary replaces the per-wave list
                self.scatter_ms += _as_float(summary.get("layer_scatter_ms"),
                                             _as_float(control.get("scatter_total")))
                self.gmm_ms += _as_float(summary.get("gmm_ms"))
                self.stage_wait_ms += _as_float(summary.get("stage_wait_ms"))
                self.h2d_bytes += _as_int(summary.get("h2d_bytes"))
                return
            self.scatter_ms += _as_float(control.get("scatter_total"))
        elif name == RESIDENT_EVENT:
            self.resident_native_calls += 1
            self.end_to_end_ms += seconds_ms
            self.pairs += _as_int(payload.get("n_tokens"))
        else:
            self.end_to_end_ms += seconds_ms
        if isinstance(per_wave, list):
            for wave in per_wave:
                if isinstance(wave, dict):
                    self.gmm_ms += _as_float(wave.get("gmm_ms"))
                    self.stage_wait_ms += _as_float(wave.get("stage_wait_ms"))
                    self.h2d_bytes += _as_int(wave.get("h2d_bytes"))

    def to_jsonable(self) -> dict[str, object]:
        return {
            "layer_id": int(self.layer_id),
            "calls": int(self.calls),
            "score_ms": round(self.score_ms, 3),
            "mean_score_ms": round(self.score_ms / self.calls if self.calls else 0.0, 3),
            "loop_ms": round(self.loop_ms, 3),
            "scatter_ms": round(self.scatter_ms, 3),
            "gmm_ms": round(self.gmm_ms, 3),
            "stage_wait_ms": round(self.stage_wait_ms, 3),
            "h2d_bytes": int(self.h2d_bytes),
            "pairs": int(self.pairs),
            "waves": int(self.waves),
            "active_experts": int(self.active_experts),
            "b2_calls": int(self.b2_calls),
            "resident_native_calls": int(self.resident_native_calls),
        }


@dataclass(frozen=True)
class PrefillResidencyPlacement:
    resident_layer_ids: tuple[int, ...]
    offloaded_layer_ids: tuple[int, ...]
    swaps: tuple[dict[str, object], ...]
    profiled_layer_ids: tuple[int, ...]
    profiled_resident_layer_ids: tuple[int, ...]
    profiled_offloaded_layer_ids: tuple[int, ...]
    reason: str

    def to_jsonable(self) -> dict[str, object]:
        return {
            "resident_layer_ids": list(self.resident_layer_ids),
            "offloaded_layer_ids": list(self.offloaded_layer_ids),
            "swaps": list(self.swaps),
            "profiled_layer_ids": list(self.profiled_layer_ids),
            "profiled_resident_layer_ids": list(self.profiled_resident_layer_ids),
            "profiled_offloaded_layer_ids": list(self.profiled_offloaded_layer_ids),
            "reason": self.reason,
        }


def load_prefill_layer_costs(profile_path: str | Path, *, strict: bool = False,
                             costs: dict[int, PrefillLayerCost] | None = None
                             ) -> dict[int, PrefillLayerCost]:
    """Per-layer costs from one profile JSONL (merged into ``costs`` when given). Lines that
    are not JSON objects, other events and negative layer ids are skipped; with ``strict`` a
    missing file or a malformed line raises."""
    path = Path(profile_path)
    merged: dict[int, PrefillLayerCost] = {} if costs is None else costs
    if not path.is_file():
        if strict:
            raise FileNotFoundError(str(path))
        return merged
    with path.open(encoding="utf-8") as fh:
        for lineno, raw in enumerate(fh, start=1):
            text = raw.strip()
            if not text:
                continue
            try:
                record = json.loads(text)
            except json.JSONDecodeError:
                if strict:
                    raise ValueError(f"Invalid JSON on {path}:{lineno}") from None
                continue
            if not isinstance(record, dict) or record.get("name") not in (B2_EVENT,
                                                                         RESIDENT_EVENT):
                continue
            lid = _as_int(record.get("layer_id"), -1)
            if lid >= 0:
                merged.setdefault(lid, PrefillLayerCost(lid)).add_event(record)
    return merged


def load_prefill_layer_costs_many(profile_paths: Iterable[str | Path], *,
                                  strict: bool = False) -> dict[int, PrefillLayerCost]:
    costs: dict[int, PrefillLayerCost] = {}
    for p in profile_paths:
        load_prefill_layer_costs(p, strict=strict, costs=costs)
    return costs


def plan_profile_guided_prefill_residency(*, num_layers: int,
                                          default_offloaded_layer_ids: Iterable[int],
                                          layer_costs: dict[int, PrefillLayerCost]
                                          ) -> PrefillResidencyPlacement:
    """Pair the default-offloaded layers in decreasing cost with the default-resident layers
    in increasing cost (profiled layers only) and swap each pair while the offloaded one
    costs strictly more. Without evidence on both sides the default plan is kept and the
    reason says which side is missing."""
    n = int(num_layers)
    offloaded = {int(x) for x in default_offloaded_layer_ids}
    profiled = sorted(int(lid) for lid, c in layer_costs.items() if 0 <= int(lid) < n
                      and c.calls > 0)

    def placement(swaps=(), reason="no_prefill_profile", p_res=(), p_off=()):
        return PrefillResidencyPlacement(
            resident_layer_ids=tuple(i for i in range(n) if i not in offloaded),
            offloaded_layer_ids=tuple(sorted(offloaded)), swaps=tuple(swaps),
            profiled_layer_ids=tuple(profiled), profiled_resident_layer_ids=tuple(p_res),
            profiled_offloaded_layer_ids=tuple(p_off), reason=reason)

    if not profiled:
        return placement()
    p_off = tuple(i for i in profiled if i in offloaded)
    p_res = tuple(i for i in profiled if i not in offloaded)
    if not p_res or not p_off:
        why = "missing_profiled_resident_layers" if p_off else "missing_profiled_offloaded_layers"
        return placement(reason=why, p_res=p_res, p_off=p_off)
    score = {i: layer_costs[i].score_ms for i in profiled}
    # stable sorts: equal scores keep ascending layer order
    expensive_offloaded = sorted(p_off, key=lambda i: score[i], reverse=True)
    cheap_resident = sorted(p_res, key=lambda i: score[i])
    swaps = []
    for off, res in zip(expensive_offloaded, cheap_resident):
        if score[off] <= score[res]:
            break
        offloaded.discard(off)
        offloaded.add(res)
        swaps.append({"make_resident": off, "make_offloaded": res,
                      "resident_gain_ms": round(score[off] - score[res], 3),
                      "old_offloaded_score_ms": round(score[off], 3),
                      "old_resident_score_ms": round(score[res], 3)})
    reason = "profile_guided_swaps" if swaps else "profile_available_no_beneficial_swap"
    return placement(swaps, reason, p_res, p_off)


# --------------------------------------------------------------------------- B200 profile source
@dataclass
class _PendingCall:
    layer_id: int
    resident: bool
    start: Any
    end: Any
    tokens: int
    pairs: int
    waves: int
    active: int
    h2d_bytes: int


@dataclass
class PrefillProfileRecorder:
    """Collects prefill layer calls as CUDA-event pairs and writes them, on :meth:`flush`, as
    JSONL records of the reference's profile schema (``b2_work_conserving_prefill`` for an
    offloaded layer, ``prefill_resident_native`` for a resident one). Recording adds two
    event records per call and no synchronisation; flush synchronises on the events."""

    path: str
    pending: list[_PendingCall] = field(default_factory=list)

    def begin(self):
        import torch

        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return ev

    def end(self, start, *, layer_id: int, resident: bool, tokens: int, pairs: int,
            waves: int = 0, active: int = 0, h2d_bytes: int = 0) -> None:
        import torch

        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.pending.append(_PendingCall(int(layer_id), bool(resident), start, ev, int(tokens),
                                         int(pairs), int(waves), int(active), int(h2d_bytes)))

    def records(self) -> list[dict[str, Any]]:
        out = []
        for c in self.pending:
            c.end.synchronize()
            ms = float(c.start.elapsed_time(c.end))
            if c.resident:
                out.append({"name": RESIDENT_EVENT, "layer_id": c.layer_id, "seconds": ms / 1e3,
                            "payload": {"n_tokens": c.tokens}})
            else:
                out.append({"name": B2_EVENT, "layer_id": c.layer_id, "seconds": ms / 1e3,
                            "payload": {"n_pairs": c.pairs, "n_waves": c.waves,
                                        "n_active": c.active,
                                        "control_ms": {"end_to_end": ms},
                                        "wave_summary": {"h2d_bytes": c.h2d_bytes}}})
        return out

    def flush(self) -> int:
        """Append the pending calls to the JSONL file; returns the number written."""
        recs = self.records()
        if recs:
            os.makedirs(os.path.dirname(os.path.abspath(self.path)), exist_ok=True)
            with open(self.path, "a", encoding="utf-8") as fh:
                for r in recs:
                    fh.write(json.dumps(r) + "\n")
        self.pending.clear()
        return len(recs)
