"""Profile-guided prefill residency, pinned to the reference's own planner and loader.

``tests/golden/residency.json`` holds profiles in the reference's JSONL schema (malformed
lines, other events and out-of-range layer ids mixed in) with the per-layer costs and the
placement the reference computed from them (``tests/golden/make_golden.py``). The vectors of
the reference's unit tests are asserted directly as well."""

import json
from pathlib import Path

import pytest

from vllm_ascend_hust_latchmoe_b200 import autoconfig as ac
from vllm_ascend_hust_latchmoe_b200.moe_offload import prefill_residency as pr

GOLDEN = Path(__file__).parent / "golden" / "residency.json"


def _write(path: Path, lines) -> str:
    path.write_text("\n".join(lines) + "\n", encoding="utf-8")
    return str(path)


def test_loader_and_planner_match_reference_golden(tmp_path):
    cases = json.loads(GOLDEN.read_text())
    assert len(cases) == 40
    for i, case in enumerate(cases):
        path = _write(tmp_path / f"p{i}.jsonl", case["lines"])
        costs = pr.load_prefill_layer_costs(path)
        assert {str(k): v.to_jsonable() for k, v in sorted(costs.items())} == case["costs"], i
        plan = pr.plan_profile_guided_prefill_residency(
            num_layers=case["num_layers"], default_offloaded_layer_ids=case["default_offloaded"],
            layer_costs=costs)
        assert json.loads(json.dumps(plan.to_jsonable())) == case["placement"], i


def test_reference_unit_vectors(tmp_path):
    # reference tests/test_autoconfig.py:713-745 (resident-native event) and :748-782 (summary)
    p = _write(tmp_path / "a.jsonl", [json.dumps({
        "name": "prefill_resident_native", "layer_id": 0, "seconds": 0.012,
        "payload": {"n_tokens": 4096}})])
    c = pr.load_prefill_layer_costs(p)[0]
    assert c.resident_native_calls == 1 and c.score_ms == pytest.approx(12.0) and c.pairs == 4096
    p = _write(tmp_path / "b.jsonl", [json.dumps({
        "name": "b2_work_conserving_prefill", "layer_id": 3, "seconds": 0.1,
        "payload": {"n_pairs": 10, "n_waves": 2, "n_active": 5,
                    "control_ms": {"end_to_end": 50.0, "loop": 40.0},
                    "wave_summary": {"gmm_ms": 23.5, "stage_wait_ms": 7.25,
                                     "h2d_bytes": 2048, "layer_scatter_ms": 1.5}}})])
    c = pr.load_prefill_layer_costs(p)[3]
    assert (c.gmm_ms, c.stage_wait_ms, c.h2d_bytes, c.scatter_ms) == (23.5, 7.25, 2048, 1.5)
    assert c.score_ms == 50.0 and c.waves == 2 and c.b2_calls == 1


def test_no_profile_strict_mode_and_many_files(tmp_path):
    plan = pr.plan_profile_guided_prefill_residency(num_layers=4,
                                                    default_offloaded_layer_ids=(1, 3),
                                                    layer_costs={})
    assert plan.reason == "no_prefill_profile" and plan.offloaded_layer_ids == (1, 3)
    assert plan.resident_layer_ids == (0, 2)
    bad = _write(tmp_path / "bad.jsonl", ["{oops"])
    assert pr.load_prefill_layer_costs(bad) == {}
    with pytest.raises(ValueError, match="Invalid JSON"):
        pr.load_prefill_layer_costs(bad, strict=True)
    with pytest.raises(FileNotFoundError):
        pr.load_prefill_layer_costs(tmp_path / "missing.jsonl", strict=True)
    a = _write(tmp_path / "x.jsonl", [json.dumps({"name": "b2_work_conserving_prefill",
                                                  "layer_id": 1, "seconds": 0.2})])
    b = _write(tmp_path / "y.jsonl", [json.dumps({"name": "prefill_resident_native",
                                                  "layer_id": 0, "seconds": 0.01})])
    costs = pr.load_prefill_layer_costs_many((a, b))
    assert sorted(costs) == [0, 1]


def test_autoconfig_applies_profile_guided_residency(tmp_path, monkeypatch):
    """Reference ``tests/test_autoconfig.py:664-711``: expensive offloaded layers 3 and 7 swap
    with the profiled resident layers 0 and 1; the number of offloaded layers is unchanged."""
    records = [("b2_work_conserving_prefill", 3, 100.0), ("b2_work_conserving_prefill", 7, 90.0),
               ("b2_work_conserving_prefill", 0, 10.0), ("b2_work_conserving_prefill", 1, 20.0)]
    profile = _write(tmp_path / "prefill_profile.jsonl", [
        json.dumps({"name": n, "layer_id": lid, "seconds": ms / 1e3,
                    "payload": {"control_ms": {"end_to_end": ms}}}) for n, lid, ms in records])
    defaults = ac.derive_prefetch_defaults(14)
    assert {3, 7} <= set(defaults["offloaded_layer_ids"])
    updated = ac.apply_profile_guided_residency(defaults, profile_path=profile)
    assert {3, 7} <= set(updated["resident_layer_ids"])
    assert {0, 1} <= set(updated["offloaded_layer_ids"])
    assert len(updated["offloaded_layer_ids"]) == len(defaults["offloaded_layer_ids"])
    assert updated["prefill_residency_plan"]["reason"] == "profile_guided_swaps"
    assert ac.apply_profile_guided_residency(defaults, profile_path=None) is defaults
    # the env route used by apply_moe_offload_defaults
    env = {ac.PREFILL_RESIDENCY_PROFILE_ENV: profile}
    ac.apply_moe_offload_defaults(14, env=env)
    resident = {int(x) for x in env["VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS"].split(",")}
    assert {3, 7} <= resident and not ({0, 1} & resident)


def test_recorder_writes_records_the_loader_reads(tmp_path):
    """The B200 profile source: event pairs become JSONL records of the reference schema."""

    class FakeEvent:
        def __init__(self, t):
            self.t = t

        def synchronize(self):
            pass

        def elapsed_time(self, other):
            return other.t - self.t

    path = tmp_path / "prof" / "run.jsonl"
    rec = pr.PrefillProfileRecorder(str(path))
    rec.pending.append(pr._PendingCall(5, False, FakeEvent(0.0), FakeEvent(42.5), 4096, 32768,
                                       4, 126, 10**9))
    rec.pending.append(pr._PendingCall(2, True, FakeEvent(1.0), FakeEvent(4.0), 4096, 32768,
                                       0, 0, 0))
    assert rec.flush() == 2 and rec.pending == []
    costs = pr.load_prefill_layer_costs(path)
    assert costs[5].score_ms == pytest.approx(42.5) and costs[5].b2_calls == 1
    assert costs[5].h2d_bytes == 10**9 and costs[5].waves == 4 and costs[5].active_experts == 126
    assert costs[2].resident_native_calls == 1 and costs[2].score_ms == pytest.approx(3.0)
    # a runtime with a profile path carries a recorder; the layer records prefill calls on it
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime

    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=4,
                                            profile_path=str(tmp_path / "p.jsonl")))
    assert isinstance(rt.prefill_profiler, pr.PrefillProfileRecorder)
    assert MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=4)).prefill_profiler is None
