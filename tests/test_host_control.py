"""Host logic of the product (planners, slot bank, runtime staging order) against the
reference's golden vectors, with the slot bank on the CPU as in the reference's tests."""

import json
from pathlib import Path

import pytest
import torch

from tests.helpers import ExpertLayer
from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
from vllm_ascend_hust_latchmoe_b200.moe_offload import phase_split as ps
from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime
from vllm_ascend_hust_latchmoe_b200.moe_offload.slot_bank import SlotState

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return json.loads((GOLDEN / name).read_text())


def test_plan_balanced_b2_waves_golden():
    for case in load("waves.json"):
        counts = {int(k): v for k, v in case["counts"].items()}
        plan = ps.plan_balanced_b2_waves(counts, case["num_slots"], slot_readiness={1: True})
        assert [list(w) for w in plan.waves] == case["waves"]


def test_async_schedule_golden():
    for case in load("schedules.json"):
        kw = dict(case["kwargs"])
        kw["h2d_bytes_by_wave"] = {int(k): v for k, v in kw["h2d_bytes_by_wave"].items()}
        kw["compute_cost_by_wave"] = {int(k): v for k, v in kw["compute_cost_by_wave"].items()}
        waves = tuple(tuple(w) for w in case["waves"])
        sched = ps.plan_b2_prefill_async_schedule(
            waves, slot_readiness={int(k): v for k, v in case["readiness"].items()}, **kw)
        assert sched.to_jsonable() == case["schedule"]
        assert [list(x) for x in ps.simulate_b2_prefill_issue_log(sched)] == case["issue_log"]


def _runtime(E, S):
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=S, async_load=False,
                                            graph_compatible_offload=True))
    layer = ExpertLayer(3, torch.zeros(E, 2, 3), torch.zeros(E, 3, 2))
    rt.register_layer_for_fixed_slots(layer, slot_device=torch.device("cpu"))
    return rt


def test_runtime_slot_traces_golden():
    for trace in load("slot_traces.json"):
        rt = _runtime(trace["num_experts"], trace["num_slots"])
        for step in trace["steps"]:
            prepared = rt.stage_fixed_slot_plan(layer_id=3, active_experts=tuple(step["active"]),
                                                num_logical_experts=trace["num_experts"])
            assert list(prepared.mapping.active_slot_ids) == step["active_slot_ids"], trace["name"]
            assert rt.log2phy_buffer(3).tolist() == step["log2phy"], trace["name"]


def test_stage_copies_expert_rows_into_slots():
    E = 6
    w13 = torch.arange(E * 2 * 3, dtype=torch.float32).reshape(E, 2, 3)
    w2 = -torch.arange(E * 3 * 2, dtype=torch.float32).reshape(E, 3, 2)
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=3))
    rt.register_layer_for_fixed_slots(ExpertLayer(1, w13, w2), slot_device=torch.device("cpu"))
    p = rt.stage_fixed_slot_plan(layer_id=1, active_experts=(4, 1), num_logical_experts=E)
    for e, s in zip(p.mapping.active_experts, p.mapping.active_slot_ids):
        assert torch.equal(p.w1[s], w13[e]) and torch.equal(p.w2[s], w2[e])


def test_compute_protected_eviction_and_lease_checks():
    rt = _runtime(8, 2)
    p = rt.stage_fixed_slot_plan(layer_id=3, active_experts=(0, 1), num_logical_experts=8)
    handle = rt.begin_slot_compute(p)
    bank = rt.slot_bank(3)
    assert all(s.state == SlotState.COMPUTING for s in bank.slots)
    rt.end_slot_compute(handle)  # CPU bank: completion is immediate
    assert all(s.state == SlotState.READY for s in bank.slots)
    p2 = rt.stage_fixed_slot_plan(layer_id=3, active_experts=(2,), num_logical_experts=8)
    assert p2.mapping.active_slot_ids == (0,)  # LRU tie -> lowest slot id
    with pytest.raises(RuntimeError, match="exceeds num_slots"):
        rt.stage_fixed_slot_plan(layer_id=3, active_experts=(3, 4, 5), num_logical_experts=8)
    with pytest.raises(ValueError):
        rt.stage_fixed_slot_plan(layer_id=3, active_experts=(9,), num_logical_experts=8)


def test_address_lock_rejects_reregistration():
    rt = _runtime(8, 2)
    assert rt.capture_safe_slot_weights(layer_id=3) is not None
    with pytest.raises(RuntimeError, match="already captured"):
        rt.register_layer_for_fixed_slots(ExpertLayer(3, torch.zeros(8, 2, 3), torch.zeros(8, 3, 2)),
                                          slot_device=torch.device("cpu"))


def test_pinned_shared_suffix_and_log2phy():
    w13 = torch.randn(6, 2, 3)
    w2 = torch.randn(6, 3, 2)
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2))
    rt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2, shared=2), slot_device=torch.device("cpu"))
    bank = rt.slot_bank(0)
    assert bank.physical_expert_count == 4 and bank.pinned_slot_ids == (2, 3)
    assert rt.log2phy_buffer(0).tolist() == [-1, -1, -1, -1, 2, 3]
    assert torch.equal(bank.w13_slots[2:], w13[4:])
    p = rt.stage_fixed_slot_plan(layer_id=0, active_experts=(3,), num_logical_experts=4)
    assert p.mapping.slot_to_expert == (3, None, 4, 5)


def test_prefill_stage_plan_positional_slots_and_d2d_hits():
    E = 8
    w13 = torch.arange(E * 2 * 3, dtype=torch.float32).reshape(E, 2, 3)
    w2 = torch.arange(E * 3 * 2, dtype=torch.float32).reshape(E, 3, 2)
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=3, b2_wave_prefill=True))
    rt.register_layer_for_fixed_slots(ExpertLayer(2, w13, w2), slot_device=torch.device("cpu"))
    rt.stage_fixed_slot_plan(layer_id=2, active_experts=(5,), num_logical_experts=E)
    stage, ready = rt.prepare_prefill_stage_plan(layer_id=2, active_experts=(1, 5, 7), buffer_index=1)
    rt.wait_prefill_stage_plan(ready)
    for pos, e in enumerate((1, 5, 7)):
        assert torch.equal(stage.w13_slots[pos], w13[e])
        assert stage.slots[pos].state == SlotState.READY
    with pytest.raises(ValueError):
        rt.prefill_stage_bank(2, 5)


def test_should_use_b2_pair_waves_gate():
    rt = _runtime(8, 2)
    assert not rt.should_use_b2_pair_waves(layer_id=3, active_expert_count=5)
    rt2 = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2, b2_wave_prefill=True))
    rt2.register_layer_for_fixed_slots(ExpertLayer(3, torch.zeros(8, 2, 3), torch.zeros(8, 3, 2)),
                                       slot_device=torch.device("cpu"))
    assert rt2.should_use_b2_pair_waves(layer_id=3, active_expert_count=3)
    assert not rt2.should_use_b2_pair_waves(layer_id=3, active_expert_count=2)


def test_tiled_layout_round_trip_and_tile_contiguity():
    from vllm_ascend_hust_latchmoe_b200.weight_layout import from_tiled, to_tiled

    w = torch.arange(2 * 256 * 128, dtype=torch.float32).reshape(2, 256, 128)
    t = to_tiled(w)
    assert t.shape == w.shape and torch.equal(from_tiled(t), w)
    flat = t.reshape(2, -1)
    # tile (n-tile 1, k-block 1) of expert 1 is one contiguous 128 x 64 block
    tile = flat[1, (1 * 2 + 1) * 8192:(1 * 2 + 2) * 8192].reshape(128, 64)
    assert torch.equal(tile, w[1, 128:256, 64:128])


def test_full_layer_prefill_plan_on_cpu_bank():
    """Full-layer fallback bank: row e holds expert e, one bank per layout reused across
    layers, payload fields, memory ledger accounting."""
    from tests.helpers import ExpertLayer
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime

    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2, b2_wave_prefill=True))
    layers = []
    for lid in (0, 1):
        w13 = torch.arange(5 * 4 * 3, dtype=torch.float32).reshape(5, 4, 3) + 100 * lid
        w2 = torch.arange(5 * 3 * 2, dtype=torch.float32).reshape(5, 3, 2) - 100 * lid
        rt.register_layer_for_fixed_slots(ExpertLayer(lid, w13, w2), slot_device=torch.device("cpu"))
        layers.append((w13, w2))
    bank0, ready0, pay0 = rt.prepare_full_layer_prefill_plan(layer_id=0)
    assert pay0["execution_mode"] == "reference_full_layer" and not pay0["pool_reused"]
    assert pay0["routed_expert_count"] == 5 and ready0.event is None
    assert torch.equal(bank0.w13_slots[:5], layers[0][0]) and torch.equal(bank0.w2_slots[:5], layers[0][1])
    rt.wait_prefill_stage_plan(ready0)  # the consumer's wait publishes the rows READY
    ledger_before = rt.memory_ledger().stage_bank_bytes
    bank1, _, pay1 = rt.prepare_full_layer_prefill_plan(layer_id=1)
    assert bank1 is bank0 and pay1["pool_reused"]
    assert torch.equal(bank1.w13_slots[:5], layers[1][0])
    assert rt.memory_ledger().stage_bank_bytes == ledger_before > 0


def test_wave_plan_qualification_raises_fallback(monkeypatch):
    from types import SimpleNamespace

    from vllm_ascend_hust_latchmoe_b200 import layer as L
    from vllm_ascend_hust_latchmoe_b200.moe_offload.phase_split import B2WaveFallback, B2WavePlan

    stub = SimpleNamespace(runtime=SimpleNamespace(config=SimpleNamespace(num_slots=2)))
    plan = L.SlotBankMoE.plan_waves_checked(stub, (3, 0, 1, 2, 5))
    assert sorted(e for w in plan.waves for e in w) == [0, 2, 3, 4]
    monkeypatch.setattr(L, "plan_balanced_b2_waves",
                        lambda counts, s: B2WavePlan(((0, 2, 3),), dict(counts)))
    try:
        L.SlotBankMoE.plan_waves_checked(stub, (3, 0, 1, 2, 5))
    except B2WaveFallback as exc:
        assert "exactly once" in str(exc)
    else:
        raise AssertionError("expected B2WaveFallback")

    def bad(counts, s):
        raise ValueError("no plan")

    monkeypatch.setattr(L, "plan_balanced_b2_waves", bad)
    try:
        L.SlotBankMoE.plan_waves_checked(stub, (1, 1))
    except B2WaveFallback as exc:
        assert "wave planning failed" in str(exc)
    else:
        raise AssertionError("expected B2WaveFallback")


def test_release_original_expert_weights_after_the_store_holds_them():
    """Opt-in release (the reference's ``release_original_expert_weights_if_ready``): only a
    non-resident layer whose store holds the experts; staging still reads the store."""
    E = 6
    w13 = torch.arange(E * 2 * 3, dtype=torch.float32).reshape(E, 2, 3)
    w2 = torch.arange(E * 3 * 2, dtype=torch.float32).reshape(E, 3, 2)

    def layer(lid):
        return ExpertLayer(lid, torch.nn.Parameter(w13.clone(), requires_grad=False),
                           torch.nn.Parameter(w2.clone(), requires_grad=False))

    off = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2))
    l0 = layer(0)
    off.register_layer_for_fixed_slots(l0, slot_device=torch.device("cpu"))
    assert off.release_original_expert_weights_if_ready(l0) == (
        False, ("release_original_expert_weights_disabled",))
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2,
                                            release_original_expert_weights=True,
                                            resident_layer_ids=frozenset({1})))
    assert rt.release_original_expert_weights_if_ready(layer(4)) == (
        False, ("host_store_missing:4",))
    l0, l1 = layer(0), layer(1)
    for lay in (l0, l1):
        rt.register_layer_for_fixed_slots(lay, slot_device=torch.device("cpu"))
    assert rt.release_original_expert_weights_if_ready(l1) == (False, ("resident_layer:1",))
    assert rt.release_original_expert_weights_if_ready(l0) == (True, ())
    assert rt.release_original_expert_weights_if_ready(l0) == (True, ())  # idempotent
    assert rt.released_original_weight_layers == (0,)
    assert tuple(l0.w13_weight.shape) == (0, 2, 3) and tuple(l0.w2_weight.shape) == (0, 3, 2)
    assert tuple(l1.w13_weight.shape) == (E, 2, 3)
    p = rt.stage_fixed_slot_plan(layer_id=0, active_experts=(4, 1), num_logical_experts=E)
    for e, s in zip(p.mapping.active_experts, p.mapping.active_slot_ids):
        assert torch.equal(p.w1[s], w13[e]) and torch.equal(p.w2[s], w2[e])


def test_stage_fixed_slot_plan_rolls_back_a_failed_load(monkeypatch):
    """A failed copy enqueue leaves every newly assigned slot EMPTY, unmapped, and log2phy
    unpublished (reference ``tests/test_prefill_stage_runtime.py:1225-1283``)."""
    from vllm_ascend_hust_latchmoe_b200.moe_offload.expert_key import ExpertKey

    E = 4
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2, async_load=True,
                                            graph_compatible_offload=True))
    rt.register_layer_for_fixed_slots(ExpertLayer(7, torch.zeros(E, 2, 3), torch.zeros(E, 3, 2)),
                                      slot_device=torch.device("cpu"))

    def fail(*args, **kwargs):
        raise RuntimeError("enqueue failed")

    monkeypatch.setattr(rt._transfer_engine, "load_many_async", fail)
    with pytest.raises(RuntimeError, match="enqueue failed"):
        rt.stage_fixed_slot_plan(layer_id=7, active_experts=(0, 1), num_logical_experts=E)
    bank = rt.slot_bank(7)
    assert all(slot.state == SlotState.EMPTY for slot in bank.slots)
    assert bank.lookup(ExpertKey(7, 0)) is None and bank.lookup(ExpertKey(7, 1)) is None
    assert rt.log2phy_buffer(7).tolist() == [-1] * E
    monkeypatch.undo()
    p = rt.stage_fixed_slot_plan(layer_id=7, active_experts=(0, 1), num_logical_experts=E)
    assert p.mapping.active_slot_ids == (0, 1)  # the slots are reusable after the rollback


def test_log2phy_updates_only_changed_active_entries(monkeypatch):
    """Only active experts whose slot changed are rewritten; an evicted expert's stale entry
    stays (it is never routed), and a hit-only stage enqueues no copy (reference
    ``tests/test_prefill_stage_runtime.py:1782-1900``)."""
    E = 4
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=3, async_load=True,
                                            graph_compatible_offload=True))
    rt.register_layer_for_fixed_slots(ExpertLayer(7, torch.zeros(E, 2, 3), torch.zeros(E, 3, 2)),
                                      slot_device=torch.device("cpu"))
    rt.stage_fixed_slot_plan(layer_id=7, active_experts=(0, 1, 2), num_logical_experts=E)
    before = rt.stage_stats["log2phy_updates"]
    p = rt.stage_fixed_slot_plan(layer_id=7, active_experts=(1, 3), num_logical_experts=E)
    assert rt.stage_stats["log2phy_updates"] - before == 1  # only expert 3 -> slot 0
    assert rt.log2phy_buffer(7).tolist() == [0, 1, 2, 0]  # expert 0's entry is stale
    assert p.mapping.active_experts == (1, 3) and p.mapping.active_slot_ids == (1, 0)

    def no_copy(*args, **kwargs):
        raise AssertionError("a hit-only stage must not enqueue a copy")

    monkeypatch.setattr(rt._transfer_engine, "load_many_async", no_copy)
    before = rt.stage_stats["log2phy_updates"]
    rt.stage_fixed_slot_plan(layer_id=7, active_experts=(1, 3), num_logical_experts=E)
    assert rt.stage_stats["log2phy_updates"] == before
    assert rt.log2phy_buffer(7).tolist() == [0, 1, 2, 0]


def test_transfer_ready_event_publishes_after_the_consumer_wait_and_rejects_stale_leases():
    """A slot becomes READY only once the consumer stream waits on the copy event, and a
    completion whose slot was reassigned meanwhile is rejected before any stream hand-off
    (reference ``tests/test_prefill_stage_runtime.py:85-157``)."""
    from vllm_ascend_hust_latchmoe_b200.moe_offload.expert_key import ExpertKey
    from vllm_ascend_hust_latchmoe_b200.moe_offload.slot_bank import ExpertSlotBank
    from vllm_ascend_hust_latchmoe_b200.moe_offload.transfer_engine import TransferReadyEvent

    bank = ExpertSlotBank(1, (1, 1), (1, 1), dtype=torch.float32, device=torch.device("cpu"))
    slot = bank.allocate_for(ExpertKey(7, 0), step_id=1)
    event = object()
    ready = TransferReadyEvent(event, ((slot, slot.lease()),))
    calls = []

    class Consumer:
        def wait_event(self, observed):
            assert observed is event and slot.state == SlotState.LOADING
            assert not ready.completed
            calls.append("wait")

    ready.install_consumer_dependency(Consumer())
    assert calls == ["wait"] and ready.consumer_wait_installed and ready.completed
    assert slot.state == SlotState.READY
    ready.mark_ready()  # idempotent

    bank2 = ExpertSlotBank(1, (1, 1), (1, 1), dtype=torch.float32, device=torch.device("cpu"))
    s2 = bank2.allocate_for(ExpertKey(7, 0), step_id=1)
    stale = TransferReadyEvent(object(), ((s2, s2.lease()),))
    bank2.clear_slot(0, force=True)  # a rolled-back load; the slot is then reassigned
    replacement = bank2.allocate_for(ExpertKey(7, 1), step_id=2)

    class NoHandOff:
        def wait_event(self, _):
            raise AssertionError("a stale completion must fail before the stream hand-off")

    with pytest.raises(RuntimeError, match="stale H2D completion"):
        stale.install_consumer_dependency(NoHandOff())
    assert replacement.state == SlotState.LOADING


def test_prefill_stage_pool_double_buffers_and_sharing_across_equal_layouts():
    """Two stage buffers never share storage; equal-layout layers share one pool and its
    release events (reference ``tests/test_prefill_stage_runtime.py:566-658``)."""
    E = 4
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=2))
    for lid in (7, 9):
        rt.register_layer_for_fixed_slots(
            ExpertLayer(lid, torch.arange(E * 6, dtype=torch.float32).reshape(E, 2, 3),
                        torch.arange(E * 6, dtype=torch.float32).reshape(E, 3, 2)),
            slot_device=torch.device("cpu"))
    first, r0 = rt.prepare_prefill_stage_plan(layer_id=7, active_experts=(0, 1), buffer_index=0)
    second, r1 = rt.prepare_prefill_stage_plan(layer_id=7, active_experts=(2, 3), buffer_index=1)
    assert first.w13_slots.data_ptr() != second.w13_slots.data_ptr()
    assert first.w2_slots.data_ptr() != second.w2_slots.data_ptr()
    with pytest.raises(RuntimeError, match="cannot be reassigned"):  # still loading
        rt.prepare_prefill_stage_plan(layer_id=9, active_experts=(3,), buffer_index=0)
    rt.wait_prefill_stage_plan(r0)
    other, _ = rt.prepare_prefill_stage_plan(layer_id=9, active_experts=(3,), buffer_index=0)
    assert other.w13_slots.data_ptr() == first.w13_slots.data_ptr()  # shared pool
    event = object()
    rt.remember_prefill_stage_buffer_release(7, 1, event)
    assert rt.prefill_stage_buffer_release_event(9, 1) is event
    with pytest.raises(ValueError, match="out of range"):
        rt.prefill_stage_bank(7, 2)
    rt.wait_prefill_stage_plan(r1)
    assert torch.equal(second.w13_slots[0], torch.arange(12, 18, dtype=torch.float32).reshape(2, 3))


def test_host_remap_fails_closed_on_an_unstaged_expert():
    """A routed expert whose log2phy entry is -1 is refused, never read from a wrong slot
    (reference ``tests/test_prefill_stage_runtime.py:2098-2111``; on the device the same
    check sets the error word inside lm_build_groups)."""
    from vllm_ascend_hust_latchmoe_b200.moe_offload.slot_mapping import ExpertSlotMapping

    m = ExpertSlotMapping(7, (1, 2), torch.tensor([-1, 0, 1, -1], dtype=torch.int32),
                          (1, 2, None, None), (0, 1))
    assert m.remap_topk_ids_host(torch.tensor([[1, 2]])).tolist() == [[0, 1]]
    assert m.physical_slot_for(2) == 1
    with pytest.raises(RuntimeError, match="not staged"):
        m.remap_topk_ids_host(torch.tensor([[2, 3]]))
    with pytest.raises(KeyError):
        m.physical_slot_for(3)


def test_slot_piece_replay_detection_follows_vllm_graph_mode(monkeypatch):
    """The overflow guard applies to token counts with a captured slot-bank MLP piece, unless
    vLLM runs the forward pass eagerly (cudagraph mode NONE)."""
    import types

    from vllm_ascend_hust_latchmoe_b200 import layer as layer_mod

    fake = types.SimpleNamespace(captured_mlp_tokens={4})
    replays = layer_mod.SlotBankMoE._slot_piece_replays
    monkeypatch.setattr(layer_mod, "_vllm_cudagraph_mode", lambda: None)
    assert replays(fake, 4) and not replays(fake, 5)
    monkeypatch.setattr(layer_mod, "_vllm_cudagraph_mode", lambda: "PIECEWISE")
    assert replays(fake, 4)
    monkeypatch.setattr(layer_mod, "_vllm_cudagraph_mode", lambda: "NONE")
    assert not replays(fake, 4)
