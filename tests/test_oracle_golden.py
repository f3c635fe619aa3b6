"""Pin the CPU oracle to the reference: golden vectors made by running the reference's own
control plane (tests/golden/make_golden.py) and the vectors its unit tests hold."""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import control as oc
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return json.loads((GOLDEN / name).read_text())


def test_waves_match_reference_golden():
    for case in load("waves.json"):
        counts = {int(k): v for k, v in case["counts"].items()}
        assert [list(w) for w in oc.plan_balanced_waves(counts, case["num_slots"])] == case["waves"]


def test_reference_unit_test_wave_vectors():
    # tests/test_phase_split_b2.py:44-63, :94-118, :120-128 of the reference
    assert oc.plan_balanced_waves({1: 10, 2: 9, 3: 8, 4: 1, 5: 1}, 2) == ((1,), (2, 5), (3, 4))
    assert oc.plan_balanced_waves({1: 10, 2: 9, 3: 8, 4: 7}, 4) == ((1, 2, 3, 4),)
    assert oc.plan_balanced_waves({5: 100, 1: 90, 2: 80, 4: 70}, 4) == ((1, 2, 4, 5),)
    assert oc.plan_balanced_waves({1: 10, 2: 100, 5: 90}, 3) == ((1, 2, 5),)


def _kw(kw):
    kw = dict(kw)
    kw["h2d_bytes_by_wave"] = {int(k): v for k, v in kw["h2d_bytes_by_wave"].items()}
    kw["compute_cost_by_wave"] = {int(k): v for k, v in kw["compute_cost_by_wave"].items()}
    return kw


def test_async_schedule_and_issue_log_match_reference_golden():
    for case in load("schedules.json"):
        waves = tuple(tuple(w) for w in case["waves"])
        ready = {int(k): v for k, v in case["readiness"].items()}
        s = oc.async_schedule(waves, ready, **_kw(case["kwargs"]))
        ref = case["schedule"]
        for key in ("compute_order", "hit_wave_indices", "staged_wave_indices",
                    "staged_issue_order", "prefetch_depth", "buffer_count",
                    "initial_stage_count", "transfer_aware"):
            got = s[key]
            assert (list(got) if isinstance(got, tuple) else got) == ref[key], key
        assert [list(x) for x in oc.simulate_issue_log(s)] == case["issue_log"]


def test_slot_allocation_matches_reference_golden():
    for trace in load("slot_traces.json"):
        alloc = oc.SlotAllocator(trace["num_slots"], trace["num_experts"])
        for step in trace["steps"]:
            got = alloc.stage(tuple(step["active"]))
            assert list(got["active_slot_ids"]) == step["active_slot_ids"], trace["name"]
            assert got["log2phy"].tolist() == step["log2phy"], trace["name"]


def test_reference_unit_test_slot_vector():
    # tests/test_fixed_slot_lifecycle.py:53-61 of the reference: S=4, (0,1) then (2,3,4)
    alloc = oc.SlotAllocator(4, 5)
    alloc.stage((0, 1))
    assert alloc.stage((2, 3, 4))["active_slot_ids"] == (2, 3, 0)


def test_pair_plans_match_reference_golden():
    for case in load("pair_plans.json"):
        ids = np.asarray(case["topk_ids"])
        plans = oc.wave_pair_plans(ids, [tuple(w) for w in case["waves"]])
        for got, ref in zip(plans, case["plans"]):
            for key in ("flat_pair_offsets", "token_indices", "physical_slot_ids"):
                assert got[key].tolist() == ref[key], key


def test_reference_device_planner_vector():
    # tests/test_phase_split_b2.py:1220-1263 of the reference
    plans = oc.wave_pair_plans(np.array([[3, 1], [2, 3], [0, 2]]), ((0, 3), (1, 2)))
    assert plans[0]["physical_slot_ids"].tolist() == [1, 1, 0]
    assert plans[1]["physical_slot_ids"].tolist() == [0, 1, 1]


def test_group_pairs_equals_concatenated_wave_plans():
    """The single device grouping (waves concatenated) reproduces the per-wave compaction."""
    for case in load("pair_plans.json"):
        ids = np.asarray(case["topk_ids"])
        waves = [tuple(w) for w in case["waves"]]
        e2g = np.full(int(ids.max()) + 1, -1)
        g = 0
        for w in waves:
            for e in w:
                e2g[e] = g
                g += 1
        off, p2r, r2p = oc.group_pairs(ids, e2g, g)
        plans = oc.wave_pair_plans(ids, waves)
        g = 0
        for w, plan in zip(waves, plans):
            rows = r2p[off[g]: off[g + len(w)]]
            assert sorted(rows.tolist()) == plan["flat_pair_offsets"].tolist()
            g += len(w)
        assert np.array_equal(p2r[r2p], np.arange(r2p.size))


def test_native_combine_index_matches_reference_golden():
    for case in load("combine_index.json"):
        idx = oc.native_combine_index([w["pair_offsets"] for w in case["waves"]],
                                      [w["local"] for w in case["waves"]], case["total_pairs"])
        assert idx.tolist() == case["index"]
    # tests/test_phase_split_b2.py:1052-1104 of the reference
    assert oc.native_combine_index([[1, 3], [0, 2]], [[1, 0], [0, 1]], 4).tolist() == [2, 1, 3, 0]


def test_bf16_rounding_known_answers():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 65504.0, 3.0e38], dtype=np.float32)
    b = f32_to_bf16_bits(x)
    assert b.tolist() == [0x3F80, 0x3F80, 0x3F81, 0xC020, 0x4780, 0x7F62]
    assert np.array_equal(round_bf16(bf16_bits_to_f32(b)), bf16_bits_to_f32(b))


def test_router_renorm_and_tie_rule():
    logits = np.array([[0.0, 2.0, 2.0, -1.0, 1.0]], dtype=np.float32)
    wb, wf, ids = orouter.route(logits, 3, renormalize=True)
    assert ids.tolist() == [[1, 2, 4]]  # tie between 1 and 2: the lower id first
    assert abs(wf.sum() - 1.0) < 1e-6
    _, wf2, _ = orouter.route(logits, 3, renormalize=False, routed_scaling_factor=2.0)
    p = np.exp(logits - logits.max()) / np.exp(logits - logits.max()).sum()
    assert np.allclose(wf2, 2.0 * p[0, [1, 2, 4]], rtol=1e-6)


def test_mlp_oracle_linear_in_combine_weights():
    rng = np.random.default_rng(0)
    T, k, E, H, I = 5, 2, 4, 32, 16
    w13 = f32_to_bf16_bits(rng.standard_normal((E, 2 * I, H)).astype(np.float32) * 0.1)
    w2 = f32_to_bf16_bits(rng.standard_normal((E, H, I)).astype(np.float32) * 0.1)
    hid = f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    ids = np.array([rng.permutation(E)[:k] for _ in range(T)])
    y = omlp.pair_outputs(hid, ids, w13, w2)
    # the union over disjoint expert subsets equals the full pass (wave keystone)
    ya = omlp.pair_outputs(hid, ids, w13, w2, experts=[0, 1])
    yb = omlp.pair_outputs(hid, ids, w13, w2, experts=[2, 3])
    assert np.array_equal(ya + yb, y)
    ones = f32_to_bf16_bits(np.ones((T, k), dtype=np.float32))
    out = omlp.combine(y, ones)
    assert np.allclose(out, round_bf16(y.reshape(T, k, H).sum(1)), atol=1e-2)


def test_native_combine_index_fails_closed_on_missing_or_duplicate_pairs():
    """The one combine must see every original top-k pair exactly once (reference
    ``tests/test_phase_split_b2.py:1106``): a missing or repeated pair is refused."""
    with pytest.raises(ValueError, match="exactly once"):
        oc.native_combine_index([[1, 3], [0]], [[1, 0], [0]], 4)  # pair 2 missing
    with pytest.raises(ValueError, match="exactly once"):
        oc.native_combine_index([[1, 3], [0, 1]], [[1, 0], [0, 1]], 4)  # pair 1 twice
    with pytest.raises(ValueError, match="pair count"):
        oc.native_combine_index([[1, 3]], [[0]], 2)


def test_router_oracle_agrees_with_vllm_torch_router():
    """Third-party cross-check of the routing semantics the oracle restates (the reference's
    own router lives in the un-vendored fork): vLLM's torch ``grouped_topk`` selects the same
    expert sets with the same weights for plain softmax + renormalise (Qwen3-MoE), softmax
    without renormalisation (DeepSeek-V2-Lite, one group) and grouped sigmoid + correction
    bias + scaling (group-limited routing). vLLM does not order the selected experts, so each
    token's (id, weight) pairs are compared sorted by id."""
    mod = pytest.importorskip("vllm.model_executor.layers.fused_moe.router.grouped_topk_router")
    grouped_topk = getattr(mod.grouped_topk, "__wrapped__", mod.grouped_topk)
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    cases = [
        dict(E=128, k=8, renorm=True, scoring="softmax", groups=1, topk_group=1, scale=1.0, bias=False),
        dict(E=64, k=6, renorm=False, scoring="softmax", groups=1, topk_group=1, scale=1.0, bias=False),
        dict(E=256, k=8, renorm=True, scoring="sigmoid", groups=8, topk_group=4, scale=2.5, bias=True),
    ]
    for c in cases:
        logits = rng.standard_normal((64, c["E"])).astype(np.float32)
        bias = rng.standard_normal(c["E"]).astype(np.float32) * 0.1 if c["bias"] else None
        _, w, ids = orouter.route(logits, c["k"], renormalize=c["renorm"],
                                  routed_scaling_factor=c["scale"], scoring_func=c["scoring"],
                                  e_score_correction_bias=bias, num_expert_group=c["groups"],
                                  topk_group=c["topk_group"])
        vw, vids = grouped_topk(torch.zeros(64, 8), torch.from_numpy(logits), c["k"], c["renorm"],
                                num_expert_group=c["groups"], topk_group=c["topk_group"],
                                scoring_func=c["scoring"], routed_scaling_factor=c["scale"],
                                e_score_correction_bias=None if bias is None else torch.from_numpy(bias))
        vw, vids = vw.float().numpy(), vids.numpy()
        for t in range(64):
            a, b = np.argsort(ids[t]), np.argsort(vids[t])
            assert ids[t][a].tolist() == vids[t][b].tolist(), (c, t)
            np.testing.assert_allclose(w[t][a], vw[t][b], rtol=1e-5, atol=1e-7)
