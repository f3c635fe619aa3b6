"""GPU parity of the whole slot-bank MoE layer (router -> stage -> MLP -> combine).

Routing ids and the slot assignment are bit-exact against the oracle (the slot allocator
oracle is pinned to the reference's own control plane); layer outputs are within the bf16
tolerance of the fp32-accumulating oracle.
"""

import numpy as np
import pytest
import torch

from oracle import control as ocontrol
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits, build_layer
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _oracle_layer(cfg, hidden, logits, w13, w2):
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=cfg.renormalize,
                               routed_scaling_factor=cfg.routed_scaling_factor,
                               scoring_func=cfg.scoring_func,
                               num_expert_group=cfg.num_expert_group, topk_group=cfg.topk_group)
    out = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
    return ids, wb, out


def _check(out, ref):
    m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m


def test_decode_slots_path_matches_oracle_and_slot_order(cuda):
    """Batch-8 decode steps (working set <= S): slots staged in sorted order, LRU reuse."""
    cfg = syn.CONFIGS["c1_decode"].with_tokens(4)
    layer, rt, (w13, w2) = build_layer(cfg, max_tokens=4)
    alloc = ocontrol.SlotAllocator(cfg.num_slots, cfg.num_experts)
    for step in range(6):
        hidden = syn.make_hidden(cfg, seed=step)
        logits = syn.make_router_logits(cfg, seed=step)
        ids_ref, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
        out = layer.forward(hidden.to(cuda), logits.to(cuda))
        torch.cuda.synchronize()
        layer.check_device_errors()
        assert np.array_equal(layer.topk_ids[:4].cpu().numpy(), ids_ref)
        exp = alloc.stage(tuple(sorted(set(ids_ref.reshape(-1).tolist()))))
        assert np.array_equal(rt.log2phy_buffer(0).cpu().numpy(), exp["log2phy"])
        _check(out, ref)


@pytest.mark.parametrize("store_on_device", [False, True])
def test_c1_decode_overflow_runs_waves(cuda, store_on_device):
    """C1: 16 tokens route to more experts than the 32 slots -> multi-wave + one combine."""
    cfg = syn.CONFIGS["c1_decode"]
    layer, rt, (w13, w2) = build_layer(cfg, store_on_device=store_on_device)
    hidden = syn.make_hidden(cfg)
    logits = syn.make_router_logits(cfg)
    ids_ref, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    assert np.array_equal(layer.topk_ids[:16].cpu().numpy(), ids_ref)
    counts = np.bincount(ids_ref.reshape(-1), minlength=cfg.num_experts)
    waves = ocontrol.plan_balanced_waves({e: int(c) for e, c in enumerate(counts)}, cfg.num_slots)
    if store_on_device:
        # HBM-resident tier: nothing is staged, a decode call groups by expert id
        assert layer.resident_wave_plan() == ()
    else:
        assert layer.last_waves.waves == waves and len(waves) >= 2
    _check(out, ref)


@pytest.mark.parametrize("store_on_device", [False, True])
def test_prefill_waves_tcgen05_matches_oracle(cuda, store_on_device):
    """C2-shaped multi-wave prefill on a 1024-token slice (>= 4 waves, one combine)."""
    cfg = syn.CONFIGS["c2_prefill"].with_tokens(1024)
    layer, rt, (w13, w2) = build_layer(cfg, store_on_device=store_on_device)
    layer.resident_wave_order = True  # the resident tier orders its groups by the plan
    hidden = syn.make_hidden(cfg)
    logits = syn.make_router_logits(cfg)
    ids_ref, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    waves = layer.resident_wave_plan() if store_on_device else layer.last_waves.waves
    assert len(waves) >= 4
    _check(out, ref)
    # Second call reuses every buffer and stage bank: same result.
    out2 = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_c4_deepseek_shaped_layer(cuda):
    cfg = syn.CONFIGS["c4_shared"]
    layer, rt, (w13, w2) = build_layer(cfg)
    hidden = syn.make_hidden(cfg)
    logits = syn.make_router_logits(cfg)
    ids_ref, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    assert np.array_equal(layer.topk_ids[:64].cpu().numpy(), ids_ref)
    _check(out, ref)


@pytest.mark.parametrize("tokens", [16, 1024])
def test_full_layer_reference_path(cuda, tokens):
    """VLLM_ASCEND_MOE_OFFLOAD_B2_REFERENCE_FULL_LAYER: every routed expert staged into the
    layout's full-layer bank, one MLP pass in the native top-k shape (decode and prefill)."""
    cfg = syn.CONFIGS["c2_prefill"].with_tokens(tokens)
    layer, rt, (w13, w2) = build_layer(cfg, reference_full_layer=True)
    hidden = syn.make_hidden(cfg)
    logits = syn.make_router_logits(cfg)
    _, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    assert layer.last_full_layer["execution_mode"] == "reference_full_layer"
    assert layer.last_full_layer["routed_expert_count"] == cfg.num_experts
    _check(out, ref)
    out2 = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    assert layer.last_full_layer["pool_reused"] and torch.equal(out, out2)


def test_wave_fallback_reruns_full_layer(cuda, monkeypatch):
    """A wave plan that fails qualification (B2WaveFallback before any wave runs) reruns the
    layer on the full-layer path with the same result."""
    from vllm_ascend_hust_latchmoe_b200.moe_offload import phase_split

    cfg = syn.CONFIGS["c2_prefill"].with_tokens(512)
    layer, rt, (w13, w2) = build_layer(cfg)
    hidden = syn.make_hidden(cfg)
    logits = syn.make_router_logits(cfg)
    _, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
    good = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    assert layer.last_fallback_reason is None
    real = phase_split.plan_balanced_b2_waves

    def drop_last_expert(counts, num_slots):  # a plan that misses an active expert
        plan = real(counts, num_slots)
        return phase_split.B2WavePlan(plan.waves[:-1] + (plan.waves[-1][:-1],),
                                      plan.token_counts_by_expert)

    monkeypatch.setattr("vllm_ascend_hust_latchmoe_b200.layer.plan_balanced_b2_waves",
                        drop_last_expert)
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    assert layer.last_fallback_reason is not None and "exactly once" in layer.last_fallback_reason
    assert layer.last_full_layer is not None
    _check(out, ref)
    m = omlp.compare(bf16_bits_to_f32(bits(out)), bf16_bits_to_f32(bits(good)))
    assert m["max_rel_err"] <= MAX_REL_ERR, m


def test_overflow_at_a_captured_size_fails_closed(cuda):
    """A slot-bank MLP piece captured at T tokens is replayed for every later T-token call,
    reading log2phy for all routed experts. When a later T-token stage call finds more active
    experts than slots it must raise (an evicted expert's stale log2phy entry would silently
    select another expert's weights), while an uncaptured size still runs its waves."""
    cfg = syn.CONFIGS["c1_decode"].with_tokens(4)
    layer, rt, (w13, w2) = build_layer(cfg, max_tokens=16, num_slots=8)
    E = cfg.num_experts
    narrow = torch.full((4, E), -5.0)
    narrow[:, :8] = torch.arange(8, 0, -1, dtype=torch.float32)  # every token: experts 0..7
    hidden4 = syn.make_hidden(cfg, seed=1).to(cuda)
    layer.forward(hidden4, narrow.to(cuda))  # 8 active experts: fits the 8 slots
    torch.cuda.synchronize()
    assert layer.stage(layer.topk_ids[:4]).mode == "slots"
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.mlp_slots(hidden4, 4)
    assert 4 in layer.captured_mlp_tokens
    wide = syn.make_router_logits(cfg, seed=2)  # 4 tokens x top-8 over many experts
    _, ids = layer.route(hidden4, wide.to(cuda))
    torch.cuda.synchronize()
    assert len(set(ids.cpu().reshape(-1).tolist())) > 8
    with pytest.raises(RuntimeError, match="replayed from a CUDA graph"):
        layer.stage(ids)
    # an uncaptured size overflows into waves as usual, with the oracle's result
    cfg5 = cfg.with_tokens(5)
    hidden5 = syn.make_hidden(cfg5, seed=3)
    logits5 = syn.make_router_logits(cfg5, seed=3)
    _, _, ref = _oracle_layer(cfg5, hidden5, logits5, w13, w2)
    out = layer.forward(hidden5.to(cuda), logits5.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    assert len(layer.last_waves.waves) >= 2
    _check(out, ref)
    del g


def test_prefill_profile_drives_residency(cuda, tmp_path):
    """Prefill calls of an offloaded layer (staged waves) and of a resident layer are recorded
    as profile records (CUDA events, read back on flush); the planner then makes the costlier
    offloaded layer resident in exchange for the cheaper resident one."""
    from vllm_ascend_hust_latchmoe_b200.moe_offload import prefill_residency as pr

    cfg = syn.CONFIGS["c2_prefill"].with_tokens(512)
    path = tmp_path / "prefill.jsonl"
    hidden = syn.make_hidden(cfg).to(cuda)
    logits = syn.make_router_logits(cfg).to(cuda)
    for lid, on_dev in ((1, False), (0, True)):
        layer, rt, _ = build_layer(cfg, store_on_device=on_dev, layer_id=lid)
        rt.prefill_profiler = pr.PrefillProfileRecorder(str(path))
        for _ in range(2):
            layer.forward(hidden, logits)
        torch.cuda.synchronize()
        layer.check_device_errors()
        assert rt.prefill_profiler.flush() == 2
    costs = pr.load_prefill_layer_costs(path)
    assert costs[1].b2_calls == 2 and costs[1].waves >= 4 and costs[1].h2d_bytes > 0
    assert costs[0].resident_native_calls == 2
    plan = pr.plan_profile_guided_prefill_residency(num_layers=2, default_offloaded_layer_ids=(1,),
                                                    layer_costs=costs)
    assert plan.reason == "profile_guided_swaps" and plan.offloaded_layer_ids == (0,)


def test_waves_reuse_main_bank_slots_device_to_device(cuda):
    """A staged layer whose main slot bank already holds some of a wave's experts (an earlier
    call fitted its slots) copies them device to device into the stage bank and stages the rest
    from the pinned store: the outputs of the slot call and of the wave call both match the
    oracle, and a slot call after the waves still does."""
    cfg = syn.LayerConfig("mix", hidden=256, num_experts=16, top_k=2, intermediate=128,
                          num_slots=8, tokens=128)
    layer, rt, (w13, w2) = build_layer(cfg)
    hidden = syn.make_hidden(cfg, seed=3)
    base = syn.make_router_logits(cfg, seed=3)
    for n_active in (6, 12, 6, 14):
        logits = base.clone()
        logits[:, n_active:] -= 100.0  # route among the first n_active experts only
        ids_ref, _, ref = _oracle_layer(cfg, hidden, logits, w13, w2)
        out = layer.forward(hidden.to(cuda), logits.to(cuda))
        torch.cuda.synchronize()
        layer.check_device_errors(f"mixed slots / waves, {n_active} experts")
        assert np.array_equal(layer.topk_ids[: cfg.tokens].cpu().numpy(), ids_ref)
        _check(out, ref)
