"""Plugin surface on CPU: register(), seam op schemas, env contract, capability descriptor
and AutoConfig (pinned to outputs of the reference's own AutoConfig)."""

import json
import os
from pathlib import Path

import pytest
import torch

import vllm_ascend_hust_latchmoe_b200 as plugin
from vllm_ascend_hust_latchmoe_b200 import autoconfig as ac
from vllm_ascend_hust_latchmoe_b200 import capabilities as cap
from vllm_ascend_hust_latchmoe_b200 import env_registry, seam_ops

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_register_is_idempotent_and_defines_the_seam_ops():
    plugin.register()
    plugin.register()
    for name, schema in seam_ops.OP_SCHEMAS.items():
        op = getattr(torch.ops.vllm, name)
        assert str(op.default._schema).startswith(f"vllm::{name}(")
    stage = torch.ops.vllm.moe_offload_stage.default._schema
    assert stage.arguments[0].alias_info is not None and stage.arguments[0].alias_info.is_write
    assert len(stage.returns) == 0


def test_fake_impls_give_shapes_without_a_device():
    from torch._subclasses.fake_tensor import FakeTensorMode

    plugin.register()
    with FakeTensorMode():
        h = torch.empty(5, 64, dtype=torch.bfloat16)
        lg = torch.empty(5, 8)
        w, ids = torch.ops.vllm.moe_router(h, lg, 2, False, True, None, None, "softmax", 1.0,
                                           None, 8)
        assert tuple(w.shape) == (5, 2) and ids.dtype == torch.int32
        out = torch.ops.vllm.moe_mlp(h, lg, w, ids, None, None, "missing", -1)
        assert tuple(out.shape) == (5, 64)


def test_env_contract_names_and_defaults(monkeypatch):
    assert len(env_registry.ENVIRONMENT_VARIABLES) == 59
    monkeypatch.delenv("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT", raising=False)
    assert env_registry.get("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT") == 2
    monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD", "yes")
    assert env_registry.get("VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD") is True
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig

    monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS", "32")
    monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS", "0, 1,2")
    cfg = MoeOffloadConfig.from_env()
    assert cfg.num_slots == 32 and cfg.resident_layer_ids == frozenset({0, 1, 2})


def test_capability_descriptor_digest_and_admission():
    qwen = {"num_experts": 128, "num_experts_per_tok": 8, "norm_topk_prob": True}
    dsv2 = {"n_routed_experts": 64, "n_shared_experts": 2, "num_experts_per_tok": 6,
            "n_group": 1, "topk_group": 1, "routed_scaling_factor": 1.0}
    d1 = cap.describe_checkpoint_config(qwen)
    d2 = cap.describe_checkpoint_config(dsv2)
    assert d1.output_contract == "routed_tensor" and d2.output_contract == "shared_routed_tuple"
    assert d1.digest() == cap.describe_checkpoint_config(dict(qwen)).digest()
    assert d1.digest() != d2.digest()
    assert cap.evaluate_support(d1).enabled and cap.evaluate_support(d2).enabled
    quant = cap.describe_checkpoint_config({**qwen, "quantization_config": {"quant_method": "fp8"}})
    with pytest.raises(cap.LatchMoECapabilityError) as err:
        cap.require_support(quant)
    payload = json.loads(str(err.value))
    assert "unsupported_weight_mode:quantized" in payload["support"]["blockers"]
    tp = cap.describe_checkpoint_config(qwen, parallel_mode="tensor_parallel")
    assert not cap.evaluate_support(tp).enabled


def test_autoconfig_matches_reference_golden(monkeypatch):
    for case in json.loads((GOLDEN / "autoconfig.json").read_text()):
        monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_BUDGET_GB", case["slot_hbm_budget_gb"])
        if case["min_net_saving_ratio"] is None:
            monkeypatch.delenv("VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_RATIO", raising=False)
        else:
            monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_RATIO",
                               case["min_net_saving_ratio"])
        pre = ac.derive_prefetch_defaults(case["offload_gb"])
        slots = ac.derive_num_slots_defaults(case["offload_gb"], None, pre,
                                             max_num_seqs=case["max_num_seqs"])
        assert list(pre["offloaded_layer_ids"]) == case["offloaded_layer_ids"]
        assert slots["num_slots"] == case["num_slots"], case
        assert slots["target_b2_waves"] == case["target_b2_waves"]
        assert slots["estimated_b2_waves"] == case["estimated_b2_waves"]


def test_autoconfig_b200_memory_model(monkeypatch):
    monkeypatch.delenv("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_BUDGET_GB", raising=False)
    hbm = (170.0, {"source": "torch.cuda.mem_get_info", "total_gib": ac.B200_HBM_GIB})
    pre = ac.derive_prefetch_defaults(14.0)
    slots = ac.derive_num_slots_defaults(14.0, None, pre, hbm=hbm)
    assert pre["estimated_offloaded_layers"] == 12 and slots["num_slots"] == 32
    assert slots["physical_slot_budget_gib"] == pytest.approx(0.12 * ac.B200_HBM_GIB)
    advice = ac.b200_residency_advice()
    assert advice["fits_resident"] and advice["expert_gib"] == pytest.approx(54.0)
    env = {}
    plan = ac.apply_moe_offload_defaults(14.0, env=env)
    assert env["VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"] == str(plan["slot_defaults"]["num_slots"])
    assert env["VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS"].startswith("0,1,2,4")


def test_autoconfig_seam_dataplane_defaults_and_release_conflict():
    """Seam data plane: its settings become the defaults (layered runtime off, originals
    released) and explicit user settings stay; the layered runtime cannot run with the
    original expert tensors released (reference ``moe_offload/autoconfig.py:83-102,700-711``)."""
    env = {"VLLM_ASCEND_MOE_OFFLOAD_SEW_DATAPLANE": "1",
           "VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS": "0,1",
           "VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT": "3"}
    plan = ac.apply_moe_offload_defaults(14.0, env=env)
    assert plan["sew_dataplane"]
    for name, value in ac.SEW_DATAPLANE_ENV_VARS.items():
        if name != "VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT":
            assert env[name] == value, name
    assert env["VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT"] == "3"
    assert env["VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS"] == "0,1"
    assert env["VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME"] == "0"
    layered = {"VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS": "1"}
    with pytest.raises(ValueError, match="LAYERED_RUNTIME=1"):
        ac.apply_moe_offload_defaults(14.0, env=layered, sew_dataplane=False)
    plain = {}
    assert not ac.apply_moe_offload_defaults(14.0, env=plain)["sew_dataplane"]
    assert plain["VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME"] == "1"
    assert "VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS" not in plain


def test_capability_admission_fails_closed_on_unimplemented_modes():
    """Anything the B200 path does not implement is refused with a named blocker, like the
    reference's admission (``tests/test_capabilities.py:95-179``): overlapped shared-expert
    streams, Python router callables, tensor / multi-GPU layouts other than the expert-
    partitioned bank, gated shared activations and unknown scoring functions."""
    import dataclasses

    base = cap.describe_checkpoint_config({"n_routed_experts": 64, "n_shared_experts": 2,
                                           "num_experts_per_tok": 6, "n_group": 1,
                                           "topk_group": 1})
    assert cap.evaluate_support(base).enabled
    cases = {
        "unsupported_overlap_mode:shared_gate_multistream":
            dataclasses.replace(base, overlap_mode="shared_gate_multistream"),
        "unsupported_router_adapter:python_callable":
            dataclasses.replace(base, router_adapter="python_callable"),
        "unsupported_parallel_mode:tensor_parallel":
            dataclasses.replace(base, parallel_mode="tensor_parallel"),
        "unsupported_shared_activation:gated":
            dataclasses.replace(base, shared_activation="gated"),
        "unsupported_scoring:sqrtsoftplus": dataclasses.replace(
            base, selection=dataclasses.replace(base.selection, scoring_function="sqrtsoftplus")),
    }
    for blocker, d in cases.items():
        support = cap.evaluate_support(d)
        assert support.state == "unsupported" and blocker in support.blockers, (blocker, support)
    ep = dataclasses.replace(base, parallel_mode="expert_parallel")
    assert cap.evaluate_support(ep).enabled


def test_fused_mix_placement_lane_is_admitted_and_the_router_widens():
    """The fused mix-placement shared lane is admitted, like the reference
    (``tests/test_capabilities.py:121-144``); it returns a routed tensor only. With
    mix_placement the router op's rows hold top_k + num_shared_experts entries."""
    import dataclasses

    from torch._subclasses.fake_tensor import FakeTensorMode

    base = cap.describe_checkpoint_config({"n_routed_experts": 64, "n_shared_experts": 2,
                                           "num_experts_per_tok": 6})
    fused = dataclasses.replace(base, shared_mode="fused_mix_placement",
                                output_contract="routed_tensor")
    assert cap.evaluate_support(fused).enabled
    tuple_out = dataclasses.replace(fused, output_contract="shared_routed_tuple")
    assert "fused_mix_placement_returns_routed_tensor" in cap.evaluate_support(tuple_out).blockers
    plugin.register()
    with FakeTensorMode():
        h = torch.empty(5, 64, dtype=torch.bfloat16)
        lg = torch.empty(5, 64)
        w, ids = torch.ops.vllm.moe_router(h, lg, 6, False, False, None, None, "softmax", 1.0,
                                           None, 64, True, 2)
        assert tuple(w.shape) == (5, 8) and tuple(ids.shape) == (5, 8)
