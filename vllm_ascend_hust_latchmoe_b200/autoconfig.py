"""AutoConfig: map an offload budget (GiB) to offloaded layers and the fixed slot count.

Restates the reference's policy (``moe_offload/autoconfig.py``: ``derive_prefetch_defaults``
:206-240, ``_target_b2_waves_for_offload`` :309, ``derive_num_slots_defaults`` :474-583;
``moe_offload/autoconfig_advisor.py``: ``suggest_num_slots`` :154-183) with the device
memory model re-derived for B200:

* offloaded layers: in groups of 4, the last ``n`` layers of every group, with ``n`` the
  budget's share of one group (at least 1);
* target prefill waves: 4 at the 14 GiB reference budget, scaled down as the budget grows,
  never below 2;
* ``num_slots = min(E, max(top_k * batch, ceil(E / target_waves)), floor(budget /
  (expert_gib * (offloaded_layers + prefill_buffers))))`` where the slot budget is the
  smallest of (a) the offloaded bytes minus a minimum net saving (25 %) and the KV /
  activation / system reserves, (b) the usable HBM reported by the device minus those
  reserves, and (c) a fixed fraction (12 %) of the physical HBM.

On a 180 GB B200 the whole Qwen3-30B-A3B expert set (54 GiB) fits in HBM, so offload is a
policy choice there; :func:`b200_residency_advice` reports that case explicitly.
"""

from __future__ import annotations

import math
import os
from typing import Any

GIB = 1024**3
GROUP_SIZE = 4
DEFAULT_TARGET_WAVES = 4
REFERENCE_OFFLOAD_GB_FOR_SLOTS = 14.0
MIN_TARGET_WAVES = 2
DEFAULT_MIN_NET_SAVING_RATIO = 0.25
DEFAULT_KV_RESERVE_SEQS = 4
DEFAULT_SYSTEM_RESERVE_GB = 2.0
DEFAULT_ACTIVATION_RESERVE_GB = 1.0
DEFAULT_SLOT_HBM_FRACTION = 0.12
B200_HBM_GIB = 183359 / 1024  # nvidia-smi memory.total of a B200, in GiB

QWEN3_30B_A3B = {
    "hidden_size": 2048, "moe_intermediate_size": 768, "num_experts": 128,
    "num_experts_per_tok": 8, "num_hidden_layers": 48, "num_attention_heads": 32,
    "num_key_value_heads": 4, "head_dim": 128, "max_position_embeddings": 40960,
    "torch_dtype": "bfloat16",
}


def _get(cfg: dict[str, Any], *keys: str, default: int = 0) -> int:
    for k in keys:
        v = cfg.get(k)
        if v is not None:
            return int(v)
    return int(default)


def _dtype_bytes(cfg: dict[str, Any]) -> int:
    d = str(cfg.get("torch_dtype", "bfloat16")).lower()
    return 1 if ("fp8" in d or "int8" in d) else (4 if "float32" in d else 2)


def _env_float(name: str) -> float | None:
    raw = os.getenv(name)
    if raw is None or not str(raw).strip():
        return None
    v = float(raw)
    if v < 0:
        raise ValueError(f"{name} must be a non-negative number, got {raw!r}")
    return v


def _env_int(name: str) -> int | None:
    raw = os.getenv(name)
    if raw is None or not str(raw).strip():
        return None
    v = int(raw)
    if v < 0:
        raise ValueError(f"{name} must be a non-negative integer, got {raw!r}")
    return v


def single_expert_gib(cfg: dict[str, Any]) -> float:
    return 3 * _get(cfg, "hidden_size") * _get(cfg, "moe_intermediate_size", "intermediate_size") \
        * _dtype_bytes(cfg) / GIB


def expert_layer_gib(cfg: dict[str, Any]) -> float:
    return single_expert_gib(cfg) * _get(cfg, "num_experts", "n_routed_experts")


def derive_prefetch_defaults(target_offload_gb: float, model_config: dict[str, Any] | None = None):
    if target_offload_gb <= 0:
        raise ValueError("target_offload_gb must be greater than 0")
    cfg = model_config or QWEN3_30B_A3B
    layers = _get(cfg, "num_hidden_layers")
    group = min(GROUP_SIZE, layers)
    groups = math.ceil(layers / group)
    layer_gb = expert_layer_gib(cfg)
    n_in_group = min(group, max(1, round(target_offload_gb / (layer_gb * groups))))
    offloaded = tuple(i for i in range(layers) if i % group >= group - n_in_group)
    resident = tuple(i for i in range(layers) if i not in set(offloaded))
    return {
        "offload_group_size": group,
        "offload_num_in_group": n_in_group,
        "offloaded_layer_ids": offloaded,
        "resident_layer_ids": resident,
        "estimated_offloaded_layers": len(offloaded),
        "estimated_offloaded_gb": len(offloaded) * layer_gb,
        "expert_layer_gb": layer_gb,
    }


def target_b2_waves_for_offload(target_offload_gb: float) -> int:
    if target_offload_gb <= 0:
        return DEFAULT_TARGET_WAVES
    scaled = math.ceil(DEFAULT_TARGET_WAVES * REFERENCE_OFFLOAD_GB_FOR_SLOTS / float(target_offload_gb))
    return max(MIN_TARGET_WAVES, int(scaled))


def device_hbm_budget(device_index: int | None = None, gpu_memory_utilization: float = 1.0):
    """Usable HBM for slots (GiB) and the physical total, from the env override or CUDA."""
    explicit = _env_float("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_BUDGET_GB")
    if explicit is not None:
        return explicit, {"source": "env_override", "slot_hbm_budget_gib": explicit}
    try:
        import torch

        if not torch.cuda.is_available():
            return None, {"source": "unavailable", "reason": "no_cuda_device"}
        free, total = torch.cuda.mem_get_info(device_index)
    except Exception as exc:  # pragma: no cover - device specific
        return None, {"source": "unavailable", "reason": type(exc).__name__}
    free_g, total_g = free / GIB, total / GIB
    used = max(0.0, total_g - free_g)
    util = min(1.0, max(0.0, float(gpu_memory_utilization)))
    usable = max(0.0, total_g * util - used)
    return usable, {"source": "torch.cuda.mem_get_info", "free_gib": free_g, "total_gib": total_g,
                    "used_gib": used, "gpu_memory_utilization": util, "slot_hbm_budget_gib": usable}


def derive_num_slots_defaults(target_offload_gb: float, model_config: dict[str, Any] | None,
                              prefetch_defaults: dict[str, Any], *, max_num_seqs: int = 1,
                              max_model_len: int | None = None, hbm: tuple | None = None):
    cfg = model_config or QWEN3_30B_A3B
    E = _get(cfg, "num_experts", "n_routed_experts", "moe_num_experts")
    top_k = _get(cfg, "num_experts_per_tok", "num_experts_per_token", "moe_top_k", "top_k", default=2)
    seq = int(max_model_len or _get(cfg, "max_position_embeddings", "seq_length", default=4096))
    waves = target_b2_waves_for_offload(target_offload_gb)
    n_off = int(prefetch_defaults["estimated_offloaded_layers"])
    off_gb = float(prefetch_defaults["estimated_offloaded_gb"])

    ratio = _env_float("VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_RATIO")
    ratio = DEFAULT_MIN_NET_SAVING_RATIO if ratio is None else min(1.0, max(0.0, ratio))
    min_gb = _env_float("VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_GB")
    min_saving = off_gb * ratio if min_gb is None else max(min_gb, off_gb * ratio)
    net_budget = max(0.0, off_gb - min_saving)

    # Reserves kept out of the slot budget: KV for a few sequences, activations, system.
    layers = _get(cfg, "num_hidden_layers")
    kv_heads = _get(cfg, "num_key_value_heads", "num_kv_heads", default=_get(cfg, "num_attention_heads"))
    head_dim = _get(cfg, "head_dim", default=_get(cfg, "hidden_size") // max(1, _get(cfg, "num_attention_heads", default=1)))
    dt = _dtype_bytes(cfg)
    kv_seqs = _env_int("VLLM_ASCEND_MOE_OFFLOAD_KV_RESERVE_SEQS")
    kv_seqs = DEFAULT_KV_RESERVE_SEQS if kv_seqs is None else kv_seqs
    kv_ctx = _env_int("VLLM_ASCEND_MOE_OFFLOAD_KV_RESERVE_CTX")
    kv_ctx = min(seq, 8192) if kv_ctx is None else kv_ctx
    kv_gib = 2 * layers * kv_heads * head_dim * max(1, kv_seqs) * max(1, kv_ctx) * dt / GIB
    act_est = 4 * _get(cfg, "hidden_size") * max(1, max_num_seqs) * seq * dt / GIB
    act_floor = _env_float("VLLM_ASCEND_MOE_OFFLOAD_ACTIVATION_RESERVE_GB")
    act_gib = max(act_est, DEFAULT_ACTIVATION_RESERVE_GB if act_floor is None else act_floor)
    sys_gib = _env_float("VLLM_ASCEND_MOE_OFFLOAD_SYSTEM_RESERVE_GB")
    sys_gib = DEFAULT_SYSTEM_RESERVE_GB if sys_gib is None else sys_gib
    bufs = _env_int("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT")
    bufs = 2 if bufs is None else bufs
    reserve = kv_gib + act_gib + sys_gib

    budget = max(0.0, net_budget - reserve)
    hbm_budget, hbm_info = hbm if hbm is not None else device_hbm_budget()
    if hbm_budget is not None:
        budget = min(budget, max(0.0, hbm_budget - reserve))
    physical = None
    if hbm_info.get("total_gib") is not None:
        frac = _env_float("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_FRACTION")
        frac = DEFAULT_SLOT_HBM_FRACTION if frac is None else min(1.0, max(0.0, frac))
        physical = float(hbm_info["total_gib"]) * frac
        budget = min(budget, physical)

    expert_gib = single_expert_gib(cfg)
    afford_layers = n_off + bufs
    slots = max(min(top_k * max(1, max_num_seqs), E), math.ceil(E / max(1, waves)), 1)
    if afford_layers > 0:
        slots = min(slots, max(1, int(budget / (expert_gib * afford_layers))))
    slots = min(slots, E)
    slot_bank = expert_gib * slots * n_off
    stage = expert_gib * slots * bufs
    return {
        "num_slots": int(slots),
        "fanout_threshold": int(slots),
        "slot_budget_gib": float(budget),
        "target_b2_waves": int(waves),
        "estimated_b2_waves": math.ceil(E / max(1, slots)),
        "decode_working_set": min(top_k * max(1, max_num_seqs), E),
        "slot_bank_gib": slot_bank,
        "b2_stage_bank_gib": stage,
        "slot_plus_b2_stage_gib": slot_bank + stage,
        "net_hbm_saving_gib": max(0.0, off_gb - slot_bank),
        "reserve_gib": {"kv": kv_gib, "activation": act_gib, "system": sys_gib,
                        "prefill_buffers": bufs},
        "hbm": hbm_info,
        "physical_slot_budget_gib": physical,
    }


# Settings of the seam data plane (fixed slots only, graph-safe staging), set as defaults when
# it is selected (reference ``moe_offload/autoconfig.py:83-102``): the original expert copies
# are unused once the host store and slot banks exist, so they are released.
SEW_DATAPLANE_ENV_VARS = {
    "VLLM_ASCEND_MOE_OFFLOAD_GRAPH_COMPATIBLE": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_B2_OVERFLOW_MODE": "multi_wave",
    "VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME": "0",
    "VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_PIN_HOST_MEMORY": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_TRANSFER_AWARE_SCHEDULE": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_PREFILL_PREFETCH_DEPTH": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT": "2",
    "VLLM_ASCEND_MOE_OFFLOAD_DEVICE_PAIR_PLANNING": "1",
    "VLLM_ASCEND_MOE_OFFLOAD_ROUTE_STATS_CACHE": "0",
    "VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS": "1",
}


def _truthy(value: Any) -> bool:
    return str(value or "").strip().lower() in ("1", "true", "yes", "on")


def check_layered_release_conflict(env: dict | None = None) -> None:
    """The layered runtime reads the full expert tensors for high-fanout batches, so it cannot
    run with those tensors released (reference ``moe_offload/autoconfig.py:700-711``)."""
    env = os.environ if env is None else env
    if (_truthy(env.get("VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME"))
            and _truthy(env.get("VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS"))):
        raise ValueError(
            "VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS=1 is incompatible with "
            "VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME=1: the layered runtime needs the full "
            "expert tensors for high-fanout batches. Unset the release or set "
            "VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME=0 for the pure fixed-slot path.")


PREFILL_RESIDENCY_PROFILE_ENV = "VLLM_ASCEND_MOE_OFFLOAD_PREFILL_RESIDENCY_PROFILE"


def apply_profile_guided_residency(defaults: dict[str, Any], *, profile_path: str | None,
                                   model_config: dict[str, Any] | None = None) -> dict[str, Any]:
    """Refine the default resident / offloaded layer split with prefill profiles
    (``os.pathsep``-separated JSONL paths; reference ``moe_offload/autoconfig.py:585-640``).
    The swap keeps the number of offloaded layers, so the offload budget is unchanged. Without
    profile evidence the defaults are returned as they are."""
    if not profile_path:
        return defaults
    from .moe_offload.prefill_residency import (load_prefill_layer_costs_many,
                                                plan_profile_guided_prefill_residency)

    paths = tuple(p.strip() for p in str(profile_path).split(os.pathsep) if p.strip())
    if not paths:
        return defaults
    cfg = model_config or QWEN3_30B_A3B
    plan = plan_profile_guided_prefill_residency(
        num_layers=_get(cfg, "num_hidden_layers"),
        default_offloaded_layer_ids=tuple(defaults["offloaded_layer_ids"]),
        layer_costs=load_prefill_layer_costs_many(paths))
    if not plan.profiled_layer_ids:
        return defaults
    out = dict(defaults)
    out.update({
        "resident_layer_ids": plan.resident_layer_ids,
        "offloaded_layer_ids": plan.offloaded_layer_ids,
        "estimated_offloaded_layers": len(plan.offloaded_layer_ids),
        "estimated_offloaded_gb": len(plan.offloaded_layer_ids) * float(defaults["expert_layer_gb"]),
        "prefill_residency_profile": os.pathsep.join(paths),
        "prefill_residency_profiles": paths,
        "prefill_residency_plan": plan.to_jsonable(),
    })
    return out


def apply_moe_offload_defaults(target_offload_gb: float, model_config: dict[str, Any] | None = None,
                               *, env: dict | None = None, max_num_seqs: int = 1,
                               max_model_len: int | None = None,
                               sew_dataplane: bool | None = None) -> dict[str, Any]:
    """Write the derived settings into ``env`` (default ``os.environ``), keeping explicit
    user overrides of NUM_SLOTS and RESIDENT_LAYER_IDS. With the seam data plane selected
    (``sew_dataplane``, default: ``VLLM_ASCEND_MOE_OFFLOAD_SEW_DATAPLANE``) its settings are
    the defaults instead of the layered ones. Returns the plan."""
    env = os.environ if env is None else env
    if sew_dataplane is None:
        sew_dataplane = _truthy(env.get("VLLM_ASCEND_MOE_OFFLOAD_SEW_DATAPLANE"))
    if sew_dataplane:
        for name, value in SEW_DATAPLANE_ENV_VARS.items():
            env.setdefault(name, value)
    pre = derive_prefetch_defaults(target_offload_gb, model_config)
    pre = apply_profile_guided_residency(pre, profile_path=env.get(PREFILL_RESIDENCY_PROFILE_ENV),
                                         model_config=model_config)
    slots = derive_num_slots_defaults(target_offload_gb, model_config, pre,
                                      max_num_seqs=max_num_seqs, max_model_len=max_model_len)
    if not env.get("VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"):
        env["VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"] = str(slots["num_slots"])
    env.setdefault("VLLM_ASCEND_MOE_OFFLOAD_FANOUT_THRESHOLD", env["VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"])
    env.setdefault("VLLM_ASCEND_MOE_OFFLOAD_ENABLED", "1")
    env.setdefault("VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL", "1")
    env.setdefault("VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD", "1")
    env.setdefault("VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME", "1")
    check_layered_release_conflict(env)
    env.setdefault("VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS",
                   ",".join(map(str, pre["resident_layer_ids"])))
    return {"prefetch_defaults": pre, "slot_defaults": slots, "sew_dataplane": bool(sew_dataplane)}


def b200_residency_advice(model_config: dict[str, Any] | None = None,
                          hbm_gib: float = B200_HBM_GIB, reserve_gib: float = 40.0) -> dict[str, Any]:
    """Whether every layer's experts can stay resident on one B200 (Regime A), leaving
    ``reserve_gib`` for attention weights, KV cache and activations."""
    cfg = model_config or QWEN3_30B_A3B
    total = expert_layer_gib(cfg) * _get(cfg, "num_hidden_layers")
    return {"expert_gib": total, "hbm_gib": hbm_gib,
            "fits_resident": total + reserve_gib <= hbm_gib,
            "headroom_gib": hbm_gib - reserve_gib - total}
