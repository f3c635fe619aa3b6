"""Environment-variable contract of the plugin (same names as the reference).

The reference keeps every setting in one inventory (``env_registry.py:56-234``) so that
vLLM can validate and propagate them; the names are part of the drop-in surface and are
kept verbatim. Values are parsed lazily on access.
"""

from __future__ import annotations

import os
from collections.abc import Callable
from typing import Any

_TRUE = {"1", "true", "yes", "on"}


def _parse(kind: str, name: str, default: str | None) -> Any:
    raw = os.getenv(name)
    if kind == "bool":
        return (raw if raw is not None else (default or "0")).strip().lower() in _TRUE
    if kind == "opt_bool":
        return None if raw is None else raw.strip().lower() in _TRUE
    if kind == "int":
        return int(raw if raw is not None and raw.strip() else (default or "0"))
    if kind == "opt_int":
        return None if raw is None or not raw.strip() else int(raw)
    if kind == "float":
        return float(raw if raw is not None and raw.strip() else (default or "0"))
    if kind == "opt_float":
        return None if raw is None or not raw.strip() else float(raw)
    return raw if raw is not None else (default or "")


# (name, kind, default)
_SPEC: tuple[tuple[str, str, str | None], ...] = (
    ("VLLM_ASCEND_MOE_B2_PROFILE_DETAILS", "bool", None),
    ("VLLM_ASCEND_MOE_COMPUTE_BUCKET_PLAN_PATH", "str", None),
    ("VLLM_ASCEND_MOE_DECODE_PROFILE_SAMPLE_RATE", "int", "1"),
    ("VLLM_ASCEND_MOE_GRAPH_REPLAY_PROFILE_SAMPLE_RATE", "int", "1024"),
    ("VLLM_ASCEND_MOE_GMM_BUCKET_PLAN_PATH", "str", None),
    ("VLLM_ASCEND_MOE_GMM_PROFILE_PATH", "str", None),
    ("VLLM_ASCEND_MOE_GMM_TRACE_PATH", "str", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_ACTIVATION_RESERVE_GB", "opt_float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_B2_AVOID_MIXED_D2D", "bool", "1"),
    ("VLLM_ASCEND_MOE_OFFLOAD_B2_DIRECT_SCATTER", "bool", "1"),
    ("VLLM_ASCEND_MOE_OFFLOAD_B2_OVERFLOW_MODE", "str", "multi_wave"),
    ("VLLM_ASCEND_MOE_OFFLOAD_B2_REFERENCE_FULL_LAYER", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_B2_REFERENCE_FULL_TOKENS", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_COMPARE_LAYER_BOUNDARY", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_COMPARE_ORIGINAL", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_COMPARE_ROUTER", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_COMPAT_ONLY", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_CPU_FIRST_LOAD", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_DEVICE_PAIR_PLANNING", "bool", "1"),
    ("VLLM_ASCEND_MOE_OFFLOAD_ENABLED", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_FANOUT_THRESHOLD", "int", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_GB", "float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_GRAPH_COMPATIBLE", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_KV_RESERVE_CTX", "opt_int", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_KV_RESERVE_SEQS", "opt_int", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME", "bool", "1"),
    ("VLLM_ASCEND_MOE_OFFLOAD_MAX_NUM_SEQS_HINT", "int", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_MAX_PHASES", "int", "2"),
    ("VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_GB", "opt_float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_RATIO", "opt_float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS", "int", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS_AUTOCONFIG_BOOTSTRAP", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_ONDEMAND_STAGE", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_PHASE_SPLIT", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_PIN_HOST_MEMORY", "opt_bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_POLICY", "str", "deadline"),
    ("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT", "int", "2"),
    ("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_PREFETCH_DEPTH", "int", "1"),
    ("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_RESIDENCY_PROFILE", "str", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_PROFILE_PATH", "str", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS", "str", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_ROUTE_STATS_CACHE", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_SEW_DATAPLANE", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_BUDGET_GB", "opt_float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_FRACTION", "opt_float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_SYSTEM_RESERVE_GB", "opt_float", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_TRACE_MAX_RECORDS", "int", "4096"),
    ("VLLM_ASCEND_MOE_OFFLOAD_TRACE_ONLY", "bool", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_TRACE_PATH", "str", None),
    ("VLLM_ASCEND_MOE_OFFLOAD_TRANSFER_AWARE_SCHEDULE", "bool", "1"),
    ("VLLM_ASCEND_MOE_PIPELINE_PROFILING", "bool", None),
    ("VLLM_ASCEND_MOE_PROFILE_EXPERT_LISTS", "bool", "1"),
    ("VLLM_ASCEND_MOE_PROFILE_FLUSH_EVERY", "int", "1"),
    ("VLLM_ASCEND_MOE_ROUTER_PARITY_MAX_TOKENS", "int", "64"),
    ("VLLM_ASCEND_MOE_ROUTER_PARITY_PATH", "str", None),
)

ENVIRONMENT_VARIABLES: dict[str, Callable[[], Any]] = {
    name: (lambda n=name, k=kind, d=default: _parse(k, n, d)) for name, kind, default in _SPEC
}

# Settings of the B200 build that the reference does not have (kept apart from the
# reference's inventory above).
_B200_SPEC: tuple[tuple[str, str, str | None], ...] = (
    ("VLLM_ASCEND_MOE_OFFLOAD_DEVICE_STAGING", "bool", None),
)

B200_ENVIRONMENT_VARIABLES: dict[str, Callable[[], Any]] = {
    name: (lambda n=name, k=kind, d=default: _parse(k, n, d)) for name, kind, default in _B200_SPEC
}

_registered = False


def register_environment_variables() -> dict[str, Callable[[], Any]]:
    """Expose the inventory through ``vllm.envs`` when vLLM is importable (idempotent)."""
    global _registered
    if _registered:
        return ENVIRONMENT_VARIABLES
    try:
        import vllm.envs as vllm_envs  # type: ignore

        table = getattr(vllm_envs, "environment_variables", None)
        if isinstance(table, dict):
            for name, loader in (*ENVIRONMENT_VARIABLES.items(),
                                 *B200_ENVIRONMENT_VARIABLES.items()):
                table.setdefault(name, loader)
    except Exception:
        pass
    _registered = True
    return ENVIRONMENT_VARIABLES


def get(name: str) -> Any:
    loader = ENVIRONMENT_VARIABLES.get(name) or B200_ENVIRONMENT_VARIABLES[name]
    return loader()
