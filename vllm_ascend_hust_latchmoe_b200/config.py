"""Frozen offload configuration read from the plugin's environment contract.

Mirrors ``moe_offload/config.py`` of the reference (``MoeOffloadConfig.from_env``
:33-133): same field names and env variables for the settings the offload hot path reads.
"""

from __future__ import annotations

from dataclasses import dataclass

from . import env_registry as env


def parse_comma_separated_ints(value: str) -> frozenset[int]:
    return frozenset(int(v) for v in str(value or "").replace(" ", "").split(",") if v)


@dataclass(frozen=True)
class MoeOffloadConfig:
    enabled: bool = False
    num_slots: int = 0
    policy: str = "deadline"
    async_load: bool = False
    resident_layer_ids: frozenset[int] = frozenset()
    graph_compatible_offload: bool = False
    offload_stage_seam: bool = False
    b2_wave_prefill: bool = False
    b2_reference_full_layer: bool = False
    release_original_expert_weights: bool = False
    # B200 addition: decode staging decided on the device (lm_slot_plan) and missed experts
    # read over PCIe by the MLP itself; no host round trip per layer.
    device_staging: bool = False
    # B200 addition: a layer whose expert store is HBM-resident still runs prefill overflow
    # through the capacity-bounded wave executor (stage banks filled device-to-device on the
    # copy stream) instead of reading every expert in place in one pass.
    stage_waves_from_hbm_store: bool = False
    # B200 addition: such waves are planned and staged on the device (device wave plan, copy
    # kernels into the stage banks, grouped MLP over each wave's groups read on the device),
    # with no host read between the router and the combine, so the layer can be captured.
    stage_waves_on_device: bool = True
    pin_host_memory: bool | None = None
    transfer_aware_wave_schedule: bool = True
    prefill_prefetch_depth: int = 1
    prefill_buffer_count: int = 2
    b2_avoid_mixed_wave_d2d: bool = True
    device_pair_planning: bool = True
    max_num_seqs_hint: int = 0
    profile_path: str = ""

    @property
    def should_pin_host_memory(self) -> bool:
        return self.async_load if self.pin_host_memory is None else bool(self.pin_host_memory)

    @property
    def effective_prefill_prefetch_depth(self) -> int:
        return max(0, int(self.prefill_prefetch_depth))

    @property
    def effective_prefill_buffer_count(self) -> int:
        return max(1, int(self.prefill_buffer_count))

    @classmethod
    def from_env(cls) -> "MoeOffloadConfig":
        return cls(
            enabled=env.get("VLLM_ASCEND_MOE_OFFLOAD_ENABLED"),
            num_slots=env.get("VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"),
            policy=env.get("VLLM_ASCEND_MOE_OFFLOAD_POLICY"),
            async_load=env.get("VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD"),
            resident_layer_ids=parse_comma_separated_ints(
                env.get("VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS")),
            graph_compatible_offload=env.get("VLLM_ASCEND_MOE_OFFLOAD_GRAPH_COMPATIBLE"),
            offload_stage_seam=env.get("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM"),
            b2_wave_prefill=env.get("VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL"),
            b2_reference_full_layer=bool(env.get("VLLM_ASCEND_MOE_OFFLOAD_B2_REFERENCE_FULL_LAYER")),
            release_original_expert_weights=bool(
                env.get("VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS")),
            device_staging=bool(env.get("VLLM_ASCEND_MOE_OFFLOAD_DEVICE_STAGING")),
            pin_host_memory=env.get("VLLM_ASCEND_MOE_OFFLOAD_PIN_HOST_MEMORY"),
            transfer_aware_wave_schedule=env.get("VLLM_ASCEND_MOE_OFFLOAD_TRANSFER_AWARE_SCHEDULE"),
            prefill_prefetch_depth=env.get("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_PREFETCH_DEPTH"),
            prefill_buffer_count=env.get("VLLM_ASCEND_MOE_OFFLOAD_PREFILL_BUFFER_COUNT"),
            b2_avoid_mixed_wave_d2d=env.get("VLLM_ASCEND_MOE_OFFLOAD_B2_AVOID_MIXED_D2D"),
            device_pair_planning=env.get("VLLM_ASCEND_MOE_OFFLOAD_DEVICE_PAIR_PLANNING"),
            max_num_seqs_hint=env.get("VLLM_ASCEND_MOE_OFFLOAD_MAX_NUM_SEQS_HINT"),
            profile_path=env.get("VLLM_ASCEND_MOE_OFFLOAD_PROFILE_PATH"),
        )
