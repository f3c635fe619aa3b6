"""Serializable capability descriptor of one MoE layer, with fail-closed admission.

Mirrors ``moe_offload/capabilities.py`` of the reference (``MoeCapabilityDescriptor``
:36-64 with its sha256 digest, ``LatchMoECapabilityError`` :79-93,
``describe_checkpoint_config`` :189-238, ``evaluate_support`` :241-281): the same field
names and JSON shape, so manifests stay comparable. The admitted set is the one this B200
data path implements: bf16 weights, softmax/sigmoid routers with optional group limiting
and correction bias, no shared experts or always-on resident shared experts returned as a
``(shared, routed)`` tuple, single GPU or expert-parallel across GPUs of one node.
"""

from __future__ import annotations

import hashlib
import json
from dataclasses import asdict, dataclass
from typing import Any, Literal

SupportState = Literal["implemented", "gpu_qualified", "unsupported"]
SCHEMA_VERSION = "latchmoe-capability-v1"


@dataclass(frozen=True)
class RouterSelection:
    top_k: int
    grouped_top_k: bool
    topk_group: int | None
    num_expert_group: int | None
    renormalize: bool
    scoring_function: str
    correction_bias: bool
    routed_scaling_factor: float


@dataclass(frozen=True)
class MoeCapabilityDescriptor:
    schema_version: str
    output_contract: str        # "routed_tensor" | "shared_routed_tuple"
    shared_mode: str            # "none" | "external_resident" | "fused_mix_placement"
    shared_activation: str
    shared_expert_count: int
    routed_expert_count: int
    router_owner: str           # "external_logits" | "internal_gate"
    router_adapter: str
    selection: RouterSelection
    combine_owner: str
    weight_lifecycle: str
    weight_mode: str
    parallel_mode: str          # "single_gpu" | "expert_parallel"
    overlap_mode: str

    def to_jsonable(self) -> dict[str, object]:
        return asdict(self)

    def fingerprint(self) -> str:
        return json.dumps(self.to_jsonable(), sort_keys=True, separators=(",", ":"))

    def digest(self) -> str:
        return hashlib.sha256(self.fingerprint().encode("utf-8")).hexdigest()


@dataclass(frozen=True)
class CapabilitySupport:
    state: SupportState
    blockers: tuple[str, ...]

    @property
    def enabled(self) -> bool:
        return self.state in ("implemented", "gpu_qualified")

    def to_jsonable(self) -> dict[str, object]:
        return {"state": self.state, "blockers": list(self.blockers)}


class LatchMoECapabilityError(RuntimeError):
    """Fail-closed rejection whose message is a JSON manifest entry."""

    def __init__(self, descriptor: MoeCapabilityDescriptor, support: CapabilitySupport) -> None:
        self.descriptor = descriptor
        self.support = support
        super().__init__(json.dumps({"event": "latchmoe_capability_rejected",
                                     "descriptor": descriptor.to_jsonable(),
                                     "support": support.to_jsonable()}, sort_keys=True))


def _pos(value: Any, default: int = 0) -> int:
    try:
        v = int(value)
    except (TypeError, ValueError):
        return int(default)
    return v if v > 0 else int(default)


def _opt(value: Any) -> int | None:
    try:
        return None if value is None else int(value)
    except (TypeError, ValueError):
        return None


def describe_checkpoint_config(config: dict[str, Any], *, parallel_mode: str = "single_gpu",
                               router_owner: str = "external_logits") -> MoeCapabilityDescriptor:
    """Descriptor from a HF ``config.json`` dict (Qwen3-MoE, DeepSeek-V2/V3 style keys)."""
    routed = _pos(config.get("n_routed_experts"), _pos(config.get("num_experts")))
    shared = _pos(config.get("n_shared_experts"))
    if shared == 0 and _pos(config.get("shared_expert_intermediate_size")):
        shared = 1
    topk_method = str(config.get("topk_method") or "")
    scoring = str(config.get("scoring_func") or ("sigmoid" if topk_method.startswith("noaux") else "softmax"))
    return MoeCapabilityDescriptor(
        schema_version=SCHEMA_VERSION,
        output_contract="shared_routed_tuple" if shared else "routed_tensor",
        shared_mode="external_resident" if shared else "none",
        shared_activation=("gated" if _pos(config.get("shared_expert_intermediate_size"))
                           else ("always_on" if shared else "none")),
        shared_expert_count=shared,
        routed_expert_count=routed,
        router_owner=router_owner,
        router_adapter="builtin",
        selection=RouterSelection(
            top_k=_pos(config.get("num_experts_per_tok")),
            grouped_top_k=config.get("topk_group") not in (None, 1),
            topk_group=_opt(config.get("topk_group")),
            num_expert_group=_opt(config.get("n_group")),
            renormalize=bool(config.get("norm_topk_prob", False)),
            scoring_function=scoring,
            correction_bias=topk_method.startswith("noaux"),
            routed_scaling_factor=float(config.get("routed_scaling_factor") or 1.0),
        ),
        combine_owner="lm_moe_combine",
        weight_lifecycle="routed_host_store_slot_bank_shared_resident",
        weight_mode=("bf16_unquantized" if not config.get("quantization_config") else "quantized"),
        parallel_mode=parallel_mode,
        overlap_mode="none",
    )


def describe_layer_capability(layer: Any) -> MoeCapabilityDescriptor:
    """Descriptor of a constructed :class:`~vllm_ascend_hust_latchmoe_b200.layer.SlotBankMoE`."""
    shared = 1 if getattr(layer, "shared_w13", None) is not None else 0
    fused = int(getattr(layer, "num_fused_shared", 0) or 0)
    n_group = int(getattr(layer, "num_expert_group", 0) or 0)
    if shared:
        shared_mode, contract, count = "external_resident", "shared_routed_tuple", shared
    elif fused:
        shared_mode, contract, count = "fused_mix_placement", "routed_tensor", fused
    else:
        shared_mode, contract, count = "none", "routed_tensor", 0
    return MoeCapabilityDescriptor(
        schema_version=SCHEMA_VERSION,
        output_contract=contract,
        shared_mode=shared_mode,
        shared_activation="always_on" if count else "none",
        shared_expert_count=count,
        routed_expert_count=int(layer.E),
        router_owner="external_logits",
        router_adapter="builtin",
        selection=RouterSelection(
            top_k=int(getattr(layer, "k_route", layer.k)), grouped_top_k=n_group > 1,
            topk_group=int(getattr(layer, "topk_group", 0) or 0) or None,
            num_expert_group=n_group or None, renormalize=bool(layer.renormalize),
            scoring_function=str(layer.scoring_func),
            correction_bias=getattr(layer, "e_bias", None) is not None,
            routed_scaling_factor=float(layer.routed_scaling_factor)),
        combine_owner="lm_moe_combine",
        weight_lifecycle="routed_host_store_slot_bank_shared_resident",
        weight_mode="bf16_unquantized",
        parallel_mode=str(getattr(layer, "parallel_mode", "single_gpu")),
        overlap_mode="none",
    )


def evaluate_support(d: MoeCapabilityDescriptor) -> CapabilitySupport:
    """Explicit support state; anything unknown is rejected."""
    b: list[str] = []
    if d.output_contract not in ("routed_tensor", "shared_routed_tuple"):
        b.append(f"unknown_output_contract:{d.output_contract}")
    if d.shared_mode not in ("none", "external_resident", "fused_mix_placement"):
        b.append(f"unsupported_shared_mode:{d.shared_mode}")
    if d.shared_mode == "fused_mix_placement" and d.output_contract != "routed_tensor":
        b.append("fused_mix_placement_returns_routed_tensor")
    if d.shared_mode == "external_resident" and d.shared_activation not in ("always_on",):
        b.append(f"unsupported_shared_activation:{d.shared_activation}")
    if d.router_owner not in ("external_logits", "internal_gate"):
        b.append(f"unsupported_router_owner:{d.router_owner}")
    if d.router_adapter != "builtin":
        b.append(f"unsupported_router_adapter:{d.router_adapter}")
    if d.selection.top_k <= 0 or d.selection.top_k > 32:
        b.append("invalid_router_top_k")
    if d.routed_expert_count <= 0 or d.routed_expert_count > 256:
        b.append("invalid_routed_expert_count")
    if d.routed_expert_count and d.selection.top_k > d.routed_expert_count:
        b.append("top_k_exceeds_experts")
    if d.selection.scoring_function not in ("softmax", "sigmoid"):
        b.append(f"unsupported_scoring:{d.selection.scoring_function}")
    if d.selection.grouped_top_k and (d.selection.num_expert_group or 0) > 32:
        b.append("unsupported_expert_group_count")
    if d.weight_mode != "bf16_unquantized":
        b.append(f"unsupported_weight_mode:{d.weight_mode}")
    if d.parallel_mode not in ("single_gpu", "expert_parallel"):
        b.append(f"unsupported_parallel_mode:{d.parallel_mode}")
    if d.overlap_mode != "none":
        b.append(f"unsupported_overlap_mode:{d.overlap_mode}")
    return CapabilitySupport("unsupported" if b else "implemented", tuple(b))


def require_support(d: MoeCapabilityDescriptor) -> CapabilitySupport:
    s = evaluate_support(d)
    if not s.enabled:
        raise LatchMoECapabilityError(d, s)
    return s
