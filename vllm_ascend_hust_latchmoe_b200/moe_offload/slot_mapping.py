"""Logical -> physical expert mapping handed from the staging controller to the MLP.

Mirrors ``moe_offload/slot_mapping.py`` of the reference (``ExpertSlotMapping`` :42,
``remap_topk_ids`` :116-141, ``PreparedSlotWeights`` :144-187). On B200 the remap
``log2phy[topk_ids]`` happens inside ``lm_build_groups`` (a -1 entry is recorded as a
device error and the pair is skipped), so this module only carries the fixed tensors.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ExpertSlotMapping:
    layer_id: int
    active_experts: tuple[int, ...]
    logical_to_physical: torch.Tensor | None
    slot_to_expert: tuple[int | None, ...]
    active_slot_ids: tuple[int, ...]

    def physical_slot_for(self, expert_id: int) -> int:
        for e, s in zip(self.active_experts, self.active_slot_ids):
            if e == int(expert_id):
                return s
        raise KeyError(f"expert {expert_id} is not staged in layer {self.layer_id}")

    def remap_topk_ids_host(self, topk_ids: torch.Tensor) -> torch.Tensor:
        """Host-side remap with the fail-closed -1 check (tests and diagnostics)."""
        table = self.logical_to_physical.to("cpu")
        out = table[topk_ids.to("cpu", torch.int64)]
        if bool((out < 0).any()):
            raise RuntimeError(f"layer {self.layer_id}: routed expert is not staged (log2phy=-1)")
        return out.to(torch.int32)


@dataclass(frozen=True)
class PreparedSlotWeights:
    """Fixed slot tensors + mapping for one layer call: ``(w1, w2, log2phy)``."""

    w1: torch.Tensor
    w2: torch.Tensor
    mapping: ExpertSlotMapping
    physical_expert_count: int

    @property
    def log2phy(self) -> torch.Tensor | None:
        return self.mapping.logical_to_physical
