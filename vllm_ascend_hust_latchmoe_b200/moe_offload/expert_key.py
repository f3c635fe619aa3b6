"""(layer, expert) identity used by the slot bank and the host store."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True, order=True)
class ExpertKey:
    layer_id: int
    expert_id: int
