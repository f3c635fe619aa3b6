"""Pinned host store of offloaded expert weights (one contiguous tensor per layer per weight).

Mirrors ``moe_offload/host_store.py`` of the reference (``HostExpertStore.register_layer``
:112-186, ``get`` :188): ``w13 [E, 2I, H]`` and ``w2 [E, H, I]`` live in page-locked host
memory so that a run of consecutive experts is one DMA-able span; expert ``e`` is row ``e``.
A layer may instead be registered on a device (an HBM-resident tier): the staging copies
are then device-to-device, and a wave whose experts all have such a copy reads them in
place.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .expert_key import ExpertKey


@dataclass(frozen=True)
class ExpertWeightBundle:
    layer_id: int
    expert_id: int
    w13: torch.Tensor
    w2: torch.Tensor

    @property
    def key(self) -> ExpertKey:
        return ExpertKey(self.layer_id, self.expert_id)


@dataclass(frozen=True)
class HostLayerBuffer:
    layer_id: int
    w13: torch.Tensor  # [E, 2I, H]
    w2: torch.Tensor   # [E, H, I]

    @property
    def num_experts(self) -> int:
        return int(self.w13.shape[0])

    @property
    def expert_bytes(self) -> int:
        return (self.w13[0].numel() + self.w2[0].numel()) * self.w13.element_size()

    @property
    def on_device(self) -> bool:
        return self.w13.is_cuda

    def bundle(self, expert_id: int) -> ExpertWeightBundle:
        return ExpertWeightBundle(self.layer_id, int(expert_id), self.w13[expert_id], self.w2[expert_id])


@dataclass(frozen=True)
class HostStoreRegisterReport:
    layer_id: int
    num_experts: int
    pin_memory_requested: bool
    pinned_tensors: int
    bytes: int

    def to_jsonable(self) -> dict[str, object]:
        return {
            "layer_id": self.layer_id,
            "num_experts": self.num_experts,
            "pin_memory_requested": self.pin_memory_requested,
            "pinned_tensors": self.pinned_tensors,
            "bytes": self.bytes,
        }


def _to_store(t: torch.Tensor, *, pin: bool, device: torch.device | None) -> torch.Tensor:
    t = t.detach()
    if device is not None and device.type == "cuda":
        return t.to(device=device, copy=True).contiguous()
    out = torch.empty(t.shape, dtype=t.dtype, pin_memory=bool(pin and torch.cuda.is_available()))
    out.copy_(t)
    return out


class HostExpertStore:
    def __init__(self) -> None:
        self._layers: dict[int, HostLayerBuffer] = {}

    def register_layer(
        self,
        layer: torch.nn.Module,
        *,
        pin_memory: bool = True,
        routed_expert_count: int | None = None,
        device: torch.device | None = None,
    ) -> HostStoreRegisterReport:
        layer_id = int(getattr(layer, "layer_id", -1))
        w13 = getattr(layer, "w13_weight")
        w2 = getattr(layer, "w2_weight")
        if w13.shape[0] != w2.shape[0]:
            raise ValueError("w13_weight and w2_weight must have the same number of experts")
        total = int(w13.shape[0])
        n = total if routed_expert_count is None else int(routed_expert_count)
        if n <= 0:
            raise ValueError("host expert store requires at least one expert")
        if n > total:
            raise ValueError(f"routed expert count exceeds materialized expert rows: routed={n}, total={total}")
        buf = HostLayerBuffer(
            layer_id,
            _to_store(w13[:n], pin=pin_memory, device=device),
            _to_store(w2[:n], pin=pin_memory, device=device),
        )
        self._layers[layer_id] = buf
        pinned = int(buf.w13.is_pinned()) + int(buf.w2.is_pinned()) if not buf.on_device else 0
        return HostStoreRegisterReport(layer_id, n, bool(pin_memory), pinned,
                                       buf.expert_bytes * n)

    def adopt_layer(self, layer_id: int, w13: torch.Tensor, w2: torch.Tensor) -> HostStoreRegisterReport:
        """Use existing store tensors ``[E, 2I, H]`` / ``[E, H, I]`` (already in the bank
        layout; pinned host memory or device memory) without copying them. Several layers
        may adopt the same tensors."""
        if w13.shape[0] != w2.shape[0]:
            raise ValueError("w13 and w2 stores must have the same number of experts")
        if not w13.is_cuda and torch.cuda.is_available() and not w13.is_pinned():
            raise ValueError("a host store must be pinned memory")
        buf = HostLayerBuffer(int(layer_id), w13, w2)
        self._layers[int(layer_id)] = buf
        return HostStoreRegisterReport(int(layer_id), buf.num_experts, not w13.is_cuda,
                                       0 if w13.is_cuda else 2, buf.expert_bytes * buf.num_experts)

    def layer(self, layer_id: int) -> HostLayerBuffer:
        try:
            return self._layers[int(layer_id)]
        except KeyError as exc:
            raise KeyError(f"layer {layer_id} is not host-managed") from exc

    def get(self, layer_id: int, expert_id: int) -> ExpertWeightBundle:
        buf = self.layer(layer_id)
        if not 0 <= int(expert_id) < buf.num_experts:
            raise KeyError(f"expert {expert_id} is not host-managed for layer {layer_id}")
        return buf.bundle(int(expert_id))

    def has_layer(self, layer_id: int) -> bool:
        return int(layer_id) in self._layers

    @property
    def total_bytes(self) -> int:
        return sum(b.expert_bytes * b.num_experts for b in self._layers.values())
