"""Shared helpers for the parity tests: seeded layers and tensor <-> numpy views."""

from __future__ import annotations

import numpy as np
import torch

from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime
from vllm_ascend_hust_latchmoe_b200.synthetic import ExpertLayer  # noqa: F401  (re-exported)

# Tolerance for bf16 outputs against the fp32-accumulating oracle.
MAX_REL_ERR = 1e-2
MIN_COSINE = 0.9999


def bits(t: torch.Tensor) -> np.ndarray:
    """Raw bf16 bit patterns of a bf16 tensor as uint16 numpy."""
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


def build_layer(cfg: syn.LayerConfig, *, seed: int = 0, max_tokens: int | None = None,
                device="cuda", store_on_device: bool = False, num_slots: int | None = None,
                experts=None, reference_full_layer: bool = False, layer_id: int = 0):
    w13, w2 = syn.make_expert_weights(cfg, seed) if experts is None else experts
    runtime = MoeOffloadRuntime(MoeOffloadConfig(
        enabled=True, num_slots=int(num_slots or cfg.num_slots), async_load=True,
        b2_wave_prefill=True, graph_compatible_offload=True,
        b2_reference_full_layer=reference_full_layer))
    runtime.register_layer_for_fixed_slots(
        ExpertLayer(layer_id, w13, w2), slot_device=torch.device(device),
        store_device=torch.device(device) if store_on_device else None)
    layer = SlotBankMoE(runtime, layer_id, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                        num_experts=cfg.num_experts, top_k=cfg.top_k,
                        max_tokens=int(max_tokens or cfg.tokens), renormalize=cfg.renormalize,
                        routed_scaling_factor=cfg.routed_scaling_factor,
                        scoring_func=cfg.scoring_func, num_expert_group=cfg.num_expert_group,
                        topk_group=cfg.topk_group, device=device)
    return layer, runtime, (w13, w2)
