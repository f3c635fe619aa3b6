"""Seam custom ops of the slot-bank MoE layer, registered under the reference's names.

The reference splits vLLM's opaque ``moe_forward`` into three ops so that the routing-
dependent staging can run eagerly between two captured graph pieces
(``ops/fused_moe/moe_router_op.py:165,312``, ``moe_offload_stage_op.py:523-529``,
``moe_mlp_op.py:232-247``):

    vllm::moe_router_indirect  ->  vllm::moe_offload_stage  ->  vllm::moe_mlp / moe_mlp_shared
      (captured piece 1)           (splitting op, eager)          (captured piece 2)

The schemas here are the reference's, with the CUDA dispatch key instead of PrivateUse1.
Layers are found through a registry (``register_moe_layer``) instead of vLLM's forward
context. ``moe_router_indirect`` returns the layer's fixed top-k buffers, so the stage and
MLP pieces always read the same addresses (what a replayed graph needs);
``moe_offload_stage`` mutates nothing but declares ``topk_ids`` mutated to keep its place
in the graph, exactly like the reference.
"""

from __future__ import annotations

import threading

import torch

from . import _lib
from .layer import PHASE_UNKNOWN, SlotBankMoE, StageDecision

_registry_lock = threading.Lock()
_LAYERS_BY_NAME: dict[str, SlotBankMoE] = {}
_LAYERS_BY_ID: dict[int, SlotBankMoE] = {}
_registered_ops = False
_lib_fragment: torch.library.Library | None = None

OP_SCHEMAS = {
    "moe_router": (
        "moe_router(Tensor hidden_states, Tensor router_logits, int top_k, bool use_grouped_topk,"
        " bool renormalize, int? topk_group, int? num_expert_group, str scoring_func,"
        " float routed_scaling_factor, Tensor? e_score_correction_bias, int num_experts,"
        " bool mix_placement=False, int num_shared_experts=0) -> (Tensor, Tensor)"),
    "moe_router_indirect": (
        "moe_router_indirect(Tensor hidden_states, Tensor router_logits, str layer_name)"
        " -> (Tensor, Tensor)"),
    "moe_offload_stage": (
        "moe_offload_stage(Tensor(a!) topk_ids, int layer_id, int num_logical_experts,"
        " int phase) -> ()"),
    "moe_mlp": (
        "moe_mlp(Tensor(a!) hidden_states, Tensor router_logits, Tensor topk_weights,"
        " Tensor topk_ids, Tensor? shared_experts_input, Tensor? input_ids, str layer_name,"
        " int hidden_dim_unpadded=-1) -> Tensor"),
    "moe_mlp_shared": (
        "moe_mlp_shared(Tensor(a!) hidden_states, Tensor router_logits, Tensor topk_weights,"
        " Tensor topk_ids, Tensor? shared_experts_input, Tensor? input_ids, str layer_name,"
        " int hidden_dim_unpadded=-1) -> (Tensor, Tensor)"),
}


def register_moe_layer(layer_name: str, layer: SlotBankMoE) -> None:
    with _registry_lock:
        _LAYERS_BY_NAME[str(layer_name)] = layer
        _LAYERS_BY_ID[int(layer.layer_id)] = layer


def unregister_moe_layer(layer_name: str) -> None:
    with _registry_lock:
        layer = _LAYERS_BY_NAME.pop(str(layer_name), None)
        if layer is not None:
            _LAYERS_BY_ID.pop(int(layer.layer_id), None)


def registered_layer_names() -> tuple[str, ...]:
    """Names of the MoE layers currently registered with the seam."""
    with _registry_lock:
        return tuple(_LAYERS_BY_NAME)


def get_layer(layer_name: str) -> SlotBankMoE:
    layer = _LAYERS_BY_NAME.get(str(layer_name))
    if layer is None:
        raise RuntimeError(f"MoE layer {layer_name!r} is not registered with the B200 seam")
    return layer


def get_layer_by_id(layer_id: int) -> SlotBankMoE:
    layer = _LAYERS_BY_ID.get(int(layer_id))
    if layer is None:
        raise RuntimeError(f"fixed-slot MoE layer {layer_id} is not registered; refusing "
                           "native-weight fallback")
    return layer


# ----------------------------------------------------------------------- implementations
def _moe_router(hidden_states, router_logits, top_k, use_grouped_topk, renormalize, topk_group,
                num_expert_group, scoring_func, routed_scaling_factor, e_score_correction_bias,
                num_experts, mix_placement=False, num_shared_experts=0):
    # mix_placement: the shared experts' ids num_experts .. num_experts + num_shared - 1 are
    # appended to every token's top-k with weight 1 (the fused shared lane's pinned suffix)
    shared = int(num_shared_experts or 0) if mix_placement else 0
    if mix_placement and shared <= 0:
        raise RuntimeError("mix_placement routing needs num_shared_experts > 0")
    T = router_logits.shape[0]
    width = int(top_k) + shared
    w = torch.empty(T, width, dtype=torch.bfloat16, device=router_logits.device)
    ids = torch.empty(T, width, dtype=torch.int32, device=router_logits.device)
    _lib.route_topk(router_logits.float().contiguous(), int(top_k), scoring_func=scoring_func,
                    renormalize=renormalize, routed_scaling_factor=routed_scaling_factor,
                    e_score_correction_bias=e_score_correction_bias,
                    num_expert_group=(num_expert_group or 0) if use_grouped_topk else 0,
                    topk_group=(topk_group or 0) if use_grouped_topk else 0,
                    weights_bf16=w, ids=ids, num_shared=shared)
    return w.to(hidden_states.dtype), ids


def _moe_router_fake(hidden_states, router_logits, top_k, use_grouped_topk=False,
                     renormalize=True, topk_group=None, num_expert_group=None,
                     scoring_func="softmax", routed_scaling_factor=1.0,
                     e_score_correction_bias=None, num_experts=0, mix_placement=False,
                     num_shared_experts=0):
    T = hidden_states.shape[0]
    width = int(top_k) + (int(num_shared_experts) if mix_placement else 0)
    return (hidden_states.new_empty((T, width)),
            torch.empty((T, width), dtype=torch.int32, device=hidden_states.device))


def _moe_router_indirect(hidden_states, router_logits, layer_name):
    layer = get_layer(layer_name)
    w, ids = layer.route(hidden_states, router_logits)
    return w, ids


def _moe_router_indirect_fake(hidden_states, router_logits, layer_name):
    T = hidden_states.shape[0]
    k = _LAYERS_BY_NAME[layer_name].k if layer_name in _LAYERS_BY_NAME else 1
    return (hidden_states.new_empty((T, k)),
            torch.empty((T, k), dtype=torch.int32, device=hidden_states.device))


def _moe_offload_stage(topk_ids, layer_id, num_logical_experts, phase):
    layer = get_layer_by_id(layer_id)
    if int(num_logical_experts) not in (layer.E, layer.E_total):
        raise RuntimeError(f"layer {layer_id}: num_logical_experts={num_logical_experts} does not "
                           f"match the registered layer ({layer.E})")
    layer.pending = layer.stage(topk_ids, int(phase))


def _moe_offload_stage_fake(topk_ids, layer_id, num_logical_experts, phase):
    return None


def _take_decision(layer: SlotBankMoE, T: int) -> StageDecision:
    if torch.cuda.is_current_stream_capturing():
        return layer.capture_decision(T)
    decision = layer.pending
    layer.pending = None
    if decision is None:
        raise RuntimeError(f"moe_mlp on layer {layer.layer_id} without a preceding "
                           "moe_offload_stage call")
    return decision


def _adopt_topk(layer: SlotBankMoE, topk_weights, topk_ids) -> None:
    """The MLP reads the layer's fixed top-k buffers; copy foreign tensors in."""
    T = topk_ids.shape[0]
    if topk_ids.data_ptr() != layer.topk_ids.data_ptr():
        layer.topk_ids[:T].copy_(topk_ids)
        layer.invalidate_router_grouping()  # ids from another router: the MLP groups them
    if topk_weights.data_ptr() != layer.topk_w.data_ptr():
        layer.topk_w[:T].copy_(topk_weights)


def _moe_mlp(hidden_states, router_logits, topk_weights, topk_ids, shared_experts_input,
             input_ids, layer_name, hidden_dim_unpadded=-1):
    layer = get_layer(layer_name)
    _adopt_topk(layer, topk_weights, topk_ids)
    out = torch.empty_like(hidden_states)
    return layer.run_mlp(hidden_states, _take_decision(layer, int(hidden_states.shape[0])), out)


def _moe_mlp_fake(hidden_states, router_logits, topk_weights, topk_ids, shared_experts_input,
                  input_ids, layer_name, hidden_dim_unpadded=-1):
    return torch.empty_like(hidden_states)


def _moe_mlp_shared(hidden_states, router_logits, topk_weights, topk_ids, shared_experts_input,
                    input_ids, layer_name, hidden_dim_unpadded=-1):
    layer = get_layer(layer_name)
    _adopt_topk(layer, topk_weights, topk_ids)
    src = shared_experts_input if shared_experts_input is not None else hidden_states
    shared_out = layer.shared_mlp(src.contiguous(), int(src.shape[0]))
    routed_out = layer.run_mlp(hidden_states, _take_decision(layer, int(hidden_states.shape[0])),
                               torch.empty_like(hidden_states))
    return shared_out, routed_out


def _moe_mlp_shared_fake(hidden_states, router_logits, topk_weights, topk_ids,
                         shared_experts_input, input_ids, layer_name, hidden_dim_unpadded=-1):
    src = shared_experts_input if shared_experts_input is not None else hidden_states
    return torch.empty_like(src), torch.empty_like(hidden_states)


_IMPLS = {
    "moe_router": (_moe_router, _moe_router_fake),
    "moe_router_indirect": (_moe_router_indirect, _moe_router_indirect_fake),
    "moe_offload_stage": (_moe_offload_stage, _moe_offload_stage_fake),
    "moe_mlp": (_moe_mlp, _moe_mlp_fake),
    "moe_mlp_shared": (_moe_mlp_shared, _moe_mlp_shared_fake),
}


def register_ops() -> tuple[str, ...]:
    """Define the seam ops in the ``vllm`` namespace (idempotent). Ops another package
    already defined under the same name are left alone. Returns the names defined here."""
    global _registered_ops, _lib_fragment
    with _registry_lock:
        if _registered_ops:
            return tuple(_IMPLS)
        _lib_fragment = torch.library.Library("vllm", "FRAGMENT")
        defined = []
        for name, schema in OP_SCHEMAS.items():
            if hasattr(torch.ops.vllm, name):
                continue
            impl, fake = _IMPLS[name]
            _lib_fragment.define(schema)
            _lib_fragment.impl(name, impl, "CUDA")
            torch.library.register_fake(f"vllm::{name}", fake, lib=_lib_fragment)
            defined.append(name)
        _registered_ops = True
        return tuple(defined)


def seam_forward(layer_name: str, hidden_states: torch.Tensor, router_logits: torch.Tensor,
                 phase: int = PHASE_UNKNOWN) -> torch.Tensor:
    """router -> stage -> MLP through the registered ops (the seam's call sequence)."""
    w, ids = torch.ops.vllm.moe_router_indirect(hidden_states, router_logits, layer_name)
    layer = get_layer(layer_name)
    torch.ops.vllm.moe_offload_stage(ids, layer.layer_id, layer.E, int(phase))
    return torch.ops.vllm.moe_mlp(hidden_states, router_logits, w, ids, None, None, layer_name, -1)
