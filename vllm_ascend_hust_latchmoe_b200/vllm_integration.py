"""vLLM (CUDA platform) integration of the slot-bank seam.

What the reference does on Ascend, done here for vLLM's CUDA platform:

* PIECEWISE graphs split at ``vllm::moe_offload_stage``, so the routing-dependent staging runs
  eagerly between the captured router piece and the captured MLP piece
  (``patches/patch_fused_moe.py:5339-5406`` ``_ensure_moe_offload_splitting_op``).
* The platform's ``check_and_update_config`` appends that splitting op once the platform has
  settled its own defaults (``patch_fused_moe.py:5310-5337``, there on ``NPUPlatform``; here on
  ``vllm.platforms.cuda.CudaPlatform``).
* ``EngineArgs.create_engine_config`` applies the AutoConfig defaults first, selects PIECEWISE
  when no graph mode was requested, retries the platform patch, and refuses a final config
  without the splitting op (``patch_fused_moe.py:5409-5445``;
  ``moe_offload/autoconfig.py:728-790``).
* The MoE runner's forward entry becomes the seam: ``moe_router_indirect`` ->
  ``moe_offload_stage`` -> ``moe_mlp`` / ``moe_mlp_shared`` instead of vLLM's opaque
  ``moe_forward`` (``patch_fused_moe.py:4917-5175``, ``AscendMoERunner._select_forward`` /
  ``_seam_forward_entry``; here ``MoERunner`` of vLLM's CUDA fused-MoE layer). A layer that was
  not attached to the slot bank is refused, never run on the native path.
* After weight loading, an unquantized ``FusedMoE`` layer is attached: its experts move into the
  host store and slot bank and the layer is registered with the seam ops (the reference's
  ``register_layer_for_fixed_slots`` call from its loader patches).

Every patch is idempotent (a marker attribute on the wrapper) and the platform / EngineArgs
patches are best-effort at install time, as in the reference: a vLLM build without the patched
class leaves the rest working. The seam only takes effect while
``VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM`` is on.
"""

from __future__ import annotations

import inspect
import json
import os
import re
from dataclasses import dataclass
from types import SimpleNamespace
from typing import Any, Callable

import torch

from . import env_registry as env

SPLITTING_OP = "vllm::moe_offload_stage"
GRAPH_CONFIG_LINE = (
    "LATCHMOE_GRAPH_CONFIG cudagraph_mode=PIECEWISE "
    "splitting_op=vllm::moe_offload_stage status=enabled")
_MARK = "_latchmoe_b200_patch"
_LAYER_ID_RE = re.compile(r"(?:^|\.)layers\.(\d+)(?:\.|$)")


def stage_seam_enabled() -> bool:
    """The seam switch (default off, like the reference's ``VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM``)."""
    return bool(env.get("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM"))


# ------------------------------------------------------------------ graph configuration
def ensure_moe_offload_splitting_op(vllm_config: Any, *, fail_closed: bool = False,
                                    create: bool = True) -> bool:
    """Put the eager staging seam into the final piecewise graph config.

    Returns True when ``vllm::moe_offload_stage`` is in ``splitting_ops``. With the seam off,
    or a graph mode that needs no piecewise split, nothing changes and the result is False.
    Any full-graph mode is refused when ``fail_closed`` (the staging would be captured and
    replayed with stale routing), as is a config without a compilation config. With
    ``create=False`` an unset (None) ``splitting_ops`` is left unset: vLLM fills in its own
    defaults (the attention ops) only while the list is None.
    """
    if not stage_seam_enabled():
        return False
    cc = getattr(vllm_config, "compilation_config", None)
    if cc is None:
        if fail_closed:
            raise RuntimeError("LatchMoE seam graph mode requires vLLM compilation_config")
        return False
    mode = getattr(cc, "cudagraph_mode", None)
    try:
        piecewise = bool(mode is not None and mode.requires_piecewise_compilation())
        full = bool(mode is not None and mode.has_full_cudagraphs())
    except Exception as exc:
        if fail_closed:
            raise RuntimeError("LatchMoE could not validate the final CUDA graph mode") from exc
        return False
    if full:
        if fail_closed:
            raise RuntimeError(
                "LatchMoE seam offload requires PIECEWISE-only CUDA graphs so "
                f"{SPLITTING_OP} executes eagerly during replay; got cudagraph_mode={mode}")
        return False
    if not piecewise:
        return False
    ops = getattr(cc, "splitting_ops", None)
    if ops is None:
        if not create:
            return False
        cc.splitting_ops = []
        ops = cc.splitting_ops
    if SPLITTING_OP not in ops:
        ops.append(SPLITTING_OP)
    present = SPLITTING_OP in ops
    if fail_closed and not present:
        raise RuntimeError("LatchMoE refused graph startup: the final splitting_ops does not "
                           f"contain {SPLITTING_OP}")
    return present


def _wrap_classmethod(cls: type, name: str, make: Callable[[Callable], Callable]) -> bool:
    """Wrap a classmethod of ``cls``, also when it is inherited (the wrapper is set on
    ``cls`` itself and calls the inherited function)."""
    current = inspect.getattr_static(cls, name, None)
    fn = getattr(current, "__func__", current)
    if fn is None or getattr(fn, _MARK, False):
        return False
    wrapped = make(fn)
    setattr(wrapped, _MARK, True)
    setattr(cls, name, classmethod(wrapped))
    return True


def patch_platform_splitting_ops(platform_cls: type | None = None) -> bool:
    """Wrap the platform's ``check_and_update_config`` so the splitting op is appended after
    the platform's own defaults. vLLM runs this hook before it fills in its default splitting
    ops, so an unset list is left to vLLM here and the EngineArgs boundary appends the op
    afterwards. Best-effort: False when the class cannot be imported or is already wrapped."""
    if platform_cls is None:
        try:
            from vllm.platforms.cuda import CudaPlatform as platform_cls
        except Exception:
            return False

    def make(original):
        def check_and_update_config(cls, vllm_config):
            original(cls, vllm_config)
            ensure_moe_offload_splitting_op(vllm_config, create=False)
        return check_and_update_config

    return _wrap_classmethod(platform_cls, "check_and_update_config", make)


# ------------------------------------------------------------------ engine arguments
def _load_model_config_dict(engine_args: Any) -> dict | None:
    model = getattr(engine_args, "model", None)
    if not model:
        return None
    path = os.path.join(str(model), "config.json")
    if not os.path.isfile(path):
        return None
    with open(path, encoding="utf-8") as f:
        cfg = json.load(f)
    return cfg.get("text_config", cfg) if isinstance(cfg, dict) else None


def set_piecewise_default(engine_args: Any) -> None:
    """Select PIECEWISE graphs when the seam is on and no graph mode was requested."""
    cc = getattr(engine_args, "compilation_config", None)
    if cc is None:
        return
    if isinstance(cc, dict):
        if cc.get("cudagraph_mode") is None:
            cc["cudagraph_mode"] = "PIECEWISE"
        return
    if getattr(cc, "cudagraph_mode", None) is not None:
        return
    from vllm.config import CUDAGraphMode

    cc.cudagraph_mode = CUDAGraphMode.PIECEWISE


def apply_engine_args_defaults(engine_args: Any) -> bool:
    """AutoConfig from ``VLLM_ASCEND_MOE_OFFLOAD_GB`` and the model's ``config.json``
    (``moe_offload/autoconfig.py:746-790``). False when no offload budget is set."""
    gb = float(env.get("VLLM_ASCEND_MOE_OFFLOAD_GB") or 0.0)
    if gb <= 0:
        return False
    from .autoconfig import apply_moe_offload_defaults

    if stage_seam_enabled():
        set_piecewise_default(engine_args)
    apply_moe_offload_defaults(
        gb, _load_model_config_dict(engine_args),
        max_num_seqs=int(getattr(engine_args, "max_num_seqs", None) or 1),
        max_model_len=getattr(engine_args, "max_model_len", None),
        sew_dataplane=True if stage_seam_enabled() else None)
    return True


def patch_engine_args(engine_args_cls: type | None = None) -> bool:
    """Wrap ``EngineArgs.create_engine_config``: defaults first, then a retry of the platform
    patch (the real ``vllm serve`` import order can miss the early one), then the original,
    then a fail-closed check of the final config."""
    if engine_args_cls is None:
        try:
            from vllm.engine.arg_utils import EngineArgs as engine_args_cls
        except Exception:
            return False
    current = engine_args_cls.__dict__.get("create_engine_config")
    if current is None or getattr(current, _MARK, False):
        return False
    original = current

    def create_engine_config(self, *args, **kwargs):
        apply_engine_args_defaults(self)
        patch_platform_splitting_ops()
        vllm_config = original(self, *args, **kwargs)
        if ensure_moe_offload_splitting_op(vllm_config, fail_closed=True):
            print(GRAPH_CONFIG_LINE, flush=True)
        return vllm_config

    setattr(create_engine_config, _MARK, True)
    engine_args_cls.create_engine_config = create_engine_config
    return True


# ------------------------------------------------------------------ MoE runner seam
@dataclass(frozen=True)
class SeamBinding:
    """What a runner's seam entry needs, fixed when its layer is attached (constants under
    tracing, so the captured pieces see the same op arguments on every replay)."""

    layer_name: str
    layer_id: int
    num_logical_experts: int
    shared: bool


def _seam_ops():
    return torch.ops.vllm


def seam_forward_entry(runner: Any, hidden_states: torch.Tensor, router_logits: torch.Tensor,
                       shared_experts_input: torch.Tensor | None, input_ids: torch.Tensor | None,
                       layer_name: Any = None, hidden_dim_unpadded: int = -1):
    """The runner's forward entry under the seam (same arguments as vLLM's ``moe_forward``).

    The phase is passed as unknown: the stage op decides from the routed counts it reads at
    run time, which stay correct for every batch a captured piece is replayed with.
    """
    binding: SeamBinding | None = getattr(runner, "_latchmoe_seam", None)
    if binding is None:
        raise RuntimeError(
            f"LatchMoE seam: MoE layer {getattr(runner, 'layer_name', '?')!r} was not attached "
            "to the slot bank; refusing native fallback")
    gate = getattr(runner, "gate", None)
    if gate is not None:
        # the runner owns the router gate (vLLM passes hidden states in the logits slot)
        router_logits, _ = gate(hidden_states)
    ops = _seam_ops()
    name = binding.layer_name
    topk_weights, topk_ids = ops.moe_router_indirect(hidden_states, router_logits, name)
    ops.moe_offload_stage(topk_ids, binding.layer_id, binding.num_logical_experts, -1)
    if binding.shared:
        return ops.moe_mlp_shared(hidden_states, router_logits, topk_weights, topk_ids,
                                  shared_experts_input, input_ids, name, int(hidden_dim_unpadded))
    return ops.moe_mlp(hidden_states, router_logits, topk_weights, topk_ids,
                       shared_experts_input, input_ids, name, int(hidden_dim_unpadded))


def patch_moe_runner(runner_cls: type | None = None) -> bool:
    """Wrap ``MoERunner._select_forward``: with the seam on, every runner built afterwards
    enters through :func:`seam_forward_entry`; with it off, vLLM's own entry is kept."""
    if runner_cls is None:
        try:
            from vllm.model_executor.layers.fused_moe.runner.moe_runner import (
                MoERunner as runner_cls,
            )
        except Exception:
            return False
    current = runner_cls.__dict__.get("_select_forward")
    if current is None or getattr(current, _MARK, False):
        return False
    original = current

    def _select_forward(self):
        if not stage_seam_enabled():
            return original(self)

        def entry(hidden_states, router_logits, shared_experts_input, input_ids,
                  layer_name=None, hidden_dim_unpadded=-1):
            return seam_forward_entry(self, hidden_states, router_logits, shared_experts_input,
                                      input_ids, layer_name, hidden_dim_unpadded)

        return entry

    setattr(_select_forward, _MARK, True)
    runner_cls._select_forward = _select_forward
    return True


# ------------------------------------------------------------------ layer attachment
def layer_id_from_name(layer_name: str) -> int:
    """Decoder-layer index of a vLLM module prefix such as ``model.layers.7.mlp.experts``."""
    m = _LAYER_ID_RE.search(str(layer_name))
    if m is None:
        raise ValueError(f"cannot derive a layer id from MoE layer name {layer_name!r}")
    return int(m.group(1))


def attach_fused_moe_layer(fused_moe: Any, *, runtime=None, layer_id: int | None = None,
                           max_tokens: int = 8192, slot_device: torch.device | None = None,
                           store_device: torch.device | None = None):
    """Move a loaded, unquantized vLLM ``FusedMoE`` layer onto the slot-bank path.

    Its experts (``w13_weight [E, 2I, H]`` with the gate rows first, ``w2_weight [E, H, I]``)
    go into the runtime's host store (or an HBM-resident store when ``store_device`` is a GPU,
    and always for the runtime's resident layers) and a slot bank; a :class:`SlotBankMoE` built with the layer's router settings is
    registered with the seam ops under the layer's name, and the layer's runner gets the
    binding its seam entry reads. With ``release_original_expert_weights`` the offloaded
    layer's original expert tensors are emptied afterwards (the store holds the copy).
    Tensor/expert-parallel layers and layers whose capability descriptor is not supported are
    refused.
    """
    from . import seam_ops
    from .capabilities import describe_layer_capability, require_support
    from .layer import SlotBankMoE
    from .moe_offload.runtime import get_moe_offload_runtime

    rt = runtime if runtime is not None else get_moe_offload_runtime()
    name = str(getattr(fused_moe, "layer_name", "") or "")
    if not name:
        raise ValueError("FusedMoE layer has no layer_name")
    if layer_id is None:
        layer_id = getattr(fused_moe, "layer_id", None)  # vLLM derives it from the name
        if layer_id is None or int(layer_id) < 0:
            layer_id = layer_id_from_name(name)
    lid = int(layer_id)
    for attr in ("tp_size", "ep_size", "dp_size"):
        if int(getattr(fused_moe, attr, 1) or 1) != 1:
            raise RuntimeError(f"LatchMoE seam supports single-GPU MoE layers; {name} has "
                               f"{attr}={getattr(fused_moe, attr)}")
    w13 = fused_moe.w13_weight.data
    w2 = fused_moe.w2_weight.data
    if w13.dtype != torch.bfloat16 or w2.dtype != torch.bfloat16:
        raise RuntimeError(f"LatchMoE seam needs bf16 unquantized experts; {name} holds "
                           f"{w13.dtype}/{w2.dtype}")
    E, two_i, H = (int(s) for s in w13.shape)
    if tuple(w2.shape) != (E, H, two_i // 2) or two_i % 2:
        raise ValueError(f"{name}: w13 {tuple(w13.shape)} and w2 {tuple(w2.shape)} do not form "
                         "an [E, 2I, H] / [E, H, I] expert pair")
    for attr, what in (("custom_routing_function", "a custom routing function"),
                       ("hash_indices_table", "hash routing"),
                       ("zero_expert_type", "zero experts")):
        if getattr(fused_moe, attr, None) is not None:
            raise RuntimeError(f"{name}: {what} is not implemented by the slot-bank router")
    if getattr(fused_moe, "apply_router_weight_on_input", False):
        raise RuntimeError(f"{name}: router weights applied to the input are not implemented")
    global_e = int(getattr(fused_moe, "global_num_experts", E) or E)
    if global_e != E:
        raise RuntimeError(f"{name}: {E} local of {global_e} experts; expert-parallel vLLM "
                           "layers are not attached")
    dev = torch.device(slot_device) if slot_device is not None else w13.device
    if store_device is None and rt.is_resident_layer(lid):
        # a layer kept resident reads its experts in place from an HBM store
        store_device = dev
    rt.register_layer_for_fixed_slots(
        SimpleNamespace(layer_id=lid, w13_weight=w13, w2_weight=w2, num_fused_shared_experts=0),
        slot_device=dev, store_device=store_device)
    use_grouped = bool(getattr(fused_moe, "use_grouped_topk", False))
    moe = SlotBankMoE(
        rt, lid, hidden_size=H, intermediate_size=two_i // 2, num_experts=E,
        top_k=int(fused_moe.top_k), max_tokens=int(max_tokens),
        renormalize=bool(getattr(fused_moe, "renormalize", True)),
        routed_scaling_factor=float(getattr(fused_moe, "routed_scaling_factor", 1.0) or 1.0),
        scoring_func=str(getattr(fused_moe, "scoring_func", "softmax") or "softmax"),
        num_expert_group=int(getattr(fused_moe, "num_expert_group", 0) or 0) if use_grouped else 0,
        topk_group=int(getattr(fused_moe, "topk_group", 0) or 0) if use_grouped else 0,
        e_score_correction_bias=getattr(fused_moe, "e_score_correction_bias", None),
        device=dev)
    require_support(describe_layer_capability(moe))
    runner = getattr(fused_moe, "runner", None)
    if runner is not None and getattr(runner, "shared_experts", None) is not None:
        raise RuntimeError(f"{name}: vLLM-owned shared experts are not attached to the seam "
                           "(install them with SlotBankMoE.set_shared_experts)")
    seam_ops.register_moe_layer(name, moe)
    if runner is not None:
        runner._latchmoe_seam = SeamBinding(name, lid, E, shared=False)
    # the seam never reads the original tensors: an offloaded layer may give their HBM back
    rt.release_original_expert_weights_if_ready(SimpleNamespace(
        layer_id=lid, w13_weight=fused_moe.w13_weight, w2_weight=fused_moe.w2_weight))
    if getattr(fused_moe, "layer_id", None) != lid:
        try:
            fused_moe.layer_id = lid
        except AttributeError:  # read-only (vLLM's FusedMoE derives it from its name)
            pass
    return moe


def patch_weight_loading(method_cls: type | None = None, *, max_tokens: Callable[[], int] | None = None,
                         attach: Callable[..., Any] = attach_fused_moe_layer) -> bool:
    """Wrap ``UnquantizedFusedMoEMethod.process_weights_after_loading`` so that, with the seam
    on, each layer is attached to the slot bank from its checkpoint-layout weights. vLLM's own
    post-processing for its fused-MoE kernels (weight shuffles, kernel set-up) is then skipped:
    the seam entry never calls those kernels and refuses to fall back to them."""
    if method_cls is None:
        try:
            from vllm.model_executor.layers.fused_moe.unquantized_fused_moe_method import (
                UnquantizedFusedMoEMethod as method_cls,
            )
        except Exception:
            return False
    current = method_cls.__dict__.get("process_weights_after_loading")
    if current is None or getattr(current, _MARK, False):
        return False
    original = current

    def process_weights_after_loading(self, layer):
        if not stage_seam_enabled():
            return original(self, layer)
        if getattr(getattr(layer, "runner", None), "_latchmoe_seam", None) is None:
            attach(layer, max_tokens=(max_tokens or _scheduler_max_tokens)())
        return None

    setattr(process_weights_after_loading, _MARK, True)
    method_cls.process_weights_after_loading = process_weights_after_loading
    return True


def _scheduler_max_tokens() -> int:
    try:
        from vllm.config import get_current_vllm_config

        n = get_current_vllm_config().scheduler_config.max_num_batched_tokens
        return int(n) if n else 8192
    except Exception:
        return 8192


def install_vllm_patches() -> dict[str, bool]:
    """Install every patch above (idempotent, best-effort per patch)."""
    return {
        "platform_splitting_ops": patch_platform_splitting_ops(),
        "engine_args": patch_engine_args(),
        "moe_runner": patch_moe_runner(),
        "weight_loading": patch_weight_loading(),
    }
