"""Third-party pin of the MLP oracle: ``oracle.mlp.moe_layer`` against vLLM's own CPU MoE.

The reference delegates its expert arithmetic to an un-vendored fork and CANN kernels, so no
reference test holds MLP values. vLLM 0.22 (installed here) ships a torch CPU MoE,
``vllm/model_executor/layers/fused_moe/cpu_fused_moe.py:cpu_fused_moe_torch``: per expert
``F.linear`` with ``w13 [2I, H]`` (gate rows first), ``SiluAndMul.forward_native`` (silu of
the first I columns times the last I), ``F.linear`` with ``w2 [H, I]``, then the top-k sum
weighted by the router weights. The oracle follows the same convention with its own rounding
points (fp32 SwiGLU, one bf16 rounding per GEMM, fp32 combine in j order), so the two agree
within the bf16 bar the GPU tests use.

vLLM's ``SiluAndMul`` CustomOp constructor needs a running vLLM config; the test puts the
static ``SiluAndMul.forward_native`` (what that constructor dispatches to on CPU) into vLLM's
activation table for the duration of the test. Everything else is vLLM's code path.
"""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

cpu_moe = pytest.importorskip("vllm.model_executor.layers.fused_moe.cpu_fused_moe")


@pytest.fixture
def vllm_silu(monkeypatch):
    from vllm.model_executor.layers.activation import SiluAndMul
    from vllm.model_executor.layers.fused_moe.activation import MoEActivation

    monkeypatch.setitem(cpu_moe._CPU_MOE_ACT_FN, MoEActivation.SILU, SiluAndMul.forward_native)


def _vllm_moe(hidden, ids, w_f32, w13, w2, num_experts):
    layer = torch.nn.Module()
    layer.w13_weight = w13
    layer.w2_weight = w2
    cpu_moe.CPUFusedMOE.init_moe_torch(None, layer)
    out = torch.empty(hidden.shape[0], w2.shape[1], dtype=torch.bfloat16)
    cpu_moe.cpu_fused_moe_torch(id(layer), out, hidden, torch.from_numpy(w_f32),
                                torch.from_numpy(ids.astype(np.int32)), "silu", num_experts)
    return out


@pytest.mark.parametrize("name,tokens,experts", [("c1_decode", 64, 0), ("c4_shared", 64, 0),
                                                 ("c5_ep", 32, 32), ("c2_prefill", 256, 0)])
def test_oracle_mlp_matches_vllm_cpu_moe(vllm_silu, name, tokens, experts):
    """Each benchmark layer shape (the Qwen3-235B one with 32 of its 128 experts, to keep the
    CPU weight generation short; H and I are what the arithmetic depends on)."""
    cfg = syn.CONFIGS[name].with_tokens(tokens)
    if experts:
        cfg = dataclasses.replace(cfg, num_experts=experts)
    w13, w2 = syn.make_expert_weights(cfg, 0)
    hidden = syn.make_hidden(cfg, 0)
    logits = syn.make_router_logits(cfg, 0)
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=cfg.renormalize,
                               routed_scaling_factor=cfg.routed_scaling_factor,
                               scoring_func=cfg.scoring_func,
                               num_expert_group=cfg.num_expert_group, topk_group=cfg.topk_group)
    got = _vllm_moe(hidden, ids, bf16_bits_to_f32(wb), w13, w2, cfg.num_experts)
    ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
    m = omlp.compare(bf16_bits_to_f32(bits(got)), ref)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m


def test_oracle_swiglu_gate_is_first_half(vllm_silu):
    """Swapping gate and up in the oracle's weights breaks the agreement: the convention
    (gate = first I rows of w13) is what is being pinned, not just the magnitudes."""
    cfg = syn.CONFIGS["c1_decode"].with_tokens(16)
    w13, w2 = syn.make_expert_weights(cfg, 0)
    hidden = syn.make_hidden(cfg, 0)
    logits = syn.make_router_logits(cfg, 0)
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=True)
    got = _vllm_moe(hidden, ids, bf16_bits_to_f32(wb), w13, w2, cfg.num_experts)
    I = cfg.intermediate
    swapped = torch.cat([w13[:, I:], w13[:, :I]], dim=1)
    ref_bad = omlp.moe_layer(bits(hidden), ids, wb, bits(swapped), bits(w2))
    m = omlp.compare(bf16_bits_to_f32(bits(got)), ref_bad)
    assert m["cosine"] < 0.99, m


def test_shared_mlp_oracle_matches_vllm_dense_swiglu(vllm_silu):
    """The fused shared-expert oracle (one MLP of intermediate n_shared * I) equals vLLM's
    MoE with a single expert that every token routes to with weight 1."""
    cfg = syn.CONFIGS["c4_shared"].with_tokens(32)
    sw13, sw2 = syn.make_shared_weights(cfg, 0)
    hidden = syn.make_hidden(cfg, 0)
    ids = np.zeros((cfg.tokens, 1), dtype=np.int32)
    w = np.ones((cfg.tokens, 1), dtype=np.float32)
    got = _vllm_moe(hidden, ids, w, sw13[None], sw2[None], 1)
    ref = omlp.shared_mlp(bits(hidden), bits(sw13), bits(sw2))
    m = omlp.compare(bf16_bits_to_f32(bits(got)), ref)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
