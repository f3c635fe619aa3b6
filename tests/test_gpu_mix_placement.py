"""GPU parity of the fused mix-placement shared lane (DeepSeek-V2-Lite shape: 64 routed experts
top-6 plus 2 shared experts of I 1408 held in the slot bank's pinned suffix).

The router appends the shared ids 64, 65 with weight 1 to every token's top-k (bit-exact
against the oracle router plus that suffix); the shared pairs run on the pinned rows on every
path -- the slot bank, the HBM-resident tier (decode and the device wave plan), the staged
multi-wave prefill (once after the routed waves, never counted against the slots) and the
full-layer fallback -- and one combine sums all k + 2 pairs in order. Outputs against the
oracle layer over the 66-expert bank: max|a-e|/max|e| <= 1e-2 and cosine >= 0.9999.
"""

import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime

pytestmark = pytest.mark.gpu

CFG = syn.CONFIGS["c4_shared"]
E, NS = CFG.num_experts, CFG.num_shared


@pytest.fixture(scope="module")
def weights():
    return syn.make_expert_weights(CFG, 0, experts=E + NS)


def _layer(cuda, weights, *, tokens, store_on_device, full_layer=False):
    w13, w2 = weights
    rt = MoeOffloadRuntime(MoeOffloadConfig(
        enabled=True, num_slots=CFG.num_slots, async_load=True, b2_wave_prefill=True,
        graph_compatible_offload=True, b2_reference_full_layer=full_layer))
    rt.register_layer_for_fixed_slots(syn.ExpertLayer(0, w13, w2, shared=NS), slot_device=cuda,
                                      store_device=cuda if store_on_device else None)
    layer = SlotBankMoE(rt, 0, hidden_size=CFG.hidden, intermediate_size=CFG.intermediate,
                        num_experts=E, top_k=CFG.top_k, max_tokens=tokens,
                        renormalize=CFG.renormalize,
                        routed_scaling_factor=CFG.routed_scaling_factor,
                        scoring_func=CFG.scoring_func, num_expert_group=CFG.num_expert_group,
                        topk_group=CFG.topk_group, device=cuda)
    return layer, rt


def _oracle(hidden, logits, weights):
    wb, _, ids = orouter.route(logits.numpy(), CFG.top_k, renormalize=CFG.renormalize,
                               routed_scaling_factor=CFG.routed_scaling_factor,
                               scoring_func=CFG.scoring_func,
                               num_expert_group=CFG.num_expert_group, topk_group=CFG.topk_group)
    T = ids.shape[0]
    shared_ids = np.tile(np.arange(E, E + NS, dtype=np.int32), (T, 1))
    ids_all = np.concatenate([ids, shared_ids], axis=1)
    w_all = np.concatenate([wb, np.full((T, NS), 0x3F80, dtype=np.uint16)], axis=1)  # bf16 1.0
    w13, w2 = weights
    return ids_all, omlp.moe_layer(bits(hidden), ids_all, w_all, bits(w13), bits(w2))


@pytest.mark.parametrize("tokens,store_on_device,full_layer", [
    (4, False, False),     # decode, working set <= slots: slot-bank path, shared on pinned rows
    (64, False, False),    # decode overflow: routed waves, shared suffix once
    (64, True, False),     # HBM-resident tier, decode grouping by expert id
    (512, True, False),    # HBM-resident tier, device wave plan (tcgen05 path)
    (512, False, False),   # staged multi-wave prefill (tcgen05 path)
    (64, False, True),     # full-layer fallback
])
def test_fused_shared_lane_matches_oracle(cuda, weights, tokens, store_on_device, full_layer):
    layer, rt = _layer(cuda, weights, tokens=tokens, store_on_device=store_on_device,
                       full_layer=full_layer)
    assert layer.num_fused_shared == NS and layer.k == CFG.top_k + NS
    cfg = CFG.with_tokens(tokens)
    hidden = syn.make_hidden(cfg, seed=tokens)
    logits = syn.make_router_logits(cfg, seed=tokens)
    ids_ref, ref = _oracle(hidden, logits, weights)
    for _ in range(2):  # a second call reuses every buffer, slot and stage bank
        out = layer.forward(hidden.to(cuda), logits.to(cuda))
        torch.cuda.synchronize()
        layer.check_device_errors("mix placement")
        assert np.array_equal(layer.topk_ids[:tokens].cpu().numpy(), ids_ref)
        m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
        assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
    if not store_on_device and not full_layer and tokens > 4:
        waves = layer.last_waves.waves
        assert len(waves) >= 2 and all(e < E for w in waves for e in w)  # shared never staged
    bank = rt.slot_bank(0)
    assert bank.pinned_slot_ids == tuple(range(CFG.num_slots, CFG.num_slots + NS))


def test_seam_router_op_appends_the_shared_suffix(cuda, weights):
    from vllm_ascend_hust_latchmoe_b200 import register

    register()
    cfg = CFG.with_tokens(16)
    hidden = syn.make_hidden(cfg, seed=1).to(cuda)
    logits = syn.make_router_logits(cfg, seed=1)
    ids_ref, _ = _oracle(hidden.cpu(), logits, weights)
    w, ids = torch.ops.vllm.moe_router(hidden, logits.to(cuda), CFG.top_k, True,
                                       CFG.renormalize, CFG.topk_group, CFG.num_expert_group,
                                       CFG.scoring_func, CFG.routed_scaling_factor, None, E,
                                       True, NS)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), ids_ref)
    assert bool((w[:, CFG.top_k:].float() == 1.0).all())
