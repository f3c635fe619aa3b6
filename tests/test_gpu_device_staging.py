"""Decode staging decided on the device (lm_slot_plan) with missed experts read over PCIe by
the MLP itself (lm_moe_mlp_decode_offload): slot assignment bit-exact against the allocator
oracle (pinned to the reference's control plane), layer outputs within the bf16 tolerance,
write-through slot contents, the working-set-above-slots case, and CUDA-graph replay."""

import numpy as np
import pytest
import torch

from oracle import control as ocontrol
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, ExpertLayer, bits
from vllm_ascend_hust_latchmoe_b200 import _lib
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime

pytestmark = pytest.mark.gpu


def _device_layer(cfg, num_slots, max_tokens, cuda):
    w13, w2 = syn.make_expert_weights(cfg, 0)
    rt = MoeOffloadRuntime(MoeOffloadConfig(
        enabled=True, num_slots=num_slots, async_load=True, b2_wave_prefill=True,
        graph_compatible_offload=True, pin_host_memory=True, device_staging=True))
    rt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2), slot_device=cuda)
    layer = SlotBankMoE(rt, 0, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                        num_experts=cfg.num_experts, top_k=cfg.top_k, max_tokens=max_tokens,
                        renormalize=cfg.renormalize, device=cuda)
    return layer, rt, (w13, w2)


def _logits_for(cfg, sets, tokens):
    """Router logits whose top-k of token t is the expert set sets[t] (exact, by margin)."""
    lg = torch.randn(tokens, cfg.num_experts, generator=torch.Generator().manual_seed(1)) * 0.1
    for t, sel in enumerate(sets):
        lg[t, list(sel)] += 8.0 + torch.arange(len(sel), dtype=torch.float32) * 0.01
    return lg


def test_slot_plan_matches_allocator_oracle(cuda):
    """40 decode calls (2 tokens, top-8, locality 0.7) on 16 slots: every slot choice,
    miss and log2phy entry equals the oracle's; LRU evictions included."""
    E, S, k = 64, 16, 8
    cfg = syn.LayerConfig("plan", hidden=256, num_experts=E, top_k=k, intermediate=128,
                          num_slots=S, tokens=2)
    seqs = [syn.locality_topk_sequence(cfg, 40, 0.7, seed=s) for s in (3, 4)]
    owner = torch.full((S,), -1, dtype=torch.int32, device=cuda)
    last = torch.full((S,), -1, dtype=torch.int64, device=cuda)
    eslot = torch.full((E,), -1, dtype=torch.int32, device=cuda)
    step = torch.zeros(1, dtype=torch.int64, device=cuda)
    log2phy = torch.full((E,), -1, dtype=torch.int32, device=cuda)
    src = torch.full((E,), -1, dtype=torch.int32, device=cuda)
    hm = torch.zeros(2, dtype=torch.int64, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    alloc = ocontrol.SlotAllocator(S, E)
    hits = misses = 0
    for t in range(40):
        ids = torch.tensor([seqs[0][t], seqs[1][t]], dtype=torch.int32)
        active = tuple(sorted(set(ids.reshape(-1).tolist())))
        _lib.slot_plan(ids.to(cuda), E, owner, last, eslot, step, log2phy, src, hm, err)
        torch.cuda.synchronize()
        assert err.item() == 0
        exp = alloc.stage(active)
        got_src = src.cpu().numpy()
        got_slots = tuple(int(got_src[e]) & ~_lib.LM_SRC_MISS for e in active)
        got_miss = tuple(e for e in active if int(got_src[e]) & _lib.LM_SRC_MISS)
        assert got_slots == exp["active_slot_ids"], t
        assert got_miss == exp["misses"], t
        assert np.array_equal(log2phy.cpu().numpy()[list(active)], exp["log2phy"][list(active)])
        assert owner.cpu().tolist() == alloc.owner
        inactive = np.setdiff1d(np.arange(E), active)
        assert (got_src[inactive] == -1).all()
        hits += len(active) - len(got_miss)
        misses += len(got_miss)
    assert hm.cpu().tolist() == [hits, misses] and misses > S  # evictions happened


def test_device_staged_layer_matches_oracle_and_fills_slots(cuda):
    """Decode steps through the layer: outputs match the oracle and every slot holds exactly
    its expert's weights after the write-through (hits read them back next step)."""
    cfg = syn.CONFIGS["c1_decode"].with_tokens(4)
    layer, rt, (w13, w2) = _device_layer(cfg, num_slots=16, max_tokens=4, cuda=cuda)
    for step in range(5):
        hidden = syn.make_hidden(cfg, seed=step)
        logits = syn.make_router_logits(cfg, seed=step % 2)  # repeats: hits on later steps
        wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=cfg.renormalize)
        out = layer.forward(hidden.to(cuda), logits.to(cuda))
        torch.cuda.synchronize()
        layer.check_device_errors()
        ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
        m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
        assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, (step, m)
    owner = layer.slot_owner.cpu().tolist()
    bank = rt.slot_bank(0)
    store = rt.host_layer(0)
    for s, e in enumerate(owner):
        if e >= 0:
            assert torch.equal(bank.w13_slots[s].cpu(), store.w13[e])
            assert torch.equal(bank.w2_slots[s].cpu(), store.w2[e])
    hits, misses = layer.hit_miss.cpu().tolist()
    assert hits > 0 and misses > 0


def test_working_set_above_slots_reads_host_and_keeps_bank(cuda):
    """More active experts than slots: outputs still exact, the bank and its state unchanged
    (the reference runs waves there and leaves the main bank alone)."""
    cfg = syn.CONFIGS["c1_decode"].with_tokens(16)  # ~33 active experts
    layer, rt, (w13, w2) = _device_layer(cfg, num_slots=8, max_tokens=16, cuda=cuda)
    small = cfg.with_tokens(1)
    h1 = syn.make_hidden(small, seed=9)
    lg1 = syn.make_router_logits(small, seed=9)
    layer.forward(h1.to(cuda), lg1.to(cuda))  # fills 8 slots
    torch.cuda.synchronize()
    owner0 = layer.slot_owner.clone()
    w0 = rt.slot_bank(0).w13_slots.clone()
    hidden = syn.make_hidden(cfg)
    logits = syn.make_router_logits(cfg)
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=cfg.renormalize)
    assert len(np.unique(ids)) > 8
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors()
    ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
    m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
    assert torch.equal(layer.slot_owner, owner0)
    assert torch.equal(rt.slot_bank(0).w13_slots, w0)


def test_device_staged_decode_piece_replays_in_a_cuda_graph(cuda):
    """The whole decode MLP piece (plan, grouping, MLP, combine) captured once and replayed
    with new routing each step equals the eager oracle."""
    cfg = syn.CONFIGS["c1_decode"].with_tokens(2)
    layer, rt, (w13, w2) = _device_layer(cfg, num_slots=20, max_tokens=2, cuda=cuda)
    hidden = torch.zeros(2, cfg.hidden, dtype=torch.bfloat16, device=cuda)
    logits = torch.zeros(2, cfg.num_experts, dtype=torch.float32, device=cuda)
    layer.route(hidden, logits)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        layer.mlp_device(hidden, 2)  # library set-up outside the capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.route(hidden, logits)
        out = layer.mlp_device(hidden, 2)
    seqs = [syn.locality_topk_sequence(cfg, 12, 0.6, seed=s) for s in (7, 8)]
    for t in range(12):
        h = syn.make_hidden(cfg, seed=100 + t)
        lg = _logits_for(cfg, [seqs[0][t], seqs[1][t]], 2)
        hidden.copy_(h.to(cuda))
        logits.copy_(lg.to(cuda))
        g.replay()
        torch.cuda.synchronize()
        layer.check_device_errors()
        wb, _, ids = orouter.route(lg.numpy(), cfg.top_k, renormalize=cfg.renormalize)
        ref = omlp.moe_layer(bits(h), ids, wb, bits(w13), bits(w2))
        m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
        assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, (t, m)
    hits, misses = layer.hit_miss.tolist()
    assert hits > 0 and misses > 20  # slots reused and evicted across replays
