"""The torch fp32 layer restatement that ``bench.py`` checks its timed outputs with agrees
with the numpy oracle (so a green bench check means what a green parity test means)."""

import numpy as np
import torch

import bench
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn


def test_torch_layer_reference_matches_oracle():
    cfg = syn.LayerConfig("t", hidden=512, num_experts=16, top_k=4, intermediate=256,
                          num_slots=8, tokens=24)
    w13, w2 = syn.make_expert_weights(cfg, 1)
    hidden = syn.make_hidden(cfg, 1)
    logits = syn.make_router_logits(cfg, 1)
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=True)
    ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
    w_t = torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16)
    got = bench.torch_layer_reference(hidden, torch.from_numpy(ids), w_t, lambda e: w13[e],
                                      lambda e: w2[e])
    m = omlp.compare(bf16_bits_to_f32(bits(got)), ref)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
    m2 = bench.compare_outputs(got, torch.from_numpy(ref))
    assert abs(m2["max_rel_err"] - m["max_rel_err"]) < 1e-9


def test_torch_route_reference_matches_oracle_router():
    cfg = syn.CONFIGS["c5_ep"].with_tokens(64)
    logits = syn.make_router_logits(cfg, 0)
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=True)
    w_t, ids_t = bench.torch_route_reference(logits, cfg.top_k)
    assert np.array_equal(ids_t.numpy(), ids)
    assert np.array_equal(bits(w_t), wb)
