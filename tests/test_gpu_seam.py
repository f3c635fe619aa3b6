"""The seam custom ops on the GPU: router -> stage -> MLP through torch.ops.vllm equals the
layer's own call, and the shared-expert tuple ABI (C4, DeepSeek-V2-Lite-shaped) matches the
oracle for both halves."""

import numpy as np
import pytest
import torch

import vllm_ascend_hust_latchmoe_b200 as plugin
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits, build_layer
from vllm_ascend_hust_latchmoe_b200 import seam_ops
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _ok(actual, expected):
    m = omlp.compare(bf16_bits_to_f32(bits(actual)), expected)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m


@pytest.mark.parametrize("name,tokens,on_device", [("c1_decode", 4, False),
                                                   ("c2_prefill", 512, True),
                                                   ("c1_decode", 16, False)])
def test_seam_ops_equal_layer_forward(cuda, name, tokens, on_device):
    plugin.register()
    cfg = syn.CONFIGS[name].with_tokens(tokens)
    layer, rt, (w13, w2) = build_layer(cfg, store_on_device=on_device)
    layer_name = f"model.layers.0.mlp.experts.{name}.{tokens}"
    seam_ops.register_moe_layer(layer_name, layer)
    try:
        h = syn.make_hidden(cfg).to(cuda)
        lg = syn.make_router_logits(cfg).to(cuda)
        via_ops = seam_ops.seam_forward(layer_name, h, lg).clone()
        direct = layer.forward(h, lg).clone()
        torch.cuda.synchronize()
        layer.check_device_errors()
        assert torch.equal(via_ops, direct)
        wb, _, ids = orouter.route(lg.cpu().numpy(), cfg.top_k)
        _ok(via_ops, omlp.moe_layer(bits(h), ids, wb, bits(w13), bits(w2)))
        # explicit-scalar router op
        w_op, ids_op = torch.ops.vllm.moe_router(h, lg, cfg.top_k, False, True, None, None,
                                                 "softmax", 1.0, None, cfg.num_experts)
        assert np.array_equal(ids_op.cpu().numpy(), ids)
    finally:
        seam_ops.unregister_moe_layer(layer_name)


def test_moe_mlp_shared_tuple_matches_oracle(cuda):
    plugin.register()
    cfg = syn.CONFIGS["c4_shared"]
    layer, rt, (w13, w2) = build_layer(cfg)
    s13, s2 = syn.make_shared_weights(cfg)
    layer.set_shared_experts(s13, s2)
    layer_name = "model.layers.3.mlp.experts"
    seam_ops.register_moe_layer(layer_name, layer)
    try:
        h = syn.make_hidden(cfg).to(cuda)
        lg = syn.make_router_logits(cfg).to(cuda)
        w, ids = torch.ops.vllm.moe_router_indirect(h, lg, layer_name)
        torch.ops.vllm.moe_offload_stage(ids, layer.layer_id, cfg.num_experts, 0)
        shared_out, routed_out = torch.ops.vllm.moe_mlp_shared(h, lg, w, ids, None, None,
                                                               layer_name, -1)
        torch.cuda.synchronize()
        layer.check_device_errors()
        wb, _, ids_ref = orouter.route(lg.cpu().numpy(), cfg.top_k, renormalize=False)
        _ok(routed_out, omlp.moe_layer(bits(h), ids_ref, wb, bits(w13), bits(w2)))
        _ok(shared_out, omlp.shared_mlp(bits(h), bits(s13), bits(s2)))
        # a prefill-sized call runs the shared MLP on the tcgen05 path
        cfg_p = cfg.with_tokens(256)
        layer_p, _, _ = build_layer(cfg_p, experts=(w13, w2))
        layer_p.set_shared_experts(s13, s2)
        hp = syn.make_hidden(cfg_p, seed=5).to(cuda)
        sp = layer_p.shared_mlp(hp, 256)
        torch.cuda.synchronize()
        _ok(sp, omlp.shared_mlp(bits(hp), bits(s13), bits(s2)))
    finally:
        seam_ops.unregister_moe_layer(layer_name)
