"""Piecewise CUDA-graph decode with the eager staging seam: replaying the captured pieces
gives the same tokens and hidden state as running the same pieces eagerly, while
offloaded layers stage their experts between pieces."""

import pytest
import torch

from vllm_ascend_hust_latchmoe_b200.decode_harness import DecoderShape, SyntheticMoEDecoder

pytestmark = pytest.mark.gpu

TINY = DecoderShape(layers=4, hidden=256, heads=2, kv_heads=1, head_dim=128, experts=16,
                    top_k=4, intermediate=128, vocab=512, num_slots=6, prompt=32, max_new=16)


def test_graph_replay_matches_eager(cuda):
    a = SyntheticMoEDecoder(TINY, offloaded_layers=(1, 3), device=cuda, seed=7,
                            teacher_forcing=True)
    b = SyntheticMoEDecoder(TINY, offloaded_layers=(1, 3), device=cuda, seed=7,
                            teacher_forcing=True)
    assert a.capture() == 3  # two stage seams -> three pieces
    a.reset_position()
    b.reset_position()
    for t in range(12):
        a.step(t)
        b.step_eager(t)
        torch.cuda.synchronize()
        for la, lb in zip(a.moe, b.moe):  # same routing and, for offloaded layers, same slots
            assert torch.equal(la.topk_ids[:1], lb.topk_ids[:1]), t
        for i in (1, 3):
            assert torch.equal(a.runtime.log2phy_buffer(i), b.runtime.log2phy_buffer(i)), t
        # hidden state after the last layer (before the next token's embedding replaced x)
        torch.testing.assert_close(a.h2.float(), b.h2.float(), rtol=2e-2, atol=2e-2)
    for layer in a.moe + b.moe:
        layer.check_device_errors()
    st = a.runtime.stage_stats
    assert st["misses"] > 0 and st["h2d_bytes"] > 0


def test_tpot_report_tiny(cuda):
    d = SyntheticMoEDecoder(TINY, offloaded_layers=(0, 2), device=cuda, seed=3)
    rep = d.run(steps=12, warmup=2)
    assert rep.graphs == 3 and rep.tpot_ms_p50 > 0 and rep.slot_hit_rate is not None
    with pytest.raises(ValueError):
        d.run(steps=TINY.max_new + 1)


def test_device_staged_decoder_is_one_graph_and_matches_host_staging(cuda):
    """Device staging: no stage seam, a token is one captured graph; it takes the same slot
    decisions as the host-staged decoder (log2phy equal every step) and the same hidden
    state."""
    a = SyntheticMoEDecoder(TINY, offloaded_layers=(1, 3), device=cuda, seed=7,
                            teacher_forcing=True, device_staging=True)
    b = SyntheticMoEDecoder(TINY, offloaded_layers=(1, 3), device=cuda, seed=7,
                            teacher_forcing=True)
    assert a.capture() == 1
    a.reset_position()
    b.reset_position()
    for t in range(12):
        a.step(t)
        b.step_eager(t)
        torch.cuda.synchronize()
        for la, lb in zip(a.moe, b.moe):
            assert torch.equal(la.topk_ids[:1], lb.topk_ids[:1]), t
        for i in (1, 3):
            assert torch.equal(a.runtime.log2phy_buffer(i), b.runtime.log2phy_buffer(i)), t
        torch.testing.assert_close(a.h2.float(), b.h2.float(), rtol=2e-2, atol=2e-2)
    for layer in a.moe + b.moe:
        layer.check_device_errors()
    rep = a.run(steps=8, warmup=2)
    assert rep.graphs == 1 and rep.tpot_ms_p50 > 0 and rep.slot_hit_rate is not None


def test_moe_share_after_a_full_run(cuda):
    """The MoE share of a token (each layer's attention and MoE piece as their own graphs):
    measured right after a run that used the whole KV cache (it starts again from the first
    generated position), between 0 and 1, and refused for a host-staged decoder."""
    d = SyntheticMoEDecoder(TINY, offloaded_layers=(1, 3), device=cuda, seed=5,
                            device_staging=True)
    d.run(steps=TINY.max_new, warmup=2)
    share = d.moe_share(steps=8, warmup=2)
    assert 0.0 < share["moe_share"] < 1.0 and share["pieces_per_token"] == 2 * TINY.layers + 1
    assert share["moe_ms_per_token_p50"] > 0
    for layer in d.moe:
        layer.check_device_errors()
    with pytest.raises(ValueError):
        d.moe_share(steps=TINY.max_new)
    host = SyntheticMoEDecoder(TINY, offloaded_layers=(1,), device=cuda, seed=5)
    with pytest.raises(ValueError):
        host.moe_share(steps=4, warmup=1)
