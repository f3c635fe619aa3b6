"""The peer exchange kernels on one GPU (world size 1: the rank is its own only owner).

Dispatch, receive, signal and combine run in stream order, so every flag a wait reads was
raised by an earlier launch: nothing waits on a concurrently running kernel. The combine of
the rows sent back unchanged equals the oracle's top-k combine. A combine whose owners never
signal (an epoch nobody raised) gives up after its bounded wait, reports
LM_DEVERR_WAIT_TIMEOUT and writes zero rows instead of reading the owners' areas.
"""

import numpy as np
import pytest
import torch

from oracle import mlp as omlp
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits
from vllm_ascend_hust_latchmoe_b200 import _lib
from vllm_ascend_hust_latchmoe_b200.expert_parallel import _DevicePtrArray

pytestmark = pytest.mark.gpu

T, K, E, H = 16, 4, 8, 256


def _setup(cuda):
    cap = T * K
    region = _lib.ep_region_alloc(_lib.ep_region_bytes(1, cap, H))
    peers = torch.tensor([region], dtype=torch.int64, device=cuda)
    off = _lib.ep_out_rows_offset(1, cap, H)
    out_rows = torch.as_tensor(_DevicePtrArray(region + off, (cap, H), "<i2"),
                               device=cuda).view(torch.bfloat16)
    rng = np.random.default_rng(3)
    ids_np = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    w = torch.from_numpy(rng.random((T, K)).astype(np.float32)).to(torch.bfloat16).to(cuda)
    ids = torch.from_numpy(ids_np).to(cuda)
    hidden = torch.randn(T, H, device=cuda).to(torch.bfloat16)
    owner = torch.zeros(E, dtype=torch.int32, device=cuda)
    offsets = torch.empty(2, dtype=torch.int32, device=cuda)
    p2r = torch.empty(cap, dtype=torch.int32, device=cuda)
    r2p = torch.empty(cap, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_lib.build_groups_scratch_elems(cap, 1), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.build_groups(ids, E, owner, 1, offsets, p2r, r2p, scratch, err)
    return dict(cap=cap, region=region, peers=peers, out_rows=out_rows, ids=ids, ids_np=ids_np,
                w=w, hidden=hidden, offsets=offsets, p2r=p2r, err=err)


def test_single_rank_exchange_round_trip_and_timeout(cuda):
    c = _setup(cuda)
    cap, err = c["cap"], c["err"]
    rows = torch.empty(cap, H, dtype=torch.bfloat16, device=cuda)
    rids = torch.empty(cap, dtype=torch.int32, device=cuda)
    total = torch.zeros(1, dtype=torch.int32, device=cuda)
    done = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
    try:
        tok_slot = torch.empty(T, dtype=torch.int32, device=cuda)
        tok_count = torch.zeros(1, dtype=torch.int32, device=cuda)
        for epoch in (1, 2):  # a second call reuses every area; epoch 2 dispatches per token
            if epoch == 1:
                _lib.ep_dispatch(c["hidden"], c["ids"], E, c["p2r"], c["offsets"], 0, 1,
                                 c["peers"], cap, epoch, done, err)
            else:
                _lib.ep_dispatch_tokens(c["hidden"], c["ids"], E, c["p2r"], c["offsets"], 0, 1,
                                        c["peers"], cap, epoch, tok_slot, tok_count, done, err)
            _lib.ep_receive(c["region"], 1, cap, H, epoch, rows, rids, total, err)
            c["out_rows"].copy_(rows)  # the "expert" returns each row unchanged
            _lib.ep_signal_outputs(c["peers"], 0, 1, cap, H, epoch)
            out.fill_(7.0)
            _lib.ep_combine(c["ids"], c["w"], E, c["p2r"], c["offsets"], 0, 1, c["peers"],
                            c["region"], cap, epoch, out, err)
            torch.cuda.synchronize()
            assert int(err.item()) == 0 and int(total.item()) == T * K
            if epoch == 2:  # one owner: every token once, in token order
                assert int(tok_count.item()) == T
                assert tok_slot.tolist() == list(range(T))
            pairs = np.repeat(bf16_bits_to_f32(bits(c["hidden"])), K, axis=0)
            ref = omlp.combine(pairs, bits(c["w"]))
            m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
            assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
        # epoch 3 was never signalled: the bounded wait gives up, nothing is read
        out.fill_(7.0)
        _lib.ep_combine(c["ids"], c["w"], E, c["p2r"], c["offsets"], 0, 1, c["peers"],
                        c["region"], cap, 3, out, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 3  # LM_DEVERR_WAIT_TIMEOUT
        assert bool((out.float() == 0).all())
    finally:
        torch.cuda.synchronize()
        c["out_rows"] = None
        _lib.ep_region_free(c["region"])


@pytest.mark.parametrize("dedupe,push", [(False, False), (True, False), (True, True)])
def test_single_rank_gather_path_matches_oracle(cuda, dedupe, push):
    """The owner path without row copies: index-only receive, the grouped MLP gathering its
    rows from the receive area, outputs left in grouped order with the pair-row table, and the
    combine reading through that table -- against the oracle layer, twice in a row. With
    ``dedupe`` each token row is stored once and all its pairs read that one row; with
    ``push`` the MLP stores every output row into the source's own area (row pointers from
    ``lm_ep_output_row_ptrs``) and the combine reads only that area."""
    from oracle import router as orouter
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import build_rank_layer

    T2, K2, E2, H2, I2 = 32, 4, 8, 256, 128
    cap = T2 * K2
    cfg = syn.LayerConfig("g", hidden=H2, num_experts=E2, top_k=K2, intermediate=I2,
                          num_slots=E2, tokens=T2)
    w13, w2 = syn.make_expert_weights(cfg, seed=9)
    layer = build_rank_layer(w13_owned=w13.to(cuda), w2_owned=w2.to(cuda), rank=0, device=cuda,
                             max_rows=cap, num_slots=E2, store_on_device=True)
    region = _lib.ep_region_alloc(_lib.ep_region_bytes(1, cap, H2))
    try:
        peers = torch.tensor([region], dtype=torch.int64, device=cuda)

        def view(off, shape, ts):
            return torch.as_tensor(_DevicePtrArray(region + off, shape, ts), device=cuda)

        recv_rows = view(_lib.ep_recv_rows_offset(1, cap, H2), (cap, H2), "<i2").view(torch.bfloat16)
        out_rows = view(_lib.ep_out_rows_offset(1, cap, H2), (cap, H2), "<i2").view(torch.bfloat16)
        pair_rows = view(_lib.ep_pair_rows_offset(1, cap, H2), (cap,), "<i4")
        slots = torch.empty(cap, dtype=torch.int32, device=cuda)
        rids = torch.empty(cap, dtype=torch.int32, device=cuda)
        total = torch.zeros(1, dtype=torch.int32, device=cuda)
        done = torch.zeros(1, dtype=torch.int32, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        owner = torch.zeros(E2, dtype=torch.int32, device=cuda)
        offsets = torch.empty(2, dtype=torch.int32, device=cuda)
        p2r = torch.empty(cap, dtype=torch.int32, device=cuda)
        r2p = torch.empty(cap, dtype=torch.int32, device=cuda)
        scratch = torch.empty(_lib.build_groups_scratch_elems(cap, 1), dtype=torch.int32,
                              device=cuda)
        out = torch.empty(T2, H2, dtype=torch.bfloat16, device=cuda)
        tok_slot = torch.empty(T2, dtype=torch.int32, device=cuda)
        tok_count = torch.zeros(1, dtype=torch.int32, device=cuda)
        for epoch, seed in ((1, 1), (2, 2)):
            hidden = syn.make_hidden(cfg, seed=seed)
            wb, _, ids_np = orouter.route(syn.make_router_logits(cfg, seed=seed).numpy(), K2)
            ids = torch.from_numpy(ids_np).to(cuda)
            w = torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16).to(cuda)
            h = hidden.to(cuda)
            _lib.build_groups(ids, E2, owner, 1, offsets, p2r, r2p, scratch, err)
            if dedupe:
                _lib.ep_dispatch_tokens(h, ids, E2, p2r, offsets, 0, 1, peers, cap, epoch,
                                        tok_slot, tok_count, done, err)
            else:
                _lib.ep_dispatch(h, ids, E2, p2r, offsets, 0, 1, peers, cap, epoch, done, err)
            _lib.ep_receive_index(region, 1, cap, H2, epoch, slots, rids, total, err)
            if push:
                def row_ptrs(row_to_pair, count, ptrs):
                    _lib.ep_output_row_ptrs(region, 1, cap, H2, 0, peers, row_to_pair, count,
                                            ptrs.shape[0], ptrs, err)

                out_rows.fill_(7.0)  # every pair's row must be rewritten
                layer.mlp_rows_gather_push(recv_rows, slots, rids, total, row_ptrs)
            else:
                layer.mlp_rows_gather_count(recv_rows, slots, rids, total, pair_rows, out_rows)
            _lib.ep_signal_outputs(peers, 0, 1, cap, H2, epoch)
            combine = _lib.ep_combine_local if push else _lib.ep_combine
            combine(ids, w, E2, p2r, offsets, 0, 1, peers, region, cap, epoch, out, err)
            torch.cuda.synchronize()
            assert int(err.item()) == 0 and int(total.item()) == cap
            if dedupe:  # the token rows sit once each at the head of the receive area
                assert int(tok_count.item()) == T2
                assert torch.equal(recv_rows[:T2], h)
            layer.check_device_errors("gather path")
            ref = omlp.moe_layer(bits(hidden), ids_np, wb, bits(w13), bits(w2))
            m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
            assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
    finally:
        torch.cuda.synchronize()
        _lib.ep_region_free(region)


def test_single_rank_device_epoch_step_replays_from_a_graph(cuda):
    """Epoch 0: every exchange kernel reads the call counter that lm_ep_advance_epoch raised
    on the device, so the whole step (advance, dispatch by token, index-only receive, gather
    MLP pushing its outputs, signal, local combine) captured once as a CUDA graph replays as a
    new call each time, with the oracle's output."""
    from oracle import router as orouter
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import build_rank_layer

    T2, K2, E2, H2, I2 = 32, 4, 8, 256, 128
    cap = T2 * K2
    cfg = syn.LayerConfig("g", hidden=H2, num_experts=E2, top_k=K2, intermediate=I2,
                          num_slots=E2, tokens=T2)
    w13, w2 = syn.make_expert_weights(cfg, seed=9)
    layer = build_rank_layer(w13_owned=w13.to(cuda), w2_owned=w2.to(cuda), rank=0, device=cuda,
                             max_rows=cap, num_slots=E2, store_on_device=True)
    region = _lib.ep_region_alloc(_lib.ep_region_bytes(1, cap, H2))
    g = None
    try:
        peers = torch.tensor([region], dtype=torch.int64, device=cuda)
        recv_rows = torch.as_tensor(_DevicePtrArray(
            region + _lib.ep_recv_rows_offset(1, cap, H2), (cap, H2), "<i2"),
            device=cuda).view(torch.bfloat16)
        slots = torch.empty(cap, dtype=torch.int32, device=cuda)
        rids = torch.empty(cap, dtype=torch.int32, device=cuda)
        total = torch.zeros(1, dtype=torch.int32, device=cuda)
        done = torch.zeros(1, dtype=torch.int32, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        owner = torch.zeros(E2, dtype=torch.int32, device=cuda)
        offsets = torch.empty(2, dtype=torch.int32, device=cuda)
        p2r = torch.empty(cap, dtype=torch.int32, device=cuda)
        r2p = torch.empty(cap, dtype=torch.int32, device=cuda)
        scratch = torch.empty(_lib.build_groups_scratch_elems(cap, 1), dtype=torch.int32,
                              device=cuda)
        tok_slot = torch.empty(T2, dtype=torch.int32, device=cuda)
        tok_count = torch.zeros(1, dtype=torch.int32, device=cuda)
        out = torch.empty(T2, H2, dtype=torch.bfloat16, device=cuda)
        hidden = syn.make_hidden(cfg, seed=4)
        wb, _, ids_np = orouter.route(syn.make_router_logits(cfg, seed=4).numpy(), K2)
        ids = torch.from_numpy(ids_np).to(cuda)
        w = torch.from_numpy(wb.view(np.int16)).view(torch.bfloat16).to(cuda)
        h = hidden.to(cuda)

        def row_ptrs(row_to_pair, count, ptrs):
            _lib.ep_output_row_ptrs(region, 1, cap, H2, 0, peers, row_to_pair, count,
                                    ptrs.shape[0], ptrs, err)

        def step():
            _lib.ep_advance_epoch(region, 1, cap, H2)
            _lib.build_groups(ids, E2, owner, 1, offsets, p2r, r2p, scratch, err)
            _lib.ep_dispatch_tokens(h, ids, E2, p2r, offsets, 0, 1, peers, cap, 0, tok_slot,
                                    tok_count, done, err)
            _lib.ep_receive_index(region, 1, cap, H2, 0, slots, rids, total, err)
            layer.mlp_rows_gather_push(recv_rows, slots, rids, total, row_ptrs)
            _lib.ep_signal_outputs(peers, 0, 1, cap, H2, 0)
            _lib.ep_combine_local(ids, w, E2, p2r, offsets, 0, 1, peers, region, cap, 0, out,
                                  err)

        ref = omlp.moe_layer(bits(hidden), ids_np, wb, bits(w13), bits(w2))
        for _ in range(2):  # eager calls, epochs 1 and 2
            step()
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
            assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(3):  # epochs 3, 4, 5: each replay waits for its own flags
            out.fill_(7.0)
            g.replay()
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            layer.check_device_errors("device epoch graph")
            m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
            assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
    finally:
        torch.cuda.synchronize()
        del g
        _lib.ep_region_free(region)

