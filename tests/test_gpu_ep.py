"""Expert-parallel layer on 2 GPUs: each rank owns half of the experts in its own slot bank
(pinned host store, staged, or HBM-resident) and the outputs match the single-GPU oracle,
with the exchange over NCCL or over peer memory (the library's dispatch / combine kernels,
the dispatch per token or per routed pair).
Skipped with fewer than 2 GPUs."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H, I, T, S = 32, 4, 2048, 768, 48, 8


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, store_on_device, transport, q):
    import datetime

    import torch.distributed as dist

    from oracle import mlp as omlp
    from oracle import router as orouter
    from oracle.bf16 import bf16_bits_to_f32
    from tests.helpers import bits
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import (ExpertParallelMoE, PeerExchange,
                                                                build_rank_layer, cuda_ops)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = syn.LayerConfig("ep", hidden=H, num_experts=E, top_k=K, intermediate=I,
                              num_slots=S, tokens=T)
        w13, w2 = syn.make_expert_weights(cfg, seed=1)
        per = E // world
        local = build_rank_layer(w13_owned=w13[rank * per:(rank + 1) * per],
                                 w2_owned=w2[rank * per:(rank + 1) * per], rank=rank,
                                 device=dev, max_rows=world * T * K, num_slots=S,
                                 store_on_device=store_on_device)
        exchange = None
        if transport.startswith("peer"):
            exchange = PeerExchange(world_size=world, rank=rank, max_tokens=T, top_k=K,
                                    hidden_size=H, device=dev,
                                    device_epoch=transport == "peer_graph")
        ep = ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, rank=rank,
                               world_size=world, device=dev, exchange=exchange,
                               dedupe_dispatch=transport in ("peer", "peer_pull", "peer_graph"),
                               push_outputs=transport in ("peer", "peer_graph"),
                               nccl_rows_per_peer=T * K if transport == "nccl_fixed" else None,
                               ops=cuda_ops(local, num_experts=E, top_k=K, max_tokens=T))
        # a call with other routing first: the checked call reuses every area and flag
        ep.forward(syn.make_hidden(cfg, seed=30 + rank).to(dev),
                   syn.make_router_logits(cfg, seed=30 + rank).to(dev))
        hidden = syn.make_hidden(cfg, seed=10 + rank)
        logits = syn.make_router_logits(cfg, seed=10 + rank)
        h_dev, lg_dev = hidden.to(dev), logits.to(dev)
        for _ in range(2):
            out = ep.forward(h_dev, lg_dev)
        graph = None
        if transport == "peer_graph":  # the step captured once, replayed as new calls
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                out = ep.forward(h_dev, lg_dev)
            for _ in range(2):
                graph.replay()
        torch.cuda.synchronize()
        local.check_device_errors("ep")
        ep.check_exchange_errors()
        if exchange is not None:
            out = out.clone()
            del graph
            exchange.close()
        wb, _, ids = orouter.route(logits.numpy(), K)
        ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
        m = omlp.compare(bf16_bits_to_f32(bits(out)), ref)
        dist.barrier()
        q.put((rank, m, ep.stats.bytes_sent))
    except Exception as exc:  # report instead of hanging the peer
        q.put((rank, {"error": repr(exc)}, 0))
        raise
    finally:
        dist.destroy_process_group()


# "peer": token-deduplicated dispatch, owners push outputs into the sources' memory;
# "peer_pull": the same dispatch, sources read the outputs from the owners;
# "peer_pairs": one row per routed pair, outputs read from the owners;
# "peer_graph": as "peer" with the epoch on the device, the step replayed from a CUDA graph
# "nccl_fixed": fixed-size all-to-all blocks, counts never read on the host
@pytest.mark.parametrize("transport", ["nccl", "nccl_fixed", "peer", "peer_pull", "peer_pairs",
                                       "peer_graph"])
@pytest.mark.parametrize("store_on_device", [False, True])
def test_ep_two_gpus_matches_oracle(store_on_device, transport):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if transport == "peer_graph" and not store_on_device:
        pytest.skip("a staged store reads its received row count on the host: not capturable")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, store_on_device, transport, q))
             for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, m, sent in results:
        assert "error" not in m, m
        assert m["max_rel_err"] <= 1e-2 and m["cosine"] >= 0.9999, (rank, m)
        assert sent > 0
    assert all(p.exitcode == 0 for p in procs)


def _edge_worker(rank, world, port, case, q):
    """Peer exchange (dispatch by token, outputs pushed by the owners) on edge routings:
    every pair owned by rank 0 (rank 1 receives nothing), one token per rank, and a rank
    with no tokens at all."""
    import datetime

    import torch.distributed as dist

    from oracle import mlp as omlp
    from oracle import router as orouter
    from oracle.bf16 import bf16_bits_to_f32
    from tests.helpers import bits
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import (ExpertParallelMoE, PeerExchange,
                                                                build_rank_layer, cuda_ops)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = syn.LayerConfig("ep", hidden=H, num_experts=E, top_k=K, intermediate=I,
                              num_slots=S, tokens=T)
        w13, w2 = syn.make_expert_weights(cfg, seed=1)
        per = E // world
        local = build_rank_layer(w13_owned=w13[rank * per:(rank + 1) * per],
                                 w2_owned=w2[rank * per:(rank + 1) * per], rank=rank,
                                 device=dev, max_rows=world * T * K, num_slots=S,
                                 store_on_device=True)
        exchange = PeerExchange(world_size=world, rank=rank, max_tokens=T, top_k=K,
                                hidden_size=H, device=dev)
        ep = ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, rank=rank,
                               world_size=world, device=dev, exchange=exchange,
                               ops=cuda_ops(local, num_experts=E, top_k=K, max_tokens=T))
        n = {"one_owner": T, "single_token": 1, "empty_rank": 0 if rank == 1 else T}[case]
        hidden = syn.make_hidden(cfg, seed=40 + rank)[:n].contiguous()
        logits = syn.make_router_logits(cfg, seed=40 + rank)[:n].contiguous()
        if case == "one_owner":
            logits[:, per:] -= 100.0  # every token's top-k among rank 0's experts
        outs = [ep.forward(hidden.to(dev), logits.to(dev)).clone() for _ in range(2)]
        torch.cuda.synchronize()
        local.check_device_errors("ep edge")
        ep.check_exchange_errors()
        received = int(exchange.total.item())
        exchange.close()
        m = {"max_rel_err": 0.0, "cosine": 1.0}
        if n:
            wb, _, ids = orouter.route(logits.numpy(), K)
            ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
            m = omlp.compare(bf16_bits_to_f32(bits(outs[1])), ref)
            assert torch.equal(outs[0], outs[1])
        dist.barrier()
        q.put((rank, m, received))
    except Exception as exc:  # report instead of hanging the peer
        q.put((rank, {"error": repr(exc)}, -1))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["one_owner", "single_token", "empty_rank"])
def test_ep_two_gpus_edge_routings(case):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_edge_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, m, _ in results:
        assert "error" not in m, m
        assert m["max_rel_err"] <= 1e-2 and m["cosine"] >= 0.9999, (rank, m)
    if case == "one_owner":  # rank 0 owns every pair of both ranks, rank 1 none
        assert results[0][2] == 2 * T * K and results[1][2] == 0
    if case == "empty_rank":
        assert results[0][2] + results[1][2] == T * K
    assert all(p.exitcode == 0 for p in procs)
