"""Expert-parallel exchange logic on CPU ranks (gloo, world sizes 2 and 4): routing -> group by owner
-> count/row/id all-to-all -> owner MLP -> reverse all-to-all -> combine in top-k order,
with the oracle supplying each compute step. Every rank's output must equal the
single-process oracle layer on that rank's tokens."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import control as oc
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32, f32_to_bf16_bits
from vllm_ascend_hust_latchmoe_b200.expert_parallel import (EPOps, ExpertParallelMoE,
                                                            balanced_expert_placement)

E, K, H, I, T = 16, 4, 64, 32, 24


def _data(rank):
    rng = np.random.default_rng(100 + rank)
    logits = (rng.standard_normal((T, E)) + np.linspace(2, -2, E)[None, :]).astype(np.float32)
    hidden = f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    wr = np.random.default_rng(7)
    w13 = f32_to_bf16_bits((wr.standard_normal((E, 2 * I, H)) * 0.1).astype(np.float32))
    w2 = f32_to_bf16_bits((wr.standard_normal((E, H, I)) * 0.1).astype(np.float32))
    return logits, hidden, w13, w2


def _bf16(bits):
    return torch.from_numpy(bf16_bits_to_f32(bits)).to(torch.bfloat16)


def _bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _oracle_ops(w13, w2, rank, per_rank):
    def route(logits):
        wb, _, ids = orouter.route(logits.numpy(), K)
        return _bf16(wb), torch.from_numpy(ids)

    def group_by_owner(ids, owner, G):
        off, p2r, r2p = oc.group_pairs(ids.numpy(), owner.numpy(), G)
        return torch.from_numpy(off), torch.from_numpy(p2r), torch.from_numpy(r2p)

    def gather_rows(hidden, rows, k):
        return hidden.index_select(0, (rows.long() // k))

    def expert_mlp(rows, local_ids):
        x = bf16_bits_to_f32(_bits(rows))
        out = np.zeros_like(x)
        for le in np.unique(local_ids.numpy()):
            sel = np.nonzero(local_ids.numpy() == le)[0]
            e = rank * per_rank + int(le)
            out[sel] = omlp.expert_mlp(x[sel], bf16_bits_to_f32(w13[e]), bf16_bits_to_f32(w2[e]))
        return torch.from_numpy(out).to(torch.bfloat16)

    def combine(back, p2r, w):
        y = bf16_bits_to_f32(_bits(back))[p2r.numpy()]
        return torch.from_numpy(omlp.combine(y, _bits(w))).to(torch.bfloat16)

    return EPOps(route, group_by_owner, gather_rows, expert_mlp, combine)


def _worker(rank, world, port, q, placed=False, rows_per_peer=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        logits, hidden, w13, w2 = _data(rank)
        if placed:
            # placement from a profiled sample (rank 0's routing), applied to the gate columns
            # and the expert bank; the layer's result must not change
            ids0 = orouter.route(_data(0)[0], K)[2]
            perm = np.asarray(balanced_expert_placement(np.bincount(ids0.reshape(-1),
                                                                    minlength=E), world))
            ep = ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, rank=rank,
                                   world_size=world, device="cpu",
                                   ops=_oracle_ops(w13[perm], w2[perm], rank, E // world))
            out = ep.forward(_bf16(hidden), torch.from_numpy(np.ascontiguousarray(logits[:, perm])))
        else:
            ep = ExpertParallelMoE(num_experts=E, top_k=K, hidden_size=H, rank=rank,
                                   world_size=world, ops=_oracle_ops(w13, w2, rank, E // world),
                                   device="cpu", nccl_rows_per_peer=rows_per_peer)
            out = ep.forward(_bf16(hidden), torch.from_numpy(logits))
            if rows_per_peer is not None:
                try:
                    ep.check_exchange_errors()
                    overflow = False
                except RuntimeError as exc:
                    overflow = "nccl_rows_per_peer" in str(exc)
                q.put((rank, overflow, ep.stats.send_rows, ep.stats.recv_rows,
                       list(ep.owned_experts())))
                if overflow:
                    return
        wb, _, ids = orouter.route(logits, K)
        ref = omlp.moe_layer(hidden, ids, wb, w13, w2)
        m = omlp.compare(bf16_bits_to_f32(_bits(out)), ref)
        if rows_per_peer is None:
            q.put((rank, m, ep.stats.send_rows, ep.stats.recv_rows, list(ep.owned_experts())))
        else:
            q.put((rank, m, 0, 0, []))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,placed", [(2, False), (4, False), (4, True)])
def test_ep_exchange_matches_single_process_oracle(world, placed):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, placed)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    per = E // world
    assert [r[4] for r in results] == [list(range(r * per, (r + 1) * per)) for r in range(world)]
    assert sum(r[2] for r in results) == sum(r[3] for r in results) == world * T * K
    for rank, m, *_ in results:
        assert m["max_rel_err"] <= 1e-2 and m["cosine"] >= 0.9999, (rank, m)


@pytest.mark.parametrize("world", [2, 4])
def test_ep_fixed_splits_match_oracle_and_report_overflow(world):
    """NCCL exchange with fixed-size blocks (no host-read counts): with room for every pair the
    output equals the oracle; with blocks smaller than some owner's share the step reports the
    overflow instead of passing it silently."""
    ctx = mp.get_context("spawn")
    for rows, expect_overflow in ((T * K, False), (3, True)):
        q = ctx.Queue()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, q, False, rows))
                 for r in range(world)]
        for p in procs:
            p.start()
        results = [q.get(timeout=120) for _ in range(2 * world if not expect_overflow else world)]
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
        flags = [r for r in results if isinstance(r[1], bool)]
        assert len(flags) == world
        if expect_overflow:
            assert any(f[1] for f in flags)
            continue
        assert not any(f[1] for f in flags)
        assert sum(f[3] for f in flags) == world * world * rows  # fixed blocks
        for rank, m, *_ in results:
            if isinstance(m, dict):
                assert m["max_rel_err"] <= 1e-2 and m["cosine"] >= 0.9999, (rank, m)


def test_balanced_placement_is_a_permutation_with_even_load():
    rng = np.random.default_rng(0)
    load = np.floor(4000.0 / np.arange(1, 129) ** 1.1)[rng.permutation(128)]
    for world in (1, 2, 4, 8):
        perm = balanced_expert_placement(load, world)
        assert sorted(perm) == list(range(128))
        per = 128 // world
        ranks = np.asarray(load)[perm].reshape(world, per).sum(1)
        # within a few percent of the lower bound (the mean, or the heaviest single expert)
        assert ranks.max() <= 1.08 * max(ranks.mean(), load.max()), (world, ranks)
        contiguous = np.asarray(load).reshape(world, per).sum(1)
        assert ranks.max() <= contiguous.max()
        for r in range(world):  # each rank's experts in id order
            assert perm[r * per:(r + 1) * per] == sorted(perm[r * per:(r + 1) * per])
    assert balanced_expert_placement([5, 5, 5, 5], 2) == [0, 2, 1, 3]  # ties: lowest rank
    with pytest.raises(ValueError):
        balanced_expert_placement(load[:10], 4)
