"""Expert-partitioned slot-bank MoE layer across the GPUs of one node (NCCL over NVLink).

The reference runs on one NPU and rejects every parallel mode
(``patches/patch_fused_moe.py:4898-4914``); this module is the B200 extension its scope
asks for. Experts are owned in contiguous blocks (``owner(e) = e // (E / G)``); each rank
keeps its own slot bank and pinned host store for the experts it owns. One layer call:

1. route the rank's tokens (``lm_route_topk``);
2. group the routed pairs by owner rank with the same stable grouping kernel the slot
   remap uses (``lm_build_groups`` with expert -> owner), gather the rows
   (``lm_permute_rows``) and the owner-local expert ids;
3. exchange per-destination counts (``all_to_all_single`` of G int64), then rows and ids
   (``all_to_all_single`` with those splits) -- the dispatch;
4. run the owner's slot-bank MLP on the received rows (top-1, unit weight: staging, waves
   and kernels exactly as a single-GPU layer);
5. send the rows back with the reverse splits -- the combine exchange -- and reduce them in
   the original top-k order with the router weights (``lm_moe_combine``, fp32).

Remote rows always land in this GPU's buffers before any kernel reads them (NCCL copies);
no kernel reads peer memory and no TMA multicast is used.

The compute steps are injectable (``ops``) so the exchange bookkeeping can be exercised on
CPU ranks with gloo against the oracle; the default ``ops`` are the CUDA kernels.

Two transports carry the exchange. ``"nccl"``: ``all_to_all_single`` of counts, rows and ids
and back (the collective library; one host sync for the counts). ``"peer"`` (a
:class:`PeerExchange`): the library's own kernels over peer memory mapped with CUDA IPC.
``lm_ep_dispatch_tokens`` stores each token's row once into every owner that holds any of
its experts (a token routed to 8 experts on 3 ranks crosses NVLink 3 times, not 8) and each
pair's owner-local id and receive-row index beside it (``lm_ep_dispatch``, the per-pair form,
stays selectable); the owner reads its rows through those indices, and ``lm_ep_combine``
reads every pair's output row from its owner and reduces it in the original top-k order
(no return collective). With an HBM-resident local store the owner's MLP takes the received
row count on the device (grouping, gather and combine read it there), so a peer step has no
host synchronisation; a staged local store reads the count once on the host to stage its
experts.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

from . import _lib
from .layer import DECODE_MAX_TOKENS


def balanced_expert_placement(expert_load, world_size: int) -> list[int]:
    """Expert placement over ``world_size`` ranks with E / world_size experts each, balancing
    the expected routed pairs per rank (longest processing time first): experts in order of
    (-load, id), each to the rank with the least load so far that still has room (lowest rank
    on a tie); each rank's experts sorted by id. Returns ``perm`` with ``perm[r * per + i]``
    the original id of rank r's i-th expert.

    The layer keeps contiguous ownership (owner = placed id // per); a placement is applied
    at load time by permuting the router's gate rows (logit columns) and the expert bank with
    ``perm``, which leaves the layer's arithmetic unchanged. Under Zipf-skewed routing,
    contiguous blocks of the original ids leave one rank with several hot experts (about 3x
    the mean load at 8 ranks on the Qwen3-30B-A3B-shaped layer); the placement evens it out.
    ``expert_load`` is a profiled per-expert pair count (or any expected load)."""
    load = [float(x) for x in expert_load]
    E, G = len(load), int(world_size)
    if G <= 0 or E % G != 0:
        raise ValueError(f"{E} experts do not split evenly over {G} ranks")
    per = E // G
    rank_load = [0.0] * G
    members: list[list[int]] = [[] for _ in range(G)]
    for e in sorted(range(E), key=lambda x: (-load[x], x)):
        r = min((r for r in range(G) if len(members[r]) < per), key=lambda r: (rank_load[r], r))
        members[r].append(e)
        rank_load[r] += load[e]
    return [e for r in range(G) for e in sorted(members[r])]


@dataclass
class EPStats:
    send_rows: int = 0
    recv_rows: int = 0
    bytes_sent: int = 0
    bytes_received: int = 0


@dataclass
class EPOps:
    """Compute steps of one EP layer call (CUDA kernels by default)."""

    route: Callable            # (logits [T,E]) -> (weights_bf16 [T,k], ids int32 [T,k])
    group_by_owner: Callable   # (ids [T,k], owner [E], G) -> (offsets [G+1], p2r [P], r2p [P])
    gather_rows: Callable      # (hidden [T,H], r2p [P], k) -> rows [P,H]
    expert_mlp: Callable       # (rows [R,H], local_ids int32 [R]) -> out [R,H]
    combine: Callable          # (rows_back [P,H], p2r [P], weights [T,k]) -> out [T,H]
    # (rows [Rmax,H], local_ids [Rmax], count int32 [1] on the device, out [Rmax,H]): the
    # owner's MLP with the received row count kept on the device (None: not available)
    expert_mlp_count: Callable | None = None
    # (receive area [Rmax,H], slot of pair [Rmax], local_ids [Rmax], count [1], pair-row table
    # out [Rmax], output rows [Rmax,H]): the owner's MLP gathering its rows straight from the
    # receive area and leaving them grouped, with the table the sources read (None: n/a)
    expert_mlp_gather: Callable | None = None
    # (receive area, slot of pair, local_ids, count, make_row_ptrs(row_to_pair, count, ptrs)):
    # the gather MLP whose outputs are stored wherever the callback points each grouped row
    # (straight into the sources' memory); None: not available
    expert_mlp_push: Callable | None = None


class _DevicePtrArray:
    """A raw device allocation seen as a tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


class PeerExchange:
    """One rank's peer-memory exchange area: its region (``lm_ep_region_alloc``) mapped into
    every rank through CUDA IPC, the device array of all ranks' region pointers, and the
    local buffers of the receive side. Ranks must be on distinct GPUs: the exchange's waits
    spin on flags written by the other ranks' kernels."""

    def __init__(self, *, world_size: int, rank: int, max_tokens: int, top_k: int,
                 hidden_size: int, device: torch.device, group=None,
                 device_epoch: bool = False) -> None:
        self.G, self.rank, self.H = int(world_size), int(rank), int(hidden_size)
        self.max_tokens = int(max_tokens)
        self.cap = self.max_tokens * int(top_k)
        self.device = torch.device(device)
        uuids = [None] * self.G
        dist.all_gather_object(uuids, str(torch.cuda.get_device_properties(self.device).uuid),
                               group=group)
        if len(set(uuids)) != self.G:
            raise RuntimeError("peer exchange needs one rank per GPU (ranks share a device)")
        nbytes = _lib.ep_region_bytes(self.G, self.cap, self.H)
        self.region = _lib.ep_region_alloc(nbytes)
        handles = [None] * self.G
        dist.all_gather_object(handles, _lib.ipc_get_handle(self.region), group=group)
        self.peer_ptrs = [self.region if r == self.rank else _lib.ipc_open_handle(handles[r])
                          for r in range(self.G)]
        self.peers = torch.tensor(self.peer_ptrs, dtype=torch.int64, device=self.device)
        rows = self.G * self.cap
        off = _lib.ep_out_rows_offset(self.G, self.cap, self.H)
        self.out_rows = torch.as_tensor(
            _DevicePtrArray(self.region + off, (rows, self.H), "<i2"),
            device=self.device).view(torch.bfloat16)
        roff = _lib.ep_recv_rows_offset(self.G, self.cap, self.H)
        self.recv_rows = torch.as_tensor(
            _DevicePtrArray(self.region + roff, (rows, self.H), "<i2"),
            device=self.device).view(torch.bfloat16)
        poff = _lib.ep_pair_rows_offset(self.G, self.cap, self.H)
        self.pair_rows = torch.as_tensor(_DevicePtrArray(self.region + poff, (rows,), "<i4"),
                                         device=self.device)
        self.slots = torch.empty(rows, dtype=torch.int32, device=self.device)
        self.rows = torch.empty(rows, self.H, dtype=torch.bfloat16, device=self.device)
        self.ids = torch.empty(rows, dtype=torch.int32, device=self.device)
        self.total = torch.zeros(1, dtype=torch.int32, device=self.device)
        # token-deduplicated dispatch: each token's slot in each owner's area, rows per owner
        self.tok_slot = torch.empty(self.max_tokens * self.G, dtype=torch.int32,
                                    device=self.device)
        self.tok_count = torch.zeros(self.G, dtype=torch.int32, device=self.device)
        self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        # device_epoch: each call raises the region's own counter on the device and the kernels
        # read it (epoch 0), so a captured step replays with a new epoch every time
        self.device_epoch = bool(device_epoch)
        self.group = group
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (collective: every rank calls it)."""
        if self.region is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for r, ptr in enumerate(self.peer_ptrs):
            if r != self.rank:
                _lib.ipc_close_handle(ptr)
        dist.barrier(group=self.group)
        self.out_rows = self.recv_rows = self.pair_rows = None
        _lib.ep_region_free(self.region)
        self.region = None


class ExpertParallelMoE:
    def __init__(self, *, num_experts: int, top_k: int, hidden_size: int, rank: int,
                 world_size: int, ops: EPOps, group: dist.ProcessGroup | None = None,
                 device: torch.device | str = "cuda",
                 exchange: PeerExchange | None = None, dedupe_dispatch: bool = True,
                 push_outputs: bool = True,
                 nccl_rows_per_peer: int | None = None) -> None:
        if num_experts % world_size != 0:
            raise ValueError(f"{num_experts} experts do not split evenly over {world_size} ranks")
        self.E = int(num_experts)
        self.k = int(top_k)
        self.H = int(hidden_size)
        self.rank = int(rank)
        self.G = int(world_size)
        self.per_rank = self.E // self.G
        self.base = self.rank * self.per_rank
        self.ops = ops
        self.group = group
        self.device = torch.device(device)
        self.owner = (torch.arange(self.E, dtype=torch.int32) // self.per_rank).to(self.device)
        self._stats = EPStats()
        # peer steps without a host sync: per-step figures accumulate on the device
        # pairs received, pairs kept local, token rows stored into other ranks
        # (a captured step adds to them on every replay: the host counts nothing per step)
        self._dev_rows = torch.zeros(4, dtype=torch.int64, device=self.device)
        self._dev_steps = 0
        self.exchange = exchange
        self.transport = "peer" if exchange is not None else "nccl"
        # peer transport: a token's row crosses to an owner once, not once per routed pair
        self.dedupe_dispatch = bool(dedupe_dispatch)
        # peer transport: owners store outputs into the sources' memory from the MLP epilogue
        # (the combine then reads only local memory) instead of the sources reading them
        self.push_outputs = bool(push_outputs)
        # nccl transport with fixed splits: every (source, owner) block holds this many rows,
        # so the all-to-alls need no host-known counts (None: exact splits, read on the host)
        self.nccl_rows_per_peer = None if nccl_rows_per_peer is None else int(nccl_rows_per_peer)
        if self.nccl_rows_per_peer is not None and self.nccl_rows_per_peer <= 0:
            raise ValueError("nccl_rows_per_peer must be positive")
        self._overflow = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def stats(self) -> EPStats:
        """Exchange totals (reads the device-side part of peer steps: synchronises)."""
        st = EPStats(**vars(self._stats))
        if self._dev_steps:
            recv, local_rows, token_rows, pairs = (int(v) for v in self._dev_rows.tolist())
            elt = 2  # bf16 rows
            st.send_rows += pairs
            st.recv_rows += recv
            # dispatch stores (token rows, or one row per remote pair) + outputs read back
            st.bytes_sent += (token_rows + pairs - local_rows) * self.H * elt
            # counted per pair: an upper bound on the dispatch side when tokens are deduplicated
            st.bytes_received += 2 * (recv - local_rows) * self.H * elt
        return st

    def owned_experts(self) -> range:
        return range(self.base, self.base + self.per_rank)

    def forward(self, hidden: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        if self.exchange is not None:
            return self._forward_peer(hidden, router_logits)
        if self.nccl_rows_per_peer is not None:
            return self._forward_fixed(hidden, router_logits)
        T = int(hidden.shape[0])
        w, ids = self.ops.route(router_logits)
        offsets, p2r, r2p = self.ops.group_by_owner(ids, self.owner, self.G)
        P = T * self.k
        send_rows = self.ops.gather_rows(hidden, r2p[:P], self.k)
        send_ids = (ids.reshape(-1).long().index_select(0, r2p[:P].long()) % self.per_rank).to(torch.int32)
        send_counts = (offsets[1:] - offsets[:-1]).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        s_split = send_counts.tolist()
        r_split = recv_counts.tolist()
        R = int(sum(r_split))
        recv_rows = torch.empty(R, self.H, dtype=hidden.dtype, device=hidden.device)
        recv_ids = torch.empty(R, dtype=torch.int32, device=hidden.device)
        dist.all_to_all_single(recv_rows, send_rows, r_split, s_split, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids, r_split, s_split, group=self.group)
        out_rows = self.ops.expert_mlp(recv_rows, recv_ids)
        back = torch.empty(P, self.H, dtype=hidden.dtype, device=hidden.device)
        dist.all_to_all_single(back, out_rows.contiguous(), s_split, r_split, group=self.group)
        st = self._stats
        elt = hidden.element_size()
        st.send_rows += P
        st.recv_rows += R
        st.bytes_sent += (P - s_split[self.rank]) * self.H * elt * 2
        st.bytes_received += (R - r_split[self.rank]) * self.H * elt * 2
        return self.ops.combine(back, p2r[:P], w)

    def _forward_fixed(self, hidden: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """NCCL exchange with fixed splits: block (source, owner) of both all-to-alls holds
        ``C = nccl_rows_per_peer`` rows (the first ``count`` real, the rest padding with local
        id -1), so counts travel as a device tensor beside the rows and no step reads them on
        the host (with the gather MLP). Pairs beyond C for one owner are not sent: they add
        nothing to the output and raise the overflow flag that :meth:`check_exchange_errors`
        reports."""
        T = int(hidden.shape[0])
        G, C, k, dev = self.G, self.nccl_rows_per_peer, self.k, hidden.device
        P = T * k
        w, ids = self.ops.route(router_logits)
        offsets, p2r, r2p = self.ops.group_by_owner(ids, self.owner, G)
        off = offsets.long()
        counts = off[1:] - off[:-1]
        self._overflow |= (counts > C).any().to(torch.int32)
        # grouped row r -> block slot q = owner * C + position (G * C: not sent)
        r = torch.arange(P, dtype=torch.int64, device=dev)
        o_r = torch.searchsorted(off[1:].contiguous(), r, right=True)
        pos = r - off[o_r]
        q_r = torch.where(pos < C, o_r * C + pos, torch.full_like(r, G * C))
        pair_of_slot = torch.zeros(G * C + 1, dtype=torch.int32, device=dev)
        pair_of_slot.index_copy_(0, q_r, r2p[:P].to(torch.int32))
        send_ids = torch.full((G * C + 1,), -1, dtype=torch.int32, device=dev)
        local_ids = (ids.reshape(-1).long().index_select(0, r2p[:P].long())
                     % self.per_rank).to(torch.int32)
        send_ids.index_copy_(0, q_r, local_ids)
        send_rows = self.ops.gather_rows(hidden, pair_of_slot[:G * C], k)
        sent = torch.minimum(counts, torch.full_like(counts, C))
        recv_counts = torch.empty_like(sent)
        dist.all_to_all_single(recv_counts, sent, group=self.group)
        recv_rows = torch.empty(G * C, self.H, dtype=hidden.dtype, device=dev)
        recv_ids = torch.empty(G * C, dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_rows, send_rows, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids[:G * C].contiguous(), group=self.group)
        # received blocks compacted in source order: slot list, ids, count (all on the device)
        q = torch.arange(G * C, dtype=torch.int64, device=dev)
        src, j = q // C, q % C
        prefix = torch.cumsum(recv_counts, 0) - recv_counts
        valid = j < recv_counts[src]
        dest = torch.where(valid, prefix[src] + j, torch.full_like(q, G * C))
        slots = torch.zeros(G * C + 1, dtype=torch.int32, device=dev)
        slots.index_copy_(0, dest, q.to(torch.int32))
        cids = torch.zeros(G * C + 1, dtype=torch.int32, device=dev)
        cids.index_copy_(0, dest, recv_ids)
        total = recv_counts.sum().to(torch.int32).reshape(1)
        n = G * C
        if self.ops.expert_mlp_gather is not None and n > DECODE_MAX_TOKENS:
            # rows gathered straight from the received blocks; outputs stay grouped
            out_rows = torch.empty(n, self.H, dtype=hidden.dtype, device=dev)
            pair_rows = torch.empty(n, dtype=torch.int32, device=dev)
            self.ops.expert_mlp_gather(recv_rows, slots[:n], cids[:n], total, pair_rows,
                                       out_rows)
        elif self.ops.expert_mlp_count is not None:
            out_rows = torch.empty(n, self.H, dtype=hidden.dtype, device=dev)
            self.ops.expert_mlp_count(recv_rows.index_select(0, slots[:n].long()), cids[:n],
                                      total, out_rows)
            pair_rows = torch.arange(n, dtype=torch.int32, device=dev)
        else:
            R = int(total.item())  # host-sized owner MLP (the injectable CPU steps)
            out_rows = torch.zeros(n, self.H, dtype=hidden.dtype, device=dev)
            if R:
                out_rows[:R] = self.ops.expert_mlp(
                    recv_rows.index_select(0, slots[:R].long()), cids[:R])
            pair_rows = torch.arange(n, dtype=torch.int32, device=dev)
        # block slot q's output row (padding slots send row 0, which nobody reads)
        d = torch.where(valid, dest, torch.zeros_like(dest))
        back_idx = torch.where(valid, pair_rows.long().index_select(0, d), torch.zeros_like(q))
        back_send = out_rows.index_select(0, back_idx)
        back = torch.empty(G * C, self.H, dtype=hidden.dtype, device=dev)
        dist.all_to_all_single(back, back_send, group=self.group)
        # pair -> its output row in the returned blocks (-1: not sent, contributes nothing)
        q_pair = torch.where(q_r < G * C, q_r, torch.full_like(q_r, -1)).index_select(
            0, p2r[:P].long()).to(torch.int32)
        st = self._stats
        elt = hidden.element_size()
        st.send_rows += P
        st.recv_rows += G * C  # block rows, padding included
        st.bytes_sent += 2 * (G - 1) * C * self.H * elt
        st.bytes_received += 2 * (G - 1) * C * self.H * elt
        return self.ops.combine(back, q_pair, w)

    def _forward_peer(self, hidden: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        x = self.exchange
        T = int(hidden.shape[0])
        if T * self.k > x.cap:
            raise ValueError(f"{T} tokens exceed the exchange capacity ({x.cap // self.k})")
        w, ids = self.ops.route(router_logits)
        offsets, p2r, _ = self.ops.group_by_owner(ids, self.owner, self.G)
        if x.device_epoch:
            _lib.ep_advance_epoch(x.region, self.G, x.cap, self.H)
            x.epoch = 0  # every kernel of the call reads the region's counter
        else:
            x.epoch += 1
        if self.dedupe_dispatch:
            _lib.ep_dispatch_tokens(hidden, ids, self.per_rank, p2r, offsets, self.rank, self.G,
                                    x.peers, x.cap, x.epoch, x.tok_slot[: T * self.G],
                                    x.tok_count, x.done, x.err)
        else:
            _lib.ep_dispatch(hidden, ids, self.per_rank, p2r, offsets, self.rank, self.G,
                             x.peers, x.cap, x.epoch, x.done, x.err)
        big = x.rows.shape[0] > DECODE_MAX_TOKENS
        push = self.push_outputs and self.ops.expert_mlp_push is not None and big
        gather = not push and self.ops.expert_mlp_gather is not None and big
        no_sync = push or gather or self.ops.expert_mlp_count is not None
        if push:
            # outputs go from the down GEMM's epilogue straight into each source's area
            _lib.ep_receive_index(x.region, self.G, x.cap, self.H, x.epoch, x.slots, x.ids,
                                  x.total, x.err)

            def row_ptrs(row_to_pair, count, ptrs):
                _lib.ep_output_row_ptrs(x.region, self.G, x.cap, self.H, self.rank, x.peers,
                                        row_to_pair, count, ptrs.shape[0], ptrs, x.err)

            self.ops.expert_mlp_push(x.recv_rows, x.slots, x.ids, x.total, row_ptrs)
        elif gather:
            # no row copies on the owner: slots only, the MLP gathers from the receive area and
            # its grouped outputs stay put; the sources read them through the pair-row table
            _lib.ep_receive_index(x.region, self.G, x.cap, self.H, x.epoch, x.slots, x.ids,
                                  x.total, x.err)
            self.ops.expert_mlp_gather(x.recv_rows, x.slots, x.ids, x.total, x.pair_rows,
                                       x.out_rows)
        else:
            _lib.ep_receive(x.region, self.G, x.cap, self.H, x.epoch, x.rows, x.ids, x.total,
                            x.err)
            if no_sync:
                # the received count stays on the device: no host round trip in the step
                self.ops.expert_mlp_count(x.rows, x.ids, x.total, x.out_rows)
            else:
                R = int(x.total.item())  # sizes (and stages) the local expert MLP
                if R:
                    self.ops.expert_mlp(x.rows[:R], x.ids[:R], out=x.out_rows[:R])
        _lib.ep_signal_outputs(x.peers, self.rank, self.G, x.cap, self.H, x.epoch)
        out = torch.empty(T, self.H, dtype=hidden.dtype, device=hidden.device)
        combine = _lib.ep_combine_local if push else _lib.ep_combine
        combine(ids, w, self.per_rank, p2r, offsets, self.rank, self.G, x.peers, x.region, x.cap,
                x.epoch, out, x.err)
        if no_sync:
            # rows received, and rows this rank kept for itself (its own experts' pairs)
            _lib.ep_step_stats(x.total, offsets, x.tok_count if self.dedupe_dispatch else None,
                               T * self.k, self.rank, self.G, self._dev_rows)
            self._dev_steps += 1
        else:
            counts = (offsets[1:] - offsets[:-1]).tolist()
            st = self._stats
            elt = hidden.element_size()
            st.send_rows += T * self.k
            st.recv_rows += R
            remote = (T * self.k - counts[self.rank]) * self.H * elt
            if self.dedupe_dispatch:
                tc = x.tok_count.tolist()
                stored = (sum(tc) - tc[self.rank]) * self.H * elt
            else:
                stored = remote
            st.bytes_sent += stored + remote  # rows stored into owners + outputs read back
            st.bytes_received += 2 * (R - int(counts[self.rank])) * self.H * elt
        return out

    def check_exchange_errors(self) -> None:
        if self.nccl_rows_per_peer is not None and int(self._overflow.item()):
            raise RuntimeError(
                f"expert-parallel rank {self.rank}: more than {self.nccl_rows_per_peer} routed "
                "pairs for one owner in a step (fixed NCCL splits); raise nccl_rows_per_peer")
        if self.exchange is not None:
            _lib.raise_on_device_error(self.exchange.err, f"expert-parallel rank {self.rank}")


def cuda_ops(local_moe, *, num_experts: int, top_k: int, renormalize: bool = True,
             routed_scaling_factor: float = 1.0, max_tokens: int) -> EPOps:
    """The CUDA kernels for one rank; ``local_moe`` is a top-1 SlotBankMoE over the rank's
    owned experts (its own slot bank and host store)."""
    dev = local_moe.device
    P = max_tokens * top_k
    wb = torch.empty(max_tokens, top_k, dtype=torch.bfloat16, device=dev)
    ids = torch.empty(max_tokens, top_k, dtype=torch.int32, device=dev)
    G_MAX = 64
    off = torch.empty(G_MAX + 1, dtype=torch.int32, device=dev)
    p2r = torch.empty(P, dtype=torch.int32, device=dev)
    r2p = torch.empty(P, dtype=torch.int32, device=dev)
    scratch = torch.empty(_lib.build_groups_scratch_elems(P, G_MAX), dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def route(logits):
        T = logits.shape[0]
        _lib.route_topk(logits.float().contiguous(), top_k, renormalize=renormalize,
                        routed_scaling_factor=routed_scaling_factor, weights_bf16=wb[:T],
                        ids=ids[:T])
        return wb[:T], ids[:T]

    def group_by_owner(i, owner, G):
        _lib.build_groups(i, num_experts, owner, G, off[: G + 1], p2r, r2p, scratch, err)
        return off[: G + 1], p2r, r2p

    def gather_rows(hidden, rows, k):
        out = torch.empty(rows.numel(), hidden.shape[1], dtype=hidden.dtype, device=hidden.device)
        _lib.permute_rows(hidden, rows, k, rows.numel(), out)
        return out

    def expert_mlp(rows, local_ids, out=None):
        R = rows.shape[0]
        if R == 0:
            return rows.new_empty((0, rows.shape[1]))
        local_moe.topk_ids[:R, 0].copy_(local_ids)
        local_moe.invalidate_router_grouping()
        local_moe.topk_w[:R].fill_(1.0)
        decision = local_moe.stage(local_moe.topk_ids[:R])
        return local_moe.run_mlp(rows, decision, out)

    def combine(back, p2r_, w):
        T = w.shape[0]
        out = torch.empty(T, back.shape[1], dtype=back.dtype, device=back.device)
        _lib.moe_combine(back, p2r_, w, out)
        return out

    expert_mlp_count = expert_mlp_gather = None
    if local_moe.runtime.host_layer(local_moe.layer_id).on_device:
        def expert_mlp_count(rows, local_ids, count, out):
            return local_moe.mlp_rows_count(rows, local_ids, count, out)

        def expert_mlp_gather(src, slots, local_ids, count, pair_rows, out):
            return local_moe.mlp_rows_gather_count(src, slots, local_ids, count, pair_rows, out)

        def expert_mlp_push(src, slots, local_ids, count, make_row_ptrs):
            return local_moe.mlp_rows_gather_push(src, slots, local_ids, count, make_row_ptrs)
    else:
        expert_mlp_push = None

    return EPOps(route, group_by_owner, gather_rows, expert_mlp, combine, expert_mlp_count,
                 expert_mlp_gather, expert_mlp_push)


def build_rank_layer(*, w13_owned: torch.Tensor, w2_owned: torch.Tensor, rank: int,
                     device: torch.device, max_rows: int, num_slots: int,
                     store_on_device: bool):
    """A top-1 SlotBankMoE over one rank's owned experts (``w13_owned [E_r, 2I, H]``,
    ``w2_owned [E_r, H, I]``, row-major). The store is pinned host memory (staged into
    ``num_slots`` slots) or HBM (read in place)."""
    from .config import MoeOffloadConfig
    from .layer import SlotBankMoE
    from .moe_offload.runtime import MoeOffloadRuntime
    from .weight_layout import to_tiled

    E_r, two_i, H = w13_owned.shape
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=int(num_slots),
                                            async_load=True, b2_wave_prefill=True,
                                            pin_host_memory=True))
    w13t, w2t = to_tiled(w13_owned), to_tiled(w2_owned)
    if store_on_device:
        w13s, w2s = w13t.to(device), w2t.to(device)
    else:
        w13s = torch.empty(w13t.shape, dtype=w13t.dtype, pin_memory=True)
        w2s = torch.empty(w2t.shape, dtype=w2t.dtype, pin_memory=True)
        w13s.copy_(w13t)
        w2s.copy_(w2t)
    rt.register_layer_with_store(rank, w13s, w2s, slot_device=device,
                                 num_slots=1 if store_on_device else int(num_slots))
    return SlotBankMoE(rt, rank, hidden_size=H, intermediate_size=two_i // 2, num_experts=E_r,
                       top_k=1, max_tokens=int(max_rows), device=device)
