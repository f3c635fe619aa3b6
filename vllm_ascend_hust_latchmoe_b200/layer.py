"""The slot-bank MoE layer on B200: router -> stage -> slot-indexed grouped MLP -> combine.

This is the executor behind the plugin's seam ops. It mirrors the reference's data path:

* router piece      -- ``ops/fused_moe/moe_router_op.py:72-278`` (K1 ``lm_route_topk``);
* stage seam        -- ``ops/fused_moe/moe_offload_stage_op.py:160-471``: eager; no-op while
                       capturing and in Regime A; reads the active set (a device histogram and
                       one 4*E-byte copy instead of copying every top-k id), defers to waves
                       when the working set exceeds the slots, else stages the slots;
* MLP piece         -- ``ops/fused_moe/moe_mlp_op.py:69-130`` + patched ``fused_experts``
                       (``patches/patch_fused_moe.py:3946-4003``): log2phy remap + grouping
                       (``lm_build_groups``), grouped MLP over the fixed slot bank
                       (``lm_moe_mlp_decode`` / ``lm_moe_mlp_prefill``), one combine. It reads
                       only fixed buffers, so it can be captured in a CUDA graph;
* multi-wave path   -- ``patches/patch_fused_moe.py:2443-3470``: canonical waves, double-
                       buffered stage banks on the copy stream, one GEMM pass per wave, and
                       ONE combine in the original top-k pair order at the end.

All buffers are allocated once for ``max_tokens`` and reused, so launches see stable
addresses. There is no CPU or eager-torch fallback for any of the math.
"""

from __future__ import annotations

import os
from dataclasses import dataclass

import torch

from . import _lib
from .moe_offload.phase_split import (
    B2WaveFallback,
    WaveIssuer,
    plan_b2_prefill_async_schedule,
    plan_balanced_b2_waves,
)
from .moe_offload.runtime import MoeOffloadRuntime

PHASE_UNKNOWN = -1
PHASE_DECODE = 0
PHASE_PREFILL = 1
PHASE_MIXED = 2

# Above this many tokens per call the grouped MLP runs on the tcgen05 GEMM; at or below it
# on the bandwidth-bound GEMV (a group never holds more rows than the call has tokens).
DECODE_MAX_TOKENS = 64


def mlp_launches(T: int) -> int:
    """Kernel launches of one grouped-MLP call: the decode path runs one persistent launch for
    both GEMMs; the prefill path runs a 2-SM and a single-SM launch per GEMM (one launch per
    GEMM with LM_UMMA_CTA_PAIR=1)."""
    if T <= DECODE_MAX_TOKENS:
        return 1
    return 2 if os.environ.get("LM_UMMA_CTA_PAIR", "") == "1" else 4


def group_launches(pairs: int) -> int:
    """Kernel launches of one lm_build_groups call: one block up to 512 pairs, else three
    passes (count, scan, scatter)."""
    return 1 if 0 < pairs <= 512 else 3


def _vllm_cudagraph_mode() -> str | None:
    """vLLM's CUDA-graph mode of the forward pass in flight ("NONE", "PIECEWISE", ...), or
    None outside a vLLM forward pass."""
    try:
        from vllm.forward_context import get_forward_context, is_forward_context_available
    except Exception:
        return None
    if not is_forward_context_available():
        return None
    mode = getattr(get_forward_context(), "cudagraph_runtime_mode", None)
    return None if mode is None else str(getattr(mode, "name", mode))


@dataclass
class StageDecision:
    mode: str  # "capturing" | "static" | "slots" | "waves" | "device_waves" | "resident" |
    #            "device" | "passthrough"
    active_experts: tuple[int, ...] = ()
    counts: tuple[int, ...] = ()
    prepared: object | None = None


@dataclass
class WaveReport:
    waves: tuple[tuple[int, ...], ...] = ()
    staged_bytes: int = 0
    zero_copy: bool = False
    launches: int = 0


class SlotBankMoE:
    def __init__(
        self,
        runtime: MoeOffloadRuntime,
        layer_id: int,
        *,
        hidden_size: int,
        intermediate_size: int,
        num_experts: int,
        top_k: int,
        max_tokens: int,
        renormalize: bool = True,
        routed_scaling_factor: float = 1.0,
        scoring_func: str = "softmax",
        num_expert_group: int = 0,
        topk_group: int = 0,
        e_score_correction_bias: torch.Tensor | None = None,
        device: torch.device | str | None = None,
    ) -> None:
        self.runtime = runtime
        self.layer_id = int(layer_id)
        self.H = int(hidden_size)
        self.I = int(intermediate_size)
        self.E = int(num_experts)
        self.k = int(top_k)
        self.max_tokens = int(max_tokens)
        self.renormalize = bool(renormalize)
        self.routed_scaling_factor = float(routed_scaling_factor)
        self.scoring_func = scoring_func
        self.k_route = self.k
        self.num_expert_group = int(num_expert_group or 0)
        self.topk_group = int(topk_group or 0)
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.e_bias = (None if e_score_correction_bias is None else
                       e_score_correction_bias.to(self.device, torch.float32).contiguous())
        bank = runtime.slot_bank(self.layer_id)
        self.E_total = runtime.total_logical_expert_count_for_layer(layer_id=self.layer_id,
                                                                    fallback=self.E)
        self.num_bank_rows = bank.physical_expert_count
        # Fused mix-placement shared lane: logical ids E .. E_total-1 are shared experts held in
        # the bank's pinned suffix; the router appends them to every token's top-k (weight 1),
        # so a pair row is k_route + num_fused_shared wide.
        self.num_fused_shared = self.E_total - self.E
        self.k = self.k_route + self.num_fused_shared
        d, i32 = self.device, torch.int32
        P = self.max_tokens * self.k
        self.G_max = max(self.E_total, self.num_bank_rows)
        self.topk_ids = torch.zeros(self.max_tokens, self.k, dtype=i32, device=d)
        self.topk_w = torch.zeros(self.max_tokens, self.k, dtype=torch.bfloat16, device=d)
        self.counts = torch.zeros(self.E_total, dtype=i32, device=d)
        self.counts_host = torch.zeros(self.E_total, dtype=i32, pin_memory=True)
        self.err = torch.zeros(1, dtype=i32, device=d)
        self.err_host = torch.zeros(1, dtype=i32, pin_memory=True)
        self.tables_host = torch.zeros(self.E_total + self.G_max, dtype=i32, pin_memory=True)
        self.tables = torch.zeros(self.E_total + self.G_max, dtype=i32, device=d)
        self.expert_to_group = self.tables[: self.E_total]
        self.group_bank_row = self.tables[self.E_total:]
        self.slot_rows = torch.arange(self.num_bank_rows, dtype=i32, device=d)
        self.group_offsets = torch.zeros(self.G_max + 1, dtype=i32, device=d)
        self.pair_to_row = torch.zeros(P, dtype=i32, device=d)
        self.row_to_pair = torch.zeros(P, dtype=i32, device=d)
        self.scratch = torch.zeros(_lib.build_groups_scratch_elems(P, self.G_max), dtype=i32, device=d)
        self.x_perm = torch.zeros(P, self.H, dtype=torch.bfloat16, device=d)
        self.act = torch.zeros(P, self.I, dtype=torch.bfloat16, device=d)
        self.y_perm = torch.zeros(P, self.H, dtype=torch.bfloat16, device=d)
        self.out = torch.zeros(self.max_tokens, self.H, dtype=torch.bfloat16, device=d)
        # Identity expert -> group table: for decode-sized calls on an HBM-resident tier the
        # wave order is irrelevant (no staging), so grouping by expert id needs no plan.
        self.identity_groups = torch.arange(self.E_total, dtype=i32, device=d)
        self.wave_offsets = torch.zeros(self.E + 1, dtype=i32, device=d)
        self.num_waves = torch.zeros(1, dtype=i32, device=d)
        # Shared experts are groups E .. E_total-1 on every path, reading the bank's pinned
        # rows; the device wave plan only writes the first E entries of these tables.
        self.pinned_rows = torch.zeros(self.E_total, dtype=i32, device=d)
        store = runtime.host_layer(self.layer_id)
        # An HBM store that holds the shared rows serves them in place (row = logical id),
        # in the same launch as the routed groups; otherwise they come from the bank's
        # pinned suffix.
        self.shared_in_store = bool(self.num_fused_shared) and store.on_device and \
            int(store.w13.shape[0]) >= self.E_total
        if self.num_fused_shared:
            if self.shared_in_store:
                pinned = list(range(self.E, self.E_total))
            else:
                pinned = [bank.pinned_slot_for_logical_id(e) for e in range(self.E, self.E_total)]
            if any(r is None for r in pinned):
                raise RuntimeError(f"layer {self.layer_id}: shared experts lack pinned slots")
            self.pinned_rows[self.E:] = torch.tensor(pinned, dtype=i32)
            self.tables[self.E:self.E_total] = torch.arange(self.E, self.E_total, dtype=i32,
                                                            device=d)
            self.tables[self.E_total + self.E:2 * self.E_total] = torch.tensor(
                pinned, dtype=i32).to(d)
        self.pinned_rows_host = self.pinned_rows.cpu()
        self.resident_tier = runtime.host_layer(self.layer_id).on_device
        # prefill on the resident tier: order the groups by the device wave plan (as a staged
        # layer's waves would run) instead of by expert id; the results are the same
        self.resident_wave_order = False
        # tokens of the last route() call whose pairs the router also grouped (None: not)
        self._grouped_by_router = None
        self.last_waves = WaveReport()
        self.last_fallback_reason: str | None = None
        # Device staging (decode): slot state kept on the GPU, see lm_slot_plan.
        self.device_staging = bool(runtime.config.device_staging) and not self.resident_tier
        if self.device_staging:
            if self.E_total != self.E:
                raise ValueError("device staging serves routed experts only (no fused shared rows)")
            S = int(runtime.config.num_slots)
            self.slot_owner = torch.full((S,), -1, dtype=i32, device=d)
            self.slot_last_used = torch.full((S,), -1, dtype=torch.int64, device=d)
            self.expert_slot = torch.full((self.E_total,), -1, dtype=i32, device=d)
            self.stage_step = torch.zeros(1, dtype=torch.int64, device=d)
            self.group_src = torch.full((self.E_total,), -1, dtype=i32, device=d)
            self.hit_miss = torch.zeros(2, dtype=torch.int64, device=d)
        self.last_full_layer: dict | None = None
        self.kernel_launches = 0
        # Token counts whose slot-bank MLP piece (mlp_slots) was captured into a CUDA graph.
        # A replayed piece reads log2phy for every routed expert, so a stage call at one of
        # these sizes must never leave the working set unstaged (see stage()).
        self.captured_mlp_tokens: set[int] = set()
        self.pending: StageDecision | None = None
        self.shared_w13 = None
        self.shared_w2 = None

    # ------------------------------------------------------------------ pieces
    def route(self, hidden: torch.Tensor, router_logits: torch.Tensor):
        """K1: fills the fixed ``topk_w`` / ``topk_ids`` buffers; returns [T, k] views."""
        T = int(router_logits.shape[0])
        self._check_tokens(T)
        logits = router_logits if router_logits.dtype == torch.float32 else router_logits.float()
        if (self.resident_tier and T <= 16 and 0 < T * self.k <= 512
                and not self.runtime.config.stage_waves_from_hbm_store):
            # experts read in place: a decode-sized call groups by expert id, which does not
            # depend on staging, so the router groups its pairs in the same launch and the
            # MLP piece (mlp_resident) skips its grouping launch. Up to 16 tokens (one per
            # warp of the block); more tokens route faster over several blocks (64 tokens:
            # 0.205 ms fused vs 0.199 ms for the C4 layer)
            _lib.route_group_small(
                logits.contiguous(), self.k_route, scoring_func=self.scoring_func,
                renormalize=self.renormalize, routed_scaling_factor=self.routed_scaling_factor,
                e_score_correction_bias=self.e_bias, num_expert_group=self.num_expert_group,
                topk_group=self.topk_group, num_shared=self.num_fused_shared,
                weights_bf16=self.topk_w[:T], ids=self.topk_ids[:T],
                num_experts_total=self.E_total, expert_to_group=self.identity_groups,
                num_groups=self.E_total, group_offsets=self.group_offsets,
                pair_to_row=self.pair_to_row, row_to_pair=self.row_to_pair, err_word=self.err)
            self.kernel_launches += 1
            self._grouped_by_router = T
            return self.topk_w[:T], self.topk_ids[:T]
        self._grouped_by_router = None
        _lib.route_topk(logits.contiguous(), self.k_route, scoring_func=self.scoring_func,
                        renormalize=self.renormalize,
                        routed_scaling_factor=self.routed_scaling_factor,
                        e_score_correction_bias=self.e_bias,
                        num_expert_group=self.num_expert_group, topk_group=self.topk_group,
                        weights_bf16=self.topk_w[:T], ids=self.topk_ids[:T],
                        num_shared=self.num_fused_shared)
        self.kernel_launches += 1
        return self.topk_w[:T], self.topk_ids[:T]

    def invalidate_router_grouping(self) -> None:
        """The top-k buffers were written by something other than :meth:`route`: the next MLP
        piece groups the pairs itself instead of using the router's grouping."""
        self._grouped_by_router = None

    def active_counts(self, topk_ids: torch.Tensor) -> tuple[int, ...]:
        """K2 histogram + one small D2H: per-expert pair counts of this call. The layer's
        device error word comes back in the same round trip and a set word raises here,
        before anything is staged or published (an out-of-range id would otherwise be
        dropped from the working set silently)."""
        _lib.expert_histogram(topk_ids, self.E_total, self.counts, self.err)
        self.kernel_launches += 1
        self.counts_host.copy_(self.counts, non_blocking=True)
        self.err_host.copy_(self.err, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        code = int(self.err_host[0])
        if code:
            raise RuntimeError(f"layer {self.layer_id}: device error {code} "
                               f"({_lib.DEVERR_NAMES.get(code, '?')}) before staging")
        # routed experts only: the pinned shared suffix is never staged
        return tuple(self.counts_host[: self.E].tolist())

    def _slot_piece_replays(self, T: int) -> bool:
        """True when the MLP piece that follows this stage call is a replay of a captured
        slot-bank piece: one was captured at this token count and the caller is not running
        vLLM's forward pass eagerly (cudagraph mode NONE)."""
        if int(T) not in self.captured_mlp_tokens:
            return False
        return _vllm_cudagraph_mode() in (None, "PIECEWISE", "FULL", "FULL_AND_PIECEWISE",
                                          "FULL_DECODE_ONLY")

    def stage(self, topk_ids: torch.Tensor, phase: int = PHASE_UNKNOWN,
              capturing: bool = False) -> StageDecision:
        """Eager staging seam between the captured router and MLP pieces."""
        rt = self.runtime
        T = int(topk_ids.shape[0])
        if self.device_staging:
            # Decode: the slot decision runs on the device inside the MLP piece (capturable).
            # Prefill: capacity-bounded waves, which never write the main bank, so the slot
            # state held on the device stays the bank's only owner.
            if T <= DECODE_MAX_TOKENS:
                return StageDecision("device")
            if capturing or torch.cuda.is_current_stream_capturing():
                raise RuntimeError("prefill-sized calls are not captured under device staging")
            counts = self.active_counts(topk_ids)
            return StageDecision("waves", tuple(e for e, c in enumerate(counts) if c > 0), counts)
        if self._device_waves(T):
            return StageDecision("device_waves")
        if capturing or torch.cuda.is_current_stream_capturing():
            if rt.should_use_fixed_slot_plan_for_layer(self.layer_id) and not rt.is_layer_registered(self.layer_id):
                raise RuntimeError(f"graph capture reached an unregistered fixed-slot MoE layer {self.layer_id}")
            return StageDecision("capturing")
        if self.resident_tier and not rt.config.stage_waves_from_hbm_store:
            # Every expert already has an HBM copy: nothing to stage, and the wave plan is
            # made on the device inside the MLP piece (no host round trip).
            return StageDecision("resident")
        if rt.is_static_residency_regime(self.E):
            # Regime A: every expert owns a slot; stage them all once, log2phy stays static.
            if not getattr(self, "_static_staged", False):
                rt.stage_full_residency_slot_plan(layer_id=self.layer_id)
                self._static_staged = True
            return StageDecision("static")
        if not rt.should_use_fixed_slot_plan_for_layer(self.layer_id):
            return StageDecision("passthrough")
        counts = self.active_counts(topk_ids)
        active = tuple(e for e, c in enumerate(counts) if c > 0)
        if len(active) > rt.config.num_slots:
            if self._slot_piece_replays(T):
                # Fail closed: the replayed piece would read log2phy for all routed experts,
                # and an evicted expert's entry still names a slot that now holds another.
                raise RuntimeError(
                    f"layer {self.layer_id}: {len(active)} active experts exceed "
                    f"num_slots={rt.config.num_slots} at {T} tokens, a size whose slot-bank "
                    "MLP piece is replayed from a CUDA graph; multi-wave execution cannot run "
                    "inside a captured piece. Raise VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS to at "
                    "least top_k * max_num_seqs, enable device staging "
                    "(VLLM_ASCEND_MOE_OFFLOAD_DEVICE_STAGING=1), or run this batch size eagerly")
            if not rt.config.b2_wave_prefill:
                raise RuntimeError(
                    f"active expert working set size {len(active)} exceeds "
                    f"num_slots={rt.config.num_slots} and multi-wave execution is disabled")
            return StageDecision("waves", active, counts)
        prepared = rt.stage_fixed_slot_plan(layer_id=self.layer_id, active_experts=active,
                                            num_logical_experts=self.E)
        return StageDecision("slots", active, counts, prepared)

    def capture_decision(self, T: int) -> StageDecision:
        """Decision for an MLP piece being captured into a CUDA graph: the path that reads
        only fixed buffers and makes no host decision for this layer's tier. An HBM-resident
        store reads experts in place; device staging decides slots on the GPU; otherwise the
        slot-bank path reads whatever the eager stage published in log2phy at replay."""
        if self._device_waves(T):
            return StageDecision("device_waves")
        if self.resident_tier:
            return StageDecision("resident")
        if self.device_staging:
            if T > DECODE_MAX_TOKENS:
                raise RuntimeError("prefill-sized calls are not captured under device staging")
            return StageDecision("device")
        return StageDecision("capturing")

    def _device_waves(self, T: int) -> bool:
        """Prefill-sized call of a layer whose HBM store is staged wave by wave, with the waves
        planned and staged on the device (no fused shared lane: its groups sit outside the
        routed plan)."""
        cfg = self.runtime.config
        return (self.resident_tier and cfg.stage_waves_from_hbm_store
                and cfg.stage_waves_on_device and T > DECODE_MAX_TOKENS
                and not self.num_fused_shared)

    def forward_waves_device(self, hidden: torch.Tensor, T: int,
                             out: torch.Tensor | None = None) -> torch.Tensor:
        """Capacity-bounded waves planned and staged on the device, for an HBM store: histogram
        -> device wave plan (canonical waves of at most S experts, stage row = position in the
        wave) -> grouping wave by wave -> row permute -> per wave: a copy kernel on the copy
        stream fills a double-buffered stage bank with the wave's experts, the grouped MLP runs
        over the wave's groups read from the device plan, and a release event frees the bank
        for the wave after next -> one combine. ceil(E / S) waves are launched; the plan
        decides how many do work. Nothing is read on the host, so it can be captured."""
        rt = self.runtime
        store = rt.host_layer(self.layer_id)
        S = rt.config.num_slots
        ids = self.topk_ids[:T]
        _lib.expert_histogram(ids, self.E_total, self.counts, self.err)
        _lib.plan_waves(self.counts[: self.E], S, self.expert_to_group, self.group_bank_row,
                        self.wave_offsets, self.num_waves, in_place_rows=False)
        _lib.build_groups(ids, self.E_total, self.expert_to_group, self.E, self.group_offsets,
                          self.pair_to_row, self.row_to_pair, self.scratch, self.err)
        _lib.permute_rows(hidden, self.row_to_pair, self.k, T * self.k, self.x_perm)
        self.resident_planned = False
        self.device_waves_planned = True
        compute = torch.cuda.current_stream()
        copy = rt.transfer_engine.stream()
        capturing = torch.cuda.is_current_stream_capturing()
        copy.wait_stream(compute)  # the plan and the tables are ready
        nbuf = rt.config.effective_prefill_buffer_count
        released: dict[int, torch.cuda.Event] = {}
        max_waves = -(-self.E // S)
        for w in range(max_waves):
            buf = w % nbuf
            bank = rt.prefill_stage_bank(self.layer_id, buf)
            prev = released.get(buf)
            if prev is None and not capturing:
                # the buffer's last consumer from an earlier call (host-driven or not)
                prev = rt.prefill_stage_buffer_release_event(self.layer_id, buf)
            if prev is not None:
                copy.wait_event(prev)
            _lib.stage_wave_copy(bank.w13_slots, store.w13, self.expert_to_group,
                                 self.wave_offsets, self.num_waves, w, stream=copy)
            _lib.stage_wave_copy(bank.w2_slots, store.w2, self.expert_to_group,
                                 self.wave_offsets, self.num_waves, w, stream=copy)
            ready = torch.cuda.Event()
            ready.record(copy)
            compute.wait_event(ready)
            _lib.moe_mlp_prefill_wave(self.x_perm, T * self.k, self.group_offsets,
                                      self.group_bank_row, self.wave_offsets, self.num_waves, w,
                                      bank.w13_slots, bank.w2_slots, self.act, self.y_perm,
                                      self.err)
            rel = torch.cuda.Event()
            rel.record(compute)
            released[buf] = rel
            if not capturing:
                rt.remember_prefill_stage_buffer_release(self.layer_id, buf, rel)
        self.kernel_launches += (2 + group_launches(T * self.k) + 1 + max_waves * 2
                                 + max_waves * mlp_launches(T) + 1)
        return self._combine(T, out)

    def device_wave_plan(self) -> tuple[tuple[int, ...], ...]:
        """The waves (expert ids in group order) of the last device-planned wave call (reads
        the plan back: synchronises)."""
        if not getattr(self, "device_waves_planned", False):
            return ()
        nw = int(self.num_waves.item())
        off = self.wave_offsets[: nw + 1].tolist()
        e2g = self.expert_to_group[: self.E].tolist()
        by_group = sorted((g, e) for e, g in enumerate(e2g) if g >= 0)
        order = [e for _, e in by_group]
        return tuple(tuple(order[off[w]:off[w + 1]]) for w in range(nw))

    def _combine(self, T: int, out: torch.Tensor | None) -> torch.Tensor:
        dst = self.out[:T] if out is None else out
        _lib.moe_combine(self.y_perm, self.pair_to_row[: T * self.k], self.topk_w[:T], dst)
        return dst

    def mlp_slots(self, hidden: torch.Tensor, T: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Captured MLP piece: log2phy remap + grouping, grouped MLP on the slot bank, combine.

        Reads only fixed addresses (slot bank, log2phy, this layer's buffers)."""
        if torch.cuda.is_current_stream_capturing():
            self.captured_mlp_tokens.add(int(T))
        rt = self.runtime
        bank = rt.slot_bank(self.layer_id)
        log2phy = rt.log2phy_buffer(self.layer_id)
        ids = self.topk_ids[:T]
        G = self.num_bank_rows
        _lib.build_groups(ids, self.E_total, log2phy, G, self.group_offsets, self.pair_to_row,
                          self.row_to_pair, self.scratch, self.err)
        if T > DECODE_MAX_TOKENS:
            # the tcgen05 MLP reads its rows in group order (the decode GEMV gathers them)
            _lib.permute_rows(hidden, self.row_to_pair, self.k, T * self.k, self.x_perm)
            self.kernel_launches += 1
        self._grouped_mlp(hidden, T, self.slot_rows, 0, G, bank.w13_slots, bank.w2_slots)
        self.kernel_launches += group_launches(T * self.k) + mlp_launches(T) + 1  # + combine
        return self._combine(T, out)

    def mlp_device(self, hidden: torch.Tensor, T: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Decode MLP piece with the staging decision on the device: slot allocation
        (``lm_slot_plan``), grouping by expert id, the MLP reading hits from their slots and
        misses from the pinned host store (written through into their slots), combine. No
        host synchronisation; fixed buffers only, so it can be captured."""
        if not self.device_staging or T > DECODE_MAX_TOKENS:
            raise RuntimeError(f"layer {self.layer_id}: device staging serves decode-sized calls")
        rt = self.runtime
        bank = rt.slot_bank(self.layer_id)
        store = rt.host_layer(self.layer_id)
        ids = self.topk_ids[:T]
        _lib.slot_plan(ids, self.E, self.slot_owner, self.slot_last_used, self.expert_slot,
                       self.stage_step, rt.log2phy_buffer(self.layer_id), self.group_src,
                       self.hit_miss, self.err)
        _lib.build_groups(ids, self.E_total, self.identity_groups, self.E, self.group_offsets,
                          self.pair_to_row, self.row_to_pair, self.scratch, self.err)
        _lib.moe_mlp_decode_offload(hidden, self.k, self.row_to_pair, self.group_offsets,
                                    self.group_src, self.identity_groups, 0, self.E, T,
                                    bank.w13_slots, bank.w2_slots, store.w13, store.w2,
                                    self.act, self.y_perm, self.err)
        # slot plan, grouping, the two offload GEMV launches, combine
        self.kernel_launches += 1 + group_launches(T * self.k) + 2 + 1
        return self._combine(T, out)

    def mlp_resident(self, hidden: torch.Tensor, T: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """MLP piece for an HBM-resident expert tier: grouping by expert id (or, with
        ``resident_wave_order``, histogram -> device wave plan -> grouping wave by wave) ->
        grouped MLP reading each expert in place -> one combine. No host synchronisation;
        fixed buffers only, so it can be captured."""
        store = self.runtime.host_layer(self.layer_id)
        ids = self.topk_ids[:T]
        if T <= DECODE_MAX_TOKENS:
            # group = expert id, bank row = expert id: no histogram or wave plan needed; the
            # router of this call may have grouped the pairs already (route_group_small)
            self.resident_planned = False
            grouped = getattr(self, "_grouped_by_router", None) == T
            self._grouped_by_router = None
            if not grouped:
                _lib.build_groups(ids, self.E_total, self.identity_groups, self.E_total,
                                  self.group_offsets, self.pair_to_row, self.row_to_pair,
                                  self.scratch, self.err)
                self.kernel_launches += group_launches(T * self.k)
            g_end = self.E_total if self.shared_in_store else self.E
            self._grouped_mlp(hidden, T, self.identity_groups, 0, g_end, store.w13, store.w2)
            if not self.shared_in_store:
                self._shared_groups_mlp(hidden, T, self.pinned_rows)
            self.kernel_launches += mlp_launches(T) + 1
            return self._combine(T, out)
        if self.resident_wave_order:
            # groups in the canonical wave order of the device planner (the order of the
            # groups changes no pair's result; the plan is kept for inspection)
            self.resident_planned = True
            _lib.expert_histogram(ids, self.E_total, self.counts, self.err)
            _lib.plan_waves(self.counts[: self.E], self.runtime.config.num_slots,
                            self.expert_to_group, self.group_bank_row, self.wave_offsets,
                            self.num_waves, in_place_rows=True)
            e2g, bank_rows, shared_rows = self.expert_to_group, self.group_bank_row, \
                self.group_bank_row
            launches = 2  # histogram, plan
        else:
            # group = expert id, bank row = expert id: nothing to plan for experts read in place
            self.resident_planned = False
            e2g, bank_rows, shared_rows = self.identity_groups, self.identity_groups, \
                self.pinned_rows
            launches = 0
        _lib.build_groups(ids, self.E_total, e2g, self.E_total, self.group_offsets,
                          self.pair_to_row, self.row_to_pair, self.scratch, self.err)
        launches += group_launches(T * self.k)
        if T > DECODE_MAX_TOKENS:
            _lib.permute_rows(hidden, self.row_to_pair, self.k, T * self.k, self.x_perm)
            launches += 1
        g_end = self.E_total if self.shared_in_store else self.E
        self._grouped_mlp(hidden, T, bank_rows, 0, g_end, store.w13, store.w2)
        if not self.shared_in_store:
            self._shared_groups_mlp(hidden, T, shared_rows)
        self.kernel_launches += launches + mlp_launches(T) + 1
        return self._combine(T, out)

    def _shared_groups_mlp(self, hidden, T, bank_rows_dev) -> None:
        """Fused mix-placement lane: the shared experts' groups (E .. E_total-1) on the
        bank's pinned rows, once per call, into the same pair rows as the routed groups (the
        single combine then sums routed and shared pairs in top-k order)."""
        if not self.num_fused_shared:
            return
        w13, w2 = self._shared_weights()
        self._grouped_mlp(hidden, T, bank_rows_dev, self.E, self.E_total, w13, w2)
        self.kernel_launches += mlp_launches(T)

    def _shared_weights(self):
        """The tensors the shared groups' rows index: the HBM store, or the slot bank."""
        if self.shared_in_store:
            store = self.runtime.host_layer(self.layer_id)
            return store.w13, store.w2
        bank = self.runtime.slot_bank(self.layer_id)
        return bank.w13_slots, bank.w2_slots

    def mlp_rows_count(self, rows: torch.Tensor, ids: torch.Tensor, count_dev: torch.Tensor,
                       out: torch.Tensor) -> torch.Tensor:
        """Top-1 MLP over the first ``count_dev`` (int32 on the device) of ``rows`` [R, H]
        with their expert ids ``ids`` [R] (HBM-resident store, experts read in place); row r's
        output (unit weight) goes to ``out[r]``. The count never reaches the host: grouping,
        row gather and combine read it on the device, the MLP is sized by R."""
        store = self.runtime.host_layer(self.layer_id)
        if self.k != 1 or not store.on_device:
            raise RuntimeError("mlp_rows_count needs a top-1 layer with an HBM-resident store")
        R = int(rows.shape[0])
        if R > self.max_tokens:
            raise ValueError(f"{R} rows exceed the layer's {self.max_tokens}")
        if getattr(self, "_unit_w", None) is None:
            self._unit_w = torch.ones(self.max_tokens, 1, dtype=torch.bfloat16, device=self.device)
        _lib.build_groups_count(ids.view(R, 1), count_dev, self.E_total, self.identity_groups,
                                self.E, self.group_offsets, self.pair_to_row, self.row_to_pair,
                                self.scratch, self.err)
        if R <= DECODE_MAX_TOKENS:
            _lib.moe_mlp_decode(rows, 1, self.row_to_pair, self.group_offsets,
                                self.identity_groups, 0, self.E, R, store.w13, store.w2,
                                self.act, self.y_perm, self.err)
        else:
            _lib.permute_rows_count(rows, self.row_to_pair, 1, R, count_dev, self.x_perm)
            _lib.moe_mlp_prefill(self.x_perm, R, self.group_offsets, self.identity_groups, 0,
                                 self.E, store.w13, store.w2, self.act, self.y_perm, self.err)
        _lib.moe_combine_count(self.y_perm, self.pair_to_row, self._unit_w[:R], count_dev, out)
        self.kernel_launches += group_launches(R) + mlp_launches(R) + 1 + (R > DECODE_MAX_TOKENS)
        return out

    def mlp_rows_gather_count(self, src_rows: torch.Tensor, pair_src: torch.Tensor,
                              ids: torch.Tensor, count_dev: torch.Tensor,
                              pair_to_row_out: torch.Tensor, y_out: torch.Tensor) -> None:
        """Top-1 MLP over the first ``count_dev`` pairs whose rows sit in ``src_rows`` at
        ``pair_src[p]`` (the receive area an exchange filled; nothing is compacted first):
        grouping by expert, a gather straight from ``src_rows`` into the grouped order, the
        tcgen05 MLP writing its rows into ``y_out`` and pair p's row index into
        ``pair_to_row_out[p]`` (the table the exchange's sources read). Needs a top-1 layer
        with an HBM-resident store and a capacity above the decode size."""
        store = self.runtime.host_layer(self.layer_id)
        R = int(ids.shape[0])
        if self.k != 1 or not store.on_device:
            raise RuntimeError("mlp_rows_gather_count needs a top-1 layer with an HBM store")
        if R > self.max_tokens or R <= DECODE_MAX_TOKENS:
            raise ValueError(f"{R} pairs outside ({DECODE_MAX_TOKENS}, {self.max_tokens}]")
        _lib.build_groups_count(ids.view(R, 1), count_dev, self.E_total, self.identity_groups,
                                self.E, self.group_offsets, pair_to_row_out, self.row_to_pair,
                                self.scratch, self.err)
        _lib.permute_rows_gather_count(src_rows, self.row_to_pair, pair_src, R, count_dev,
                                       self.x_perm)
        _lib.moe_mlp_prefill(self.x_perm, R, self.group_offsets, self.identity_groups, 0,
                             self.E, store.w13, store.w2, self.act, y_out, self.err)
        self.kernel_launches += group_launches(R) + 1 + mlp_launches(R)

    def mlp_rows_gather_push(self, src_rows: torch.Tensor, pair_src: torch.Tensor,
                             ids: torch.Tensor, count_dev: torch.Tensor, make_row_ptrs) -> None:
        """:meth:`mlp_rows_gather_count` whose output rows go wherever
        ``make_row_ptrs(row_to_pair, count_dev, row_ptrs)`` points them: after grouping, the
        callback fills ``row_ptrs`` (int64 device addresses, one per grouped row, from the
        row's pair index) and the down GEMM's epilogue stores each row there -- an exchange
        uses it to store every output straight into its source's memory."""
        store = self.runtime.host_layer(self.layer_id)
        R = int(ids.shape[0])
        if self.k != 1 or not store.on_device:
            raise RuntimeError("mlp_rows_gather_push needs a top-1 layer with an HBM store")
        if R > self.max_tokens or R <= DECODE_MAX_TOKENS:
            raise ValueError(f"{R} pairs outside ({DECODE_MAX_TOKENS}, {self.max_tokens}]")
        if getattr(self, "_row_ptrs", None) is None:
            self._row_ptrs = torch.empty(self.max_tokens, dtype=torch.int64, device=self.device)
            self._pair_rows_scratch = torch.empty(self.max_tokens, dtype=torch.int32,
                                                  device=self.device)
        _lib.build_groups_count(ids.view(R, 1), count_dev, self.E_total, self.identity_groups,
                                self.E, self.group_offsets, self._pair_rows_scratch[:R],
                                self.row_to_pair, self.scratch, self.err)
        make_row_ptrs(self.row_to_pair, count_dev, self._row_ptrs[:R])
        _lib.permute_rows_gather_count(src_rows, self.row_to_pair, pair_src, R, count_dev,
                                       self.x_perm)
        _lib.moe_mlp_prefill_rows(self.x_perm, R, self.group_offsets, self.identity_groups, 0,
                                  self.E, store.w13, store.w2, self.act, self._row_ptrs[:R],
                                  self.err)
        self.kernel_launches += group_launches(R) + 2 + mlp_launches(R)

    def resident_wave_plan(self) -> tuple[tuple[int, ...], ...]:
        """Read back the last device wave plan (synchronises; diagnostics and tests). Empty
        after a decode-sized resident call, which groups by expert id without waves."""
        if not getattr(self, "resident_planned", False):
            return ()
        nw = int(self.num_waves.item())
        off = self.wave_offsets[: nw + 1].tolist()
        rows = self.group_bank_row.tolist()
        return tuple(tuple(rows[off[w]:off[w + 1]]) for w in range(nw))

    def _grouped_mlp(self, hidden, T, bank_rows_dev, g0, g1, w13_bank, w2_bank) -> None:
        if T <= DECODE_MAX_TOKENS:
            _lib.moe_mlp_decode(hidden, self.k, self.row_to_pair, self.group_offsets,
                                bank_rows_dev, g0, g1, T, w13_bank, w2_bank, self.act,
                                self.y_perm, self.err)
        else:
            _lib.moe_mlp_prefill(self.x_perm, T * self.k, self.group_offsets, bank_rows_dev,
                                 g0, g1, w13_bank, w2_bank, self.act, self.y_perm, self.err)

    def forward_waves(self, hidden: torch.Tensor, T: int, counts: tuple[int, ...],
                      out: torch.Tensor | None = None) -> torch.Tensor:
        """Capacity-bounded waves with one combine at the end (eager). A wave plan that does
        not qualify (``B2WaveFallback``, raised before any wave runs) reruns the layer on the
        full-layer path, as does ``b2_reference_full_layer``."""
        rt = self.runtime
        cfg = rt.config
        self.last_fallback_reason = None
        if cfg.b2_reference_full_layer and not rt.host_layer(self.layer_id).on_device:
            return self.forward_full_layer(hidden, T, out)
        try:
            plan = self.plan_waves_checked(counts)
        except B2WaveFallback as exc:
            self.last_fallback_reason = f"{type(exc).__name__}: {exc}"
            return self.forward_full_layer(hidden, T, out)
        return self._run_waves(hidden, T, plan, out)

    def plan_waves_checked(self, counts: tuple[int, ...]):
        """Canonical wave plan, qualified before anything runs: every active expert in
        exactly one wave, no wave above the slot count (reference: ``patch_fused_moe.py``
        :2540-2548, ``phase_split.py:1790-1856``). Failures raise ``B2WaveFallback``."""
        S = int(self.runtime.config.num_slots)
        active = {e: int(c) for e, c in enumerate(counts) if c > 0}
        try:
            plan = plan_balanced_b2_waves(active, S)
        except ValueError as exc:
            raise B2WaveFallback(f"wave planning failed: {exc}") from exc
        members = [e for w in plan.waves for e in w]
        if sorted(members) != sorted(active) or any(len(w) > S for w in plan.waves):
            raise B2WaveFallback(
                f"B2 waves must cover every active expert exactly once within {S} slots: "
                f"covered={len(members)} active={len(active)}")
        return plan

    def forward_full_layer(self, hidden: torch.Tensor, T: int,
                           out: torch.Tensor | None = None) -> torch.Tensor:
        """Recoverable fallback: all routed experts staged into the full-layer bank (row e =
        expert e), then one grouped MLP pass in the native top-k shape and the combine
        (reference ``_run_b2_full_layer_reference``, ``patch_fused_moe.py:3472-3650``)."""
        rt = self.runtime
        bank, ready, payload = rt.prepare_full_layer_prefill_plan(layer_id=self.layer_id)
        rt.wait_prefill_stage_plan(ready, torch.cuda.current_stream())
        ids = self.topk_ids[:T]
        _lib.build_groups(ids, self.E_total, self.identity_groups, self.E_total,
                          self.group_offsets, self.pair_to_row, self.row_to_pair, self.scratch,
                          self.err)
        launches = group_launches(T * self.k)
        if T > DECODE_MAX_TOKENS:
            _lib.permute_rows(hidden, self.row_to_pair, self.k, T * self.k, self.x_perm)
            launches += 1
        self._grouped_mlp(hidden, T, self.identity_groups, 0, self.E, bank.w13_slots,
                          bank.w2_slots)
        self._shared_groups_mlp(hidden, T, self.pinned_rows)
        launches += mlp_launches(T) + 1
        self.kernel_launches += launches
        self.last_full_layer = payload
        self.last_waves = WaveReport(waves=(tuple(range(self.E)),),
                                     staged_bytes=int(payload["h2d_bytes"]), launches=launches)
        return self._combine(T, out)

    def _run_waves(self, hidden: torch.Tensor, T: int, plan, out: torch.Tensor | None):
        rt = self.runtime
        cfg = rt.config
        waves = plan.waves
        store = rt.host_layer(self.layer_id)
        zero_copy = store.on_device and not cfg.stage_waves_from_hbm_store
        e2g = self.tables_host[: self.E_total]
        e2g.fill_(-1)
        rows = self.tables_host[self.E_total:]
        wave_groups: list[tuple[int, int]] = []
        g = 0
        for wave in waves:
            g0 = g
            for pos, e in enumerate(wave):
                e2g[e] = g
                rows[g] = e if zero_copy else pos
                g += 1
            wave_groups.append((g0, g))
        g_routed = g
        if self.num_fused_shared:
            # fused shared lane: groups E .. E_total-1 (as on every path) on the pinned rows
            for e in range(self.E, self.E_total):
                e2g[e] = e
                rows[e] = int(self.pinned_rows_host[e])
            g = self.E_total
        self.tables.copy_(self.tables_host, non_blocking=True)
        ids = self.topk_ids[:T]
        _lib.build_groups(ids, self.E_total, self.expert_to_group, g, self.group_offsets,
                          self.pair_to_row, self.row_to_pair, self.scratch, self.err)
        launches = group_launches(T * self.k)
        if T > DECODE_MAX_TOKENS:
            _lib.permute_rows(hidden, self.row_to_pair, self.k, T * self.k, self.x_perm)
            launches += 1
        report = WaveReport(waves=waves, zero_copy=zero_copy)
        if zero_copy:
            # Every expert already has an HBM copy: read it in place, all waves in one pass.
            self._grouped_mlp(hidden, T, self.group_bank_row, 0, g_routed, store.w13, store.w2)
            launches += mlp_launches(T)
        else:
            main = rt.slot_bank(self.layer_id)
            ready = main.ready_slot_ids(self.layer_id, [e for w in waves for e in w])
            h2d = {i: sum(store.expert_bytes for e in w if e not in ready) for i, w in enumerate(waves)}
            cost = {i: float(plan.wave_tokens(w)) for i, w in enumerate(waves)}
            schedule = plan_b2_prefill_async_schedule(
                waves, slot_readiness={}, prefetch_depth=cfg.effective_prefill_prefetch_depth,
                buffer_count=cfg.effective_prefill_buffer_count, h2d_bytes_by_wave=h2d,
                compute_cost_by_wave=cost, transfer_aware=cfg.transfer_aware_wave_schedule)
            pending = {}
            compute_stream = torch.cuda.current_stream()
            for kind, w, buf in WaveIssuer(schedule).events():
                if kind == "issue_stage":
                    pending[w] = rt.prepare_prefill_stage_plan(
                        layer_id=self.layer_id, active_experts=waves[w], buffer_index=buf,
                        wait_event=rt.prefill_stage_buffer_release_event(self.layer_id, buf))
                    report.staged_bytes += pending[w][1].bytes
                elif kind == "compute":
                    stage_bank, ready_ev = pending.pop(w)
                    rt.wait_prefill_stage_plan(ready_ev, compute_stream)
                    g0, g1 = wave_groups[w]
                    self._grouped_mlp(hidden, T, self.group_bank_row, g0, g1,
                                      stage_bank.w13_slots, stage_bank.w2_slots)
                    launches += mlp_launches(T)
                    release = torch.cuda.Event()
                    release.record(compute_stream)
                    rt.remember_prefill_stage_buffer_release(self.layer_id, buf, release)
        if self.num_fused_shared:
            # the pinned shared suffix once, after the routed waves (never counted against
            # the slots, never repeated per wave)
            sw13, sw2 = self._shared_weights()
            self._grouped_mlp(hidden, T, self.group_bank_row, self.E, self.E_total, sw13, sw2)
            launches += mlp_launches(T)
        dst = self._combine(T, out)
        launches += 1
        report.launches = launches
        self.last_waves = report
        self.kernel_launches += launches
        return dst

    # ------------------------------------------------------------------ shared experts
    def set_shared_experts(self, w13: torch.Tensor, w2: torch.Tensor) -> None:
        """Always-resident shared expert(s) fused into one MLP: ``w13 [2*Is, H]`` (gate rows
        then up rows) and ``w2 [H, Is]``; applied to every token by :meth:`shared_mlp`."""
        from .weight_layout import to_tiled

        Is = int(w2.shape[-1])
        if tuple(w13.shape) != (2 * Is, self.H) or tuple(w2.shape) != (self.H, Is):
            raise ValueError(f"shared expert shapes {tuple(w13.shape)}, {tuple(w2.shape)} do not "
                             f"match hidden {self.H}")
        self.shared_w13 = to_tiled(w13.to(self.device, torch.bfloat16))[None].contiguous()
        self.shared_w2 = to_tiled(w2.to(self.device, torch.bfloat16))[None].contiguous()
        d, i32 = self.device, torch.int32
        self.shared_rows = torch.arange(self.max_tokens, dtype=i32, device=d)
        self.shared_bank_row = torch.zeros(1, dtype=i32, device=d)
        self.shared_offsets = torch.zeros(2, dtype=i32, device=d)
        self.shared_act = torch.zeros(self.max_tokens, Is, dtype=torch.bfloat16, device=d)

    def shared_mlp(self, hidden: torch.Tensor, T: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Resident shared-expert MLP over all T tokens (one group of T rows)."""
        if self.shared_w13 is None:
            raise RuntimeError(f"layer {self.layer_id} has no shared experts")
        out = torch.empty(T, self.H, dtype=torch.bfloat16, device=self.device) if out is None else out
        self.shared_offsets[1:].fill_(T)
        if T <= DECODE_MAX_TOKENS:
            _lib.moe_mlp_decode(hidden, 1, self.shared_rows, self.shared_offsets,
                                self.shared_bank_row, 0, 1, T, self.shared_w13, self.shared_w2,
                                self.shared_act, out, self.err)
        else:
            _lib.moe_mlp_prefill(hidden, T, self.shared_offsets, self.shared_bank_row, 0, 1,
                                 self.shared_w13, self.shared_w2, self.shared_act, out, self.err)
        self.kernel_launches += mlp_launches(T)
        return out

    def run_mlp(self, hidden: torch.Tensor, decision: StageDecision,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """MLP piece for a stage decision (the seam's second captured piece, or eager)."""
        T = int(hidden.shape[0])
        if decision.mode == "device":
            return self.mlp_device(hidden, T, out)
        if decision.mode == "device_waves":
            return self.forward_waves_device(hidden, T, out)
        if decision.mode == "waves":
            return self.forward_waves(hidden, T, decision.counts, out)
        if decision.mode == "resident":
            return self.mlp_resident(hidden, T, out)
        if decision.mode not in ("slots", "static", "capturing"):
            raise RuntimeError(f"layer {self.layer_id} is not offloaded under fixed slots")
        rt = self.runtime
        rt.capture_safe_slot_weights(layer_id=self.layer_id)
        handle = rt.begin_slot_compute(decision.prepared) if decision.prepared is not None else None
        result = self.mlp_slots(hidden, T, out)
        rt.end_slot_compute(handle)
        return result

    # ------------------------------------------------------------------ whole layer
    def forward(self, hidden: torch.Tensor, router_logits: torch.Tensor,
                phase: int = PHASE_UNKNOWN) -> torch.Tensor:
        """Eager layer call: route -> stage -> slot MLP or multi-wave MLP -> combine."""
        T = int(hidden.shape[0])
        self._check_tokens(T)
        if hidden.dtype != torch.bfloat16 or not hidden.is_contiguous():
            raise ValueError("hidden_states must be a contiguous bf16 tensor")
        _, ids = self.route(hidden, router_logits)
        prof = self.runtime.prefill_profiler
        if prof is None or T <= DECODE_MAX_TOKENS:
            return self.run_mlp(hidden, self.stage(ids, phase))
        # prefill call recorded for profile-guided residency (events only; no sync here)
        start = prof.begin()
        decision = self.stage(ids, phase)
        out = self.run_mlp(hidden, decision)
        resident = decision.mode == "resident"
        host_waves = decision.mode == "waves"  # device-planned waves are not read back here
        prof.end(start, layer_id=self.layer_id, resident=resident, tokens=T, pairs=T * self.k,
                 waves=len(self.last_waves.waves) if host_waves else 0,
                 active=len(decision.active_experts),
                 h2d_bytes=int(self.last_waves.staged_bytes) if host_waves else 0)
        return out

    def check_device_errors(self, where: str = "SlotBankMoE") -> None:
        _lib.raise_on_device_error(self.err, f"{where} layer {self.layer_id}")

    def _check_tokens(self, T: int) -> None:
        if T <= 0 or T > self.max_tokens:
            raise ValueError(f"token count {T} outside (0, {self.max_tokens}]")

