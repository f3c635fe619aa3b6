"""Decode-TPOT harness: a Qwen3-30B-A3B-shaped decoder stack replayed as piecewise CUDA graphs
split at the staging seam, with routed experts served by slot banks (offloaded layers) or
read in place from HBM (resident layers).

Per decode token, layer ``i`` runs attention (RMSNorm, QKV, RoPE, GQA over a fixed-size KV
cache with a position mask, output projection) and the MoE block (RMSNorm, router, grouped
expert MLP, residual). The router's logits come from a seeded temporal-locality process
(each of the previous top-k experts kept with probability 0.7) so the staging traffic is
the one the offload path is meant to absorb; the attention weights and KV contents are
random. Graph pieces end right after the router of every offloaded layer; between pieces
the eager stage seam runs (the reference's PIECEWISE split at ``vllm::moe_offload_stage``,
``patches/patch_fused_moe.py:5339-5406``): device histogram -> 512-byte D2H -> slot
allocation -> H2D of the misses on the copy stream -> consumer wait -> log2phy publish, and
the next piece replays the captured slot-bank MLP against the fixed slot/log2phy addresses.
The attention and dense pieces are plain PyTorch (not the hot path).

Memory: resident layers own a device expert store each; all offloaded layers share ONE
pinned host store (the expert values do not matter for timing, and 24 private 1.2 GB
pinned copies would not fit many hosts), each with its own HBM slot bank.
"""

from __future__ import annotations

import math
import statistics
import time
from dataclasses import dataclass, field

import torch

from .config import MoeOffloadConfig
from .layer import PHASE_DECODE, SlotBankMoE
from .moe_offload.runtime import MoeOffloadRuntime
from .synthetic import LayerConfig, locality_topk_sequence


@dataclass(frozen=True)
class DecoderShape:
    layers: int = 48
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    intermediate: int = 768
    vocab: int = 151936
    num_slots: int = 32
    prompt: int = 1024
    max_new: int = 256
    rope_theta: float = 1_000_000.0

    @property
    def max_len(self) -> int:
        return self.prompt + self.max_new


@dataclass
class TpotReport:
    steps: int
    tpot_ms_p50: float
    tpot_ms_p95: float
    tpot_ms_mean: float
    offloaded_layers: int
    h2d_bytes_per_step: float
    h2d_gbs_during_stage: float | None
    slot_hit_rate: float | None
    graphs: int
    stage_ms_per_step: float
    extra: dict = field(default_factory=dict)


def _rand(shape, device, std=0.02, gen=None):
    return (torch.randn(*shape, device=device, generator=gen) * std).to(torch.bfloat16)


class SyntheticMoEDecoder:
    def __init__(self, shape: DecoderShape, offloaded_layers, device, seed: int = 0,
                 keep_prob: float = 0.7, host_store=None, teacher_forcing: bool = False,
                 device_staging: bool = False):
        self.s = s = shape
        self.device = d = torch.device(device)
        self.offloaded = sorted(set(int(i) for i in offloaded_layers))
        g = torch.Generator(device=d)
        g.manual_seed(seed)
        H, L = s.hidden, s.layers
        qd, kvd = s.heads * s.head_dim, s.kv_heads * s.head_dim
        self.embed = _rand((s.vocab, H), d, gen=g)
        self.lm_head = _rand((s.vocab, H), d, gen=g)
        self.final_norm = torch.ones(H, device=d, dtype=torch.bfloat16)
        self.ln1 = [torch.ones(H, device=d, dtype=torch.bfloat16) for _ in range(L)]
        self.ln2 = [torch.ones(H, device=d, dtype=torch.bfloat16) for _ in range(L)]
        self.wqkv = [_rand((qd + 2 * kvd, H), d, gen=g) for _ in range(L)]
        self.wo = [_rand((H, qd), d, gen=g) for _ in range(L)]
        self.kcache = [torch.randn(s.max_len, s.kv_heads, s.head_dim, device=d, generator=g)
                       .to(torch.bfloat16) for _ in range(L)]
        self.vcache = [torch.randn(s.max_len, s.kv_heads, s.head_dim, device=d, generator=g)
                       .to(torch.bfloat16) for _ in range(L)]
        inv = 1.0 / (s.rope_theta ** (torch.arange(0, s.head_dim, 2, device=d, dtype=torch.float32)
                                      / s.head_dim))
        ang = torch.arange(s.max_len, device=d, dtype=torch.float32)[:, None] * inv[None, :]
        self.rope_cos = torch.cos(ang)  # [max_len, head_dim / 2]
        self.rope_sin = torch.sin(ang)

        # experts: resident layers own an HBM store; offloaded layers share one pinned store
        I = s.intermediate
        # device_staging: offloaded layers decide their staging on the GPU and read missed
        # experts over PCIe inside the MLP piece, so a whole token is one graph.
        self.device_staging = bool(device_staging)
        self.runtime = MoeOffloadRuntime(MoeOffloadConfig(
            enabled=True, num_slots=s.num_slots, async_load=True, b2_wave_prefill=True,
            graph_compatible_offload=True, pin_host_memory=True,
            device_staging=self.device_staging))
        if self.offloaded:
            if host_store is None:
                w13 = torch.empty(s.experts, 2 * I, H, dtype=torch.bfloat16, pin_memory=True)
                w2 = torch.empty(s.experts, H, I, dtype=torch.bfloat16, pin_memory=True)
                for e in range(s.experts):  # fill through the GPU generator, expert by expert
                    w13[e].copy_(_rand((2 * I, H), d, gen=g))
                    w2[e].copy_(_rand((H, I), d, gen=g))
                host_store = (w13, w2)
        self.host_store = host_store
        self.moe: list[SlotBankMoE] = []
        for i in range(L):
            if i in self.offloaded:
                self.runtime.register_layer_with_store(i, host_store[0], host_store[1],
                                                       slot_device=d)
            else:
                self.runtime.register_layer_with_store(
                    i, _rand((s.experts, 2 * I, H), d, gen=g), _rand((s.experts, H, I), d, gen=g),
                    slot_device=d, num_slots=1)
            self.moe.append(SlotBankMoE(self.runtime, i, hidden_size=H, intermediate_size=I,
                                        num_experts=s.experts, top_k=s.top_k, max_tokens=1,
                                        device=d))

        # static decode state
        self.x = torch.zeros(1, H, device=d, dtype=torch.bfloat16)
        self.h2 = torch.zeros(1, H, device=d, dtype=torch.bfloat16)
        self.pos = torch.full((1,), s.prompt, device=d, dtype=torch.int64)
        self.token = torch.zeros(1, device=d, dtype=torch.int64)
        # With teacher forcing the next input token is set by the host (``forced``) instead
        # of the greedy argmax, so two runs cannot diverge through a near-tied argmax.
        self.teacher_forcing = bool(teacher_forcing)
        self.forced = torch.zeros(1, device=d, dtype=torch.int64)
        self.logits = torch.zeros(L, s.experts, device=d, dtype=torch.float32)
        self.positions = torch.arange(s.max_len, device=d)

        # routing with temporal locality, one sequence per layer
        cfg = LayerConfig("router", hidden=H, num_experts=s.experts, top_k=s.top_k,
                          intermediate=I, num_slots=s.num_slots, tokens=1)
        steps = s.max_new
        table = torch.randn(steps, L, s.experts, generator=torch.Generator().manual_seed(seed)) * 0.1
        for i in range(L):
            for t, sel in enumerate(locality_topk_sequence(cfg, steps, keep_prob, seed=1000 + i)):
                table[t, i, list(sel)] += 8.0
        self.logit_table = table.pin_memory()
        self.graphs: list[tuple[torch.cuda.CUDAGraph, int | None]] = []

    # ------------------------------------------------------------------ pieces
    @staticmethod
    def _rms(x, w, eps=1e-6):
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), w, eps)

    def _rope(self, t, n_heads, cos, sin):
        t = t.view(1, n_heads, self.s.head_dim // 2, 2).float()
        a, b = t[..., 0], t[..., 1]
        out = torch.stack((a * cos - b * sin, a * sin + b * cos), dim=-1)
        return out.view(1, n_heads, self.s.head_dim).to(torch.bfloat16)

    def _attention(self, i):
        s = self.s
        qd, kvd = s.heads * s.head_dim, s.kv_heads * s.head_dim
        h = self._rms(self.x, self.ln1[i])
        qkv = h @ self.wqkv[i].t()
        cos = self.rope_cos.index_select(0, self.pos)
        sin = self.rope_sin.index_select(0, self.pos)
        q = self._rope(qkv[:, :qd], s.heads, cos, sin)
        k = self._rope(qkv[:, qd:qd + kvd], s.kv_heads, cos, sin)
        v = qkv[:, qd + kvd:].view(1, s.kv_heads, s.head_dim)
        self.kcache[i].index_copy_(0, self.pos, k.view(1, s.kv_heads, s.head_dim))
        self.vcache[i].index_copy_(0, self.pos, v)
        mask = (self.positions <= self.pos).view(1, 1, 1, -1)
        o = torch.nn.functional.scaled_dot_product_attention(
            q.view(1, s.heads, 1, s.head_dim), self.kcache[i].permute(1, 0, 2)[None],
            self.vcache[i].permute(1, 0, 2)[None], attn_mask=mask, enable_gqa=True)
        self.x.add_(o.reshape(1, qd) @ self.wo[i].t())
        self.h2.copy_(self._rms(self.x, self.ln2[i]))
        self.moe[i].route(self.h2, self.logits[i:i + 1])

    def _moe(self, i):
        layer = self.moe[i]
        if i not in self.offloaded:
            out = layer.mlp_resident(self.h2, 1)
        elif self.device_staging:
            out = layer.mlp_device(self.h2, 1)
        else:
            out = layer.mlp_slots(self.h2, 1)
        self.x.add_(out)

    def _head(self):
        h = self._rms(self.x, self.final_norm)
        self.token.copy_((h @ self.lm_head.t()).argmax(-1))
        self.x.copy_(self.embed.index_select(0, self.forced if self.teacher_forcing else self.token))
        self.pos.add_(1)

    # ------------------------------------------------------------------ graphs
    def _segments(self):
        """Lists of callables between eager stage points; each segment ends after the
        router of an offloaded layer (whose stage runs eagerly) or at the LM head."""
        segs, cur = [], []
        for i in range(self.s.layers):
            cur.append(lambda i=i: self._attention(i))
            if i in self.offloaded and not self.device_staging:
                segs.append((cur, i))
                cur = []
            cur.append(lambda i=i: self._moe(i))
        cur.append(self._head)
        segs.append((cur, None))
        return segs

    def _stage_all(self, segs):
        for _, stage_layer in segs:
            if stage_layer is not None:
                self.moe[stage_layer].stage(self.moe[stage_layer].topk_ids[:1], PHASE_DECODE)

    def capture(self) -> int:
        """Warm up eagerly (staging every offloaded layer once), then capture one graph per
        segment. Returns the number of graphs."""
        segs = self._segments()
        self.logits.copy_(self.logit_table[0].to(self.device))
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):  # lazy library init happens outside the capture
            for _ in range(2):
                for fns, stage_layer in segs:
                    for fn in fns:
                        fn()
                    if stage_layer is not None:
                        self.moe[stage_layer].stage(self.moe[stage_layer].topk_ids[:1],
                                                    PHASE_DECODE)
        torch.cuda.synchronize()
        self.reset_position()
        pool = torch.cuda.graph_pool_handle()
        self.graphs = []
        for fns, stage_layer in segs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                for fn in fns:
                    fn()
            self.graphs.append((g, stage_layer))
        torch.cuda.synchronize()
        self.reset_position()
        return len(self.graphs)

    def step_eager(self, t: int) -> None:
        """The same token step without graphs (reference for the captured path)."""
        rt = self.runtime
        self.forced.fill_(t % self.s.vocab)
        self.logits.copy_(self.logit_table[t % self.logit_table.shape[0]], non_blocking=True)
        for fns, stage_layer in self._segments():
            for fn in fns:
                fn()
            if stage_layer is not None:
                layer = self.moe[stage_layer]
                decision = layer.stage(layer.topk_ids[:1], PHASE_DECODE)
                handle = rt.begin_slot_compute(decision.prepared)
                rt.end_slot_compute(handle)

    def reset_position(self) -> None:
        """Back to the first generated position with the start token's embedding as input."""
        self.pos.fill_(self.s.prompt)
        self.forced.zero_()
        self.token.zero_()
        self.x.copy_(self.embed[0:1])
        self.h2.zero_()

    def step(self, t: int) -> float:
        """One decode token by graph replay; returns the host time spent in stage seams."""
        rt = self.runtime
        self.forced.fill_(t % self.s.vocab)
        self.logits.copy_(self.logit_table[t % self.logit_table.shape[0]], non_blocking=True)
        stage_s = 0.0
        pending = None
        for g, stage_layer in self.graphs:
            g.replay()
            if pending is not None:
                rt.end_slot_compute(pending)
                pending = None
            if stage_layer is not None:
                t0 = time.perf_counter()
                layer = self.moe[stage_layer]
                decision = layer.stage(layer.topk_ids[:1], PHASE_DECODE)
                if decision.mode != "slots":
                    raise RuntimeError(f"decode stage of layer {stage_layer} chose {decision.mode}")
                pending = rt.begin_slot_compute(decision.prepared)
                stage_s += time.perf_counter() - t0
        rt.end_slot_compute(pending)
        return stage_s

    def moe_share(self, steps: int = 32, warmup: int = 4) -> dict:
        """Device time of the MoE blocks in a decode token beside the rest of the token.

        Each layer's attention piece and MoE piece (router output -> grouped expert MLP ->
        residual) is captured as its own graph and the pieces are replayed in token order
        with an event after each; a token of MoE piece times is summed. Needs a decoder
        without host stage seams (every layer resident or device-staged), so the host
        enqueues whole tokens ahead of the GPU and the intervals hold device time only. The
        per-piece split adds launch gaps the token graphs do not have; the share, not the
        absolute, is the figure."""
        if self.offloaded and not self.device_staging:
            raise ValueError("moe_share needs resident or device-staged layers")
        s = self.s
        if steps + 2 > s.max_new or warmup + 2 > s.max_new:
            raise ValueError(f"at most {s.max_new - 2} decode steps fit the KV cache")
        # every pass below starts from the first generated position (a previous run() may
        # have left the position at the end of the KV cache)
        self.reset_position()
        pieces = []
        for i in range(s.layers):
            pieces.append(("attn", lambda i=i: self._attention(i)))
            pieces.append(("moe", lambda i=i: self._moe(i)))
        pieces.append(("head", self._head))
        self.logits.copy_(self.logit_table[0].to(self.device))
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(2):
                for _, fn in pieces:
                    fn()
        torch.cuda.synchronize()
        self.reset_position()
        pool = torch.cuda.graph_pool_handle()
        graphs = []
        for kind, fn in pieces:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                fn()
            graphs.append((kind, g))
        torch.cuda.synchronize()
        self.reset_position()

        def token(t, evs=None):
            self.forced.fill_(t % s.vocab)
            self.logits.copy_(self.logit_table[t % self.logit_table.shape[0]], non_blocking=True)
            if evs is not None:
                evs[0].record()
            for n, (_, g) in enumerate(graphs):
                g.replay()
                if evs is not None:
                    evs[n + 1].record()

        for t in range(warmup):
            token(t)
        torch.cuda.synchronize()
        self.reset_position()
        moe_ms, tok_ms = [], []
        for t in range(steps):
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(graphs) + 1)]
            token(t, evs)
            evs[-1].synchronize()
            gaps = [evs[n].elapsed_time(evs[n + 1]) for n in range(len(graphs))]
            moe_ms.append(sum(x for x, (kind, _) in zip(gaps, graphs) if kind == "moe"))
            tok_ms.append(sum(gaps))
        del graphs
        self.reset_position()
        moe = statistics.median(moe_ms)
        tok = statistics.median(tok_ms)
        return {"moe_ms_per_token_p50": moe, "token_ms_split_p50": tok,
                "moe_share": moe / tok if tok else None, "steps": steps,
                "pieces_per_token": 2 * s.layers + 1}

    def _stage_counts(self) -> dict:
        """Hits, misses and H2D bytes so far (device counters under device staging)."""
        if not self.device_staging:
            return dict(self.runtime.stage_stats)
        hits = misses = 0
        for i in self.offloaded:
            h, m = self.moe[i].hit_miss.tolist()
            hits, misses = hits + h, misses + m
        per_expert = self.host_store[0][0].nbytes + self.host_store[1][0].nbytes
        return {"hits": hits, "misses": misses, "h2d_bytes": misses * per_expert}

    def run(self, steps: int | None = None, warmup: int = 8) -> TpotReport:
        steps = int(steps or self.s.max_new)
        if steps > self.s.max_new or warmup > self.s.max_new:
            raise ValueError(f"at most {self.s.max_new} decode steps fit the KV cache")
        if not self.graphs:
            self.capture()
        for t in range(warmup):
            self.step(t)
        torch.cuda.synchronize()
        self.reset_position()
        st = self._stage_counts()
        h0, m0, c0 = st["h2d_bytes"], st["misses"], st["hits"]
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        evs[0].record()
        stage_total = 0.0
        for t in range(steps):
            stage_total += self.step(t)
            evs[t + 1].record()
        torch.cuda.synchronize()
        ms = [evs[t].elapsed_time(evs[t + 1]) for t in range(steps)]
        st = self._stage_counts()
        h2d = (st["h2d_bytes"] - h0) / steps
        misses, hits = st["misses"] - m0, st["hits"] - c0
        srt = sorted(ms)
        return TpotReport(
            steps=steps, tpot_ms_p50=statistics.median(ms),
            tpot_ms_p95=srt[min(len(srt) - 1, math.ceil(0.95 * len(srt)) - 1)],
            tpot_ms_mean=statistics.mean(ms), offloaded_layers=len(self.offloaded),
            h2d_bytes_per_step=h2d, h2d_gbs_during_stage=None,
            slot_hit_rate=(hits / (hits + misses)) if (hits + misses) else None,
            graphs=len(self.graphs), stage_ms_per_step=1e3 * stage_total / steps)
