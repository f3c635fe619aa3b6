"""Seeded synthetic inputs for the slot-bank MoE layer (no dataset or checkpoint needed).

Shapes follow the benchmark configurations of the offload path (Qwen3-30B-A3B-,
DeepSeek-V2-Lite- and Qwen3-235B-A22B-shaped MoE layers). Every tensor is drawn from a
CPU ``torch.Generator`` with its own sub-seed in a fixed order, so the CPU oracle and the
GPU path see bit-identical inputs on any machine:

* expert weights bf16 ~ N(0, 0.02): ``w13 [E, 2I, H]`` (rows 0..I-1 gate, I..2I-1 up) and
  ``w2 [E, H, I]``; shared experts (if any) fused into one MLP of intermediate
  ``num_shared * I``;
* activations bf16 ~ N(0, 1): ``hidden [T, H]``;
* router logits fp32 = N(0, 1) + Zipf(s) bias, ``bias_e = -s * ln(rank_e)`` with ``rank`` a
  seeded permutation of 1..E (a few hot experts, a long tail).
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch


@dataclass(frozen=True)
class LayerConfig:
    name: str
    hidden: int
    num_experts: int
    top_k: int
    intermediate: int
    num_slots: int
    tokens: int
    renormalize: bool = True
    routed_scaling_factor: float = 1.0
    scoring_func: str = "softmax"
    num_expert_group: int = 0
    topk_group: int = 0
    num_shared: int = 0
    zipf_s: float = 1.1

    @property
    def expert_bytes(self) -> int:
        """bf16 bytes of one routed expert (w13 + w2) = 6 * H * I."""
        return 6 * self.hidden * self.intermediate

    @property
    def flops_per_pair(self) -> int:
        return 6 * self.hidden * self.intermediate

    def with_tokens(self, tokens: int) -> "LayerConfig":
        return replace(self, tokens=int(tokens))


QWEN3_30B = dict(hidden=2048, num_experts=128, top_k=8, intermediate=768)
CONFIGS: dict[str, LayerConfig] = {
    # C1: decode layer, 16 tokens, 32 slots.
    "c1_decode": LayerConfig("qwen3-30b-a3b/decode-t16-s32", tokens=16, num_slots=32, **QWEN3_30B),
    # C2: multi-wave prefill, 4096 tokens, 32 slots (working set > capacity -> >= 4 waves).
    "c2_prefill": LayerConfig("qwen3-30b-a3b/prefill-t4096-s32", tokens=4096, num_slots=32,
                              **QWEN3_30B),
    # C4: DeepSeek-V2-Lite-shaped shared-expert layer.
    "c4_shared": LayerConfig("deepseek-v2-lite/decode-t64-s24", hidden=2048, num_experts=64,
                             top_k=6, intermediate=1408, num_slots=24, tokens=64,
                             renormalize=False, num_expert_group=1, topk_group=1,
                             num_shared=2),
    # C5: Qwen3-235B-A22B-shaped layer for the expert-partitioned multi-GPU bank.
    "c5_ep": LayerConfig("qwen3-235b-a22b/decode-t256", hidden=4096, num_experts=128, top_k=8,
                         intermediate=1536, num_slots=48, tokens=256),
}


class ExpertLayer(torch.nn.Module):
    """The attributes the runtime reads from a MoE layer when it registers the layer's
    experts (``register_layer_for_fixed_slots``): ``layer_id``, ``w13_weight [E, 2I, H]``,
    ``w2_weight [E, H, I]`` and ``num_fused_shared_experts``. Stands in for a loaded model's
    FusedMoE module when the weights are synthetic."""

    def __init__(self, layer_id: int, w13: torch.Tensor, w2: torch.Tensor, shared: int = 0):
        super().__init__()
        self.layer_id = layer_id
        self.w13_weight = w13
        self.w2_weight = w2
        self.num_fused_shared_experts = shared


def _gen(seed: int, index: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed) * 1_000_003 + int(index))
    return g


def zipf_bias(num_experts: int, s: float, seed: int) -> torch.Tensor:
    rank = torch.randperm(num_experts, generator=_gen(seed, 1)).to(torch.float64) + 1.0
    return (-s * torch.log(rank)).to(torch.float32)


def make_router_logits(cfg: LayerConfig, seed: int = 0, tokens: int | None = None,
                       bias_seed: int | None = None) -> torch.Tensor:
    """Router logits: N(0, 1) noise from ``seed`` plus the Zipf bias of ``bias_seed``
    (default ``seed``). Ranks of one expert-parallel model share the bias seed (the experts'
    popularity is a property of the model) and differ in the noise (their tokens)."""
    T = cfg.tokens if tokens is None else int(tokens)
    noise = torch.randn(T, cfg.num_experts, generator=_gen(seed, 2), dtype=torch.float32)
    bseed = seed if bias_seed is None else bias_seed
    return noise + zipf_bias(cfg.num_experts, cfg.zipf_s, bseed)[None, :]


def make_hidden(cfg: LayerConfig, seed: int = 0, tokens: int | None = None) -> torch.Tensor:
    T = cfg.tokens if tokens is None else int(tokens)
    return torch.randn(T, cfg.hidden, generator=_gen(seed, 3), dtype=torch.float32).to(
        torch.bfloat16)


def make_expert_weights(cfg: LayerConfig, seed: int = 0, experts: int | None = None,
                        std: float = 0.02) -> tuple[torch.Tensor, torch.Tensor]:
    E = cfg.num_experts if experts is None else int(experts)
    H, I = cfg.hidden, cfg.intermediate
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16)
    g = _gen(seed, 4)
    # Expert by expert keeps the fp32 staging buffer small for large layers.
    for e in range(E):
        w13[e] = (torch.randn(2 * I, H, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)
        w2[e] = (torch.randn(H, I, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)
    return w13, w2


def make_shared_weights(cfg: LayerConfig, seed: int = 0,
                        std: float = 0.02) -> tuple[torch.Tensor, torch.Tensor]:
    """Resident shared experts fused into one MLP: ``[2*Is, H]`` and ``[H, Is]``, Is = n_shared*I."""
    Is = cfg.num_shared * cfg.intermediate
    g = _gen(seed, 5)
    w13 = (torch.randn(2 * Is, cfg.hidden, generator=g) * std).to(torch.bfloat16)
    w2 = (torch.randn(cfg.hidden, Is, generator=g) * std).to(torch.bfloat16)
    return w13, w2


def locality_topk_sequence(cfg: LayerConfig, steps: int, keep_prob: float = 0.7,
                           seed: int = 0) -> list[tuple[int, ...]]:
    """Decode-time expert sets with temporal locality (batch 1): each step keeps each of the
    previous top-k ids with probability ``keep_prob`` and redraws the rest without
    replacement from the Zipf-biased router distribution."""
    g = _gen(seed, 6)
    probs = torch.softmax(zipf_bias(cfg.num_experts, cfg.zipf_s, seed).double(), dim=0)
    prev = tuple(sorted(torch.multinomial(probs, cfg.top_k, generator=g).tolist()))
    out = [prev]
    for _ in range(steps - 1):
        keep = [e for e in prev if torch.rand((), generator=g).item() < keep_prob]
        p = probs.clone()
        if keep:
            p[list(keep)] = 0.0
        need = cfg.top_k - len(keep)
        new = torch.multinomial(p / p.sum(), need, generator=g).tolist() if need else []
        prev = tuple(sorted(keep + new))
        out.append(prev)
    return out


def active_union(topk_ids: torch.Tensor) -> int:
    return int(torch.unique(topk_ids).numel())


def roofline_bytes_decode(cfg: LayerConfig, active_experts: int) -> int:
    """Algorithmic HBM bytes of one decode layer call: each active expert's weights once,
    plus hidden in/out, fp32 logits and the top-k tables."""
    T = cfg.tokens
    return (active_experts * cfg.expert_bytes + 2 * T * cfg.hidden * 2 + T * cfg.num_experts * 4
            + T * cfg.top_k * 8)


def ceil_div(a: int, b: int) -> int:
    return -(-int(a) // int(b))
