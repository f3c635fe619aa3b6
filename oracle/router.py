"""Router oracle: expert selection on the CPU in numpy (parity unpinned, see package doc).

Follows the call-site semantics of the reference router seam:
  * ``ops/fused_moe/moe_router_op.py:98-124`` -- ``select_experts`` with top_k, grouped
    selection, renormalize, scoring_func, routed_scaling_factor, correction bias;
  * ``patches/patch_fused_moe.py:597-637`` -- the gating fallback: scores -> top-k, then,
    if ``renorm``, ``w / clamp_min(sum(w), finfo(fp32).eps)``;
  * ``ops/fused_moe/moe_router_op.py:143-150`` -- weights are cast to the hidden dtype
    (bf16) and ids to int32.
Selection order: highest score first, the lower expert id wins a tie.
"""

from __future__ import annotations

import numpy as np

from .bf16 import f32_to_bf16_bits

FP32_EPS = np.float32(np.finfo(np.float32).eps)


def scores_of(logits: np.ndarray, scoring_func: str = "softmax") -> np.ndarray:
    logits = np.asarray(logits, dtype=np.float32)
    if scoring_func == "softmax":
        m = logits.max(axis=1, keepdims=True)
        ex = np.exp(logits - m, dtype=np.float32)
        return (ex / ex.sum(axis=1, keepdims=True, dtype=np.float32)).astype(np.float32)
    if scoring_func == "sigmoid":
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-logits, dtype=np.float32))).astype(
            np.float32
        )
    raise ValueError(f"unsupported scoring_func {scoring_func!r}")


def _ranked(values: np.ndarray, count: int) -> np.ndarray:
    """Indices of the `count` largest values, descending, ties toward the lower index."""
    idx = np.arange(values.shape[-1])
    order = np.lexsort((idx, -values.astype(np.float64)))
    return order[:count]


def route(
    logits: np.ndarray,
    top_k: int,
    *,
    renormalize: bool = True,
    routed_scaling_factor: float = 1.0,
    scoring_func: str = "softmax",
    e_score_correction_bias: np.ndarray | None = None,
    num_expert_group: int = 0,
    topk_group: int = 0,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Return ``(topk_weights_bf16_bits[T,k] uint16, topk_weights_f32[T,k], topk_ids[T,k] int32)``."""
    logits = np.asarray(logits, dtype=np.float32)
    T, E = logits.shape
    scores = scores_of(logits, scoring_func)
    choice = scores if e_score_correction_bias is None else (
        scores + np.asarray(e_score_correction_bias, dtype=np.float32)[None, :]
    )
    ids = np.zeros((T, top_k), dtype=np.int32)
    w = np.zeros((T, top_k), dtype=np.float32)
    grouped = num_expert_group and num_expert_group > 1 and topk_group < num_expert_group
    for t in range(T):
        c = choice[t].copy()
        if grouped:
            gsize = E // num_expert_group
            groups = c.reshape(num_expert_group, gsize)
            if e_score_correction_bias is None:
                gscore = groups.max(axis=1)
            else:
                top2 = -np.sort(-groups, axis=1)[:, :2]
                gscore = top2.sum(axis=1)
            keep = _ranked(gscore, topk_group)
            mask = np.ones(num_expert_group, dtype=bool)
            mask[keep] = False
            c = c.copy()
            c.reshape(num_expert_group, gsize)[mask] = -np.inf
        sel = _ranked(c, top_k)
        ids[t] = sel
        w[t] = scores[t, sel]
    if renormalize:
        s = w.sum(axis=1, keepdims=True, dtype=np.float32)
        w = (w / np.maximum(s, FP32_EPS)).astype(np.float32)
    w = (w * np.float32(routed_scaling_factor)).astype(np.float32)
    return f32_to_bf16_bits(w), w, ids


def route_by_logit_order(logits: np.ndarray, top_k: int) -> np.ndarray:
    """Top-k ids ranked on the raw logits (lower id wins ties). Softmax and sigmoid are
    monotone, so this equals the score ranking unless two different logits round to the
    same fp32 score; tests use it to show the seeded inputs contain no such tie."""
    logits = np.asarray(logits, dtype=np.float32)
    return np.stack([_ranked(row, top_k) for row in logits]).astype(np.int32)
