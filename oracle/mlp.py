"""Expert MLP + combine oracle in numpy (parity unpinned for values, see package doc).

Restates the layer arithmetic the reference delegates to its host apply path
(``moe_offload/phase_split.py:2167`` unified_apply_mlp; ``patches/patch_fused_moe.py:
4249-4302`` two grouped matmuls + swiglu; ``phase_split.py:1765-1856`` and
``patch_fused_moe.py:3340-3366`` one top-k combine in the original pair order):

  y1[p]  = bf16( x[token(p)] . W13[e(p)]^T )              fp32 accumulate, bf16 output
  act[p] = bf16( silu(y1[p, :I]) * y1[p, I:] )             gate = first I columns
  y2[p]  = bf16( act[p] . W2[e(p)]^T )
  out[t] = bf16( sum_{j<k} f32(w_bf16[t, j]) * y2[t*k + j] )  fp32, in j order

Weights use the slot-bank layout of this build: W13 ``[E, 2I, H]`` and W2 ``[E, H, I]``
(K-major rows, the checkpoint layout of ``moe_offload/cpu_first_loader.py:64-82``).
"""

from __future__ import annotations

import numpy as np

from .bf16 import bf16_bits_to_f32, round_bf16


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x, dtype=np.float32))).astype(np.float32)


def expert_mlp(x: np.ndarray, w13: np.ndarray, w2: np.ndarray) -> np.ndarray:
    """One expert on rows ``x [n, H]`` (fp32 values of bf16 data) -> ``y2 [n, H]`` (bf16 values)."""
    inter = w2.shape[1]
    y1 = round_bf16(x @ w13.T)
    act = round_bf16(silu(y1[:, :inter]) * y1[:, inter:])
    return round_bf16(act @ w2.T)


def _as_f32(w: np.ndarray) -> np.ndarray:
    """bf16 bit patterns (uint16) -> fp32 values; fp32 arrays (pre-converted) pass through."""
    return bf16_bits_to_f32(w) if w.dtype == np.uint16 else w


def pair_outputs(hidden_bits: np.ndarray, topk_ids: np.ndarray, w13_bits: np.ndarray,
                 w2_bits: np.ndarray, experts: np.ndarray | None = None) -> np.ndarray:
    """y2 for every routed pair, ``[T*k, H]`` fp32 (bf16 values), in flat pair order.

    Weights are bf16 bit patterns or their fp32 values (converted once, like loaded
    parameters). ``experts`` optionally restricts the computation to a subset (pairs of
    other experts stay zero); the union over disjoint subsets equals the full result.
    """
    x_all = bf16_bits_to_f32(hidden_bits)
    T, k = topk_ids.shape
    H = x_all.shape[1]
    flat = topk_ids.reshape(-1)
    out = np.zeros((T * k, H), dtype=np.float32)
    todo = np.unique(flat) if experts is None else np.asarray(experts)
    for e in todo:
        pairs = np.nonzero(flat == e)[0]
        if pairs.size == 0:
            continue
        x = x_all[pairs // k]
        out[pairs] = expert_mlp(x, _as_f32(w13_bits[e]), _as_f32(w2_bits[e]))
    return out


def combine(y2_pairs: np.ndarray, topk_weights_bits: np.ndarray) -> np.ndarray:
    """Weighted top-k combine in the original pair order; returns bf16 values (fp32)."""
    T, k = topk_weights_bits.shape
    w = bf16_bits_to_f32(topk_weights_bits)
    y = y2_pairs.reshape(T, k, -1)
    acc = np.zeros((T, y.shape[-1]), dtype=np.float32)
    for j in range(k):
        acc = (acc + w[:, j : j + 1] * y[:, j, :]).astype(np.float32)
    return round_bf16(acc)


def moe_layer(hidden_bits, topk_ids, topk_weights_bits, w13_bits, w2_bits) -> np.ndarray:
    """Full routed-expert layer output ``[T, H]`` (bf16 values as fp32)."""
    return combine(pair_outputs(hidden_bits, topk_ids, w13_bits, w2_bits), topk_weights_bits)


def shared_mlp(hidden_bits, w13_shared_bits, w2_shared_bits) -> np.ndarray:
    """Resident shared expert(s) fused into one MLP, applied to every token."""
    return expert_mlp(bf16_bits_to_f32(hidden_bits), bf16_bits_to_f32(w13_shared_bits),
                      bf16_bits_to_f32(w2_shared_bits))


def compare(actual: np.ndarray, expected: np.ndarray) -> dict[str, float]:
    """Tolerance metrics used by the parity tests: max |a-e| / max |e| and cosine."""
    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    e = np.asarray(expected, dtype=np.float64).reshape(-1)
    denom = max(float(np.abs(e).max()), 1e-30)
    max_rel = float(np.abs(a - e).max()) / denom
    cos = float(a @ e / max(np.linalg.norm(a) * np.linalg.norm(e), 1e-30))
    return {"max_rel_err": max_rel, "cosine": cos}
