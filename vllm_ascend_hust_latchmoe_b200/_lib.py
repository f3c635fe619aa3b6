"""ctypes binding of liblatchmoe_b200.so (the C ABI declared in include/latchmoe_b200.h).

Every wrapper takes torch tensors, passes raw pointers and the current CUDA stream across
the C boundary, and raises ``RuntimeError`` with the library's message on a negative
return code. There is no fallback: if the library is missing the import of this module
fails loudly, so no CPU or eager path can silently stand in for the kernels.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

from ._build import LIB_PATH

LM_OK = 0
LM_SCORING_SOFTMAX = 0
LM_SCORING_SIGMOID = 1
LM_COPY_H2D = 1
LM_COPY_D2D = 3

DEVERR_NAMES = {
    0: "none",
    1: "top-k id outside [0, num_experts)",
    2: "expert routed but unmapped (log2phy/group entry is -1)",
    3: "bounded device wait timed out",
    4: "group table inconsistent with the pair table",
}

# Every symbol include/latchmoe_b200.h declares, with (restype, argtypes).
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F32 = ctypes.c_float
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "lm_abi_version": (ctypes.c_int, []),
    "lm_last_error": (ctypes.c_char_p, []),
    "lm_route_topk": (
        ctypes.c_int,
        [_P, _I64, _I32, _I32, _I32, _I32, _F32, _P, _I32, _I32, _P, _P, _P, _P],
    ),
    "lm_route_topk_shared": (
        ctypes.c_int,
        [_P, _I64, _I32, _I32, _I32, _I32, _F32, _P, _I32, _I32, _I32, _P, _P, _P, _P],
    ),
    "lm_route_group_small": (
        ctypes.c_int,
        [_P, _I64, _I32, _I32, _I32, _I32, _F32, _P, _I32, _I32, _I32, _P, _P, _P, _I32, _P,
         _I32, _P, _P, _P, _P, _P],
    ),
    "lm_expert_histogram": (ctypes.c_int, [_P, _I64, _I32, _P, _P, _P]),
    "lm_decode_counter_sets": (ctypes.c_int, [_P, _P, _P, _P]),
    "lm_ep_region_bytes": (ctypes.c_int64, [_I32, _I32, _I32]),
    "lm_ep_out_rows_offset": (ctypes.c_int64, [_I32, _I32, _I32]),
    "lm_ep_region_alloc": (ctypes.c_int, [_I64, ctypes.POINTER(ctypes.c_void_p)]),
    "lm_ep_region_free": (ctypes.c_int, [_P]),
    "lm_ipc_get_handle": (ctypes.c_int, [_P, _P]),
    "lm_ipc_open_handle": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    "lm_ipc_close_handle": (ctypes.c_int, [_P]),
    "lm_ep_dispatch": (
        ctypes.c_int,
        [_P, _I64, _I32, _I32, _P, _I32, _P, _P, _I32, _I32, _P, _I32, _I64, _P, _P, _P],
    ),
    "lm_ep_dispatch_tokens": (
        ctypes.c_int,
        [_P, _I64, _I32, _I32, _P, _I32, _P, _P, _I32, _I32, _P, _I32, _I64, _P, _P, _P, _P, _P],
    ),
    "lm_ep_receive": (ctypes.c_int, [_P, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P]),
    "lm_ep_signal_outputs": (ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _I64, _P]),
    "lm_ep_receive_index": (ctypes.c_int, [_P, _I32, _I32, _I32, _I64, _P, _P, _P, _P, _P]),
    "lm_ep_recv_rows_offset": (ctypes.c_int64, [_I32, _I32, _I32]),
    "lm_ep_pair_rows_offset": (ctypes.c_int64, [_I32, _I32, _I32]),
    "lm_permute_rows_gather_count": (ctypes.c_int, [_P, _I32, _P, _P, _I64, _P, _P, _P]),
    "lm_ep_advance_epoch": (ctypes.c_int, [_P, _I32, _I32, _I32, _P]),
    "lm_ep_step_stats": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _P, _P]),
    "lm_ep_output_row_ptrs": (
        ctypes.c_int, [_P, _I32, _I32, _I32, _I32, _P, _P, _P, _I32, _P, _P, _P]),
    "lm_ep_combine_local": (
        ctypes.c_int,
        [_P, _P, _I64, _I32, _I32, _I32, _P, _P, _I32, _I32, _P, _P, _I32, _I64, _P, _P, _P],
    ),
    "lm_ep_combine": (
        ctypes.c_int,
        [_P, _P, _I64, _I32, _I32, _I32, _P, _P, _I32, _I32, _P, _P, _I32, _I64, _P, _P, _P],
    ),
    "lm_slot_plan": (ctypes.c_int, [_P, _I64, _I32, _I32, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "lm_moe_mlp_decode_offload": (
        ctypes.c_int,
        [_P, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _P, _P, _I32, _P, _P, _I32, _I32, _I32,
         _P, _P, _P, _P],
    ),
    "lm_plan_waves": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _P, _P, _P, _P]),
    "lm_build_groups_scratch_elems": (ctypes.c_int64, [_I64, _I32]),
    "lm_build_groups": (
        ctypes.c_int,
        [_P, _I64, _I32, _P, _I32, _P, _P, _P, _P, _I64, _P, _P],
    ),
    "lm_build_groups_noalloc": (
        ctypes.c_int,
        [_P, _I64, _I32, _P, _I32, _P, _P, _P, _P, _P],
    ),
    "lm_permute_rows": (ctypes.c_int, [_P, _I32, _P, _I32, _I64, _P, _P]),
    "lm_permute_rows_count": (ctypes.c_int, [_P, _I32, _P, _I32, _I64, _P, _P, _P]),
    "lm_build_groups_count": (
        ctypes.c_int,
        [_P, _I64, _P, _I32, _P, _I32, _P, _P, _P, _P, _I64, _P, _P],
    ),
    "lm_moe_combine_count": (ctypes.c_int, [_P, _P, _P, _I64, _P, _I32, _I32, _P, _P]),
    "lm_moe_mlp_decode": (
        ctypes.c_int,
        [_P, _I32, _P, _P, _P, _I32, _I32, _I32, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P],
    ),
    "lm_moe_mlp_prefill": (
        ctypes.c_int,
        [_P, _I64, _P, _P, _I32, _I32, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P],
    ),
    "lm_moe_mlp_prefill_rows": (
        ctypes.c_int,
        [_P, _I64, _P, _P, _I32, _I32, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P],
    ),
    "lm_stage_wave_copy": (
        ctypes.c_int, [_P, _I64, _I32, _P, _I64, _I32, _I64, _P, _P, _P, _I32, _P]),
    "lm_moe_mlp_prefill_wave": (
        ctypes.c_int,
        [_P, _I64, _P, _P, _P, _P, _I32, _P, _P, _I64, _I32, _I32, _P, _P, _P, _P],
    ),
    "lm_moe_combine": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _P, _P]),
    "lm_stage_copy": (
        ctypes.c_int,
        [_P, _I64, _P, _I64, _P, _P, _I32, _I64, _I32, _P],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load the library once and bind every declared symbol (raises if absent)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        lib_path = Path(path) if path is not None else LIB_PATH
        if not lib_path.exists():
            raise RuntimeError(
                f"{lib_path.name} is not built at {lib_path}; run "
                "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a). "
                "There is no CPU fallback for the MoE data path."
            )
        lib = ctypes.CDLL(str(lib_path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.lm_abi_version() != 1:
            raise RuntimeError("liblatchmoe_b200.so ABI version mismatch")
        _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load()


def _check(name: str, rc: int) -> int:
    if rc < 0:
        msg = lib().lm_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed ({rc}): {msg}")
    return rc


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _require_cuda(*tensors: torch.Tensor | None) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("liblatchmoe_b200 kernels take CUDA tensors only")


def route_group_small(logits, top_k, *, scoring_func="softmax", renormalize=True,
                      routed_scaling_factor=1.0, e_score_correction_bias=None,
                      num_expert_group=None, topk_group=None, num_shared=0, weights_bf16,
                      ids, num_experts_total, expert_to_group, num_groups, group_offsets,
                      pair_to_row, row_to_pair, err_word=None, weights_f32=None) -> None:
    """Routing and grouping of a decode-sized call in one launch (same outputs as
    :func:`route_topk` followed by :func:`build_groups`)."""
    _require_cuda(logits, weights_bf16, ids, expert_to_group, group_offsets, pair_to_row,
                  row_to_pair)
    assert logits.dtype == torch.float32 and logits.is_contiguous()
    T, E = logits.shape
    scoring = {"softmax": LM_SCORING_SOFTMAX, "sigmoid": LM_SCORING_SIGMOID}.get(scoring_func)
    if scoring is None:
        raise ValueError(f"unsupported scoring_func {scoring_func!r}")
    if ids.shape[-1] != top_k + num_shared or weights_bf16.shape[-1] != top_k + num_shared:
        raise ValueError("outputs need top_k + num_shared columns")
    _check(
        "lm_route_group_small",
        lib().lm_route_group_small(
            _ptr(logits), T, E, int(top_k), scoring, int(bool(renormalize)),
            float(routed_scaling_factor), _ptr(e_score_correction_bias),
            int(num_expert_group or 0), int(topk_group or 0), int(num_shared),
            _ptr(weights_bf16), _ptr(weights_f32), _ptr(ids), int(num_experts_total),
            _ptr(expert_to_group), int(num_groups), _ptr(group_offsets), _ptr(pair_to_row),
            _ptr(row_to_pair), _ptr(err_word), _stream(),
        ),
    )


def route_topk(
    logits: torch.Tensor,
    top_k: int,
    *,
    scoring_func: str = "softmax",
    renormalize: bool = True,
    routed_scaling_factor: float = 1.0,
    e_score_correction_bias: torch.Tensor | None = None,
    num_expert_group: int | None = None,
    topk_group: int | None = None,
    weights_bf16: torch.Tensor,
    ids: torch.Tensor,
    weights_f32: torch.Tensor | None = None,
    num_shared: int = 0,
) -> None:
    """Top-k routing into ``weights_bf16`` / ``ids`` ``[T, top_k]``; with ``num_shared`` > 0
    the rows are ``top_k + num_shared`` wide and end with the fused shared experts' ids
    (``E .. E + num_shared - 1``, weight 1)."""
    _require_cuda(logits, weights_bf16, ids, weights_f32, e_score_correction_bias)
    assert logits.dtype == torch.float32 and logits.is_contiguous()
    T, E = logits.shape
    scoring = {"softmax": LM_SCORING_SOFTMAX, "sigmoid": LM_SCORING_SIGMOID}.get(scoring_func)
    if scoring is None:
        raise ValueError(f"unsupported scoring_func {scoring_func!r}")
    if num_shared:
        if ids.shape[-1] != top_k + num_shared or weights_bf16.shape[-1] != top_k + num_shared:
            raise ValueError("mix-placement outputs need top_k + num_shared columns")
        _check(
            "lm_route_topk_shared",
            lib().lm_route_topk_shared(
                _ptr(logits), T, E, int(top_k), scoring, int(bool(renormalize)),
                float(routed_scaling_factor), _ptr(e_score_correction_bias),
                int(num_expert_group or 0), int(topk_group or 0), int(num_shared),
                _ptr(weights_bf16), _ptr(weights_f32), _ptr(ids), _stream(),
            ),
        )
        return
    _check(
        "lm_route_topk",
        lib().lm_route_topk(
            _ptr(logits), T, E, int(top_k), scoring, int(bool(renormalize)),
            float(routed_scaling_factor), _ptr(e_score_correction_bias),
            int(num_expert_group or 0), int(topk_group or 0),
            _ptr(weights_bf16), _ptr(weights_f32), _ptr(ids), _stream(),
        ),
    )


def expert_histogram(ids: torch.Tensor, num_experts: int, counts: torch.Tensor,
                     err_word: torch.Tensor | None = None) -> None:
    _require_cuda(ids, counts, err_word)
    _check(
        "lm_expert_histogram",
        lib().lm_expert_histogram(_ptr(ids), ids.numel(), int(num_experts), _ptr(counts),
                                  _ptr(err_word), _stream()),
    )


def plan_waves(counts: torch.Tensor, num_slots: int, expert_to_group: torch.Tensor,
               group_bank_row: torch.Tensor, wave_offsets: torch.Tensor,
               num_waves: torch.Tensor, *, in_place_rows: bool = True) -> None:
    _require_cuda(counts, expert_to_group, group_bank_row, wave_offsets, num_waves)
    _check(
        "lm_plan_waves",
        lib().lm_plan_waves(_ptr(counts), counts.numel(), int(num_slots),
                            0 if in_place_rows else 1, _ptr(expert_to_group),
                            _ptr(group_bank_row), _ptr(wave_offsets), _ptr(num_waves),
                            _stream()),
    )


def build_groups_scratch_elems(num_pairs: int, num_groups: int) -> int:
    return int(lib().lm_build_groups_scratch_elems(int(num_pairs), int(num_groups)))


def build_groups(ids: torch.Tensor, num_experts: int, expert_to_group: torch.Tensor,
                 num_groups: int, group_offsets: torch.Tensor, pair_to_row: torch.Tensor,
                 row_to_pair: torch.Tensor, scratch: torch.Tensor,
                 err_word: torch.Tensor | None = None) -> None:
    _require_cuda(ids, expert_to_group, group_offsets, pair_to_row, row_to_pair, scratch)
    _check(
        "lm_build_groups",
        lib().lm_build_groups(
            _ptr(ids), ids.numel(), int(num_experts), _ptr(expert_to_group), int(num_groups),
            _ptr(group_offsets), _ptr(pair_to_row), _ptr(row_to_pair), _ptr(scratch),
            scratch.numel(), _ptr(err_word), _stream(),
        ),
    )


def build_groups_noalloc(ids: torch.Tensor, num_experts: int, expert_to_group: torch.Tensor,
                         num_groups: int, group_offsets: torch.Tensor, pair_to_row: torch.Tensor,
                         row_to_pair: torch.Tensor, err_word: torch.Tensor | None = None) -> None:
    """lm_build_groups with the library's built-in static scratch (no device allocation by
    the caller or the library); see include/latchmoe_b200.h for its size limit."""
    _require_cuda(ids, expert_to_group, group_offsets, pair_to_row, row_to_pair)
    _check(
        "lm_build_groups_noalloc",
        lib().lm_build_groups_noalloc(
            _ptr(ids), ids.numel(), int(num_experts), _ptr(expert_to_group), int(num_groups),
            _ptr(group_offsets), _ptr(pair_to_row), _ptr(row_to_pair), _ptr(err_word),
            _stream(),
        ),
    )


def build_groups_count(ids: torch.Tensor, num_pairs_dev: torch.Tensor, num_experts: int,
                       expert_to_group: torch.Tensor, num_groups: int,
                       group_offsets: torch.Tensor, pair_to_row: torch.Tensor,
                       row_to_pair: torch.Tensor, scratch: torch.Tensor,
                       err_word: torch.Tensor | None = None) -> None:
    """lm_build_groups over the first ``num_pairs_dev`` (int32 on the device) of ``ids``."""
    _require_cuda(ids, num_pairs_dev, expert_to_group, group_offsets, pair_to_row, row_to_pair,
                  scratch)
    _check(
        "lm_build_groups_count",
        lib().lm_build_groups_count(
            _ptr(ids), ids.numel(), _ptr(num_pairs_dev), int(num_experts),
            _ptr(expert_to_group), int(num_groups), _ptr(group_offsets), _ptr(pair_to_row),
            _ptr(row_to_pair), _ptr(scratch), scratch.numel(), _ptr(err_word), _stream(),
        ),
    )


def permute_rows_count(hidden: torch.Tensor, row_to_pair: torch.Tensor, top_k: int,
                       max_rows: int, num_rows_dev: torch.Tensor, x_perm: torch.Tensor) -> None:
    """lm_permute_rows over the first ``num_rows_dev`` (device int32) of ``max_rows`` rows."""
    _require_cuda(hidden, row_to_pair, num_rows_dev, x_perm)
    _check(
        "lm_permute_rows_count",
        lib().lm_permute_rows_count(_ptr(hidden), hidden.shape[-1], _ptr(row_to_pair),
                                    int(top_k), int(max_rows), _ptr(num_rows_dev), _ptr(x_perm),
                                    _stream()),
    )


def moe_combine_count(y_perm, pair_to_row, topk_weights_bf16, num_tokens_dev, out) -> None:
    """lm_moe_combine over the first ``num_tokens_dev`` (device int32) tokens of
    ``topk_weights_bf16`` / ``out``."""
    _require_cuda(y_perm, pair_to_row, topk_weights_bf16, num_tokens_dev, out)
    T, k = topk_weights_bf16.shape
    _check(
        "lm_moe_combine_count",
        lib().lm_moe_combine_count(_ptr(y_perm), _ptr(pair_to_row), _ptr(topk_weights_bf16), T,
                                   _ptr(num_tokens_dev), k, out.shape[-1], _ptr(out),
                                   _stream()),
    )


def permute_rows(hidden: torch.Tensor, row_to_pair: torch.Tensor, top_k: int, num_rows: int,
                 x_perm: torch.Tensor) -> None:
    _require_cuda(hidden, row_to_pair, x_perm)
    _check(
        "lm_permute_rows",
        lib().lm_permute_rows(_ptr(hidden), hidden.shape[-1], _ptr(row_to_pair), int(top_k),
                              int(num_rows), _ptr(x_perm), _stream()),
    )


def moe_mlp_decode(hidden, top_k, row_to_pair, group_offsets, group_bank_row, group_begin,
                   group_end, max_rows_per_group, w13_bank, w2_bank, act, y_perm,
                   err_word=None) -> None:
    _require_cuda(hidden, row_to_pair, group_offsets, group_bank_row, w13_bank, w2_bank, act,
                  y_perm)
    H = hidden.shape[-1]
    I = w2_bank.shape[-1]
    _check(
        "lm_moe_mlp_decode",
        lib().lm_moe_mlp_decode(
            _ptr(hidden), int(top_k), _ptr(row_to_pair), _ptr(group_offsets),
            _ptr(group_bank_row), int(group_begin), int(group_end), int(max_rows_per_group),
            _ptr(w13_bank), _ptr(w2_bank), w13_bank.shape[0], H, I, _ptr(act), _ptr(y_perm),
            _ptr(err_word), _stream(),
        ),
    )


def moe_mlp_prefill(x_perm, total_rows, group_offsets, group_bank_row, group_begin, group_end,
                    w13_bank, w2_bank, act, y_perm, err_word=None) -> None:
    _require_cuda(x_perm, group_offsets, group_bank_row, w13_bank, w2_bank, act, y_perm)
    H = x_perm.shape[-1]
    I = w2_bank.shape[-1]
    _check(
        "lm_moe_mlp_prefill",
        lib().lm_moe_mlp_prefill(
            _ptr(x_perm), int(total_rows), _ptr(group_offsets), _ptr(group_bank_row),
            int(group_begin), int(group_end), _ptr(w13_bank), _ptr(w2_bank),
            w13_bank.shape[0], H, I, _ptr(act), _ptr(y_perm), _ptr(err_word), _stream(),
        ),
    )


def moe_mlp_prefill_rows(x_perm, total_rows, group_offsets, group_bank_row, group_begin,
                         group_end, w13_bank, w2_bank, act, y_row_ptrs, err_word=None) -> None:
    """The prefill MLP with output row r stored at the address ``y_row_ptrs[r]`` (int64)."""
    _require_cuda(x_perm, group_offsets, group_bank_row, w13_bank, w2_bank, act, y_row_ptrs)
    H = x_perm.shape[-1]
    I = w2_bank.shape[-1]
    _check(
        "lm_moe_mlp_prefill_rows",
        lib().lm_moe_mlp_prefill_rows(
            _ptr(x_perm), int(total_rows), _ptr(group_offsets), _ptr(group_bank_row),
            int(group_begin), int(group_end), _ptr(w13_bank), _ptr(w2_bank),
            w13_bank.shape[0], H, I, _ptr(act), _ptr(y_row_ptrs), _ptr(err_word), _stream(),
        ),
    )


def stage_wave_copy(dst: torch.Tensor, src: torch.Tensor, expert_to_group, wave_offsets,
                    num_waves, wave: int, stream: torch.cuda.Stream | None = None) -> None:
    """Copy the experts a device wave plan put in wave ``wave`` from ``src`` (row e = expert
    e) into ``dst`` rows 0.. in group order (no host read of the plan)."""
    _require_cuda(dst, src, expert_to_group, wave_offsets, num_waves)
    row_bytes = dst[0].numel() * dst.element_size()
    if src[0].numel() * src.element_size() != row_bytes or src.dtype != dst.dtype:
        raise ValueError("stage_wave_copy: source and destination rows differ")
    _check("lm_stage_wave_copy", lib().lm_stage_wave_copy(
        _ptr(dst), dst.stride(0) * dst.element_size(), dst.shape[0], _ptr(src),
        src.stride(0) * src.element_size(), src.shape[0], row_bytes, _ptr(expert_to_group),
        _ptr(wave_offsets), _ptr(num_waves), int(wave), _stream(stream)))


def moe_mlp_prefill_wave(x_perm, total_rows, group_offsets, group_bank_row, wave_offsets,
                         num_waves, wave, w13_bank, w2_bank, act, y_perm, err_word=None) -> None:
    """The prefill MLP over the groups of wave ``wave`` of a device wave plan."""
    _require_cuda(x_perm, group_offsets, group_bank_row, wave_offsets, num_waves, w13_bank,
                  w2_bank, act, y_perm)
    _check("lm_moe_mlp_prefill_wave", lib().lm_moe_mlp_prefill_wave(
        _ptr(x_perm), int(total_rows), _ptr(group_offsets), _ptr(group_bank_row),
        _ptr(wave_offsets), _ptr(num_waves), int(wave), _ptr(w13_bank), _ptr(w2_bank),
        w13_bank.shape[0], x_perm.shape[-1], w2_bank.shape[-1], _ptr(act), _ptr(y_perm),
        _ptr(err_word), _stream()))


def ep_region_bytes(world: int, cap: int, hidden: int) -> int:
    return int(lib().lm_ep_region_bytes(int(world), int(cap), int(hidden)))


def ep_out_rows_offset(world: int, cap: int, hidden: int) -> int:
    return int(lib().lm_ep_out_rows_offset(int(world), int(cap), int(hidden)))


def ep_region_alloc(nbytes: int) -> int:
    out = ctypes.c_void_p()
    _check("lm_ep_region_alloc", lib().lm_ep_region_alloc(int(nbytes), ctypes.byref(out)))
    return int(out.value)


def ep_region_free(ptr: int) -> None:
    _check("lm_ep_region_free", lib().lm_ep_region_free(ptr))


def ipc_get_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(64)
    _check("lm_ipc_get_handle", lib().lm_ipc_get_handle(ptr, buf))
    return buf.raw


def ipc_open_handle(handle: bytes) -> int:
    buf = ctypes.create_string_buffer(bytes(handle), 64)
    out = ctypes.c_void_p()
    _check("lm_ipc_open_handle", lib().lm_ipc_open_handle(buf, ctypes.byref(out)))
    return int(out.value)


def ipc_close_handle(ptr: int) -> None:
    _check("lm_ipc_close_handle", lib().lm_ipc_close_handle(ptr))


def ep_dispatch(hidden, topk_ids, experts_per_rank, pair_to_row, send_offsets, rank, world,
                peer_regions, cap, epoch, done_counter, err_word=None) -> None:
    T, k = topk_ids.shape
    _check("lm_ep_dispatch", lib().lm_ep_dispatch(
        _ptr(hidden), T, k, hidden.shape[-1], _ptr(topk_ids), int(experts_per_rank),
        _ptr(pair_to_row), _ptr(send_offsets), int(rank), int(world), _ptr(peer_regions),
        int(cap), int(epoch), _ptr(done_counter), _ptr(err_word), _stream()))


def ep_dispatch_tokens(hidden, topk_ids, experts_per_rank, pair_to_row, send_offsets, rank,
                       world, peer_regions, cap, epoch, tok_slot, tok_count, done_counter,
                       err_word=None) -> None:
    """Token-deduplicated dispatch: each token row goes once to each owner holding any of its
    experts (tok_slot [T * world], tok_count [world] are written, on the device)."""
    T, k = topk_ids.shape
    _check("lm_ep_dispatch_tokens", lib().lm_ep_dispatch_tokens(
        _ptr(hidden), T, k, hidden.shape[-1], _ptr(topk_ids), int(experts_per_rank),
        _ptr(pair_to_row), _ptr(send_offsets), int(rank), int(world), _ptr(peer_regions),
        int(cap), int(epoch), _ptr(tok_slot), _ptr(tok_count), _ptr(done_counter),
        _ptr(err_word), _stream()))


def ep_receive(region: int, world, cap, hidden_size, epoch, rows_out, ids_out, total_out,
               err_word=None) -> None:
    _check("lm_ep_receive", lib().lm_ep_receive(
        region, int(world), int(cap), int(hidden_size), int(epoch), _ptr(rows_out),
        _ptr(ids_out), _ptr(total_out), _ptr(err_word), _stream()))


def ep_receive_index(region: int, world, cap, hidden_size, epoch, slot_out, ids_out, total_out,
                     err_word=None) -> None:
    _check("lm_ep_receive_index", lib().lm_ep_receive_index(
        region, int(world), int(cap), int(hidden_size), int(epoch), _ptr(slot_out),
        _ptr(ids_out), _ptr(total_out), _ptr(err_word), _stream()))


def ep_recv_rows_offset(world, cap, hidden_size) -> int:
    return int(lib().lm_ep_recv_rows_offset(int(world), int(cap), int(hidden_size)))


def ep_pair_rows_offset(world, cap, hidden_size) -> int:
    return int(lib().lm_ep_pair_rows_offset(int(world), int(cap), int(hidden_size)))


def permute_rows_gather_count(src, row_to_pair, pair_src, max_rows, count_dev, x_perm) -> None:
    """x_perm[r] = src[pair_src[row_to_pair[r]]] for r < *count_dev (rows read at L2)."""
    _require_cuda(src, row_to_pair, pair_src, count_dev, x_perm)
    _check("lm_permute_rows_gather_count", lib().lm_permute_rows_gather_count(
        _ptr(src), src.shape[-1], _ptr(row_to_pair), _ptr(pair_src), int(max_rows),
        _ptr(count_dev), _ptr(x_perm), _stream()))


def ep_signal_outputs(peer_regions, rank, world, cap, hidden_size, epoch) -> None:
    _check("lm_ep_signal_outputs", lib().lm_ep_signal_outputs(
        _ptr(peer_regions), int(rank), int(world), int(cap), int(hidden_size), int(epoch),
        _stream()))


def ep_advance_epoch(region: int, world, cap, hidden_size) -> None:
    """Raise the region's device-side call counter (the epoch of calls given epoch 0)."""
    _check("lm_ep_advance_epoch", lib().lm_ep_advance_epoch(
        region, int(world), int(cap), int(hidden_size), _stream()))


def ep_step_stats(total, send_offsets, tok_count, num_pairs, rank, world, stats) -> None:
    """Accumulate one exchange step's figures into ``stats`` (int64 [4], on the device)."""
    _check("lm_ep_step_stats", lib().lm_ep_step_stats(
        _ptr(total), _ptr(send_offsets), _ptr(tok_count), int(num_pairs), int(rank), int(world),
        _ptr(stats), _stream()))


def ep_output_row_ptrs(region: int, world, cap, hidden_size, rank, peer_regions, row_to_pair,
                       count_dev, max_rows, row_ptrs_out, err_word=None) -> None:
    """Row pointers (int64 tensor) of an owner's grouped output rows in the sources' areas."""
    _check("lm_ep_output_row_ptrs", lib().lm_ep_output_row_ptrs(
        region, int(world), int(cap), int(hidden_size), int(rank), _ptr(peer_regions),
        _ptr(row_to_pair), _ptr(count_dev), int(max_rows), _ptr(row_ptrs_out), _ptr(err_word),
        _stream()))


def ep_combine_local(topk_ids, topk_weights_bf16, experts_per_rank, pair_to_row, send_offsets,
                     rank, world, peer_regions, local_region: int, cap, epoch, out,
                     err_word=None) -> None:
    """Combine of outputs the owners pushed into this rank's own output area."""
    T, k = topk_ids.shape
    _check("lm_ep_combine_local", lib().lm_ep_combine_local(
        _ptr(topk_ids), _ptr(topk_weights_bf16), T, k, out.shape[-1], int(experts_per_rank),
        _ptr(pair_to_row), _ptr(send_offsets), int(rank), int(world), _ptr(peer_regions),
        local_region, int(cap), int(epoch), _ptr(out), _ptr(err_word), _stream()))


def ep_combine(topk_ids, topk_weights_bf16, experts_per_rank, pair_to_row, send_offsets, rank,
               world, peer_regions, local_region: int, cap, epoch, out, err_word=None) -> None:
    T, k = topk_ids.shape
    _check("lm_ep_combine", lib().lm_ep_combine(
        _ptr(topk_ids), _ptr(topk_weights_bf16), T, k, out.shape[-1], int(experts_per_rank),
        _ptr(pair_to_row), _ptr(send_offsets), int(rank), int(world), _ptr(peer_regions),
        local_region, int(cap), int(epoch), _ptr(out), _ptr(err_word), _stream()))


LM_SRC_MISS = 0x40000000
LM_SRC_HOST = -2


def slot_plan(topk_ids, num_experts, slot_owner, slot_last_used, expert_slot, step_counter,
              log2phy, group_src, hit_miss=None, err_word=None) -> None:
    """Device-side stage decision (see ``lm_slot_plan``); all state tensors on the device."""
    _require_cuda(topk_ids, slot_owner, slot_last_used, expert_slot, step_counter, log2phy,
                  group_src)
    _check(
        "lm_slot_plan",
        lib().lm_slot_plan(
            _ptr(topk_ids), topk_ids.numel(), int(num_experts), slot_owner.numel(),
            _ptr(slot_owner), _ptr(slot_last_used), _ptr(expert_slot), _ptr(step_counter),
            _ptr(log2phy), _ptr(group_src), _ptr(hit_miss), _ptr(err_word), _stream(),
        ),
    )


def decode_counter_sets() -> dict:
    """Counter sets of the persistent decode kernel on the current device."""
    u, p = ctypes.c_int32(0), ctypes.c_int32(0)
    r, f = ctypes.c_int64(0), ctypes.c_int64(0)
    _check("lm_decode_counter_sets", lib().lm_decode_counter_sets(
        ctypes.byref(u), ctypes.byref(p), ctypes.byref(r), ctypes.byref(f)))
    return {"in_use": u.value, "pinned": p.value, "recycled": r.value, "fallbacks": f.value}


def moe_mlp_decode_offload(hidden, top_k, row_to_pair, group_offsets, group_src, group_expert,
                           group_begin, group_end, max_rows_per_group, w13_slots, w2_slots,
                           w13_host, w2_host, act, y_perm, err_word=None) -> None:
    """Decode MLP reading each group's weights from a slot or the pinned host store."""
    _require_cuda(hidden, row_to_pair, group_offsets, group_src, group_expert, w13_slots,
                  w2_slots, act, y_perm)
    H = hidden.shape[-1]
    I = w2_slots.shape[-1]
    _check(
        "lm_moe_mlp_decode_offload",
        lib().lm_moe_mlp_decode_offload(
            _ptr(hidden), int(top_k), _ptr(row_to_pair), _ptr(group_offsets), _ptr(group_src),
            _ptr(group_expert), int(group_begin), int(group_end), int(max_rows_per_group),
            _ptr(w13_slots), _ptr(w2_slots), w13_slots.shape[0], _ptr(w13_host), _ptr(w2_host),
            w13_host.shape[0], H, I, _ptr(act), _ptr(y_perm), _ptr(err_word), _stream(),
        ),
    )


def moe_combine(y_perm, pair_to_row, topk_weights_bf16, out) -> None:
    _require_cuda(y_perm, pair_to_row, topk_weights_bf16, out)
    T, k = topk_weights_bf16.shape
    _check(
        "lm_moe_combine",
        lib().lm_moe_combine(_ptr(y_perm), _ptr(pair_to_row), _ptr(topk_weights_bf16), T, k,
                             out.shape[-1], _ptr(out), _stream()),
    )


def stage_copy(dst: torch.Tensor, src: torch.Tensor, src_rows: list[int], dst_rows: list[int],
               stream: torch.cuda.Stream | None = None) -> int:
    """Copy expert rows src[src_rows[i]] -> dst[dst_rows[i]] (first dim = expert/slot row)."""
    if len(src_rows) != len(dst_rows):
        raise ValueError("src_rows and dst_rows must have the same length")
    n = len(src_rows)
    if n == 0:
        return 0
    if not dst.is_cuda:
        raise RuntimeError("stage_copy destination must be a CUDA tensor")
    if src.is_cuda:
        kind = LM_COPY_D2D
    else:
        if not src.is_pinned():
            raise RuntimeError("stage_copy host source must be pinned (cudaHostAlloc) memory")
        kind = LM_COPY_H2D
    row_bytes = dst[0].numel() * dst.element_size()
    if src[0].numel() * src.element_size() != row_bytes or src.dtype != dst.dtype:
        raise ValueError("stage_copy: source and destination rows differ in size or dtype")
    arr = ctypes.c_int32 * n
    src_arr = arr(*[int(r) for r in src_rows])
    dst_arr = arr(*[int(r) for r in dst_rows])
    return _check(
        "lm_stage_copy",
        lib().lm_stage_copy(
            _ptr(dst), dst.stride(0) * dst.element_size(), _ptr(src),
            src.stride(0) * src.element_size(), src_arr, dst_arr, n, row_bytes, kind,
            _stream(stream),
        ),
    )


def read_err_word(err_word: torch.Tensor) -> int:
    return int(err_word.item())


def raise_on_device_error(err_word: torch.Tensor, where: str) -> None:
    code = read_err_word(err_word)
    if code != 0:
        raise RuntimeError(f"{where}: device error {code} ({DEVERR_NAMES.get(code, '?')})")
