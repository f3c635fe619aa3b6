"""Time the host control plane of the REFERENCE beside this package's (CPU, this machine).

    python tests/golden/time_control_plane.py <reference checkout>

Imports the reference through the same two-module stand-in as ``make_golden.py`` and times,
on the seeded benchmark inputs:

* ``plan_balanced_b2_waves`` on the 4096-token C2 routing histogram (126 active experts,
  32 slots);
* ``MoeOffloadRuntime.stage_fixed_slot_plan`` over the 64-step decode locality trace (128
  experts, 32 slots, top-8; the slot bank on the CPU with tiny expert rows, so the figure is
  the decision logic and the bookkeeping, not weight copies).

Each is also timed with this package's host implementation of the same function. The GPU
counterparts (``lm_plan_waves``, ``lm_slot_plan``) are timed by ``bench.py``'s launch lists.
Prints one JSON object; the numbers go into the baseline notes.
"""

from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1]))

from make_golden import _install_reference  # noqa: E402


def _best_us(fn, repeats: int = 5, inner: int = 20) -> float:
    best = float("inf")
    for _ in range(repeats):
        t0 = time.perf_counter()
        for _ in range(inner):
            fn()
        best = min(best, (time.perf_counter() - t0) / inner)
    return best * 1e6


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LATCHMOE_REFERENCE_ROOT", "")
    if not root:
        raise SystemExit("usage: time_control_plane.py <reference checkout>")
    _install_reference(root)
    import torch

    from oracle import router as orouter
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig as OurConfig
    from vllm_ascend_hust_latchmoe_b200.moe_offload import phase_split as our_ps
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime as OurRuntime
    from vllm_moe_offload_ascend.moe_offload import phase_split as ref_ps
    from vllm_moe_offload_ascend.moe_offload.config import MoeOffloadConfig as RefConfig
    from vllm_moe_offload_ascend.moe_offload.runtime import MoeOffloadRuntime as RefRuntime

    cfg = syn.CONFIGS["c2_prefill"]
    ids = orouter.route(syn.make_router_logits(cfg, seed=0).numpy(), cfg.top_k)[2]
    hist = torch.bincount(torch.from_numpy(ids.reshape(-1)).long(), minlength=cfg.num_experts)
    counts = {e: int(c) for e, c in enumerate(hist.tolist()) if c}
    out = {"threads": torch.get_num_threads(), "cpu_count": os.cpu_count()}
    out["plan_balanced_b2_waves_us"] = {
        "reference": _best_us(lambda: ref_ps.plan_balanced_b2_waves(counts, 32)),
        "ours": _best_us(lambda: our_ps.plan_balanced_b2_waves(counts, 32)),
        "input": f"C2 histogram, {len(counts)} active experts, 32 slots"}

    class Layer(torch.nn.Module):
        def __init__(self, E):
            super().__init__()
            self.layer_id = 3
            self.w13_weight = torch.nn.Parameter(torch.zeros(E, 2, 3))
            self.w2_weight = torch.nn.Parameter(torch.zeros(E, 3, 2))

    trace = syn.locality_topk_sequence(syn.CONFIGS["c1_decode"], 64, keep_prob=0.7, seed=0)

    def run_trace(runtime_cls, config_cls):
        rt = runtime_cls(config_cls(enabled=True, num_slots=32, async_load=False,
                                    graph_compatible_offload=True))
        rt.register_layer_for_fixed_slots(Layer(128), slot_device=torch.device("cpu"))
        t0 = time.perf_counter()
        for active in trace:
            rt.stage_fixed_slot_plan(layer_id=3, active_experts=tuple(active),
                                     num_logical_experts=128)
        return (time.perf_counter() - t0) / len(trace) * 1e6

    out["stage_fixed_slot_plan_us_per_step"] = {
        "reference": min(run_trace(RefRuntime, RefConfig) for _ in range(5)),
        "ours": min(run_trace(OurRuntime, OurConfig) for _ in range(5)),
        "input": "64-step decode locality trace, 128 experts, 32 slots, top-8 (CPU bank)"}
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
