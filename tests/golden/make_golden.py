"""Generate golden control-plane vectors by running the REFERENCE's own Python code.

Run in a container that has the reference checkout (read-only) at REFERENCE_ROOT:

    python tests/golden/make_golden.py [REFERENCE_ROOT]

It imports ``vllm_moe_offload_ascend`` (slot bank, runtime, phase_split) with a two-module
stand-in for ``vllm_ascend.envs`` (the reference reads its settings through that module;
the stand-in answers from the reference's own ``env_registry``), drives it on seeded
inputs with the slot bank on the CPU (as the reference's unit tests do), and writes the
results as JSON next to this script. Tests never import the reference; they compare the
oracle and the product host logic against these files.
"""

from __future__ import annotations

import json
import os
import random
import sys
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _install_reference(root: str) -> None:
    sys.path.insert(0, root)
    from importlib import import_module

    envreg = import_module("vllm_moe_offload_ascend.env_registry")

    class _Envs(types.ModuleType):
        def __getattr__(self, name):
            loader = envreg.ENVIRONMENT_VARIABLES.get(name)
            if loader is None:
                raise AttributeError(name)
            return loader()

    pkg = types.ModuleType("vllm_ascend")
    envs = _Envs("vllm_ascend.envs")
    pkg.envs = envs
    sys.modules["vllm_ascend"] = pkg
    sys.modules["vllm_ascend.envs"] = envs


def _wave_cases(ps):
    rng = random.Random(1234)
    cases = [({1: 10, 2: 9, 3: 8, 4: 1, 5: 1}, 2), ({1: 10, 2: 9, 3: 8, 4: 7}, 4),
             ({5: 100, 1: 90, 2: 80, 4: 70}, 4), ({1: 10, 2: 100, 5: 90}, 3),
             ({e: 1 for e in range(128)}, 32), ({0: 5}, 1)]
    for _ in range(60):
        E = rng.choice([8, 64, 128])
        S = rng.choice([1, 2, 3, 7, 24, 32])
        counts = {e: rng.choice([0, 0, 1, 2, 3, 10, 50, rng.randint(1, 4096)]) for e in range(E)}
        cases.append((counts, S))
    # routing histograms of the seeded benchmark configurations
    import torch

    sys.path.insert(0, str(REPO))
    from oracle import router as orouter
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    for name in ("c1_decode", "c2_prefill", "c4_shared", "c5_ep"):
        cfg = syn.CONFIGS[name]
        logits = syn.make_router_logits(cfg, seed=0)
        _, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=cfg.renormalize)
        counts = torch.bincount(torch.from_numpy(ids.reshape(-1)).long(), minlength=cfg.num_experts)
        cases.append(({e: int(c) for e, c in enumerate(counts.tolist())}, cfg.num_slots))
    out = []
    for counts, S in cases:
        plan = ps.plan_balanced_b2_waves(counts, S)
        out.append({"counts": {str(k): int(v) for k, v in counts.items()}, "num_slots": S,
                    "waves": [list(w) for w in plan.waves]})
    return out


def _schedule_cases(ps):
    rng = random.Random(99)
    out = []
    for _ in range(40):
        n = rng.randint(1, 6)
        waves = tuple(tuple(range(i * 4, i * 4 + rng.randint(1, 4))) for i in range(n))
        ready = {e: rng.random() < 0.4 for w in waves for e in w}
        kw = dict(prefetch_depth=rng.randint(0, 3), buffer_count=rng.randint(1, 3),
                  h2d_bytes_by_wave={i: rng.randint(0, 10) * 1000 for i in range(n)},
                  compute_cost_by_wave={i: float(rng.randint(0, 9)) for i in range(n)},
                  transfer_aware=rng.random() < 0.6)
        sched = ps.plan_b2_prefill_async_schedule(waves, slot_readiness=ready, **kw)
        out.append({
            "waves": [list(w) for w in waves],
            "readiness": {str(k): v for k, v in ready.items()},
            "kwargs": {**kw, "h2d_bytes_by_wave": {str(k): v for k, v in kw["h2d_bytes_by_wave"].items()},
                       "compute_cost_by_wave": {str(k): v for k, v in kw["compute_cost_by_wave"].items()}},
            "schedule": sched.to_jsonable(),
            "issue_log": [list(x) for x in ps.simulate_b2_prefill_issue_log(sched)],
        })
    return out


def _slot_traces():
    import torch
    from vllm_moe_offload_ascend.moe_offload.config import MoeOffloadConfig
    from vllm_moe_offload_ascend.moe_offload.runtime import MoeOffloadRuntime

    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    class Layer(torch.nn.Module):
        def __init__(self, E):
            super().__init__()
            self.layer_id = 3
            self.w13_weight = torch.nn.Parameter(torch.zeros(E, 2, 3))
            self.w2_weight = torch.nn.Parameter(torch.zeros(E, 3, 2))

    traces = []
    rng = random.Random(7)
    seqs = [
        ("reference_test_S4", 5, 4, [(0, 1), (2, 3, 4)]),
        ("locality_k8_S32", 128, 32,
         syn.locality_topk_sequence(syn.CONFIGS["c1_decode"], 64, keep_prob=0.7, seed=0)),
        ("random_S8", 32, 8, [tuple(sorted(rng.sample(range(32), rng.randint(1, 8))))
                              for _ in range(50)]),
        ("evict_later_active_S3", 8, 3, [(5, 6, 7), (0, 5), (1, 2, 6), (0, 1, 7)]),
    ]
    for name, E, S, steps in seqs:
        rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=S, async_load=False,
                                                graph_compatible_offload=True))
        rt.register_layer_for_fixed_slots(Layer(E), slot_device=torch.device("cpu"))
        rec = []
        for active in steps:
            prepared = rt.stage_fixed_slot_plan(layer_id=3, active_experts=tuple(active),
                                                num_logical_experts=E)
            rec.append({"active": list(active),
                        "active_slot_ids": list(prepared.mapping.active_slot_ids),
                        "log2phy": rt.log2phy_buffer(3).tolist()})
        traces.append({"name": name, "num_experts": E, "num_slots": S, "steps": rec})
    return traces


def _pair_plans(ps):
    import torch

    rng = random.Random(5)
    out = []
    cases = [(torch.tensor([[3, 1], [2, 3], [0, 2]]), ((0, 3), (1, 2)))]
    for _ in range(12):
        E = rng.choice([8, 16, 128])
        k = rng.choice([1, 2, 6, 8])
        T = rng.randint(1, 40)
        ids = torch.tensor([rng.sample(range(E), k) for _ in range(T)])
        counts = {int(e): int(c) for e, c in zip(*torch.unique(ids, return_counts=True))}
        waves = ps.plan_balanced_b2_waves(counts, rng.choice([1, 2, 4, 8])).waves
        cases.append((ids, waves))
    for ids, waves in cases:
        E = int(ids.max()) + 1
        active = tuple(sorted(set(ids.reshape(-1).tolist())))
        plans = ps.build_b2_device_wave_microbatch_plans(
            ids, waves, num_logical_experts=E, active_experts=active,
            wave_pair_counts=tuple(int(sum(int((ids == e).sum()) for e in w)) for w in waves))
        out.append({"topk_ids": ids.tolist(), "waves": [list(w) for w in waves],
                    "plans": [{"flat_pair_offsets": p.flat_pair_offsets.tolist(),
                               "token_indices": p.token_indices.tolist(),
                               "physical_slot_ids": p.physical_slot_ids.tolist()} for p in plans]})
    return out


def _combine_index(ps):
    import torch
    from dataclasses import dataclass

    @dataclass(frozen=True)
    class Meta:
        x: int = 0

    rng = random.Random(11)
    out = []
    for case in range(10):
        total = rng.randint(1, 24)
        perm = list(range(total))
        rng.shuffle(perm)
        n_w = rng.randint(1, min(4, total))
        cuts = sorted(rng.sample(range(1, total), n_w - 1)) if n_w > 1 else []
        parts = [perm[a:b] for a, b in zip([0] + cuts, cuts + [total])]
        payloads = []
        for w, offs in enumerate(parts):
            local = list(range(len(offs)))
            rng.shuffle(local)
            payloads.append(ps.B2DirectScatterPayload(
                permuted_tokens=torch.arange(len(offs), dtype=torch.float32).reshape(-1, 1),
                expanded_row_idx=torch.tensor(local, dtype=torch.int32),
                topk_weights=torch.ones(len(offs), 1),
                restore_token_indices=torch.zeros(len(offs), dtype=torch.long),
                pair_offsets=torch.tensor(sorted(offs)), combine_metadata=Meta(), wave_index=w))
        _, index, _ = ps.build_b2_native_combine_inputs(tuple(payloads), total_pairs=total)
        out.append({"total_pairs": total,
                    "waves": [{"pair_offsets": sorted(o), "local": p.expanded_row_idx.tolist()}
                              for o, p in zip(parts, payloads)],
                    "index": index.tolist()})
    return out


def _autoconfig_cases():
    import os
    from types import SimpleNamespace

    from vllm_moe_offload_ascend.moe_offload import autoconfig as ac

    out = []
    cfg = dict(ac._DEFAULT_QWEN3_30B_A3B_CONFIG)
    keys = ("VLLM_ASCEND_MOE_OFFLOAD_SLOT_HBM_BUDGET_GB", "VLLM_ASCEND_MOE_OFFLOAD_MIN_NET_SAVING_RATIO")
    saved = {k: os.environ.get(k) for k in keys}
    try:
        for gb in (7.0, 14.0, 21.0, 28.0, 48.0):
            for budget in ("80", "20"):
                for ratio in (None, "0.75"):
                    for seqs in (1, 8):
                        os.environ[keys[0]] = budget
                        if ratio is None:
                            os.environ.pop(keys[1], None)
                        else:
                            os.environ[keys[1]] = ratio
                        pre = ac.derive_prefetch_defaults(gb, cfg)
                        slots = ac.derive_num_slots_defaults(
                            gb, cfg, pre, SimpleNamespace(max_num_seqs=seqs, max_model_len=None))
                        out.append({"offload_gb": gb, "slot_hbm_budget_gb": budget,
                                    "min_net_saving_ratio": ratio, "max_num_seqs": seqs,
                                    "offloaded_layer_ids": list(pre["offloaded_layer_ids"]),
                                    "num_slots": slots["num_slots"],
                                    "target_b2_waves": slots["target_b2_waves"],
                                    "estimated_b2_waves": slots["estimated_b2_waves"]})
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return out


def _residency_cases():
    """Profiles in the reference's JSONL schema (with malformed lines, other events and bad
    layer ids mixed in) -> the reference loader's per-layer costs and its placement."""
    import tempfile

    from vllm_moe_offload_ascend.moe_offload import prefill_residency as pr

    rng = random.Random(4242)
    out = []
    for case in range(40):
        layers = rng.choice([4, 12, 48])
        offloaded = sorted(rng.sample(range(layers), rng.randint(1, layers - 1)))
        lines = []
        for _ in range(rng.randint(0 if case < 2 else 1, 30)):
            kind = rng.random()
            lid = rng.randrange(-1, layers + 2)
            if kind < 0.45:
                payload = {"n_pairs": rng.randint(0, 32768), "n_waves": rng.randint(1, 6),
                           "n_active": rng.randint(1, 128),
                           "control_ms": {"end_to_end": round(rng.uniform(1, 200), 3)}
                           if rng.random() < 0.8 else {},
                           "waves": [{"gmm_ms": rng.uniform(0, 9), "stage_wait_ms":
                                      rng.uniform(0, 3), "h2d_bytes": rng.randint(0, 10**9)}
                                     for _ in range(rng.randint(0, 3))]}
                if rng.random() < 0.5:
                    payload["wave_summary"] = {"gmm_ms": rng.uniform(0, 50),
                                               "stage_wait_ms": rng.uniform(0, 9),
                                               "h2d_bytes": rng.randint(0, 10**10)}
                    payload["control_ms"]["loop"] = rng.uniform(0, 5)
                rec = {"name": "b2_work_conserving_prefill", "layer_id": lid,
                       "seconds": rng.uniform(0.001, 0.3), "payload": payload}
            elif kind < 0.8:
                rec = {"name": "prefill_resident_native", "layer_id": lid,
                       "seconds": rng.uniform(0.001, 0.3),
                       "payload": {"n_tokens": rng.randint(1, 8192)}}
            elif kind < 0.9:
                rec = {"name": "decode_step", "layer_id": lid, "seconds": 0.5}
            else:
                lines.append("{not json")
                continue
            lines.append(json.dumps(rec))
        with tempfile.NamedTemporaryFile("w", suffix=".jsonl", delete=False) as fh:
            fh.write("\n".join(lines) + "\n")
            path = fh.name
        try:
            costs = pr.load_prefill_layer_costs(path)
        finally:
            os.unlink(path)
        plan = pr.plan_profile_guided_prefill_residency(
            num_layers=layers, default_offloaded_layer_ids=tuple(offloaded), layer_costs=costs)
        out.append({"lines": lines, "num_layers": layers, "default_offloaded": offloaded,
                    "costs": {str(k): v.to_jsonable() for k, v in sorted(costs.items())},
                    "placement": plan.to_jsonable()})
    return out


def main() -> None:
    # the reference checkout: first argument, else LATCHMOE_REFERENCE_ROOT
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LATCHMOE_REFERENCE_ROOT", "")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout> "
                         "(or set LATCHMOE_REFERENCE_ROOT)")
    _install_reference(root)
    sys.path.insert(0, str(REPO))
    from vllm_moe_offload_ascend.moe_offload import phase_split as ps

    blobs = {
        "waves.json": _wave_cases(ps),
        "schedules.json": _schedule_cases(ps),
        "slot_traces.json": _slot_traces(),
        "pair_plans.json": _pair_plans(ps),
        "combine_index.json": _combine_index(ps),
        "autoconfig.json": _autoconfig_cases(),
        "residency.json": _residency_cases(),
    }
    for name, data in blobs.items():
        (HERE / name).write_text(json.dumps(data, separators=(",", ":")) + "\n")
        print(name, len(data))


if __name__ == "__main__":
    main()
