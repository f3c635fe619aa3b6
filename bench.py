"""Benchmark of the B200 slot-bank MoE hot path (one JSON line on stdout, rank 0).

Workload (N=1): the multi-wave prefill layer on synthetic Qwen3-30B-A3B-shaped data
(4096 tokens x hidden 2048, 128 experts, top-8, moe_intermediate 768, bf16 weights, 32 slots:
the routed working set exceeds the slots, so the layer runs >= 4 capacity-bounded waves and
one final combine). One step = one full layer call.

* ``value``: layer tokens/s with hidden states, router logits and the layer's experts already
  in HBM (an HBM-resident expert tier: each wave's experts are read in place).
* ``e2e``: the same layer through the public layer API from HOST buffers: pinned hidden
  states and logits copied in, every expert staged from the pinned host store into the
  double-buffered stage banks on the copy stream (the offload path), the output copied out.
* ``roofline``: the grouped expert MLP (``lm_moe_mlp_prefill``: gate_up+SiLU*mul and down
  launches of the tcgen05 kernel), algorithmic FLOPs = pairs * 6 * H * I per call, timed with
  CUDA events on its stream inside the timed region, against the measured bf16 peak.
* ``cpu_baseline``: the numpy oracle (a restatement of the reference path) on a bounded
  token sample on the host cores.

``--impl reference`` times that CPU implementation alone (the reference ships no native or
GPU code for this path; its arithmetic runs in an absent Ascend stack), prints the same line
with ``"impl": "reference"`` and exits. Under torchrun only rank 0 runs it.
N > 1: one independent replica of the layer per GPU (weak scaling, no data-path collective);
timing is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "moe_layer_tokens_per_s"
UNIT = "tokens/s"
CONFIG_NAME = "c2_prefill"


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


def _clock_process(conn, bus: str, index: int, period: float) -> None:
    """Child process body: polls NVML between "start" and "stop" messages (its own
    interpreter, so the launch loop's GIL cannot starve it)."""
    import time

    import pynvml

    pynvml.nvmlInit()
    try:
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
    except Exception:
        h = pynvml.nvmlDeviceGetHandleByIndex(index)
    conn.send(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
    while conn.recv() == "start":
        samples = []
        while True:
            try:
                samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))))
            except Exception:
                pass
            if conn.poll():
                break
            time.sleep(period)
        conn.recv()
        conn.send(samples)
    pynvml.nvmlShutdown()


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML every millisecond while the timed
    region runs, from a spawned child process (the timed region is often only tens of ms)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, cuda_index: int, period_s: float = 0.001) -> None:
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._proc = None
        self._conn = None

    def __enter__(self):
        import multiprocessing as mp

        import torch

        try:
            p = torch.cuda.get_device_properties(self.cuda_index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            ctx = mp.get_context("spawn")
            self._conn, child = ctx.Pipe()
            self._proc = ctx.Process(target=_clock_process,
                                     args=(child, bus, self.cuda_index, self.period), daemon=True)
            self._proc.start()
            if not self._conn.poll(60):
                raise TimeoutError("clock sampler did not start")
            self.max_mhz = self._conn.recv()
            self._conn.send("start")
        except Exception:
            self._stop_proc()
        return self

    def _stop_proc(self):
        if self._proc is not None:
            self._proc.join(timeout=5)
            if self._proc.is_alive():
                self._proc.kill()
        self._proc = None

    def __exit__(self, *exc):
        if self._proc is None:
            return
        try:
            self._conn.send("stop")
            if self._conn.poll(10):
                self.samples = self._conn.recv()
            self._conn.send("quit")
        except Exception:
            pass
        self._stop_proc()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml"}
        seen = 0
        for _, r in self.samples:
            seen |= r
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz,
                "reasons": sorted(n for n, bit in self.REASONS.items() if seen & bit),
                "samples": len(self.samples), "source": "nvml (1 ms, separate process)"}


def _profiled_traffic(name: str) -> int | None:
    """DRAM bytes (read + write) per call from a committed ncu summary under profiles/: the
    value of its ``traffic_bytes_per_call:`` line."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_call:"):
            return int(line.split(":", 1)[1].strip().split()[0])
    return None


# --------------------------------------------------------------------------- CPU arm
def use_all_host_threads() -> int:
    """Give the CPU arm every host core, whatever the launcher set: torchrun exports
    OMP_NUM_THREADS=1 when it starts more than one process, which numpy's BLAS and torch
    both honour. Returns the BLAS thread count in effect."""
    cores = os.cpu_count() or 1
    import torch

    torch.set_num_threads(cores)
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=cores)
        blas = [int(i["num_threads"]) for i in threadpool_info()
                if i.get("user_api") == "blas" and i.get("num_threads")]
        return max(blas) if blas else cores
    except Exception:
        return cores


def cpu_reference_step(cfg, tokens: int, w13, w2, hidden_bits, logits_np) -> float:
    """One bounded oracle pass (router + grouped MLP + combine) on `tokens` tokens; expert
    weights are fp32 arrays indexed by expert id (converted once, like loaded parameters)."""
    from oracle import mlp as omlp
    from oracle import router as orouter

    t0 = time.perf_counter()
    wb, _, ids = orouter.route(logits_np[:tokens], cfg.top_k, renormalize=cfg.renormalize,
                               routed_scaling_factor=cfg.routed_scaling_factor,
                               scoring_func=cfg.scoring_func,
                               num_expert_group=cfg.num_expert_group, topk_group=cfg.topk_group)
    omlp.moe_layer(hidden_bits[:tokens], ids, wb, w13, w2)
    return time.perf_counter() - t0


def _bits(t):
    import numpy as np
    import torch

    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def cpu_inputs(cfg, tokens: int):
    """The GPU arm's own seeded inputs (weights, hidden, logits), weights as fp32 numpy."""
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    w13, w2 = syn.make_expert_weights(cfg, 0)
    hidden = syn.make_hidden(cfg, 0, tokens=tokens)
    logits = syn.make_router_logits(cfg, 0, tokens=tokens)
    return w13.float().numpy(), w2.float().numpy(), _bits(hidden), logits.numpy()


def cpu_inputs_routed(cfg, tokens: int):
    """Inputs for a timing sample of a large layer: seeded hidden states and logits, and
    N(0, 0.02) fp32 weights for only the experts the sample routes to (the CPU pass touches
    no other expert), so a Qwen3-235B-shaped sample does not materialise all 128 experts."""
    import numpy as np
    import torch

    from oracle import router as orouter
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    logits = syn.make_router_logits(cfg, 0, tokens=tokens).numpy()
    hidden = _bits(syn.make_hidden(cfg, 0, tokens=tokens))
    ids = orouter.route(logits, cfg.top_k, renormalize=cfg.renormalize)[2]
    g = torch.Generator().manual_seed(0)
    H, I = cfg.hidden, cfg.intermediate
    w13, w2 = {}, {}
    for e in np.unique(ids).tolist():
        w13[e] = (torch.randn(2 * I, H, generator=g) * 0.02).numpy()
        w2[e] = (torch.randn(H, I, generator=g) * 0.02).numpy()
    return w13, w2, hidden, logits


# CPU samples of the other benchmark layers: (config, tokens per timed pass)
CPU_CONFIG_SAMPLES = (("c1_decode", 16), ("c4_shared", 64), ("c5_ep", 64))


def cpu_config_times(headline: dict, repeats: int = 3) -> dict:
    """Median wall time of the CPU pass of each benchmark layer on the host cores; the C2
    entry is the headline figure measured by the caller (`headline`)."""
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    out = {}
    for name, tokens in CPU_CONFIG_SAMPLES:
        cfg = syn.CONFIGS[name]
        tokens = min(tokens, cfg.tokens)
        ins = cpu_inputs_routed(cfg, tokens)
        cpu_reference_step(cfg, tokens, *ins)
        tt = sorted(cpu_reference_step(cfg, tokens, *ins) for _ in range(repeats))
        ms = 1e3 * tt[len(tt) // 2]
        out[name] = {"workload": cfg.name, "tokens": tokens, "full_tokens": cfg.tokens,
                     "ms_per_pass": ms, "tokens_per_s": tokens / (ms / 1e3),
                     "weights": "seeded N(0,0.02) fp32 for the routed experts"}
        del ins
    out["c2_prefill"] = headline
    return out


def run_reference(args, cfg) -> dict:
    """The CPU implementation of the path, timed on the host cores (bounded samples)."""
    cores = os.cpu_count() or 1
    threads = use_all_host_threads()
    sample = args.cpu_sample_tokens
    w13, w2, hid, lg = cpu_inputs(cfg, sample)
    for _ in range(max(0, args.warmup)):
        cpu_reference_step(cfg, sample, w13, w2, hid, lg)
    times = [cpu_reference_step(cfg, sample, w13, w2, hid, lg) for _ in range(args.steps)]
    del w13, w2
    total = sum(times)
    value = sample * len(times) / total
    per_config = cpu_config_times({"workload": cfg.name, "tokens": sample,
                                   "full_tokens": cfg.tokens,
                                   "ms_per_pass": 1e3 * total / len(times),
                                   "tokens_per_s": value,
                                   "weights": "the GPU arm's seeded bf16 weights as fp32"})
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) bf16 weights, Zipf-biased router)",
        "config": {"workload": cfg.name, "tokens_per_step": sample, "full_tokens": cfg.tokens,
                   "same_config": False,
                   "sample_rule": "each step is the first 1024 of the 4096 tokens (same seeded "
                                  "inputs as the GPU arm); tokens/s normalises the sample",
                   "hidden": cfg.hidden, "experts": cfg.num_experts, "top_k": cfg.top_k,
                   "moe_intermediate": cfg.intermediate, "num_slots": cfg.num_slots},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "threads": threads,
                         "kind": "port",
                         "sample": f"{sample} of {cfg.tokens} tokens per step, numpy fp32 BLAS",
                         "per_config": per_config},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# --------------------------------------------------------------------------- layer check
def torch_layer_reference(hidden, ids, weights_bf16, w13_of, w2_of):
    """fp32 torch restatement of the routed layer, used by the bench to check the outputs it
    times (the numpy oracle is reserved for the tests and the CPU arm): per routed pair
    y1 = bf16(x . W13^T), act = bf16(silu(y1[:, :I]) * y1[:, I:]), y2 = bf16(act . W2^T);
    out[t] = bf16(sum_j f32(w[t, j]) * y2[t, j]) accumulated in fp32 in j order.
    ``w13_of(e)`` / ``w2_of(e)`` return expert e's row-major bf16 weights."""
    import torch

    T, k = ids.shape
    H = hidden.shape[1]
    x = hidden.float()
    y = torch.zeros(T, k, H, dtype=torch.float32, device=hidden.device)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for e in torch.unique(ids).tolist():
            t_idx, j_idx = (ids == e).nonzero(as_tuple=True)
            w13 = w13_of(e).float()
            w2 = w2_of(e).float()
            inter = w2.shape[1]
            y1 = (x[t_idx] @ w13.T).to(torch.bfloat16).float()
            gate = y1[:, :inter]
            act = (gate / (1.0 + torch.exp(-gate)) * y1[:, inter:]).to(torch.bfloat16).float()
            y[t_idx, j_idx] = (act @ w2.T).to(torch.bfloat16).float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    w = weights_bf16.float()
    acc = torch.zeros(T, H, dtype=torch.float32, device=hidden.device)
    for j in range(k):
        acc = acc + w[:, j:j + 1] * y[:, j]
    return acc.to(torch.bfloat16)


def torch_route_reference(logits, top_k: int, renormalize: bool = True):
    """softmax(fp32) -> top-k -> w / max(sum w, eps) -> bf16 weights, int32 ids."""
    import torch

    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, top_k, dim=-1)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True).clamp_min(torch.finfo(torch.float32).eps)
    return w.to(torch.bfloat16), ids.to(torch.int32)


def compare_outputs(actual, expected) -> dict:
    """max |a - e| / max |e| and cosine, in fp64."""
    a = actual.double().reshape(-1)
    e = expected.double().reshape(-1)
    denom = max(float(e.abs().max()), 1e-30)
    cos = float(a @ e / max(float(a.norm() * e.norm()), 1e-30))
    return {"max_rel_err": float((a - e).abs().max()) / denom, "cosine": cos}


# --------------------------------------------------------------------------- C5 (N > 1)
def ep_expert_weights(e: int, cfg, dev):
    """Expert e of the expert-partitioned layer: bf16 N(0, 0.02), seeded per expert so any
    rank can rebuild any expert (its owner's bank, or a checker on another rank)."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(7000 + int(e))
    I, H = cfg.intermediate, cfg.hidden
    w13 = (torch.randn(2 * I, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(H, I, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    return w13, w2


EP_CHECK_TOKENS = 8  # tokens per rank checked against the torch reference after timing
EP_MAX_REL_ERR = 1e-2
EP_MIN_COSINE = 0.9999


def run_expert_parallel(dist, rank: int, world: int, dev, args) -> dict:
    """Qwen3-235B-A22B-shaped layer with the expert bank partitioned over the ranks: 256
    decode tokens per step in total (256 / N per rank). Cases: HBM-resident store with the
    exchange over NCCL (exact splits read on the host, or fixed-size blocks sized from the
    routing with no host read) and over peer memory (the library's dispatch / combine kernels), and a
    pinned-host store staged into half as many slots as the rank owns experts (peer
    exchange). Times are the max over ranks; `hbm_gbs_per_rank` counts the weights of the
    rank's active experts read once per step. After timing, each case's output for the
    rank's first tokens is checked against the torch fp32 restatement of the layer (the
    1-GPU semantics), worst case over ranks."""
    import torch

    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import (ExpertParallelMoE, PeerExchange,
                                                                build_rank_layer, cuda_ops)

    cfg = syn.CONFIGS["c5_ep"]
    T = cfg.tokens // world
    per = cfg.num_experts // world
    I, H = cfg.intermediate, cfg.hidden
    owned = [ep_expert_weights(rank * per + i, cfg, dev) for i in range(per)]
    w13 = torch.stack([a for a, _ in owned])
    w2 = torch.stack([b for _, b in owned])
    del owned
    hidden = syn.make_hidden(cfg, seed=rank, tokens=T).to(dev)
    all_logits = syn.make_router_logits(cfg, seed=0, tokens=cfg.tokens)
    logits = all_logits[rank * T:(rank + 1) * T].to(dev)
    ids_all = torch.topk(all_logits, cfg.top_k, dim=1).indices
    owned_ids = ids_all[(ids_all // per) == rank]
    active_owned = int(torch.unique(owned_ids).numel())
    # fixed NCCL block size: the largest (source, owner) pair count of this routing, plus a
    # quarter (the capacity an expert-parallel deployment provisions from a profile)
    block_counts = torch.stack([torch.bincount((ids_all[r * T:(r + 1) * T] // per).reshape(-1),
                                               minlength=world) for r in range(world)])
    rows_per_peer = min(T * cfg.top_k, -(-int(block_counts.max()) * 5 // 4))
    expert_bytes = 6 * H * I
    n_chk = min(EP_CHECK_TOKENS, T)
    w_ref, ids_ref = torch_route_reference(logits[:n_chk], cfg.top_k)
    cache: dict[int, tuple] = {}

    def weights_of(e):
        if e not in cache:
            cache[e] = ep_expert_weights(e, cfg, dev)
        return cache[e]

    ref = torch_layer_reference(hidden[:n_chk], ids_ref, w_ref, lambda e: weights_of(e)[0],
                                lambda e: weights_of(e)[1])
    cache.clear()
    out = {"workload": cfg.name, "tokens_per_step": cfg.tokens, "tokens_per_rank": T,
           "experts_per_rank": per, "active_experts_rank": active_owned}
    cases = (("resident_nccl", True, per, "nccl"), ("resident_nccl_fixed", True, per, "nccl_fixed"),
             ("resident_peer", True, per, "peer"),
             ("offloaded_peer", False, max(1, per // 2), "peer"))
    for name, on_dev, slots, transport in cases:
        local = build_rank_layer(w13_owned=w13 if on_dev else w13.cpu(),
                                 w2_owned=w2 if on_dev else w2.cpu(), rank=rank, device=dev,
                                 max_rows=cfg.tokens * cfg.top_k, num_slots=slots,
                                 store_on_device=on_dev)
        exchange = None
        if transport == "peer":
            exchange = PeerExchange(world_size=world, rank=rank, max_tokens=T,
                                    top_k=cfg.top_k, hidden_size=H, device=dev)
        ep = ExpertParallelMoE(num_experts=cfg.num_experts, top_k=cfg.top_k, hidden_size=H,
                               rank=rank, world_size=world, device=dev, exchange=exchange,
                               ops=cuda_ops(local, num_experts=cfg.num_experts, top_k=cfg.top_k,
                                            max_tokens=T),
                               nccl_rows_per_peer=rows_per_peer
                               if transport == "nccl_fixed" else None)
        for _ in range(3):
            ep.forward(hidden, logits)
        torch.cuda.synchronize()
        dist.barrier()
        sent0 = ep.stats.bytes_sent
        h2d0 = local.runtime.transfer_engine.stats.bytes_h2d
        steps = 10
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            ep.forward(hidden, logits)
        e.record()
        torch.cuda.synchronize()
        local.check_device_errors("bench ep")
        ep.check_exchange_errors()
        ms = torch.tensor([s.elapsed_time(e) / steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        t_ms = float(ms.item())
        nv = (ep.stats.bytes_sent - sent0) / steps
        h2d = (local.runtime.transfer_engine.stats.bytes_h2d - h2d0) / steps
        # correctness of what was timed: one more call, its first tokens against the reference
        got = ep.forward(hidden, logits)
        torch.cuda.synchronize()
        local.check_device_errors("bench ep check")
        ep.check_exchange_errors()
        m = compare_outputs(got[:n_chk], ref)
        worst = torch.tensor([m["max_rel_err"], -m["cosine"]], dtype=torch.float64, device=dev)
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
        parity = {"max_rel_err": float(worst[0]), "cosine": -float(worst[1]),
                  "tokens_checked_per_rank": n_chk, "ranks": world,
                  "bar": {"max_rel_err": EP_MAX_REL_ERR, "cosine": EP_MIN_COSINE},
                  "reference": "torch fp32 restatement of the 1-GPU layer"}
        parity["ok"] = parity["max_rel_err"] <= EP_MAX_REL_ERR and parity["cosine"] >= EP_MIN_COSINE
        out[name] = {"transport": transport, "ms_per_step": t_ms,
                     "tokens_per_s": cfg.tokens / (t_ms / 1e3),
                     "nvlink_bytes_per_rank_step": nv,
                     "hbm_gbs_per_rank": active_owned * expert_bytes / (t_ms / 1e3) / 1e9,
                     "slots_per_rank": slots if not on_dev else None,
                     "h2d_bytes_rank0_step": int(h2d), "parity": parity}
        if transport == "nccl_fixed":
            out[name]["rows_per_peer"] = rows_per_peer
        if exchange is not None:
            exchange.close()
        del ep, local
        torch.cuda.empty_cache()
    return out


def run_value(args, cfg, make_layer, hidden, logits, dist, dev, world, local_rank, peaks,
              barrier):
    """``value``: the C2 layer with hidden states, logits and the expert store in HBM. The
    layer step (route, grouping by expert id, row permute, grouped MLP, combine; no host
    synchronisation on this tier) is captured once as a CUDA graph, as vLLM's
    piecewise capture runs it, and replayed `steps` times. The grouped MLP alone is captured
    as a second graph and replayed right after the timed steps, bracketed by CUDA events on
    the replay stream: its mean duration is the roofline's kernel time."""
    import torch

    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    layer = make_layer(True)
    T = cfg.tokens
    for _ in range(args.warmup):
        layer.forward(hidden, logits)
    torch.cuda.synchronize()
    layer.check_device_errors("bench warmup")
    store = layer.runtime.host_layer(layer.layer_id)
    launches0 = layer.kernel_launches
    g_layer, g_mlp = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_layer):
        layer.route(hidden, logits)
        layer.mlp_resident(hidden, T)
    launches_per_step = layer.kernel_launches - launches0
    bank_rows = layer.group_bank_row if layer.resident_planned else layer.identity_groups
    with torch.cuda.graph(g_mlp):
        layer._grouped_mlp(hidden, T, bank_rows, 0, layer.E, store.w13, store.w2)
    for _ in range(3):
        g_layer.replay()
        g_mlp.replay()
    torch.cuda.synchronize()
    layer.check_device_errors("bench graph warmup")

    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    m_start, m_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        t_start.record()
        for _ in range(args.steps):
            g_layer.replay()
        t_end.record()
        barrier()
        m_start.record()
        for _ in range(args.steps):
            g_mlp.replay()
        m_end.record()
        torch.cuda.synchronize()
    layer.check_device_errors("bench")
    ms_total = t_start.elapsed_time(t_end)
    mlp_ms = m_start.elapsed_time(m_end) / args.steps
    waves = len(layer.resident_wave_plan())
    del g_layer, g_mlp

    if dist is not None:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = world * cfg.tokens * args.steps / (ms_total / 1e3)

    pairs = cfg.tokens * cfg.top_k
    flops_call = pairs * cfg.flops_per_pair
    achieved_tflops = flops_call / (mlp_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved_tflops, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved_tflops / peaks["bf16_tflops"],
                "frac_of_sustained": achieved_tflops / peaks["bf16_tflops_sustained"],
                "peak_source": peaks["source"], "traffic": None,
                "kernel": "lm_moe_mlp_prefill (tcgen05 grouped MLP: gate_up + SiLU*mul and "
                          "down; 2-SM tiles for groups of more than 128 rows beside single-SM "
                          "tiles for the rest)",
                "timing": f"CUDA-graph replays of the grouped MLP call x{args.steps}, CUDA "
                          "events on the replay stream",
                "ms_per_call": mlp_ms, "flops_per_call": flops_call}
    if cfg.tokens == syn.CONFIGS[CONFIG_NAME].tokens:
        roofline["traffic"] = _profiled_traffic("umma_grouped_kernel_c2_t4096.md")
        roofline["traffic_source"] = "ncu dram__bytes_read.sum + dram__bytes_write.sum, " \
                                     "all launches of one call"
        dram_bytes = roofline["traffic"]
        if dram_bytes:
            roofline["hbm_frac_of_traffic"] = dram_bytes / (mlp_ms / 1e3) / 1e9 / peaks["hbm_gbs"]
    del layer
    torch.cuda.empty_cache()
    return value, ms_step, roofline, int(launches_per_step * args.steps), waves, clocks


# --------------------------------------------------------------------------- wave executor
def run_waves_hbm(args, cfg, w13, w2, dev) -> dict:
    """The capacity-bounded wave executor on the device: the C2 layer with its store in HBM but
    staged wave by wave (canonical waves of at most 32 experts, double-buffered stage banks
    filled device-to-device on the copy stream, one tcgen05 pass per wave, stage-buffer
    release events, one combine). The waves are planned and staged on the device (no host
    read); the same layer with the host-planned executor (one 4*E-byte count read-back per
    call, copies issued per wave) is timed after it. CUDA events around the steps."""
    import torch

    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
    from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime
    from vllm_ascend_hust_latchmoe_b200.synthetic import ExpertLayer

    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=cfg.num_slots,
                                            async_load=True, b2_wave_prefill=True,
                                            graph_compatible_offload=True,
                                            stage_waves_from_hbm_store=True))
    rt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2), slot_device=dev, store_device=dev)
    layer = SlotBankMoE(rt, 0, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                        num_experts=cfg.num_experts, top_k=cfg.top_k, max_tokens=cfg.tokens,
                        renormalize=cfg.renormalize, device=dev)
    hidden = syn.make_hidden(cfg, seed=0).to(dev)
    logits = syn.make_router_logits(cfg, seed=0).to(dev)
    for _ in range(args.warmup):
        layer.forward(hidden, logits)
    torch.cuda.synchronize()
    layer.check_device_errors("bench waves")
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        layer.forward(hidden, logits)
    b.record()
    torch.cuda.synchronize()
    layer.check_device_errors("bench waves")
    ms = a.elapsed_time(b) / args.steps
    waves = layer.device_wave_plan()  # the device plan of the last call (reads it back)
    staged = sum(len(w) for w in waves) * cfg.expert_bytes
    # the same layer with the waves planned and staged by the host (count read-back, host
    # wave plan, copies issued per wave), for comparison
    del layer, rt
    torch.cuda.empty_cache()
    hrt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=cfg.num_slots,
                                             async_load=True, b2_wave_prefill=True,
                                             graph_compatible_offload=True,
                                             stage_waves_from_hbm_store=True,
                                             stage_waves_on_device=False))
    hrt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2), slot_device=dev,
                                       store_device=dev)
    hlayer = SlotBankMoE(hrt, 0, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                         num_experts=cfg.num_experts, top_k=cfg.top_k, max_tokens=cfg.tokens,
                         renormalize=cfg.renormalize, device=dev)
    for _ in range(args.warmup):
        hlayer.forward(hidden, logits)
    torch.cuda.synchronize()
    a.record()
    for _ in range(args.steps):
        hlayer.forward(hidden, logits)
    b.record()
    torch.cuda.synchronize()
    hlayer.check_device_errors("bench waves (host plan)")
    host_ms = a.elapsed_time(b) / args.steps
    host_waves = hlayer.last_waves.waves
    res = {"workload": cfg.name + ", store in HBM, staged wave by wave",
           "ms_per_step": ms, "tokens_per_s": cfg.tokens / (ms / 1e3),
           "waves": len(waves), "wave_sizes": [len(w) for w in waves],
           "staged_bytes_per_step": int(staged),
           "d2d_gbs": staged / (ms / 1e3) / 1e9,
           "plan": "device wave plan; copy kernels into the stage banks; per-wave group ranges "
                   "read on the device; no host read between router and combine",
           "host_plan": {"ms_per_step": host_ms, "same_waves": [tuple(w) for w in host_waves]
                         == [tuple(w) for w in waves],
                         "plan": "count read-back, host wave plan, stage copies issued per "
                                 "wave by the host"},
           "timing": f"eager layer calls x{args.steps}, CUDA events"}
    del hlayer, hrt
    torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------------- N > 1 value
def run_value_ep(args, cfg, dist, dev, rank, world, local_rank, peaks, barrier):
    """``value`` at N > 1: the same C2 layer (Qwen3-30B-A3B shape, 4096 tokens per rank: weak
    scaling) with its 128 experts partitioned over the N GPUs. Experts are placed on ranks by
    a load-balanced placement of a profiled routing sample (the router's gate columns and the
    expert bank permuted together at load time); each rank holds its E / N experts in HBM.
    One step on every rank: route its tokens, store each token's row once into every owner that
    holds any of its experts over NVLink (peer memory), with each pair's owner-local id and
    receive-row index; the owner's grouped MLP gathers its rows from the receive area (the row
    count stays on the device) and its down GEMM stores every output row into the source's
    memory; signal, and combine every token's pairs from local memory in top-k order. The
    rank's step is captured once as a CUDA graph (the exchange's epoch is advanced on the
    device) and replayed. Time = max over ranks; after timing, each rank's first tokens are
    checked against the torch fp32 restatement of the 1-GPU layer. Also returns the same step
    from host buffers (``e2e``)."""
    import torch

    from vllm_ascend_hust_latchmoe_b200.layer import group_launches
    from vllm_ascend_hust_latchmoe_b200 import _lib
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import (ExpertParallelMoE, PeerExchange,
                                                                balanced_expert_placement,
                                                                build_rank_layer, cuda_ops)

    T, E, k, H, I = cfg.tokens, cfg.num_experts, cfg.top_k, cfg.hidden, cfg.intermediate
    per = E // world
    prof = torch.topk(syn.make_router_logits(cfg, seed=0, tokens=1024), k, dim=1).indices
    perm = torch.tensor(balanced_expert_placement(
        torch.bincount(prof.reshape(-1), minlength=E).tolist(), world))
    w13, w2 = syn.make_expert_weights(cfg, 0)
    owned = perm[rank * per:(rank + 1) * per]
    local = build_rank_layer(w13_owned=w13[owned].to(dev), w2_owned=w2[owned].to(dev),
                             rank=rank, device=dev, max_rows=world * T * k, num_slots=per,
                             store_on_device=True)
    exchange = PeerExchange(world_size=world, rank=rank, max_tokens=T, top_k=k, hidden_size=H,
                            device=dev, device_epoch=True)
    ep = ExpertParallelMoE(num_experts=E, top_k=k, hidden_size=H, rank=rank, world_size=world,
                           device=dev, exchange=exchange,
                           ops=cuda_ops(local, num_experts=E, top_k=k, max_tokens=T))
    hidden_cpu = syn.make_hidden(cfg, seed=rank)
    logits_cpu = syn.make_router_logits(cfg, seed=rank, bias_seed=0)
    placed_cpu = logits_cpu[:, perm].contiguous()
    hidden, logits = hidden_cpu.to(dev), placed_cpu.to(dev)
    for _ in range(args.warmup):
        ep.forward(hidden, logits)
    torch.cuda.synchronize()
    local.check_device_errors("bench ep value warmup")
    ep.check_exchange_errors()
    # the step captured once as a CUDA graph on every rank (the exchange's epoch lives on the
    # device, so each replay is a new call) and replayed; the capture executes nothing
    launches0 = local.kernel_launches
    g_step = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        ep.forward(hidden, logits)
    owner_launches = local.kernel_launches - launches0
    for _ in range(2):
        g_step.replay()
    torch.cuda.synchronize()
    local.check_device_errors("bench ep value graph warmup")
    ep.check_exchange_errors()
    sent0 = ep.stats.bytes_sent
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        t0.record()
        for _ in range(args.steps):
            g_step.replay()
        t1.record()
        barrier()
    local.check_device_errors("bench ep value")
    ep.check_exchange_errors()
    ms = torch.tensor([t0.elapsed_time(t1)], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms_total = float(ms.item())
    ms_step = ms_total / args.steps
    value = world * T * args.steps / (ms_total / 1e3)
    nvlink = (ep.stats.bytes_sent - sent0) / args.steps
    # per step: route, owner grouping, epoch, dispatch (token slots + stores when
    # deduplicated), receive (wait + index), the owner MLP's grouping / row pointers / gather /
    # grouped MLP, signal, combine (wait + reduce), step figures
    dispatch_launches = 2 if ep.dedupe_dispatch else 1
    launches_per_step = (1 + group_launches(T * k) + 1 + dispatch_launches + 2 + owner_launches
                         + 1 + 2 + 1)

    # correctness of what was timed: one more call, first tokens against the reference
    got = ep.forward(hidden, logits)
    torch.cuda.synchronize()
    local.check_device_errors("bench ep value check")
    ep.check_exchange_errors()
    n_chk = EP_CHECK_TOKENS
    w_ref, ids_ref = torch_route_reference(logits_cpu[:n_chk].to(dev), k)
    ref = torch_layer_reference(hidden[:n_chk], ids_ref, w_ref, lambda e: w13[e].to(dev),
                                lambda e: w2[e].to(dev))
    m = compare_outputs(got[:n_chk], ref)
    worst = torch.tensor([m["max_rel_err"], -m["cosine"]], dtype=torch.float64, device=dev)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    parity = {"max_rel_err": float(worst[0]), "cosine": -float(worst[1]),
              "tokens_checked_per_rank": n_chk, "ranks": world,
              "bar": {"max_rel_err": EP_MAX_REL_ERR, "cosine": EP_MIN_COSINE},
              "reference": "torch fp32 restatement of the 1-GPU layer (original expert order)"}
    parity["ok"] = parity["max_rel_err"] <= EP_MAX_REL_ERR and parity["cosine"] >= EP_MIN_COSINE

    # the owner's grouped MLP alone on the rows it received in the last step (roofline)
    x = exchange
    rows_recv = int(x.total.item())
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # the gather path the step runs (every rank's combine of the last step has completed: the
    # all-reduce above follows it in each rank's stream; the rewrite stores the same values)
    def row_ptrs(row_to_pair, count, ptrs):
        _lib.ep_output_row_ptrs(x.region, world, x.cap, H, rank, x.peers, row_to_pair, count,
                                ptrs.shape[0], ptrs, x.err)

    def owner_mlp():
        if ep.push_outputs:  # outputs stored into the sources' areas (same values again)
            local.mlp_rows_gather_push(x.recv_rows, x.slots, x.ids, x.total, row_ptrs)
        else:
            local.mlp_rows_gather_count(x.recv_rows, x.slots, x.ids, x.total, x.pair_rows,
                                        x.out_rows)

    for _ in range(3):
        owner_mlp()
    a.record()
    for _ in range(args.steps):
        owner_mlp()
    b.record()
    torch.cuda.synchronize()
    mlp_ms = a.elapsed_time(b) / args.steps
    local.check_device_errors("bench ep owner mlp")
    flops = rows_recv * cfg.flops_per_pair
    achieved = flops / (mlp_ms / 1e3) / 1e12
    loads = torch.tensor([rows_recv], dtype=torch.float64, device=dev)
    gathered = [torch.zeros_like(loads) for _ in range(world)]
    dist.all_gather(gathered, loads)
    rows_all = [float(g.item()) for g in gathered]
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
                "peak_source": peaks["source"], "traffic": None,
                "kernel": "rank 0's grouped MLP (owner side: grouping, gather from the receive "
                          "area, tcgen05 MLP whose down-GEMM epilogue stores each output row "
                          "into its source's memory over NVLink) on the rows it received"
                          if ep.push_outputs else
                          "rank 0's grouped MLP (owner side: grouping, gather from the receive "
                          "area, lm_moe_mlp_prefill) on the rows it received",
                "ms_per_call": mlp_ms, "flops_per_call": flops, "rows_rank0": rows_recv}

    # e2e: the same step from pinned host buffers (inputs in, output out, every step). The
    # copies run on two copy streams, double-buffered: step i+1's inputs go up and step i-1's
    # output comes down while step i computes (what a serving loop does); the timed region
    # opens before the first upload and closes after the last download.
    h_host = hidden_cpu.pin_memory()
    lg_host = placed_cpu.pin_memory()
    out_host = [torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    h_dev = [torch.empty_like(hidden) for _ in range(2)]
    lg_dev = [torch.empty_like(logits) for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    c_in, c_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    buf_free = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        j = i % 2
        if i >= 2:
            c_in.wait_event(buf_free[j])  # step i-2 has finished reading buffer j
        with torch.cuda.stream(c_in):
            h_dev[j].copy_(h_host, non_blocking=True)
            lg_dev[j].copy_(lg_host, non_blocking=True)
        in_ready[j].record(c_in)

    def e2e_run(n):
        c_in.wait_event(a)
        upload(0)
        for i in range(n):
            j = i % 2
            if i + 1 < n:
                upload(i + 1)
            comp.wait_event(in_ready[j])
            o = ep.forward(h_dev[j], lg_dev[j])
            buf_free[j].record(comp)
            c_out.wait_stream(comp)
            with torch.cuda.stream(c_out):
                out_host[j].copy_(o, non_blocking=True)
            o.record_stream(c_out)
        comp.wait_stream(c_out)
        comp.wait_stream(c_in)

    e2e_steps = max(3, min(args.steps, 10))
    a.record()
    e2e_run(3)  # warm-up of the pipelined loop
    torch.cuda.synchronize()
    barrier()
    a.record()
    e2e_run(e2e_steps)
    b.record()
    barrier()
    ep.check_exchange_errors()
    e_ms = torch.tensor([a.elapsed_time(b)], device=dev)
    dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e_ms.item()) / e2e_steps
    e2e = {"value": world * T / (e2e_ms / 1e3), "unit": UNIT,
           "h2d_bytes_per_step": int(h_host.numel() * 2 + lg_host.numel() * 4),
           "d2h_bytes_per_step": int(out_host[0].numel() * 2), "ms_per_step": e2e_ms,
           "path": "ExpertParallelMoE.forward per rank from pinned host buffers; uploads and "
                   "downloads on two copy streams, overlapped with the neighbouring steps"}
    ep_info = {"placement": "load-balanced (profiled routing sample; gate columns and expert "
                            "bank permuted at load time)",
               "experts_per_rank": per, "rows_received_per_rank": rows_all,
               "rank_load_max_over_mean": max(rows_all) / (sum(rows_all) / world),
               "nvlink_bytes_sent_rank0_per_step": nvlink, "transport": "peer memory (IPC)",
               "dispatch": "token-deduplicated (one row per token and owner)"
                           if ep.dedupe_dispatch else "one row per routed pair",
               "parity": parity}
    del g_step  # its kernels name the exchange region
    exchange.close()
    del ep, local
    torch.cuda.empty_cache()
    return value, ms_step, roofline, int(launches_per_step * args.steps), clocks, e2e, ep_info


def run_c5_single(args, dev) -> dict:
    """Single-GPU baseline of the Qwen3-235B-A22B-shaped layer of the expert-partitioned
    configuration: all 128 experts (4.8 GB) HBM-resident on one GPU, 256 tokens per step,
    the layer (route, wave plan, grouping, permute, tcgen05 MLP, combine) captured as a CUDA
    graph and replayed; its first tokens checked against the torch fp32 restatement."""
    import torch

    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
    from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime
    from vllm_ascend_hust_latchmoe_b200.weight_layout import to_tiled

    cfg = syn.CONFIGS["c5_ep"]
    E, H, I, T = cfg.num_experts, cfg.hidden, cfg.intermediate, cfg.tokens
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=dev)
    for e in range(E):
        w13[e], w2[e] = ep_expert_weights(e, cfg, dev)
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=cfg.num_slots,
                                            async_load=True, b2_wave_prefill=True))
    rt.register_layer_with_store(0, to_tiled(w13), to_tiled(w2), slot_device=dev, num_slots=1)
    layer = SlotBankMoE(rt, 0, hidden_size=H, intermediate_size=I, num_experts=E,
                        top_k=cfg.top_k, max_tokens=T, device=dev)
    hidden = syn.make_hidden(cfg, seed=0).to(dev)
    logits = syn.make_router_logits(cfg, seed=0).to(dev)
    for _ in range(3):
        layer.forward(hidden, logits)
    torch.cuda.synchronize()
    layer.check_device_errors("bench c5 single")
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.route(hidden, logits)
        layer.mlp_resident(hidden, T)
    for _ in range(3):
        g.replay()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(50):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / 50
    out = layer.out[:T]
    n_chk = EP_CHECK_TOKENS
    w_ref, ids_ref = torch_route_reference(logits[:n_chk], cfg.top_k)
    ref = torch_layer_reference(hidden[:n_chk], ids_ref, w_ref, lambda e: w13[e],
                                lambda e: w2[e])
    m = compare_outputs(out[:n_chk], ref)
    active = int((torch.bincount(layer.topk_ids[:T].reshape(-1).long(), minlength=E) > 0).sum())
    del g
    res = {"workload": cfg.name + " on one GPU (all 128 experts in HBM)", "ms_per_step": ms,
           "tokens_per_s": T / (ms / 1e3), "active_experts": active,
           "hbm_gbs": active * cfg.expert_bytes / (ms / 1e3) / 1e9,
           "timing": "CUDA-graph replay x50 of the whole layer",
           "parity": dict(m, tokens_checked=n_chk,
                          ok=m["max_rel_err"] <= EP_MAX_REL_ERR and m["cosine"] >= EP_MIN_COSINE)}
    del layer, rt, w13, w2
    torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------------- GPU arm
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--cpu-sample-tokens", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tpot", action="store_true", help="skip the 48-layer decode TPOT section")
    ap.add_argument("--tokens", type=int, default=0,
                    help="profiling override of the layer's token count (default: the config's)")
    ap.add_argument("--sections", default="all",
                    help="comma list of value,decode,c4,tpot,e2e,ep,cpu,waves (profiling runs "
                         "use one)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        # before numpy / torch load their thread pools (torchrun sets 1 thread per process)
        for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
            os.environ[var] = str(os.cpu_count() or 1)
    every = {"value", "decode", "c4", "tpot", "e2e", "ep", "cpu", "waves"}
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    # at N > 1 the single-GPU sections (decode, C4, TPOT) would only repeat BENCH's figures
    default = every if world_env == 1 else {"value", "e2e", "ep"}
    sec = default if args.sections == "all" else set(args.sections.split(","))
    if not sec <= every:
        ap.error(f"unknown sections {sorted(sec - every)}")
    if args.no_tpot:
        sec.discard("tpot")
    if args.no_cpu_baseline:
        sec.discard("cpu")

    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

    cfg = syn.CONFIGS[CONFIG_NAME]
    if args.tokens:
        cfg = cfg.with_tokens(args.tokens)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args, cfg)), flush=True)
        return

    import torch

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from vllm_ascend_hust_latchmoe_b200 import _lib
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
    from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime
    from vllm_ascend_hust_latchmoe_b200.synthetic import ExpertLayer

    _lib.load()
    peaks = _peaks()
    w13, w2 = syn.make_expert_weights(cfg, 0)
    hidden_cpu = syn.make_hidden(cfg, seed=rank)
    logits_cpu = syn.make_router_logits(cfg, seed=rank)

    def make_layer(store_on_device: bool) -> SlotBankMoE:
        rt = MoeOffloadRuntime(MoeOffloadConfig(
            enabled=True, num_slots=cfg.num_slots, async_load=True, b2_wave_prefill=True,
            graph_compatible_offload=True, pin_host_memory=True))
        rt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2), slot_device=dev,
                                          store_device=dev if store_on_device else None)
        return SlotBankMoE(rt, 0, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                           num_experts=cfg.num_experts, top_k=cfg.top_k, max_tokens=cfg.tokens,
                           renormalize=cfg.renormalize, device=dev)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ----------------------------------------------------------------- value (HBM inputs)
    hidden = hidden_cpu.to(dev)
    logits = logits_cpu.to(dev)
    value = ms_step = roofline = None
    launches = waves = 0
    clocks = ClockSampler(local_rank)
    ep_value = e2e_ep = None
    if "value" in sec and world == 1:
        value, ms_step, roofline, launches, waves, clocks = run_value(
            args, cfg, make_layer, hidden, logits, dist, dev, world, local_rank, peaks, barrier)
    elif "value" in sec:
        value, ms_step, roofline, launches, clocks, e2e_ep, ep_value = run_value_ep(
            args, cfg, dist, dev, rank, world, local_rank, peaks, barrier)
    waves_hbm = None
    if "waves" in sec:
        waves_hbm = run_waves_hbm(args, cfg, w13, w2, dev)
    # ----------------------------------------------------------------- decode layer (C1)
    decode = None
    if "decode" in sec:
        dcfg = syn.CONFIGS["c1_decode"]
        drt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=dcfg.num_slots,
                                                 async_load=True, b2_wave_prefill=True))
        drt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2), slot_device=dev, store_device=dev)
        dl = SlotBankMoE(drt, 0, hidden_size=dcfg.hidden, intermediate_size=dcfg.intermediate,
                         num_experts=dcfg.num_experts, top_k=dcfg.top_k, max_tokens=dcfg.tokens,
                         device=dev)
        dh = syn.make_hidden(dcfg, seed=rank).to(dev)
        dlg = syn.make_router_logits(dcfg, seed=rank).to(dev)
        T1 = dcfg.tokens
        for _ in range(args.warmup):
            dl.forward(dh, dlg)
        torch.cuda.synchronize()
        # eager calls (host-issued launches; includes any host launch gaps)
        d_steps = 50
        s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(d_steps):
            dl.forward(dh, dlg)
        e0.record()
        torch.cuda.synchronize()
        eager_ms = s0.elapsed_time(e0) / d_steps
        # device time: the layer (route -> grouping -> MLP -> combine) and the MLP alone, each
        # captured once as a CUDA graph and replayed back to back
        store = drt.host_layer(0)
        g_layer, g_mlp = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_layer):
            dl.route(dh, dlg)
            dl.mlp_resident(dh, T1)
        with torch.cuda.graph(g_mlp):
            dl._grouped_mlp(dh, T1, dl.identity_groups, 0, dl.E, store.w13, store.w2)

        def replay_ms(graph) -> float:
            for _ in range(3):
                graph.replay()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(d_steps):
                graph.replay()
            b.record()
            torch.cuda.synchronize()
            return a.elapsed_time(b) / d_steps

        layer_graph_ms = replay_ms(g_layer)
        d_mlp_ms = replay_ms(g_mlp)
        del g_layer, g_mlp
        dl.check_device_errors("bench decode")
        # The same layer on the slot bank: pinned host store, 64 slots (the 16 tokens route to
        # 33 experts, one more than 32 slots hold), every active expert staged once, then the
        # router + captured slot-bank MLP piece (log2phy remap, grouping, MLP, combine)
        # replayed: all hits.
        srt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=64, async_load=True,
                                                 b2_wave_prefill=True,
                                                 graph_compatible_offload=True,
                                                 pin_host_memory=True))
        srt.register_layer_for_fixed_slots(ExpertLayer(0, w13, w2), slot_device=dev)
        sl = SlotBankMoE(srt, 0, hidden_size=dcfg.hidden, intermediate_size=dcfg.intermediate,
                         num_experts=dcfg.num_experts, top_k=dcfg.top_k, max_tokens=dcfg.tokens,
                         device=dev)
        for _ in range(2):
            sl.forward(dh, dlg)
        torch.cuda.synchronize()
        assert sl.stage(sl.topk_ids[:T1]).mode == "slots"
        g_slots = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_slots):
            sl.route(dh, dlg)
            sl.mlp_slots(dh, T1)
        slot_layer_ms = replay_ms(g_slots)
        del g_slots
        sl.check_device_errors("bench decode slots")
        del sl, srt
        from vllm_ascend_hust_latchmoe_b200.moe_offload.phase_split import plan_balanced_b2_waves

        d_counts = torch.bincount(dl.topk_ids[: dcfg.tokens].reshape(-1).long().cpu(),
                                  minlength=dcfg.num_experts).tolist()
        d_active = sum(1 for c in d_counts if c > 0)
        d_plan = plan_balanced_b2_waves({e: c for e, c in enumerate(d_counts) if c}, dcfg.num_slots).waves
        d_bytes = d_active * dcfg.expert_bytes
        decode = {"workload": dcfg.name, "layer_ms": layer_graph_ms, "timing":
                  "CUDA-graph replay x50 (layer: route, grouping, MLP, combine; MLP: the "
                  "lm_moe_mlp_decode launch alone)", "layer_eager_ms": eager_ms,
                  "layer_hbm_frac": d_bytes / (layer_graph_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                  "mlp_ms": d_mlp_ms, "active_experts": d_active,
                  "waves_if_staged": len(d_plan),
                  "tier": "HBM-resident experts read in place (grouped by expert id)",
                  "mlp_hbm_gbs": d_bytes / (d_mlp_ms / 1e3) / 1e9,
                  "mlp_frac_hbm": d_bytes / (d_mlp_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                  "algorithmic_bytes_per_call": d_bytes,
                  "slot_bank": {"layer_ms": slot_layer_ms,
                                "layer_hbm_frac":
                                    d_bytes / (slot_layer_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                                "num_slots": 64,
                                "timing": "router + captured slot-bank MLP piece (log2phy "
                                          "remap, grouping, MLP, combine), graph replay x50; "
                                          "every active expert a slot hit"},
                  "kernel": "gemv_persistent_kernel (lm_moe_mlp_decode: gate_up and down in one "
                            "persistent launch)"}
        del dl, drt
        torch.cuda.empty_cache()

    # ----------------------------------------------------------------- shared-expert layer (C4)
    c4 = None
    if "c4" in sec:
        ccfg = syn.CONFIGS["c4_shared"]
        cw13, cw2 = syn.make_expert_weights(ccfg, 0)
        sw13, sw2 = syn.make_shared_weights(ccfg, 0)
        crt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=ccfg.num_slots,
                                                 async_load=True, b2_wave_prefill=True))
        crt.register_layer_for_fixed_slots(ExpertLayer(0, cw13, cw2), slot_device=dev,
                                           store_device=dev)
        cl = SlotBankMoE(crt, 0, hidden_size=ccfg.hidden, intermediate_size=ccfg.intermediate,
                         num_experts=ccfg.num_experts, top_k=ccfg.top_k, max_tokens=ccfg.tokens,
                         renormalize=ccfg.renormalize,
                         routed_scaling_factor=ccfg.routed_scaling_factor,
                         scoring_func=ccfg.scoring_func, num_expert_group=ccfg.num_expert_group,
                         topk_group=ccfg.topk_group, device=dev)
        cl.set_shared_experts(sw13, sw2)
        ch = syn.make_hidden(ccfg, seed=rank).to(dev)
        clg = syn.make_router_logits(ccfg, seed=rank).to(dev)
        Tc = ccfg.tokens
        shared_out = torch.empty(Tc, ccfg.hidden, dtype=torch.bfloat16, device=dev)
        for _ in range(args.warmup):
            cl.forward(ch, clg)
            cl.shared_mlp(ch, Tc, shared_out)
        torch.cuda.synchronize()
        g_c4 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_c4):
            cl.route(ch, clg)
            cl.mlp_resident(ch, Tc)
            cl.shared_mlp(ch, Tc, shared_out)
        for _ in range(3):
            g_c4.replay()
        a4, b4 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a4.record()
        for _ in range(50):
            g_c4.replay()
        b4.record()
        torch.cuda.synchronize()
        c4_ms = a4.elapsed_time(b4) / 50
        del g_c4
        cl.check_device_errors("bench c4")
        c_active = int((torch.bincount(cl.topk_ids[:Tc].reshape(-1).long(),
                                       minlength=ccfg.num_experts) > 0).sum())
        c_bytes = c_active * ccfg.expert_bytes + ccfg.num_shared * ccfg.expert_bytes
        ext_out = (cl.out[:Tc].float() + shared_out.float()).to(torch.bfloat16)
        # The same layer through the fused mix-placement lane: the 2 shared experts become
        # logical experts 64, 65 (each one I=1408 slice of the fused shared MLP), held in the
        # HBM store beside the routed ones, appended to every token's top-k by the router and
        # run in the same grouped-MLP launch; one combine.
        Is = ccfg.intermediate
        sh13 = torch.stack([torch.cat([sw13[s * Is:(s + 1) * Is], sw13[2 * Is + s * Is:
                                                                       2 * Is + (s + 1) * Is]])
                            for s in range(ccfg.num_shared)])
        sh2 = torch.stack([sw2[:, s * Is:(s + 1) * Is] for s in range(ccfg.num_shared)])
        frt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=ccfg.num_slots,
                                                 async_load=True, b2_wave_prefill=True))
        frt.register_layer_for_fixed_slots(
            ExpertLayer(0, torch.cat([cw13, sh13]), torch.cat([cw2, sh2]), shared=ccfg.num_shared),
            slot_device=dev, store_device=dev)
        fl = SlotBankMoE(frt, 0, hidden_size=ccfg.hidden, intermediate_size=Is,
                         num_experts=ccfg.num_experts, top_k=ccfg.top_k, max_tokens=Tc,
                         renormalize=ccfg.renormalize,
                         routed_scaling_factor=ccfg.routed_scaling_factor,
                         scoring_func=ccfg.scoring_func, num_expert_group=ccfg.num_expert_group,
                         topk_group=ccfg.topk_group, device=dev)
        for _ in range(args.warmup):
            fl.forward(ch, clg)
        torch.cuda.synchronize()
        g_f = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_f):
            fl.route(ch, clg)
            fl.mlp_resident(ch, Tc)
        for _ in range(3):
            g_f.replay()
        a4.record()
        for _ in range(50):
            g_f.replay()
        b4.record()
        torch.cuda.synchronize()
        fused_ms = a4.elapsed_time(b4) / 50
        fl.check_device_errors("bench c4 fused lane")
        fused_vs_external = compare_outputs(fl.out[:Tc], ext_out)
        del g_f, fl, frt
        c4 = {"workload": ccfg.name + " + 2 resident shared experts", "layer_ms": c4_ms,
              "fused_lane": {"layer_ms": fused_ms,
                             "frac_hbm": c_bytes / (fused_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                             "lane": "mix placement: shared experts as groups 64, 65 of the "
                                     "same grouped-MLP launch (HBM store), one combine",
                             "vs_external_lane": fused_vs_external},
              "timing": "CUDA-graph replay x50: route, grouping, routed MLP (experts read in "
                        "place), combine, shared-expert MLP",
              "active_experts": c_active, "algorithmic_bytes_per_call": c_bytes,
              "hbm_gbs": c_bytes / (c4_ms / 1e3) / 1e9,
              "frac_hbm": c_bytes / (c4_ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
        del cl, crt, cw13, cw2
        torch.cuda.empty_cache()

    # ----------------------------------------------------------------- decode TPOT (C3)
    tpot = None
    if "tpot" in sec:
        from vllm_ascend_hust_latchmoe_b200.decode_harness import DecoderShape, SyntheticMoEDecoder

        shape = DecoderShape()
        offl = [i for i in range(shape.layers) if i % 2 == 1]
        dec = SyntheticMoEDecoder(shape, offloaded_layers=offl, device=dev, seed=rank)
        rep = dec.run(shape.max_new, warmup=8)
        for lay in dec.moe:
            lay.check_device_errors("bench tpot")
        del dec
        torch.cuda.empty_cache()
        dec = SyntheticMoEDecoder(shape, offloaded_layers=offl, device=dev, seed=rank,
                                  device_staging=True)
        rep_dev = dec.run(shape.max_new, warmup=8)
        for lay in dec.moe:
            lay.check_device_errors("bench tpot (device staging)")
        share_dev = dec.moe_share()
        del dec
        torch.cuda.empty_cache()
        dec = SyntheticMoEDecoder(shape, offloaded_layers=[], device=dev, seed=rank)
        rep_res = dec.run(shape.max_new, warmup=8)
        share_res = dec.moe_share()
        del dec
        torch.cuda.empty_cache()
        tpot = {"workload": "qwen3-30b-a3b-shaped 48-layer decoder, batch 1, 1024-token context, "
                            "256 new tokens, piecewise CUDA-graph replay, router locality 0.7",
                "offloaded_layers": len(offl), "num_slots": shape.num_slots,
                "tpot_ms_p50": rep.tpot_ms_p50, "tpot_ms_p95": rep.tpot_ms_p95,
                "h2d_bytes_per_token": rep.h2d_bytes_per_step,
                "h2d_gbs_per_token_time": rep.h2d_bytes_per_step / (rep.tpot_ms_p50 / 1e3) / 1e9,
                "slot_hit_rate": rep.slot_hit_rate, "graphs_per_token": rep.graphs,
                "stage_host_ms_per_token": rep.stage_ms_per_step,
                "device_staging": {
                    "tpot_ms_p50": rep_dev.tpot_ms_p50, "tpot_ms_p95": rep_dev.tpot_ms_p95,
                    "h2d_bytes_per_token": rep_dev.h2d_bytes_per_step,
                    "h2d_gbs_per_token_time":
                        rep_dev.h2d_bytes_per_step / (rep_dev.tpot_ms_p50 / 1e3) / 1e9,
                    "slot_hit_rate": rep_dev.slot_hit_rate, "graphs_per_token": rep_dev.graphs,
                    "staging": "slot decision on the GPU (lm_slot_plan); misses read over "
                               "PCIe by the MLP and written through into their slots",
                    "moe_share": share_dev},
                "all_resident_tpot_ms_p50": rep_res.tpot_ms_p50,
                "all_resident_tpot_ms_p95": rep_res.tpot_ms_p95,
                "all_resident_moe_share": share_res,
                "moe_share_method": "each layer's attention and MoE piece captured as its own "
                                    "graph, replayed in token order with an event after each; "
                                    "MoE piece times summed per token (median over 32 tokens)",
                "data": "random-init weights and KV; synthetic routing"}

    # ----------------------------------------------------------------- e2e (host buffers)
    e2e = e2e_ep
    if "e2e" in sec and world == 1:
        off = make_layer(False)
        h_host = hidden_cpu.pin_memory()
        lg_host = logits_cpu.pin_memory()
        out_host = torch.empty(cfg.tokens, cfg.hidden, dtype=torch.bfloat16, pin_memory=True)
        h_dev = torch.empty_like(hidden)
        lg_dev = torch.empty_like(logits)

        def e2e_step():
            h_dev.copy_(h_host, non_blocking=True)
            lg_dev.copy_(lg_host, non_blocking=True)
            out = off.forward(h_dev, lg_dev)
            out_host.copy_(out, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        staged0 = off.runtime.transfer_engine.stats.bytes_h2d
        e2e_steps = max(3, min(args.steps, 10))
        barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(e2e_steps):
            e2e_step()
        e.record()
        barrier()
        off.check_device_errors("bench e2e")
        e2e_ms = s.elapsed_time(e)
        staged = (off.runtime.transfer_engine.stats.bytes_h2d - staged0) / e2e_steps
        if dist is not None:
            t = torch.tensor([e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e_value = world * cfg.tokens * e2e_steps / (e2e_ms / 1e3)
        io_in = h_host.numel() * 2 + lg_host.numel() * 4
        e2e = {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(io_in + staged),
               "d2h_bytes_per_step": int(out_host.numel() * 2),
               "h2d_breakdown": {"activations_and_logits": int(io_in), "expert_staging": int(staged)},
               "h2d_gbs": (io_in + staged) / (e2e_ms / e2e_steps / 1e3) / 1e9,
               "pcie_gen5_x16_gbs": 64.0, "ms_per_step": e2e_ms / e2e_steps}

    # ----------------------------------------------------------------- expert parallel (C5)
    ep_report = None
    if dist is not None and "ep" in sec:
        ep_report = run_expert_parallel(dist, rank, world, dev, args)
    elif "ep" in sec:
        ep_report = {"single_gpu": run_c5_single(args, dev)}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    cpu = None
    if "cpu" in sec:
        threads = use_all_host_threads()
        sample = args.cpu_sample_tokens
        w13b, w2b, hid, lg = cpu_inputs(cfg, sample)
        cpu_reference_step(cfg, sample, w13b, w2b, hid, lg)
        tt = [cpu_reference_step(cfg, sample, w13b, w2b, hid, lg) for _ in range(2)]
        del w13b, w2b
        cpu_value = sample * len(tt) / sum(tt)
        cpu = {"value": cpu_value, "unit": UNIT, "cores": os.cpu_count(),
               "threads": threads, "kind": "port",
               "sample": f"{sample} of {cfg.tokens} tokens, numpy fp32 BLAS",
               "per_config": cpu_config_times({
                   "workload": cfg.name, "tokens": sample, "full_tokens": cfg.tokens,
                   "ms_per_pass": 1e3 * sum(tt) / len(tt), "tokens_per_s": cpu_value,
                   "weights": "the GPU arm's seeded bf16 weights as fp32"})}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) bf16 weights, Zipf-biased router)",
        "config": {"workload": cfg.name, "global_batch": world * cfg.tokens, "tokens": cfg.tokens,
                   "hidden": cfg.hidden, "experts": cfg.num_experts, "top_k": cfg.top_k,
                   "moe_intermediate": cfg.intermediate,
                   "tier": "HBM-resident experts read in place (no staging)",
                   "group_order": ("expert id: experts read in place need no wave plan; "
                                   "all groups in one grouped-MLP pass" if not waves else
                                   f"device wave plan ({waves} waves of at most "
                                   f"{cfg.num_slots}), all groups in one grouped-MLP pass")
                                  if world == 1 else None,
                   "launch": ("layer step captured once as a CUDA graph, replayed per step"
                              if world == 1 else "the rank's step (route, exchange, owner MLP, "
                              "combine) captured once as a CUDA graph per rank and replayed; "
                              "the exchange epoch is advanced on the device"),
                   "parallelism": ("single GPU" if world == 1 else
                                   f"expert-partitioned x{world}: 128 experts over {world} GPUs, "
                                   "4096 tokens per rank, dispatch/combine over NVLink peer "
                                   "memory"),
                   "expert_partition": ep_value,
                   "l2": "weights 1.2 GB per step > 126 MB L2 (no flush needed)"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "decode": decode, "c4": c4, "tpot": tpot,
        "expert_parallel": ep_report, "wave_executor": waves_hbm,
        "clocks": clocks.summary(), "gpu_launches": int(launches),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
