"""GPU parity at the sizes the benchmark runs, not slices of them.

* The full C2 layer (4096 tokens, Qwen3-30B-A3B shape, 32 slots, seed 0: exactly the
  inputs ``bench.py`` times) through the public layer API, on the HBM-resident tier (device
  wave plan, experts read in place) and on the offload tier (waves staged from the pinned
  host store): top-k ids bit-exact, the wave plan equal to the canonical plan, the output
  within the bf16 bar of the oracle.
* The Qwen3-235B-A22B layer shape of the expert-partitioned configuration (H 4096, I 1536,
  128 experts, top-8): the decode GEMV and the tcgen05 prefill MLP on a whole 256-token step
  (2048 pairs), and the owner-side top-1 MLP with a device-held row count on both paths.

Bar: integer tables bit-exact; bf16 values max|a-e|/max|e| <= 1e-2 and cosine >= 0.9999
(fp32-accumulating oracle, ``oracle/mlp.py``).
"""

import numpy as np
import pytest
import torch

from oracle import control as ocontrol
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits, build_layer
from vllm_ascend_hust_latchmoe_b200 import _lib
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
from vllm_ascend_hust_latchmoe_b200.weight_layout import to_tiled

pytestmark = pytest.mark.gpu


def _check(actual_bf16: torch.Tensor, ref: np.ndarray) -> dict:
    m = omlp.compare(bf16_bits_to_f32(bits(actual_bf16)), ref)
    assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
    return m


@pytest.fixture(scope="module")
def c2_case():
    cfg = syn.CONFIGS["c2_prefill"]
    w13, w2 = syn.make_expert_weights(cfg, 0)
    hidden = syn.make_hidden(cfg, seed=0)
    logits = syn.make_router_logits(cfg, seed=0)
    wb, _, ids = orouter.route(logits.numpy(), cfg.top_k, renormalize=cfg.renormalize)
    ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
    counts = np.bincount(ids.reshape(-1), minlength=cfg.num_experts)
    waves = ocontrol.plan_balanced_waves({e: int(c) for e, c in enumerate(counts) if c},
                                         cfg.num_slots)
    return cfg, (w13, w2), hidden, logits, ids, ref, waves


@pytest.mark.parametrize("store_on_device", [True, False], ids=["resident", "staged"])
def test_c2_full_layer_4096_tokens(cuda, c2_case, store_on_device):
    cfg, experts, hidden, logits, ids_ref, ref, waves = c2_case
    layer, rt, _ = build_layer(cfg, store_on_device=store_on_device, experts=experts)
    layer.resident_wave_order = True  # groups in the device wave plan's order (checked below)
    out = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    layer.check_device_errors("c2 full")
    assert np.array_equal(layer.topk_ids[: cfg.tokens].cpu().numpy(), ids_ref)
    got_waves = layer.resident_wave_plan() if store_on_device else layer.last_waves.waves
    assert [tuple(w) for w in got_waves] == [tuple(w) for w in waves] and len(waves) >= 4
    _check(out, ref)
    # the timed loop calls the layer again and again on the same buffers
    out2 = layer.forward(hidden.to(cuda), logits.to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    if store_on_device:  # groups by expert id (the default): the same output, bit for bit
        layer.resident_wave_order = False
        out3 = layer.forward(hidden.to(cuda), logits.to(cuda))
        torch.cuda.synchronize()
        layer.check_device_errors("c2 full, expert-id order")
        assert torch.equal(out, out3) and layer.resident_wave_plan() == ()


# ----------------------------------------------------------------------------- C5 shape
C5 = syn.CONFIGS["c5_ep"]


class _ExpertBits:
    """Per-expert bf16 bit patterns of a device weight bank, fetched on first use (the oracle
    touches only the routed experts; the whole bank is 4.8 GB)."""

    def __init__(self, w: torch.Tensor) -> None:
        self.w = w
        self.cache: dict[int, np.ndarray] = {}

    def __getitem__(self, e) -> np.ndarray:
        e = int(e)
        if e not in self.cache:
            self.cache[e] = bits(self.w[e])
        return self.cache[e]


@pytest.fixture(scope="module")
def c5_bank():
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(235)
    E, H, I = C5.num_experts, C5.hidden, C5.intermediate
    w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(E, H, I, dtype=torch.bfloat16, device=dev)
    for e in range(E):
        w13[e] = torch.randn(2 * I, H, generator=g, device=dev) * 0.02
        w2[e] = torch.randn(H, I, generator=g, device=dev) * 0.02
    W13, W2 = to_tiled(w13), to_tiled(w2)
    yield w13, w2, W13, W2
    del w13, w2, W13, W2
    torch.cuda.empty_cache()


def _c5_mlp(cuda, bank, T, use_prefill):
    w13, w2, W13, W2 = bank
    E, H, I, k = C5.num_experts, C5.hidden, C5.intermediate, C5.top_k
    cfg = C5.with_tokens(T)
    hidden = syn.make_hidden(cfg, seed=5)
    logits = syn.make_router_logits(cfg, seed=5)
    wb, _, ids = orouter.route(logits.numpy(), k, renormalize=True)
    active = np.unique(ids)
    e2g = np.full(E, -1, dtype=np.int32)
    e2g[active] = np.arange(active.size)
    Gn, P = active.size, T * k
    off = torch.empty(Gn + 1, dtype=torch.int32, device=cuda)
    p2r = torch.empty(P, dtype=torch.int32, device=cuda)
    r2p = torch.empty(P, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_lib.build_groups_scratch_elems(P, Gn), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.build_groups(torch.from_numpy(ids).to(cuda), E, torch.from_numpy(e2g).to(cuda), Gn,
                      off, p2r, r2p, scratch, err)
    bank_row = torch.from_numpy(active.astype(np.int32)).to(cuda)
    h = hidden.to(cuda)
    act = torch.zeros(P, I, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(P, H, dtype=torch.bfloat16, device=cuda)
    if use_prefill:
        x = torch.empty(P, H, dtype=torch.bfloat16, device=cuda)
        _lib.permute_rows(h, r2p, k, P, x)
        _lib.moe_mlp_prefill(x, P, off, bank_row, 0, Gn, W13, W2, act, y, err)
    else:
        _lib.moe_mlp_decode(h, k, r2p, off, bank_row, 0, Gn, T, W13, W2, act, y, err)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
    _lib.moe_combine(y, p2r, torch.from_numpy(bf16_bits_to_f32(wb)).to(torch.bfloat16).to(cuda),
                     out)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref_pairs = omlp.pair_outputs(bits(hidden), ids, _ExpertBits(w13), _ExpertBits(w2))
    _check(y[p2r.long()], ref_pairs)
    _check(out, omlp.combine(ref_pairs, wb))


@pytest.mark.parametrize("T", [1, 32])
def test_c5_shape_decode_mlp(cuda, c5_bank, T):
    _c5_mlp(cuda, c5_bank, T, use_prefill=False)


def test_c5_shape_prefill_mlp_whole_step(cuda, c5_bank):
    """One 256-token step of the C5 layer on one GPU: 2048 pairs over the active experts."""
    _c5_mlp(cuda, c5_bank, C5.tokens, use_prefill=True)


@pytest.mark.parametrize("R,live", [(48, 41), (2048, 1777)])
def test_c5_shape_owner_rows_count(cuda, c5_bank, R, live):
    """The expert-partitioned owner's top-1 MLP at the C5 shape (16 owned experts, as at 8
    GPUs), its received row count held on the device: decode path (R <= 64) and tcgen05 path."""
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import build_rank_layer

    w13, w2, _, _ = c5_bank
    E_r = C5.num_experts // 8
    layer = build_rank_layer(w13_owned=w13[:E_r], w2_owned=w2[:E_r], rank=0, device=cuda,
                             max_rows=R, num_slots=E_r, store_on_device=True)
    rng = np.random.default_rng(R + live)
    ids_np = rng.integers(0, E_r, size=R).astype(np.int32)
    ids_np[live:] = 1000  # past the count: never read
    cfg = C5.with_tokens(R)
    rows = syn.make_hidden(cfg, seed=6)
    out = torch.zeros(R, C5.hidden, dtype=torch.bfloat16, device=cuda)
    layer.mlp_rows_count(rows.to(cuda), torch.from_numpy(ids_np).to(cuda),
                         torch.tensor([live], dtype=torch.int32, device=cuda), out)
    torch.cuda.synchronize()
    layer.check_device_errors("c5 owner")
    unit = np.full((live, 1), 0x3F80, dtype=np.uint16)  # bf16 1.0
    ref = omlp.moe_layer(bits(rows)[:live], ids_np[:live, None], unit, _ExpertBits(w13),
                         _ExpertBits(w2))
    _check(out[:live], ref)


@pytest.mark.parametrize("on_device", [False, True], ids=["host_plan", "device_plan"])
def test_c2_waves_staged_from_hbm_store(cuda, c2_case, on_device):
    """The capacity-bounded wave executor with an HBM-resident store (stage banks filled
    device-to-device, one GEMM pass per wave on its stage bank, one combine): the canonical
    waves, each within the 32 slots, and the oracle's output -- planned and staged by the
    host, or planned on the device with copy kernels and per-wave group ranges read on the
    device (then also replayed from a CUDA graph)."""
    from vllm_ascend_hust_latchmoe_b200.config import MoeOffloadConfig
    from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE
    from vllm_ascend_hust_latchmoe_b200.moe_offload.runtime import MoeOffloadRuntime

    cfg, (w13, w2), hidden, logits, ids_ref, ref, waves = c2_case
    rt = MoeOffloadRuntime(MoeOffloadConfig(enabled=True, num_slots=cfg.num_slots,
                                            async_load=True, b2_wave_prefill=True,
                                            graph_compatible_offload=True,
                                            stage_waves_from_hbm_store=True,
                                            stage_waves_on_device=on_device))
    rt.register_layer_for_fixed_slots(syn.ExpertLayer(0, w13, w2), slot_device=cuda,
                                      store_device=cuda)
    layer = SlotBankMoE(rt, 0, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                        num_experts=cfg.num_experts, top_k=cfg.top_k, max_tokens=cfg.tokens,
                        device=cuda)
    h, lg = hidden.to(cuda), logits.to(cuda)
    for _ in range(2):
        out = layer.forward(h, lg)
        torch.cuda.synchronize()
        layer.check_device_errors("c2 staged waves")
        if on_device:
            assert [tuple(w) for w in layer.device_wave_plan()] == [tuple(w) for w in waves]
        else:
            assert not layer.last_waves.zero_copy
            assert [tuple(w) for w in layer.last_waves.waves] == [tuple(w) for w in waves]
            assert layer.last_waves.staged_bytes == sum(len(w) for w in waves) * cfg.expert_bytes
        _check(out, ref)
    if on_device:  # no host step: the whole layer replays from a CUDA graph, same output
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer.route(h, lg)
            gout = layer.run_mlp(h, layer.stage(layer.topk_ids[: cfg.tokens]))
        for _ in range(2):
            gout.zero_()
            g.replay()
            torch.cuda.synchronize()
            layer.check_device_errors("c2 device waves, graph")
            assert torch.equal(gout, out)
