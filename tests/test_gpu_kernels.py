"""GPU parity of the individual C-ABI kernels against the CPU oracle (seeded inputs).

Bar: integer outputs (top-k ids, group offsets, pair<->row tables) bit-exact; bf16 values
within max|a-e|/max|e| <= 1e-2 and cosine >= 0.9999 (fp32 accumulation on both sides).
"""

import numpy as np
import pytest
import torch

from oracle import control as ocontrol
from oracle import mlp as omlp
from oracle import router as orouter
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits
from vllm_ascend_hust_latchmoe_b200 import _lib
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
from vllm_ascend_hust_latchmoe_b200.weight_layout import to_tiled

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,tokens", [("c1_decode", 16), ("c2_prefill", 4096),
                                         ("c4_shared", 64), ("c5_ep", 256)])
def test_router_ids_bit_exact(cuda, name, tokens):
    cfg = syn.CONFIGS[name]
    logits = syn.make_router_logits(cfg, seed=0, tokens=tokens)
    wb_ref, wf_ref, ids_ref = orouter.route(
        logits.numpy(), cfg.top_k, renormalize=cfg.renormalize,
        routed_scaling_factor=cfg.routed_scaling_factor, scoring_func=cfg.scoring_func,
        num_expert_group=cfg.num_expert_group, topk_group=cfg.topk_group)
    # The seeded logits hold no score ties, so the logit order is the score order.
    assert np.array_equal(orouter.route_by_logit_order(logits.numpy(), cfg.top_k), ids_ref)
    T = logits.shape[0]
    wb = torch.empty(T, cfg.top_k, dtype=torch.bfloat16, device=cuda)
    wf = torch.empty(T, cfg.top_k, dtype=torch.float32, device=cuda)
    ids = torch.empty(T, cfg.top_k, dtype=torch.int32, device=cuda)
    _lib.route_topk(logits.to(cuda), cfg.top_k, scoring_func=cfg.scoring_func,
                    renormalize=cfg.renormalize,
                    routed_scaling_factor=cfg.routed_scaling_factor,
                    num_expert_group=cfg.num_expert_group, topk_group=cfg.topk_group,
                    weights_bf16=wb, ids=ids, weights_f32=wf)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), ids_ref)
    got = wf.cpu().numpy()
    assert np.abs(got - wf_ref).max() <= 1e-6 * max(1.0, np.abs(wf_ref).max())
    gb = bf16_bits_to_f32(bits(wb))
    eb = bf16_bits_to_f32(wb_ref)
    assert np.abs(gb - eb).max() <= 2.0 ** -8 * np.abs(eb).max()
    assert (bits(wb) == wb_ref).mean() > 0.99


def test_router_grouped_and_sigmoid_bias(cuda):
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((97, 64)).astype(np.float32)
    bias = (rng.standard_normal(64) * 0.1).astype(np.float32)
    for kw in (dict(scoring_func="sigmoid", num_expert_group=8, topk_group=3,
                    e_score_correction_bias=bias, renormalize=True, routed_scaling_factor=2.5),
               dict(scoring_func="softmax", num_expert_group=4, topk_group=2, renormalize=False)):
        _, wf_ref, ids_ref = orouter.route(logits, 6, **kw)
        wb = torch.empty(97, 6, dtype=torch.bfloat16, device=cuda)
        wf = torch.empty(97, 6, dtype=torch.float32, device=cuda)
        ids = torch.empty(97, 6, dtype=torch.int32, device=cuda)
        gkw = dict(kw)
        if gkw.get("e_score_correction_bias") is not None:
            gkw["e_score_correction_bias"] = torch.from_numpy(bias).to(cuda)
        _lib.route_topk(torch.from_numpy(logits).to(cuda), 6, weights_bf16=wb, ids=ids,
                        weights_f32=wf, **gkw)
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), ids_ref), kw
        assert np.abs(wf.cpu().numpy() - wf_ref).max() < 1e-5


def _groups_case(cuda, ids_np, e2g_np, G, E):
    ids = torch.from_numpy(ids_np.astype(np.int32)).to(cuda)
    e2g = torch.from_numpy(e2g_np.astype(np.int32)).to(cuda)
    P = ids_np.size
    off = torch.full((G + 1,), -7, dtype=torch.int32, device=cuda)
    p2r = torch.full((max(P, 1),), -7, dtype=torch.int32, device=cuda)
    r2p = torch.full((max(P, 1),), -7, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_lib.build_groups_scratch_elems(P, G), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.build_groups(ids, E, e2g, G, off, p2r, r2p, scratch, err)
    torch.cuda.synchronize()
    ref_off, ref_p2r, ref_r2p = ocontrol.group_pairs(ids_np, e2g_np, G)
    assert np.array_equal(off.cpu().numpy(), ref_off)
    if P:
        assert np.array_equal(p2r.cpu().numpy()[:P], ref_p2r)
        assert np.array_equal(r2p.cpu().numpy()[: ref_r2p.size], ref_r2p)
    return int(err.item())


@pytest.mark.parametrize("T,k,E,G", [(16, 8, 128, 32), (4096, 8, 128, 122), (1, 8, 128, 8),
                                     (1000, 6, 64, 64), (513, 8, 128, 128), (4096, 8, 128, 1),
                                     (64, 8, 128, 1024), (64, 8, 128, 128), (65, 8, 128, 128)])
def test_build_groups_bit_exact(cuda, T, k, E, G):
    rng = np.random.default_rng(T * 31 + G)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    experts = np.unique(ids)
    e2g = np.full(E, -1, dtype=np.int64)
    # map the active experts onto G groups (several experts may share a group)
    e2g[experts] = rng.permutation(np.arange(experts.size)) % G
    assert _groups_case(cuda, ids, e2g, G, E) == 0


def test_build_groups_empty_and_unmapped(cuda):
    assert _groups_case(cuda, np.zeros((0, 8), dtype=np.int32), np.zeros(128), 4, 128) == 0
    ids = np.array([[0, 1], [2, 3]], dtype=np.int32)
    e2g = np.array([0, -1, 1, 1], dtype=np.int64)
    assert _groups_case(cuda, ids, e2g, 2, 4) == 2  # LM_DEVERR_UNMAPPED_EXPERT


@pytest.mark.parametrize("T,k,E,P", [(16, 8, 128, 0), (1, 8, 128, 0), (64, 8, 128, 0),
                                     (20, 6, 64, 2), (40, 4, 16, 0)])
def test_route_group_small_equals_route_then_group(cuda, T, k, E, P):
    """The one-launch router + grouping of a decode-sized call writes exactly what
    lm_route_topk(_shared) followed by lm_build_groups writes (identity expert -> group)."""
    g = torch.Generator().manual_seed(T * 131 + E)
    logits = (torch.randn(T, E, generator=g) * 2.0).to(cuda)
    Et = E + P
    ident = torch.arange(Et, dtype=torch.int32, device=cuda)
    n = T * (k + P)

    def bufs():
        return (torch.zeros(T, k + P, dtype=torch.bfloat16, device=cuda),
                torch.zeros(T, k + P, dtype=torch.int32, device=cuda),
                torch.full((Et + 1,), -7, dtype=torch.int32, device=cuda),
                torch.full((n,), -7, dtype=torch.int32, device=cuda),
                torch.full((n,), -7, dtype=torch.int32, device=cuda),
                torch.zeros(1, dtype=torch.int32, device=cuda))

    w1, i1, o1, p1, r1, e1 = bufs()
    _lib.route_topk(logits, k, weights_bf16=w1, ids=i1, num_shared=P)
    scratch = torch.empty(_lib.build_groups_scratch_elems(n, Et), dtype=torch.int32, device=cuda)
    _lib.build_groups(i1, Et, ident, Et, o1, p1, r1, scratch, e1)
    w2, i2, o2, p2, r2, e2 = bufs()
    _lib.route_group_small(logits, k, num_shared=P, weights_bf16=w2, ids=i2,
                           num_experts_total=Et, expert_to_group=ident, num_groups=Et,
                           group_offsets=o2, pair_to_row=p2, row_to_pair=r2, err_word=e2)
    torch.cuda.synchronize()
    assert int(e1.item()) == 0 and int(e2.item()) == 0
    for a, b in ((w1, w2), (i1, i2), (o1, o2), (p1, p2), (r1, r2)):
        assert torch.equal(a, b)


def test_histogram(cuda):
    rng = np.random.default_rng(5)
    ids = rng.integers(0, 128, size=(4096, 8)).astype(np.int32)
    counts = torch.empty(128, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.expert_histogram(torch.from_numpy(ids).to(cuda), 128, counts, err)
    assert np.array_equal(counts.cpu().numpy(), np.bincount(ids.reshape(-1), minlength=128))
    assert err.item() == 0
    bad = torch.tensor([[0, 200]], dtype=torch.int32, device=cuda)
    _lib.expert_histogram(bad, 128, counts, err)
    assert err.item() == 1


def _mlp_case(cuda, T, k, E, H, I, G, use_prefill, seed=0, skewed=False, ids=None):
    rng = np.random.default_rng(seed)
    cfg = syn.LayerConfig("t", hidden=H, num_experts=E, top_k=k, intermediate=I, num_slots=G,
                          tokens=T, zipf_s=2.0)
    w13, w2 = syn.make_expert_weights(cfg, seed=seed, experts=E)
    hidden = syn.make_hidden(cfg, seed=seed)
    if ids is not None:
        ids_np = ids
    elif skewed:  # Zipf-biased routing: a few groups span many m-tiles, most span one
        ids_np = orouter.route(syn.make_router_logits(cfg, seed=seed).numpy(), k)[2]
    else:
        ids_np = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    wts = torch.from_numpy(rng.random((T, k)).astype(np.float32)).to(torch.bfloat16)
    active = np.unique(ids_np)
    e2g = np.full(E, -1, dtype=np.int64)
    e2g[active] = np.arange(active.size)
    Gn = active.size
    bank_row = torch.from_numpy(active.astype(np.int32)).to(cuda)
    d_ids = torch.from_numpy(ids_np).to(cuda)
    P = T * k
    off = torch.empty(Gn + 1, dtype=torch.int32, device=cuda)
    p2r = torch.empty(P, dtype=torch.int32, device=cuda)
    r2p = torch.empty(P, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_lib.build_groups_scratch_elems(P, Gn), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.build_groups(d_ids, E, torch.from_numpy(e2g.astype(np.int32)).to(cuda), Gn, off, p2r,
                      r2p, scratch, err)
    h = hidden.to(cuda)
    W13, W2 = to_tiled(w13).to(cuda), to_tiled(w2).to(cuda)
    act = torch.zeros(P, I, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(P, H, dtype=torch.bfloat16, device=cuda)
    if use_prefill:
        x = torch.empty(P, H, dtype=torch.bfloat16, device=cuda)
        _lib.permute_rows(h, r2p, k, P, x)
        _lib.moe_mlp_prefill(x, P, off, bank_row, 0, Gn, W13, W2, act, y, err)
    else:
        _lib.moe_mlp_decode(h, k, r2p, off, bank_row, 0, Gn, T, W13, W2, act, y, err)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=cuda)
    _lib.moe_combine(y, p2r, wts.to(cuda), out)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref_pairs = omlp.pair_outputs(bits(hidden), ids_np, bits(w13), bits(w2))
    ref_out = omlp.combine(ref_pairs, bits(wts))
    # per-pair outputs (rows are permuted: undo with pair_to_row)
    got_pairs = bf16_bits_to_f32(bits(y))[p2r.cpu().numpy()]
    m_pairs = omlp.compare(got_pairs, ref_pairs)
    m_out = omlp.compare(bf16_bits_to_f32(bits(out)), ref_out)
    assert m_pairs["max_rel_err"] <= MAX_REL_ERR and m_pairs["cosine"] >= MIN_COSINE, m_pairs
    assert m_out["max_rel_err"] <= MAX_REL_ERR and m_out["cosine"] >= MIN_COSINE, m_out


@pytest.mark.parametrize("T,k,E,H,I", [(16, 8, 128, 2048, 768), (1, 8, 128, 2048, 768),
                                       (64, 6, 64, 2048, 1408), (40, 8, 16, 256, 128),
                                       (150, 2, 4, 512, 192)])
def test_decode_mlp_matches_oracle(cuda, T, k, E, H, I):
    _mlp_case(cuda, T, k, E, H, I, 32, use_prefill=False)


def test_decode_mlp_concurrent_streams(cuda):
    """The persistent decode kernel keeps its work queue and pass counters per stream: two
    layers' decode calls running at the same time on two streams give exactly what each gives
    alone, call after call (a shared counter set would mix their queues)."""
    E, H, I, k = 64, 512, 256, 8
    g = torch.Generator().manual_seed(11)
    W13 = to_tiled((torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)).to(cuda)
    W2 = to_tiled((torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)).to(cuda)
    ident = torch.arange(E, dtype=torch.int32, device=cuda)
    cases = []
    for T, seed in ((16, 1), (40, 2)):
        rng = np.random.default_rng(seed)
        ids = torch.from_numpy(np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)).to(cuda)
        h = (torch.randn(T, H, generator=g)).to(torch.bfloat16).to(cuda)
        P = T * k
        off = torch.empty(E + 1, dtype=torch.int32, device=cuda)
        p2r = torch.empty(P, dtype=torch.int32, device=cuda)
        r2p = torch.empty(P, dtype=torch.int32, device=cuda)
        scratch = torch.empty(_lib.build_groups_scratch_elems(P, E), dtype=torch.int32, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        _lib.build_groups(ids, E, ident, E, off, p2r, r2p, scratch, err)
        act = torch.zeros(P, I, dtype=torch.bfloat16, device=cuda)
        y = torch.zeros(P, H, dtype=torch.bfloat16, device=cuda)
        cases.append(dict(T=T, h=h, off=off, r2p=r2p, act=act, y=y, err=err))

    def run(c):
        _lib.moe_mlp_decode(c["h"], k, c["r2p"], c["off"], ident, 0, E, c["T"], W13, W2, c["act"],
                            c["y"], c["err"])

    for c in cases:  # alone, on the default stream
        run(c)
    torch.cuda.synchronize()
    refs = [c["y"].clone() for c in cases]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for _ in range(20):
        for c, st in zip(cases, streams):
            c["y"].zero_()
        torch.cuda.synchronize()
        for c, st in zip(cases, streams):
            with torch.cuda.stream(st):
                run(c)
        torch.cuda.synchronize()
        for c, ref in zip(cases, refs):
            assert int(c["err"].item()) == 0
            assert torch.equal(c["y"], ref)


def test_decode_counter_sets_move_between_streams(cuda):
    """More streams than counter sets, each used eagerly in turn: a set whose stream's last
    launch has finished moves to the next stream, so every launch stays on the persistent
    kernel (no fallback) and gives the same output."""
    E, H, I, k, T = 16, 256, 128, 8, 4
    g = torch.Generator().manual_seed(5)
    W13 = to_tiled((torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)).to(cuda)
    W2 = to_tiled((torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)).to(cuda)
    ident = torch.arange(E, dtype=torch.int32, device=cuda)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    h = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16).to(cuda)
    off = torch.empty(E + 1, dtype=torch.int32, device=cuda)
    p2r = torch.empty(T * k, dtype=torch.int32, device=cuda)
    r2p = torch.empty(T * k, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_lib.build_groups_scratch_elems(T * k, E), dtype=torch.int32,
                          device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.build_groups(ids.to(cuda), E, ident, E, off, p2r, r2p, scratch, err)
    act = torch.empty(T * k, I, dtype=torch.bfloat16, device=cuda)
    y = torch.empty(T * k, H, dtype=torch.bfloat16, device=cuda)
    _lib.moe_mlp_decode(h, k, r2p, off, ident, 0, E, T, W13, W2, act, y, err)
    torch.cuda.synchronize()
    ref = y.clone()
    before = _lib.decode_counter_sets()
    streams = [torch.cuda.Stream() for _ in range(20)]  # kept alive: distinct handles
    for st in streams:
        y.zero_()
        torch.cuda.synchronize()
        with torch.cuda.stream(st):
            _lib.moe_mlp_decode(h, k, r2p, off, ident, 0, E, T, W13, W2, act, y, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0 and torch.equal(y, ref)
    after = _lib.decode_counter_sets()
    assert after["fallbacks"] == before["fallbacks"], (before, after)
    assert after["recycled"] >= before["recycled"] + 4, (before, after)
    assert after["in_use"] <= 16


@pytest.mark.parametrize("T,k,E,H,I", [(256, 8, 32, 2048, 768), (300, 8, 128, 2048, 768),
                                       (129, 2, 4, 256, 128), (512, 6, 64, 2048, 1408)])
def test_prefill_tcgen05_mlp_matches_oracle(cuda, T, k, E, H, I):
    _mlp_case(cuda, T, k, E, H, I, 32, use_prefill=True)


@pytest.mark.parametrize("T,k,E", [(2048, 4, 32), (1500, 8, 128), (700, 2, 8)])
def test_prefill_tcgen05_skewed_groups(cuda, T, k, E):
    """Heavy (multi-m-tile) and light (single-m-tile) groups in one launch: exercises the
    merged heavy/light tile order of the persistent scheduler."""
    _mlp_case(cuda, T, k, E, 2048, 768, 32, use_prefill=True, skewed=True)


@pytest.mark.parametrize("H,I", [(512, 256), (2048, 768)])
def test_prefill_group_size_boundaries(cuda, H, I):
    """Group sizes on every boundary of the two tile kinds: groups of at most 128 rows run on
    single-SM tiles (row loads trimmed to 16 / 32 / 64 / 128), larger ones on 256-row 2-SM
    tiles; 1-row, exact-multiple and one-past groups."""
    sizes = [1, 15, 16, 17, 31, 32, 33, 63, 64, 65, 100, 127, 128, 129, 255, 256, 257, 300, 513]
    ids = np.concatenate([np.full(n, e, dtype=np.int32) for e, n in enumerate(sizes)])
    ids = np.random.default_rng(5).permutation(ids).reshape(-1, 1)
    _mlp_case(cuda, ids.shape[0], 1, len(sizes), H, I, 32, use_prefill=True, ids=ids)


def test_stage_copy_coalesces_runs(cuda):
    src = torch.arange(10 * 64, dtype=torch.float32).reshape(10, 64).pin_memory()
    dst = torch.zeros(6, 64, dtype=torch.float32, device=cuda)
    n = _lib.stage_copy(dst, src, [3, 4, 5, 9, 0], [0, 1, 2, 4, 5])
    torch.cuda.synchronize()
    assert n == 3  # one run of 3 + two singles
    assert torch.equal(dst[[0, 1, 2, 4, 5]].cpu(), src[[3, 4, 5, 9, 0]])


def test_stage_copy_device_to_device_kernel(cuda):
    """D2D staging runs as a copy kernel (one launch per 64 rows) and moves exactly the rows
    asked for, rows larger than one CTA's chunk included; a copy whose row size is not a
    multiple of 16 bytes goes through cudaMemcpyAsync."""
    g = torch.Generator().manual_seed(3)
    src = torch.randn(10, 100_003 * 4, generator=g).to(cuda)  # 1.6 MB rows, many chunks
    dst = torch.zeros(6, src.shape[1], device=cuda)
    n = _lib.stage_copy(dst, src, [3, 4, 5, 9, 0], [0, 1, 2, 4, 5])
    torch.cuda.synchronize()
    assert n == 1
    assert torch.equal(dst[[0, 1, 2, 4, 5]], src[[3, 4, 5, 9, 0]])
    assert bool((dst[3] == 0).all())
    many_src = torch.randn(200, 64, generator=g).to(cuda)
    many_dst = torch.zeros(200, 64, device=cuda)
    rows = list(range(199, -1, -1))
    assert _lib.stage_copy(many_dst, many_src, rows, list(range(200))) == 4  # 64 rows a launch
    torch.cuda.synchronize()
    assert torch.equal(many_dst, many_src.flip(0))
    odd_src = torch.randn(4, 5, generator=g).to(cuda)  # 20-byte rows
    odd_dst = torch.zeros(4, 5, device=cuda)
    assert _lib.stage_copy(odd_dst, odd_src, [1, 2], [2, 3]) == 1  # one memcpy of the run
    torch.cuda.synchronize()
    assert torch.equal(odd_dst[2:], odd_src[1:3])


def test_device_wave_planner_matches_reference_golden(cuda):
    """lm_plan_waves reproduces the reference's canonical wave plans bit for bit."""
    import json
    from pathlib import Path

    cases = json.loads((Path(__file__).parent / "golden" / "waves.json").read_text())
    for case in cases:
        counts_d = {int(k): int(v) for k, v in case["counts"].items()}
        E = max(counts_d) + 1
        counts = torch.zeros(E, dtype=torch.int32)
        for e, c in counts_d.items():
            counts[e] = c
        e2g = torch.empty(E, dtype=torch.int32, device=cuda)
        rows = torch.empty(E, dtype=torch.int32, device=cuda)
        woff = torch.empty(E + 1, dtype=torch.int32, device=cuda)
        nw = torch.empty(1, dtype=torch.int32, device=cuda)
        _lib.plan_waves(counts.to(cuda), case["num_slots"], e2g, rows, woff, nw, in_place_rows=True)
        n = int(nw.item())
        off = woff[: n + 1].tolist()
        r = rows.tolist()
        got = [r[off[w]:off[w + 1]] for w in range(n)]
        assert got == case["waves"], case["num_slots"]
        # expert_to_group numbers groups wave by wave, members by id
        g = e2g.tolist()
        flat = [e for w in case["waves"] for e in w]
        assert [g[e] for e in flat] == list(range(len(flat)))
        # positional rows (stage-bank mode)
        _lib.plan_waves(counts.to(cuda), case["num_slots"], e2g, rows, woff, nw, in_place_rows=False)
        r = rows.tolist()
        assert [r[off[w]:off[w + 1]] for w in range(n)] == [list(range(len(w))) for w in case["waves"]]


def test_prefill_single_sm_tiles_match_oracle_in_subprocess(cuda):
    """Every group on single-SM tiles over all SMs (LM_UMMA_CTA_PAIR=1, set per process; the
    default splits the groups between 2-SM and single-SM tiles) passes the same parity
    cases."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, LM_UMMA_CTA_PAIR="1")
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-m", "gpu",
         str(root / "tests" / "test_gpu_kernels.py"), "-k", "prefill_tcgen05 or boundaries"],
        cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-2000:]
