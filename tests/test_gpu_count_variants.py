"""GPU parity of the device-count entry points (grouping, row gather, combine and the top-1
resident MLP that read their live row count from device memory).

Each case fills the rows past the live count with ids no grouping accepts and rows of
sentinel values: a kernel that read past the count would raise the device error word or
change an output it must leave alone. Integer tables bit-exact against the CPU oracle on
the live prefix; bf16 values within max|a-e|/max|e| <= 1e-2 and cosine >= 0.9999.
"""

import numpy as np
import pytest
import torch

from oracle import control as ocontrol
from oracle import mlp as omlp
from oracle.bf16 import bf16_bits_to_f32
from tests.helpers import MAX_REL_ERR, MIN_COSINE, bits
from vllm_ascend_hust_latchmoe_b200 import _lib
from vllm_ascend_hust_latchmoe_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

SENTINEL = -12345  # int16 view of a bf16 value no kernel writes here


def _dev_count(cuda, n):
    return torch.tensor([n], dtype=torch.int32, device=cuda)


@pytest.mark.parametrize("R,live,E,G", [(64, 0, 16, 16), (64, 1, 16, 16), (64, 63, 16, 16),
                                        (700, 513, 32, 32), (4096, 4096, 128, 128),
                                        (4096, 2999, 128, 40)])
def test_build_groups_count_reads_only_the_live_prefix(cuda, R, live, E, G):
    rng = np.random.default_rng(R + live)
    ids_np = rng.integers(0, E, size=(R, 1)).astype(np.int32)
    ids_np[live:] = 10 * E  # out of range: reading one sets the device error word
    e2g_np = (np.arange(E) % G).astype(np.int64)
    ids = torch.from_numpy(ids_np).to(cuda)
    e2g = torch.from_numpy(e2g_np.astype(np.int32)).to(cuda)
    off = torch.full((G + 1,), -7, dtype=torch.int32, device=cuda)
    p2r = torch.full((R,), -7, dtype=torch.int32, device=cuda)
    r2p = torch.full((R,), -7, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_lib.build_groups_scratch_elems(R, G), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    _lib.build_groups_count(ids, _dev_count(cuda, live), E, e2g, G, off, p2r, r2p, scratch, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref_off, ref_p2r, ref_r2p = ocontrol.group_pairs(ids_np[:live], e2g_np, G)
    assert np.array_equal(off.cpu().numpy(), ref_off)
    assert np.array_equal(p2r.cpu().numpy()[:live], ref_p2r)
    assert np.array_equal(r2p.cpu().numpy()[:live], ref_r2p[:live])


@pytest.mark.parametrize("R,live,H", [(64, 17, 2048), (1024, 1000, 512), (512, 0, 256)])
def test_permute_and_combine_count(cuda, R, live, H):
    rng = np.random.default_rng(R * 7 + live)
    perm = rng.permutation(R).astype(np.int32)  # row -> pair over the whole capacity
    r2p = torch.from_numpy(perm).to(cuda)
    p2r = torch.from_numpy(np.argsort(perm).astype(np.int32)).to(cuda)
    hidden = torch.randn(R, H, device=cuda).to(torch.bfloat16)
    x_perm = torch.full((R, H), SENTINEL, dtype=torch.int16, device=cuda).view(torch.bfloat16)
    _lib.permute_rows_count(hidden, r2p, 1, R, _dev_count(cuda, live), x_perm)
    y_perm = torch.randn(R, H, device=cuda).to(torch.bfloat16)
    w = torch.ones(R, 1, dtype=torch.bfloat16, device=cuda)
    out = torch.full((R, H), SENTINEL, dtype=torch.int16, device=cuda).view(torch.bfloat16)
    _lib.moe_combine_count(y_perm, p2r, w, _dev_count(cuda, live), out)
    torch.cuda.synchronize()
    xs, hs = x_perm.view(torch.int16).cpu(), hidden.view(torch.int16).cpu()
    assert torch.equal(xs[:live], hs[torch.from_numpy(perm[:live]).long()])
    assert bool((xs[live:] == SENTINEL).all())
    os_, ys = out.view(torch.int16).cpu(), y_perm.view(torch.int16).cpu()
    rows = torch.from_numpy(np.argsort(perm)[:live].astype(np.int64))
    assert torch.equal(os_[:live], ys[rows])  # unit weight: the row itself
    assert bool((os_[live:] == SENTINEL).all())


@pytest.mark.parametrize("R,live", [(48, 37), (48, 0), (600, 517)])
def test_mlp_rows_count_matches_oracle(cuda, R, live):
    """Top-1 owner MLP of the expert-parallel layer: rows sized by capacity, count live."""
    from vllm_ascend_hust_latchmoe_b200.expert_parallel import build_rank_layer

    E_r, H, I = 8, 2048, 768
    cfg = syn.LayerConfig("cnt", hidden=H, num_experts=E_r, top_k=1, intermediate=I,
                          num_slots=E_r, tokens=R)
    w13, w2 = syn.make_expert_weights(cfg, seed=3)
    layer = build_rank_layer(w13_owned=w13, w2_owned=w2, rank=0, device=cuda, max_rows=R,
                             num_slots=E_r, store_on_device=True)
    rng = np.random.default_rng(R + live)
    ids_np = rng.integers(0, E_r, size=R).astype(np.int32)
    ids_np[live:] = 1000  # never read
    rows = syn.make_hidden(cfg, seed=4)
    out = torch.full((R, H), SENTINEL, dtype=torch.int16, device=cuda).view(torch.bfloat16)
    for _ in range(2):  # a second call reuses every buffer
        layer.mlp_rows_count(rows.to(cuda), torch.from_numpy(ids_np).to(cuda),
                             _dev_count(cuda, live), out)
    torch.cuda.synchronize()
    layer.check_device_errors("mlp_rows_count")
    assert bool((out.view(torch.int16)[live:] == SENTINEL).all())
    if live:
        unit = np.full((live, 1), 0x3F80, dtype=np.uint16)  # bf16 1.0
        ref = omlp.moe_layer(bits(rows)[:live], ids_np[:live, None], unit, bits(w13), bits(w2))
        m = omlp.compare(bf16_bits_to_f32(bits(out[:live])), ref)
        assert m["max_rel_err"] <= MAX_REL_ERR and m["cosine"] >= MIN_COSINE, m
