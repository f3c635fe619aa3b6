"""lm_build_groups_noalloc: the grouping entry point for callers that cannot allocate
device memory (a host whose own pool already owns all free HBM, or a foreign-language
binding without a device allocator). It must give exactly what lm_build_groups gives with
caller-owned scratch, call after call, although every call reuses one static array.

Collected last on purpose (file name), and self-contained so it also passes alone in a
fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from vllm_ascend_hust_latchmoe_b200 import _lib

pytestmark = pytest.mark.gpu

NOALLOC_LIMIT = 131072  # LM_NOALLOC_GROUP_SCRATCH_ELEMS in include/latchmoe_b200.h


def _case(rng, T, k, E, G, dev):
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    active = np.unique(ids)
    e2g = np.full(E, -1, dtype=np.int32)
    e2g[active] = (rng.permutation(active.size) % G).astype(np.int32)
    return torch.from_numpy(ids).to(dev), torch.from_numpy(e2g).to(dev)


def _outputs(P, G, dev):
    return (torch.full((G + 1,), -9, dtype=torch.int32, device=dev),
            torch.full((P,), -9, dtype=torch.int32, device=dev),
            torch.full((P,), -9, dtype=torch.int32, device=dev),
            torch.zeros(1, dtype=torch.int32, device=dev))


def test_noalloc_matches_caller_scratch_on_consecutive_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    rng = np.random.default_rng(2024)
    # Two calls in a row with different shapes, then a third that is smaller than the
    # second, so stale scratch from the earlier call would show up as a mismatch.
    for T, k, E, G in ((4096, 8, 128, 122), (1000, 6, 64, 40), (16, 8, 128, 33)):
        ids, e2g = _case(rng, T, k, E, G, dev)
        P = ids.numel()
        ref = _outputs(P, G, dev)
        got = _outputs(P, G, dev)
        scratch = torch.empty(_lib.build_groups_scratch_elems(P, G), dtype=torch.int32, device=dev)
        _lib.build_groups(ids, E, e2g, G, ref[0], ref[1], ref[2], scratch, ref[3])
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = lib.lm_build_groups_noalloc(ids.data_ptr(), P, E, e2g.data_ptr(), G,
                                         got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(),
                                         got[3].data_ptr(), stream)
        assert rc == 0, lib.lm_last_error()
        torch.cuda.synchronize()
        for a, b in zip(got, ref):  # integer tables: bit-exact
            assert torch.equal(a, b)
        assert int(got[3].item()) == 0


def test_noalloc_rejects_sizes_beyond_its_array():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    G = 1024
    P = 64 * 512 + 1  # 65 tiles x 1024 groups x 2 > NOALLOC_LIMIT
    assert _lib.build_groups_scratch_elems(P, G) > NOALLOC_LIMIT
    ids = torch.zeros(P, dtype=torch.int32, device=dev)
    e2g = torch.zeros(G, dtype=torch.int32, device=dev)
    off, p2r, r2p, err = _outputs(P, G, dev)
    rc = lib.lm_build_groups_noalloc(ids.data_ptr(), P, G, e2g.data_ptr(), G, off.data_ptr(),
                                     p2r.data_ptr(), r2p.data_ptr(), err.data_ptr(), None)
    assert rc == -1
    assert b"built-in array" in lib.lm_last_error()
