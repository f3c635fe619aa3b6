"""The C-ABI library loads without a GPU and exports every symbol include/*.h declares."""

import ctypes
import re
from pathlib import Path

from vllm_ascend_hust_latchmoe_b200 import _build, _lib

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(lm_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    path = _build.build()
    lib = ctypes.CDLL(str(path))
    names = declared_symbols()
    assert len(names) >= 10
    for name in sorted(names):
        assert hasattr(lib, name), name
    assert names == set(_lib.SIGNATURES), names ^ set(_lib.SIGNATURES)


def test_abi_version_and_error_strings_without_gpu():
    lib = _lib.load()
    assert lib.lm_abi_version() == 1
    # argument validation happens on the host, before any CUDA call
    rc = lib.lm_route_topk(None, 4, 999, 8, 0, 1, 1.0, None, 0, 0, None, None, None, None)
    assert rc == -1
    assert b"num_experts" in lib.lm_last_error()
    rc = lib.lm_stage_copy(None, 16, None, 16, None, None, 1, 16, 7, None)
    assert rc == -1 and b"kind" in lib.lm_last_error()
    # an empty call may pass empty (null) tensors: nothing to do, no CUDA call
    assert lib.lm_route_topk(None, 0, 128, 8, 0, 1, 1.0, None, 0, 0, None, None, None,
                             None) == 0
    rc = lib.lm_ep_dispatch_tokens(None, 10, 8, 2048, None, 16, None, None, 0, 2, None, 160, 1,
                                   None, None, None, None, None)
    assert rc == -1  # tokens present: every pointer is required


def test_ep_exchange_capacity_is_checked_on_the_host():
    """More routed pairs than the exchange capacity are refused before any launch (a C-ABI
    caller could otherwise address rows past an owner's receive area)."""
    lib = _lib.load()
    fake = ctypes.c_void_p(0x1000)
    # 10 tokens x top-8 = 80 pairs > cap 64
    rc = lib.lm_ep_dispatch(fake, 10, 8, 2048, fake, 16, fake, fake, 0, 2, fake, 64, 1, fake,
                            None, None)
    assert rc == -1 and b"capacity" in lib.lm_last_error()
    rc = lib.lm_ep_combine(fake, fake, 10, 8, 2048, 16, fake, fake, 0, 2, fake, fake, 64, 1,
                           fake, None, None)
    assert rc == -1 and b"capacity" in lib.lm_last_error()
    rc = lib.lm_ep_dispatch_tokens(fake, 10, 8, 2048, fake, 16, fake, fake, 0, 2, fake, 64, 1,
                                   fake, fake, fake, None, None)
    assert rc == -1 and b"capacity" in lib.lm_last_error()
    rc = lib.lm_ep_combine_local(fake, fake, 10, 8, 2048, 16, fake, fake, 0, 2, fake, fake, 64,
                                 1, fake, None, None)
    assert rc == -1 and b"capacity" in lib.lm_last_error()
    # epoch 0 selects the region's device-side counter; a negative epoch is refused
    rc = lib.lm_ep_dispatch_tokens(fake, 4, 8, 2048, fake, 16, fake, fake, 0, 2, fake, 64, -1,
                                   fake, fake, fake, None, None)
    assert rc == -1 and b"bad arguments" in lib.lm_last_error()
    rc = lib.lm_ep_signal_outputs(fake, 0, 2, 64, 2048, -1, None)
    assert rc == -1
    rc = lib.lm_ep_advance_epoch(None, 2, 64, 2048, None)
    assert rc == -1 and b"null region" in lib.lm_last_error()
