"""CPU oracle for the slot-bank MoE hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy and plain Python, what the reference
(vLLM-HUST/vllm-ascend-hust-LatchMoE, package ``vllm_moe_offload_ascend``) computes on
the MoE offload path, so the CUDA data path can be checked against it:

* ``router``  -- expert selection (softmax/sigmoid -> top-k -> renorm -> scale -> bf16),
* ``mlp``     -- grouped expert MLP (gate_up GEMM, SiLU*mul, down GEMM) and the weighted
                 top-k combine in the original pair order, fp32 accumulation,
* ``control`` -- the integer control plane: slot allocation (first EMPTY, else LRU READY),
                 canonical capacity-bounded wave planning, the async stage schedule, the
                 stable pair grouping and the native-combine index.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import this package, and only as the checker or the timed CPU
baseline. The product path (``vllm_ascend_hust_latchmoe_b200``) never imports it.

Pinning: the control-plane functions are pinned against golden vectors produced by
running the reference's own Python control plane (``tests/golden/make_golden.py``) and
against the vectors its unit tests hold. The MLP and router numerics of the reference
live in an un-vendored fork (vllm-ascend-hust @ 4806367) and CANN kernels; no reference
test pins their values, so those two functions are "parity unpinned": they restate the
documented call-site semantics cited in each docstring.
"""
