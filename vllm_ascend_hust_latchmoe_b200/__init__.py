"""B200-native slot-bank MoE offload hot path (drop-in for the LatchMoE offload path).

``register()`` is the ``vllm.general_plugins`` entry point, like the reference's
``vllm_moe_offload_ascend.register`` (``__init__.py:38-58``): it registers the environment
contract first, then the seam custom ops. It is idempotent and can be retried after a
failure.
"""

from __future__ import annotations

import threading

__all__ = ["register", "__version__"]
__version__ = "0.1.0"

_lock = threading.Lock()
_registered = False


def register() -> None:
    global _registered
    with _lock:
        if _registered:
            return
        from . import env_registry

        env_registry.register_environment_variables()
        from . import seam_ops

        seam_ops.register_ops()
        if env_registry.get("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM"):
            # vLLM CUDA integration: PIECEWISE split at the stage op, runner seam entry,
            # attachment after weight loading (each patch best-effort and idempotent)
            from . import vllm_integration

            vllm_integration.install_vllm_patches()
        _registered = True
