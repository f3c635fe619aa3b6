"""vLLM's own CUDA ``FusedMoE`` layer on the slot-bank seam: the layer is built by vLLM (its
``MoERunner`` picks the seam entry because the patch is installed and the seam switch is on),
its checkpoint-layout weights are attached to the host store and slot bank, and
``FusedMoE.forward`` then runs router -> stage -> grouped MLP -> combine through the seam ops.
Top-k ids must equal the oracle's and outputs stay within the bf16 tolerance, on a decode call
with more active experts than slots (waves) and on a prefill-sized call, after vLLM's own
copies of the expert tensors were released (the seam reads only the store and slot bank).

The vLLM part runs in a child process: it initialises vLLM's distributed state and its global
config, which must not leak into the other tests of this session.
"""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _child(port: int) -> None:
    sys.path.insert(0, str(ROOT))
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM"] = "1"
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_ENABLED"] = "1"
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"] = "32"
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD"] = "1"
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL"] = "1"
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_GRAPH_COMPATIBLE"] = "1"
    os.environ["VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS"] = "1"
    import torch

    import vllm_ascend_hust_latchmoe_b200 as plugin
    from oracle import mlp as omlp
    from oracle import router as orouter
    from oracle.bf16 import bf16_bits_to_f32
    from tests.helpers import bits
    from vllm_ascend_hust_latchmoe_b200 import seam_ops
    from vllm_ascend_hust_latchmoe_b200 import synthetic as syn
    from vllm_ascend_hust_latchmoe_b200 import vllm_integration as vi

    plugin.register()  # seam on: installs the vLLM patches
    from vllm.config import VllmConfig, set_current_vllm_config
    from vllm.distributed import init_distributed_environment, initialize_model_parallel
    from vllm.model_executor.layers.fused_moe.layer import FusedMoE

    cfg = syn.CONFIGS["c1_decode"]
    w13, w2 = syn.make_expert_weights(cfg, 0)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    name = "model.layers.0.mlp.experts"
    result = {}
    with set_current_vllm_config(VllmConfig()):
        init_distributed_environment(world_size=1, rank=0, local_rank=0, backend="nccl",
                                     distributed_init_method=f"tcp://127.0.0.1:{port}")
        initialize_model_parallel(1, 1)
        with torch.device(dev):
            layer = FusedMoE(num_experts=cfg.num_experts, top_k=cfg.top_k,
                             hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
                             params_dtype=torch.bfloat16, renormalize=True, prefix=name)
        result["entry_is_seam"] = layer.runner._forward_entry.__qualname__.endswith("entry")
        layer.w13_weight.data.copy_(w13.to(dev))
        layer.w2_weight.data.copy_(w2.to(dev))
        moe = vi.attach_fused_moe_layer(layer, max_tokens=1024)
        result["layer_id"] = moe.layer_id
        # offloaded layer: vLLM's own expert tensors were emptied, the seam reads the store
        result["released_shapes"] = [list(layer.w13_weight.shape), list(layer.w2_weight.shape)]
        cases = []
        for tokens, seed in ((16, 0), (16, 1), (512, 2)):
            c = cfg.with_tokens(tokens)
            hidden = syn.make_hidden(c, seed=seed)
            logits = syn.make_router_logits(c, seed=seed)
            out = layer.forward(hidden.to(dev), logits.to(dev))
            torch.cuda.synchronize()
            moe.check_device_errors("vllm seam")
            wb, _, ids = orouter.route(logits.numpy(), c.top_k, renormalize=True)
            got_ids = seam_ops.get_layer(name).topk_ids[:tokens].cpu().numpy()
            ref = omlp.moe_layer(bits(hidden), ids, wb, bits(w13), bits(w2))
            m = omlp.compare(bf16_bits_to_f32(bits(out.cpu())), ref)
            cases.append({"tokens": tokens, "ids_equal": bool((got_ids == ids).all()),
                          "waves": len(moe.last_waves.waves) if moe.last_waves else 0, **m})
        result["cases"] = cases
    print("RESULT " + json.dumps(result), flush=True)


def test_vllm_fused_moe_layer_runs_through_the_seam(cuda):
    pytest.importorskip("vllm")
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    proc = subprocess.run([sys.executable, str(Path(__file__).resolve()), str(_free_port())],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")]
    assert proc.returncode == 0 and lines, proc.stdout[-3000:] + proc.stderr[-4000:]
    res = json.loads(lines[-1][len("RESULT "):])
    from tests.helpers import MAX_REL_ERR, MIN_COSINE

    assert res["entry_is_seam"] and res["layer_id"] == 0
    assert res["released_shapes"] == [[0, 1536, 2048], [0, 2048, 768]]
    for case in res["cases"]:
        assert case["ids_equal"], case
        assert case["max_rel_err"] <= MAX_REL_ERR and case["cosine"] >= MIN_COSINE, case
    assert res["cases"][0]["waves"] >= 2  # 33 active experts on 32 slots


if __name__ == "__main__":
    _child(int(sys.argv[1]))
