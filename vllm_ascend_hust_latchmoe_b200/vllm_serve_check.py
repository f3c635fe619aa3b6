"""Serve a synthetic Qwen3-30B-A3B-shaped model through vLLM with the slot-bank seam.

    python -m vllm_ascend_hust_latchmoe_b200.vllm_serve_check --layers 4 --new-tokens 64

What it exercises, end to end inside vLLM's own engine (in-process, one GPU):

* ``register()`` with ``VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM=1`` installs the vLLM patches; the
  engine config must come out PIECEWISE with ``vllm::moe_offload_stage`` as a splitting op;
* vLLM builds ``Qwen3MoeForCausalLM`` (random "dummy" weights, no checkpoint or tokenizer);
  every ``FusedMoE`` layer is attached to the slot bank while vLLM post-processes weights
  (odd layers offloaded to the pinned host store, their original expert tensors released;
  even layers on an HBM-resident store);
* vLLM compiles the model, captures PIECEWISE CUDA graphs for the decode batch sizes and
  generates greedily: router and MLP pieces replay from graphs, the stage op runs eagerly.

Prints one JSON line: build time, prefill (TTFT) and decode (TPOT) times, tokens generated,
whether two identical requests produced identical tokens, the staging counters and the final
graph configuration. Random weights: the tokens mean nothing; this checks the integration.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from pathlib import Path


def qwen3_moe_config(layers: int, vocab: int) -> dict:
    """Qwen3-30B-A3B shapes (hidden 2048, 32 q / 4 kv heads of 128, 128 experts top-8, expert
    intermediate 768) with ``layers`` decoder layers."""
    return {
        "architectures": ["Qwen3MoeForCausalLM"], "model_type": "qwen3_moe",
        "hidden_size": 2048, "intermediate_size": 6144, "moe_intermediate_size": 768,
        "num_hidden_layers": layers, "num_attention_heads": 32, "num_key_value_heads": 4,
        "head_dim": 128, "num_experts": 128, "num_experts_per_tok": 8, "norm_topk_prob": True,
        "decoder_sparse_step": 1, "mlp_only_layers": [], "vocab_size": vocab,
        "max_position_embeddings": 8192, "rope_theta": 1000000.0, "rms_norm_eps": 1e-6,
        "hidden_act": "silu", "attention_bias": False, "attention_dropout": 0.0,
        "tie_word_embeddings": False, "torch_dtype": "bfloat16", "use_sliding_window": False,
        "sliding_window": None, "output_router_logits": False, "router_aux_loss_coef": 0.001,
        "bos_token_id": 1, "eos_token_id": 2,
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=32768)
    ap.add_argument("--prompt-tokens", type=int, default=512)
    ap.add_argument("--new-tokens", type=int, default=64)
    ap.add_argument("--slots", type=int, default=32)
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.4)
    args = ap.parse_args(argv)

    resident = ",".join(str(i) for i in range(0, args.layers, 2))
    os.environ.update({
        "VLLM_ENABLE_V1_MULTIPROCESSING": "0",  # the engine core runs in this process
        "VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM": "1",
        "VLLM_ASCEND_MOE_OFFLOAD_ENABLED": "1",
        "VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS": str(args.slots),
        "VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD": "1",
        "VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL": "1",
        "VLLM_ASCEND_MOE_OFFLOAD_GRAPH_COMPATIBLE": "1",
        "VLLM_ASCEND_MOE_OFFLOAD_PIN_HOST_MEMORY": "1",
        "VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS": resident,
        "VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS": "1",
    })
    import vllm_ascend_hust_latchmoe_b200 as plugin

    plugin.register()
    import numpy as np
    from vllm import LLM, SamplingParams

    from . import seam_ops
    from .moe_offload.runtime import get_moe_offload_runtime

    model_dir = Path(tempfile.mkdtemp(prefix="latchmoe_qwen3moe_"))
    (model_dir / "config.json").write_text(json.dumps(qwen3_moe_config(args.layers, args.vocab)))
    t0 = time.perf_counter()
    llm = LLM(model=str(model_dir), load_format="dummy", dtype="bfloat16",
              skip_tokenizer_init=True, seed=0, max_num_seqs=1,
              max_model_len=args.prompt_tokens + args.new_tokens + 64,
              max_num_batched_tokens=max(args.prompt_tokens, 256),
              enable_prefix_caching=False,
              gpu_memory_utilization=args.gpu_memory_utilization,
              compilation_config={"cudagraph_mode": "PIECEWISE",
                                  "cudagraph_capture_sizes": [1, 2, 4]})
    build_s = time.perf_counter() - t0

    rng = np.random.default_rng(0)
    prompt = {"prompt_token_ids": rng.integers(3, args.vocab, args.prompt_tokens).tolist()}

    def run(n: int):
        sp = SamplingParams(max_tokens=n, temperature=0.0, ignore_eos=True, detokenize=False)
        t = time.perf_counter()
        out = llm.generate([prompt], sp, use_tqdm=False)
        return time.perf_counter() - t, list(out[0].outputs[0].token_ids)

    run(4)  # warm-up
    rt = get_moe_offload_runtime()
    stats0 = dict(rt.stage_stats)
    t1, _ = run(1)
    tn, ids_a = run(args.new_tokens)
    _, ids_b = run(args.new_tokens)
    stats = {k: rt.stage_stats[k] - stats0.get(k, 0) for k in rt.stage_stats}
    try:
        cc = llm.llm_engine.vllm_config.compilation_config
        graph = {"cudagraph_mode": str(cc.cudagraph_mode),
                 "splitting_ops": list(cc.splitting_ops or [])}
    except Exception as exc:  # introspection only
        graph = {"unavailable": repr(exc)}
    print(json.dumps({
        "model": f"qwen3-30b-a3b-shaped, {args.layers} layers, dummy weights",
        "attached_moe_layers": len(seam_ops.registered_layer_names()),
        "offloaded_layers": args.layers - len(resident.split(",")),
        "released_original_expert_layers": list(rt.released_original_weight_layers),
        "num_slots": args.slots,
        "engine_build_s": round(build_s, 1),
        "prompt_tokens": args.prompt_tokens,
        "ttft_ms": round(t1 * 1e3, 2),
        "tpot_ms": round((tn - t1) / max(1, args.new_tokens - 1) * 1e3, 3),
        "generated_tokens": len(ids_a),
        "repeatable": ids_a == ids_b,
        "stage_stats_3_requests": stats,
        "graph": graph,
    }), flush=True)
    return 0 if len(ids_a) == args.new_tokens and ids_a == ids_b else 1


if __name__ == "__main__":
    sys.exit(main())
