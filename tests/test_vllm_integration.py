"""vLLM CUDA integration on CPU: PIECEWISE splitting at ``vllm::moe_offload_stage``, the
platform and EngineArgs patches, vLLM's own graph splitter on a traced seam call, the MoE
runner's seam entry and the weight-loading attachment hook. Mirrors the reference's
``tests/test_patch_fused_moe.py:760-880`` on vLLM's CUDA classes."""

import json
from types import SimpleNamespace

import pytest
import torch

import vllm_ascend_hust_latchmoe_b200 as plugin
from vllm_ascend_hust_latchmoe_b200 import autoconfig as ac
from vllm_ascend_hust_latchmoe_b200 import vllm_integration as vi

CUDAGraphMode = pytest.importorskip("vllm.config").CUDAGraphMode


def _config(mode, ops=None):
    return SimpleNamespace(compilation_config=SimpleNamespace(cudagraph_mode=mode,
                                                              splitting_ops=ops))


@pytest.fixture
def seam_on(monkeypatch):
    monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM", "1")


def test_splitting_op_added_for_piecewise_only(seam_on):
    cfg = _config(CUDAGraphMode.PIECEWISE, [])
    assert vi.ensure_moe_offload_splitting_op(cfg, fail_closed=True)
    assert vi.ensure_moe_offload_splitting_op(cfg, fail_closed=True)  # no duplicate
    assert cfg.compilation_config.splitting_ops == [vi.SPLITTING_OP]
    cfg = _config(CUDAGraphMode.PIECEWISE, None)
    assert vi.ensure_moe_offload_splitting_op(cfg)
    assert cfg.compilation_config.splitting_ops == [vi.SPLITTING_OP]
    none = _config(CUDAGraphMode.NONE, [])
    assert not vi.ensure_moe_offload_splitting_op(none, fail_closed=True)
    assert none.compilation_config.splitting_ops == []
    with pytest.raises(RuntimeError, match="compilation_config"):
        vi.ensure_moe_offload_splitting_op(SimpleNamespace(), fail_closed=True)


def test_seam_off_leaves_the_config_alone(monkeypatch):
    monkeypatch.delenv("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM", raising=False)
    cfg = _config(CUDAGraphMode.FULL, [])
    assert not vi.ensure_moe_offload_splitting_op(cfg, fail_closed=True)
    assert cfg.compilation_config.splitting_ops == []


@pytest.mark.parametrize("mode", [CUDAGraphMode.FULL, CUDAGraphMode.FULL_AND_PIECEWISE,
                                  CUDAGraphMode.FULL_DECODE_ONLY])
def test_stage_seam_fails_closed_for_any_full_graph(seam_on, mode):
    with pytest.raises(RuntimeError, match="requires PIECEWISE-only"):
        vi.ensure_moe_offload_splitting_op(_config(mode, []), fail_closed=True)
    assert not vi.ensure_moe_offload_splitting_op(_config(mode, []))


def test_platform_patch_appends_after_platform_defaults(seam_on):
    calls = []

    class FakePlatformBase:
        @classmethod
        def check_and_update_config(cls, vllm_config):
            calls.append(cls)
            if vllm_config.compilation_config.splitting_ops is not None:
                vllm_config.compilation_config.splitting_ops.append("vllm::unified_attention")

    class FakeCudaPlatform(FakePlatformBase):  # inherits the hook, like vLLM's CUDA classes
        pass

    assert vi.patch_platform_splitting_ops(FakeCudaPlatform)
    assert not vi.patch_platform_splitting_ops(FakeCudaPlatform)  # idempotent
    cfg = _config(CUDAGraphMode.PIECEWISE, [])
    FakeCudaPlatform.check_and_update_config(cfg)
    assert calls == [FakeCudaPlatform]
    assert cfg.compilation_config.splitting_ops == ["vllm::unified_attention", vi.SPLITTING_OP]
    # an unset list stays unset: vLLM fills in its attention ops only while it is None
    unset = _config(CUDAGraphMode.PIECEWISE, None)
    FakeCudaPlatform.check_and_update_config(unset)
    assert unset.compilation_config.splitting_ops is None
    FakePlatformBase.check_and_update_config(cfg)  # the base class itself is not wrapped
    assert calls[-1] is FakePlatformBase


def test_engine_args_final_config_boundary(seam_on, monkeypatch, tmp_path, capsys):
    events = []
    (tmp_path / "config.json").write_text(json.dumps({
        "num_hidden_layers": 48, "num_experts": 128, "num_experts_per_tok": 8,
        "hidden_size": 2048, "moe_intermediate_size": 768, "torch_dtype": "bfloat16"}))

    class FakeEngineArgs:
        model = str(tmp_path)
        max_num_seqs = 1
        max_model_len = 4096

        def __init__(self):
            self.compilation_config = {}

        def create_engine_config(self):
            events.append("create")
            return _config(CUDAGraphMode[self.compilation_config["cudagraph_mode"]], [])

    monkeypatch.setattr(vi, "patch_platform_splitting_ops", lambda *a: events.append("retry"))
    monkeypatch.setenv("VLLM_ASCEND_MOE_OFFLOAD_GB", "14")
    for name in ("VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS", "VLLM_ASCEND_MOE_OFFLOAD_ENABLED",
                 "VLLM_ASCEND_MOE_OFFLOAD_RESIDENT_LAYER_IDS",
                 "VLLM_ASCEND_MOE_OFFLOAD_FANOUT_THRESHOLD",
                 "VLLM_ASCEND_MOE_OFFLOAD_B2_WAVE_PREFILL", "VLLM_ASCEND_MOE_OFFLOAD_ASYNC_LOAD",
                 "VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME", *ac.SEW_DATAPLANE_ENV_VARS):
        if name != "VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM":
            monkeypatch.delenv(name, raising=False)
    assert vi.patch_engine_args(FakeEngineArgs)
    assert not vi.patch_engine_args(FakeEngineArgs)
    args = FakeEngineArgs()
    cfg = args.create_engine_config()
    assert events == ["retry", "create"]
    assert args.compilation_config["cudagraph_mode"] == "PIECEWISE"  # seam default
    assert cfg.compilation_config.splitting_ops == [vi.SPLITTING_OP]
    assert vi.GRAPH_CONFIG_LINE in capsys.readouterr().out
    import os

    assert int(os.environ["VLLM_ASCEND_MOE_OFFLOAD_NUM_SLOTS"]) > 0  # AutoConfig applied
    assert os.environ["VLLM_ASCEND_MOE_OFFLOAD_ENABLED"] == "1"
    # the seam selects the fixed-slot data plane defaults
    assert os.environ["VLLM_ASCEND_MOE_OFFLOAD_RELEASE_ORIGINAL_EXPERT_WEIGHTS"] == "1"
    assert os.environ["VLLM_ASCEND_MOE_OFFLOAD_LAYERED_RUNTIME"] == "0"

    class FullGraphArgs(FakeEngineArgs):
        def __init__(self):
            self.compilation_config = {"cudagraph_mode": "FULL"}

    with pytest.raises(RuntimeError, match="requires PIECEWISE-only"):
        FullGraphArgs().create_engine_config()


def test_stage_custom_op_is_a_top_level_splitting_graph():
    from torch.fx.experimental.proxy_tensor import make_fx
    from vllm.compilation.backends import split_graph

    plugin.register()

    def model(x):
        routed = x + 1
        torch.ops.vllm.moe_offload_stage(routed, 0, 128, 0)
        return routed * 2

    graph = make_fx(model, tracing_mode="fake")(torch.ones(2, dtype=torch.int32))
    _, items = split_graph(graph, [vi.SPLITTING_OP])
    splitting = [item for item in items if item.is_splitting_graph]
    assert len(splitting) == 1
    targets = [n.target for n in splitting[0].graph.graph.nodes if n.op == "call_function"]
    assert torch.ops.vllm.moe_offload_stage.default in targets
    assert len(items) == 3  # router piece | eager stage | MLP piece


class _Recorder:
    def __init__(self):
        self.calls = []

    def moe_router_indirect(self, h, lg, name):
        self.calls.append(("router", name))
        return "w", "ids"

    def moe_offload_stage(self, ids, layer_id, n, phase):
        self.calls.append(("stage", ids, layer_id, n, phase))

    def moe_mlp(self, h, lg, w, ids, shared_in, input_ids, name, unpadded):
        self.calls.append(("mlp", w, ids, name, unpadded))
        return "routed"


def test_runner_seam_entry_routes_through_the_seam_ops(seam_on, monkeypatch):
    class FakeRunner:
        layer_name = "model.layers.3.mlp.experts"

        def __init__(self):
            self._forward_entry = self._select_forward()

        def _select_forward(self):
            return "native"

    assert vi.patch_moe_runner(FakeRunner)
    assert not vi.patch_moe_runner(FakeRunner)
    rec = _Recorder()
    monkeypatch.setattr(vi, "_seam_ops", lambda: rec)
    runner = FakeRunner()
    with pytest.raises(RuntimeError, match="refusing native fallback"):
        runner._forward_entry("h", "lg", None, None, "from_forward_context", -1)
    runner._latchmoe_seam = vi.SeamBinding(FakeRunner.layer_name, 3, 128, shared=False)
    assert runner._forward_entry("h", "lg", None, None, "from_forward_context", -1) == "routed"
    assert rec.calls == [("router", FakeRunner.layer_name), ("stage", "ids", 3, 128, -1),
                         ("mlp", "w", "ids", FakeRunner.layer_name, -1)]
    monkeypatch.delenv("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM")
    assert FakeRunner()._forward_entry == "native"


def test_layer_ids_and_attachment_guards():
    assert vi.layer_id_from_name("model.layers.7.mlp.experts") == 7
    assert vi.layer_id_from_name("layers.0.experts") == 0
    with pytest.raises(ValueError):
        vi.layer_id_from_name("model.mlp.experts")
    w13 = torch.zeros(4, 256, 128, dtype=torch.bfloat16)
    w2 = torch.zeros(4, 128, 128, dtype=torch.bfloat16)

    def layer(**kw):
        base = dict(layer_name="model.layers.1.mlp.experts", w13_weight=w13, w2_weight=w2,
                    top_k=2, global_num_experts=4, tp_size=1, ep_size=1, dp_size=1)
        base.update(kw)
        return SimpleNamespace(**base)

    with pytest.raises(RuntimeError, match="single-GPU"):
        vi.attach_fused_moe_layer(layer(tp_size=2), runtime=object())
    with pytest.raises(RuntimeError, match="bf16 unquantized"):
        vi.attach_fused_moe_layer(layer(w2_weight=w2.float()), runtime=object())
    with pytest.raises(ValueError, match="expert pair"):
        vi.attach_fused_moe_layer(layer(w2_weight=w2[:, :, :64]), runtime=object())
    with pytest.raises(RuntimeError, match="expert-parallel"):
        vi.attach_fused_moe_layer(layer(global_num_experts=8), runtime=object())


def test_weight_loading_hook_attaches_once_and_skips_native_setup(seam_on, monkeypatch):
    events = []

    class FakeMethod:
        def process_weights_after_loading(self, layer):
            events.append(("vllm", layer.name))

    def attach(layer, max_tokens):
        events.append(("attach", layer.name, max_tokens))
        layer.runner._latchmoe_seam = object()

    assert vi.patch_weight_loading(FakeMethod, max_tokens=lambda: 512, attach=attach)
    assert not vi.patch_weight_loading(FakeMethod)
    layer = SimpleNamespace(name="l0", runner=SimpleNamespace())
    FakeMethod().process_weights_after_loading(layer)
    FakeMethod().process_weights_after_loading(layer)  # already attached: not again
    assert events == [("attach", "l0", 512)]
    monkeypatch.delenv("VLLM_ASCEND_MOE_OFFLOAD_STAGE_SEAM")
    FakeMethod().process_weights_after_loading(SimpleNamespace(name="l1", runner=None))
    assert events[-1] == ("vllm", "l1")  # seam off: vLLM's own post-processing


def test_seam_entry_applies_the_runner_gate(seam_on, monkeypatch):
    rec = _Recorder()
    monkeypatch.setattr(vi, "_seam_ops", lambda: rec)
    seen = []

    def gate(h):
        seen.append(h)
        return "logits", None

    orig_router = rec.moe_router_indirect

    def router(h, lg, name):
        seen.append(lg)
        return orig_router(h, lg, name)

    rec.moe_router_indirect = router
    runner = SimpleNamespace(gate=gate, _latchmoe_seam=vi.SeamBinding("x.layers.0.e", 0, 8, False))
    assert vi.seam_forward_entry(runner, "h", "h", None, None) == "routed"
    assert seen == ["h", "logits"]


def test_traced_seam_entry_splits_into_router_stage_and_mlp_pieces():
    """The runner's seam entry traced with fake tensors (what vLLM's compiler sees) splits
    at the stage op into a router piece, the eager stage and the MLP piece."""
    from torch.fx.experimental.proxy_tensor import make_fx
    from vllm.compilation.backends import split_graph

    plugin.register()
    runner = SimpleNamespace(layer_name="model.layers.5.mlp.experts",
                             _latchmoe_seam=vi.SeamBinding("model.layers.5.mlp.experts", 5, 128,
                                                           shared=False))

    def forward(h, lg):
        return vi.seam_forward_entry(runner, h, lg, None, None, "from_forward_context", 0)

    graph = make_fx(forward, tracing_mode="fake")(torch.empty(4, 256, dtype=torch.bfloat16),
                                                  torch.empty(4, 128))
    ops = [n.target for n in graph.graph.nodes if n.op == "call_function"
           and "vllm" in str(n.target)]
    assert [str(o) for o in ops] == ["vllm.moe_router_indirect.default",
                                     "vllm.moe_offload_stage.default", "vllm.moe_mlp.default"]
    _, items = split_graph(graph, [vi.SPLITTING_OP])
    pieces = [[str(n.target) for n in it.graph.graph.nodes if n.op == "call_function"]
              for it in items]
    assert [it.is_splitting_graph for it in items] == [False, True, False]
    assert any("moe_router_indirect" in t for t in pieces[0])
    assert pieces[1] == ["vllm.moe_offload_stage.default"]
    assert any("moe_mlp" in t for t in pieces[2])


def test_captured_mlp_piece_takes_the_path_of_its_layer_tier(monkeypatch):
    """While vLLM captures an MLP piece, the seam records the path that reads only fixed
    buffers for the layer's tier: in-place reads for an HBM store, the device slot plan under
    device staging, the slot bank otherwise; prefill-sized captures under device staging are
    refused. Outside capture the eager stage decision is consumed once."""
    from vllm_ascend_hust_latchmoe_b200 import seam_ops
    from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE, StageDecision

    def layer(resident, device, waves_from_store=False):
        lay = SlotBankMoE.__new__(SlotBankMoE)
        lay.resident_tier, lay.device_staging, lay.layer_id, lay.pending = resident, device, 0, None
        lay.num_fused_shared = 0
        lay.runtime = SimpleNamespace(config=SimpleNamespace(
            stage_waves_from_hbm_store=waves_from_store, stage_waves_on_device=True))
        return lay

    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    assert seam_ops._take_decision(layer(True, False), 4).mode == "resident"
    # an HBM store staged wave by wave: prefill sizes plan and stage their waves on the device
    assert seam_ops._take_decision(layer(True, False, True), 512).mode == "device_waves"
    assert seam_ops._take_decision(layer(True, False, True), 4).mode == "resident"
    assert seam_ops._take_decision(layer(False, True), 4).mode == "device"
    assert seam_ops._take_decision(layer(False, False), 4).mode == "capturing"
    with pytest.raises(RuntimeError, match="not captured under device staging"):
        seam_ops._take_decision(layer(False, True), 512)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)
    lay = layer(False, False)
    lay.pending = StageDecision("slots")
    assert seam_ops._take_decision(lay, 4).mode == "slots" and lay.pending is None
    with pytest.raises(RuntimeError, match="without a preceding"):
        seam_ops._take_decision(lay, 4)


def test_serve_check_model_config_is_a_qwen3_moe_config():
    """The synthetic model the serving check hands vLLM parses as a transformers Qwen3-MoE
    config with Qwen3-30B-A3B's expert shapes."""
    transformers = pytest.importorskip("transformers")
    from vllm_ascend_hust_latchmoe_b200.vllm_serve_check import qwen3_moe_config

    raw = qwen3_moe_config(4, 32768)
    cfg = transformers.AutoConfig.for_model(raw.pop("model_type"), **raw)
    assert type(cfg).__name__ == "Qwen3MoeConfig"
    assert (cfg.num_hidden_layers, cfg.hidden_size, cfg.moe_intermediate_size) == (4, 2048, 768)
    assert (cfg.num_experts, cfg.num_experts_per_tok, cfg.norm_topk_prob) == (128, 8, True)
    assert (cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim) == (32, 4, 128)


def test_foreign_topk_ids_drop_the_routers_grouping():
    """When the MLP op receives top-k tensors from another router, it copies them into the
    layer's buffers and the layer groups the pairs again (the one-launch router grouping of
    the previous route() call no longer describes them)."""
    from vllm_ascend_hust_latchmoe_b200 import seam_ops
    from vllm_ascend_hust_latchmoe_b200.layer import SlotBankMoE

    lay = SlotBankMoE.__new__(SlotBankMoE)
    lay.topk_ids = torch.zeros(4, 2, dtype=torch.int32)
    lay.topk_w = torch.zeros(4, 2, dtype=torch.bfloat16)
    lay._grouped_by_router = 4
    seam_ops._adopt_topk(lay, lay.topk_w[:4], lay.topk_ids[:4])  # the layer's own buffers
    assert lay._grouped_by_router == 4
    seam_ops._adopt_topk(lay, torch.ones(4, 2, dtype=torch.bfloat16),
                         torch.ones(4, 2, dtype=torch.int32))
    assert lay._grouped_by_router is None and int(lay.topk_ids.sum()) == 8

