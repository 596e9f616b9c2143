"""The drop-in boundary, checked against the reference's own model code.

With the unmodified reference installed in baseline/_ref (these tests skip
without it), a fresh process applies the one change INTEGRATION.md asks a
maintainer to make -- nanovllm.layers.moe's ExpertParallelMoE and
MOE_MAX_GRAPH_TOKENS_PER_RANK rebound to this package's -- and then drives
the reference's Qwen3-MoE model and model runner on the CPU:
  * the names the model and runner bound at import are this package's
    (qwen3_moe.py:10, model_runner.py:33), and the layer picks up nano-vLLM's
    own process groups and forward context (dist_env);
  * the model builds every sparse layer with this class
    (Qwen3MoeDecoderLayer, qwen3_moe.py:60-80) and its state_dict keys and
    shapes equal the reference class's;
  * the isinstance sites route through it: expert weight loading
    (should_load_weight / load_weight, qwen3_moe.py:286-331), the piecewise
    prefill runner's "moe" pieces (:222), get_expert_diagnostics (:343-390)
    and the runner's relocate_moe_experts (model_runner.py:670-683).
Expert math runs on the oracle-backed CPU stand-in of the kernels (no GPU).
"""

import multiprocessing as mp
import os
import socket
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(REPO, "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF_DIR, "nanovllm")),
                                reason="reference not installed in baseline/_ref")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config():
    from transformers import Qwen3MoeConfig
    return Qwen3MoeConfig(hidden_size=64, intermediate_size=128, moe_intermediate_size=32,
                          num_experts=8, num_experts_per_tok=2, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                          vocab_size=128, decoder_sparse_step=1, norm_topk_prob=True)


def _worker(port: int, queue) -> None:
    try:
        sys.path.insert(0, REF_DIR)
        sys.path.insert(0, REPO)
        import torch
        import torch.distributed as dist

        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0,
                                world_size=1)
        from nanovllm.distributed.parallel_state import initialize_model_parallel
        initialize_model_parallel(1, 1, True)
        import nanovllm.layers.moe as ref_moe
        original = ref_moe.ExpertParallelMoE
        import extend_nano_vllm_b200 as b2
        # The maintainer's patch at the end of nanovllm/layers/moe.py.
        ref_moe.ExpertParallelMoE = b2.ExpertParallelMoE
        ref_moe.MOE_MAX_GRAPH_TOKENS_PER_RANK = b2.MOE_MAX_GRAPH_TOKENS_PER_RANK
        from nanovllm.engine import model_runner
        from nanovllm.models import qwen3_moe
        from extend_nano_vllm_b200 import dist_env
        from oracle.cpu_ops import CpuOps

        checks = {}
        checks["names"] = (qwen3_moe.ExpertParallelMoE is b2.ExpertParallelMoE
                           and model_runner.ExpertParallelMoE is b2.ExpertParallelMoE
                           and model_runner.MOE_MAX_GRAPH_TOKENS_PER_RANK == 512)
        from nanovllm.utils.context import get_context
        checks["groups"] = (dist_env._ps is not None and dist_env.get_tp_world_size() == 1
                            and dist_env.get_context() is get_context())

        cfg = _config()
        torch.manual_seed(0)
        model = qwen3_moe.Qwen3MoeForCausalLM(cfg).to(torch.bfloat16)
        with torch.no_grad():
            for parameter in model.parameters():
                parameter.normal_(0.0, 0.02)
        moes = [layer.mlp for layer in model.model.layers.values()]
        checks["layers"] = all(type(m) is b2.ExpertParallelMoE for m in moes)
        ref_layer = original(cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts,
                             cfg.num_experts_per_tok, cfg.norm_topk_prob)
        ours = {k: tuple(v.shape) for k, v in moes[0].state_dict().items()}
        theirs = {k: tuple(v.shape) for k, v in ref_layer.state_dict().items()}
        checks["state_dict"] = ours == theirs

        # Expert weight routing through the model's isinstance-guarded loader.
        w = torch.randn(cfg.moe_intermediate_size, cfg.hidden_size).to(torch.bfloat16)
        name = "model.layers.1.mlp.experts.5.up_proj.weight"
        loaded = model.should_load_weight(name) and model.load_weight(name, w)
        checks["load_weight"] = bool(loaded) and torch.equal(
            moes[1].gate_up_proj.data[5, cfg.moe_intermediate_size:], w)

        # An EP shard of the same model: ownership decides what loads.
        shard = qwen3_moe.Qwen3MoeForCausalLM(
            cfg, ep_rank=1, ep_size=2, dispatch_backend="all_to_all_nvlink",
            expert_placement={"0": (0, 1) * 4, "1": (1, 1, 1, 1, 0, 0, 0, 0)})
        checks["ownership"] = (
            shard.should_load_weight("model.layers.0.mlp.experts.3.gate_proj.weight")
            and not shard.should_load_weight("model.layers.0.mlp.experts.2.gate_proj.weight")
            and shard.should_load_weight("model.layers.1.mlp.experts.0.down_proj.weight")
            and not shard.should_load_weight("model.layers.1.mlp.experts.7.down_proj.weight")
            and shard.model.layers["0"].mlp.local_expert_ids == (1, 3, 5, 7))

        # The piecewise prefill runner tags these layers as "moe" pieces.
        for m in moes:
            m._ops = CpuOps()
        tokens = 5
        kinds, outs = [], []

        def runner(kind, module, *args):
            if kind == "embed":
                return torch.randn(tokens, cfg.hidden_size).to(torch.bfloat16)
            if kind == "pre":
                return None, None, None, args[2]
            if kind == "attention":
                return None
            if kind == "post":
                return torch.randn(tokens, cfg.hidden_size).to(torch.bfloat16), args[1]
            if kind in ("moe", "mlp"):
                kinds.append(kind)
                out = module(args[0])
                outs.append(tuple(out.shape))
                return out
            return args[0], None

        model.model.forward_prefill_piece(torch.arange(tokens), torch.arange(tokens), runner)
        checks["prefill_pieces"] = (kinds == ["moe", "moe"]
                                    and outs == [(tokens, cfg.hidden_size)] * 2)
        diag = model.get_expert_diagnostics()
        checks["diagnostics"] = (diag["total_assignment_count"] == 2 * tokens * 2
                                 and diag["dispatch_assignment_count"] == 2 * tokens * 2
                                 and diag["num_local_experts"] == 8
                                 and diag["local_expert_ids"] == list(range(8)))

        # The runner's relocation entry point reaches relocate_experts.
        dyn = qwen3_moe.Qwen3MoeForCausalLM(cfg, dynamic_placement=True)
        runner_obj = model_runner.ModelRunner.__new__(model_runner.ModelRunner)

        class _Cfg:
            moe_dynamic_placement = True
            moe_placement_by_layer = {}

        runner_obj.config = _Cfg()
        runner_obj.model = dyn
        runner_obj.world_size = 1
        runner_obj.rank = 0
        gathered = runner_obj.relocate_moe_experts({"0": (0,) * 8, "1": (0,) * 8})
        checks["relocate"] = gathered == [{"0": 0, "1": 0}]
        queue.put(checks)
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        import traceback
        queue.put(traceback.format_exc())


@pytest.mark.timeout(300)
def test_reference_model_and_runner_use_the_drop_in():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    proc = ctx.Process(target=_worker, args=(_free_port(), queue))
    proc.start()
    try:
        result = queue.get(timeout=240)
    finally:
        proc.join(timeout=30)
        if proc.is_alive():
            proc.terminate()
    assert isinstance(result, dict), result
    failed = [name for name, ok in result.items() if not ok]
    assert not failed, result
