"""Host side of the end-to-end harness (bench.py --e2e), on CPU: the
config-only model directory loads through transformers as the reference
engine loads it, and the import-time swap makes every nanovllm module that
imported the reference's ExpertParallelMoE build this library's class, with
the engine's cross-DP all-gather backend mapped to the NVLink exchange."""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(REPO, "baseline", "_ref")


def _bench():
    sys.path.insert(0, REPO)
    import bench
    return bench


def test_model_directory_loads_like_a_checkpoint(tmp_path):
    from transformers import AutoConfig, AutoTokenizer

    bench = _bench()
    bench.e2e_model_dir(str(tmp_path), 4)
    config = AutoConfig.from_pretrained(str(tmp_path))
    assert config.model_type == "qwen3_moe"
    assert (config.num_hidden_layers, config.hidden_size, config.num_experts,
            config.num_experts_per_tok, config.moe_intermediate_size,
            config.num_attention_heads, config.num_key_value_heads, config.head_dim,
            config.vocab_size) == (4, 2048, 128, 8, 768, 32, 4, 128, 151936)
    tok = AutoTokenizer.from_pretrained(str(tmp_path), use_fast=True)
    assert tok.eos_token_id == 151645
    assert tok.decode([5, 151935]) == "t5 t151935"


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "nanovllm")),
                    reason="the reference is not installed in baseline/_ref")
def test_engine_modules_get_this_layer():
    bench = _bench()
    added = REF not in sys.path
    if added:
        sys.path.insert(0, REF)
    import nanovllm.engine.model_runner as runner
    import nanovllm.layers.moe as ref_moe
    import nanovllm.models.qwen3_moe as qwen3_moe

    from extend_nano_vllm_b200.moe import ExpertParallelMoE

    original = ref_moe.ExpertParallelMoE
    try:
        bench.e2e_install_b200_layer()
        for module in (ref_moe, qwen3_moe, runner):
            assert issubclass(module.ExpertParallelMoE, ExpertParallelMoE)
        layer = qwen3_moe.ExpertParallelMoE(
            hidden_size=64, intermediate_size=32, num_experts=8, top_k=2, norm_topk_prob=True,
            ep_rank=0, ep_size=2, dispatch_backend="allgather_reduce", graph_safe_decode=True)
        assert layer.dispatch_backend == "all_to_all_nvlink"
    finally:
        # Later tests (and the processes they spawn, which inherit sys.path)
        # run the library standalone, without the reference's groups.
        if added:
            sys.path.remove(REF)
        for module in list(sys.modules.values()):
            if getattr(module, "__name__", "").startswith("nanovllm") and \
                    getattr(module, "ExpertParallelMoE", None) is not None and \
                    module.ExpertParallelMoE is not original and \
                    issubclass(module.ExpertParallelMoE, ExpertParallelMoE):
                module.ExpertParallelMoE = original
