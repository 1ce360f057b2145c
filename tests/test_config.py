import argparse

import pytest
import yaml

from kunserve_b200.config import KunServeConfig, ModelConfig, ParallelConfig, add_cli_args, get_cli_args, parse_args


def test_cli_defaults_match_reference():
    cfg = parse_args([])
    e = cfg.engine_config
    assert (e.block_size, e.max_batch_size, e.max_batch_tokens, e.gpu_util, e.chunked_prefill_budget) == \
        (256, 256, 131072, 0.9, 4096)
    assert e.preempt_method == "recompute" and e.dtype == "bf16"
    b = cfg.balloon_config
    assert (b.exchange_batch_size, b.max_balloon_memory_ratio, b.max_restore_memory_ratio) == (8, 0.5, 0.8)
    assert cfg.dispatch_config.dispatch_strategy == "round-robin"


def test_yaml_overrides_cli(tmp_path):
    y = {"engine_config": {"ngroups": 2, "group_size": 2, "pp": 1, "tp": 2, "max_batch_size": 64,
                           "max_batch_tokens": 8192, "block_size": 16, "chunked_prefill_budget": 2048},
         "balloon_config": {"balloon_mode": "livereshard", "max_balloon_memory_ratio": 0.4,
                            "max_restore_memory_ratio": 0.7, "restore_memory_threshold": 0.5,
                            "exchange_batch_size": 4},
         "dispatch_config": {"dispatch_strategy": "load"},
         "bench_config": {"model": "llama-2-13b", "qps": 2.5, "zigzag_chunk_limit": 8, "dispatch_strategy": "memory",
                          "duplicate_server": True}}
    f = tmp_path / "c.yaml"
    f.write_text(yaml.safe_dump(y))
    cfg = parse_args(["-c", str(f), "--tp", "1", "--qps", "9"])
    assert cfg.engine_config.tp == 2 and cfg.engine_config.group_size == 2
    assert cfg.balloon_config.enable_balloon and cfg.balloon_config.balloon_mode == "livereshard"
    assert cfg.dispatch_config.dispatch_strategy == "load"
    # the three YAML keys the reference mis-read
    assert cfg.bench_config.zigzag_chunk_limit == 8
    assert cfg.bench_config.server_dispatch_strategy == "memory"
    assert cfg.bench_config.duplicate_server is True
    assert cfg.bench_config.qps == 2.5
    d = cfg.to_dict()
    assert d["engine_config"]["tp"] == 2


@pytest.mark.parametrize("argv", [["--gpu-util", "1.5"], ["--balloon-mode", "bogus"], ["--dispatch-strategy", "x"]])
def test_validation(argv):
    with pytest.raises((ValueError, SystemExit)):
        parse_args(argv)


def test_model_config_shapes():
    mc = ModelConfig("llama-3-70b")
    pc = ParallelConfig(tensor_parallel_size=4, pipeline_parallel_size=2)
    assert (mc.get_q_heads(pc), mc.get_num_heads(pc), mc.get_num_layers(pc)) == (16, 2, 40)
    assert mc.get_kv_bytes_per_token() == 2 * 80 * 8 * 128 * 2
    assert ModelConfig("meta-llama/Meta-Llama-3-8B").arch.num_hidden_layers == 32
    with pytest.raises(ValueError):
        ModelConfig("no-such-model")
