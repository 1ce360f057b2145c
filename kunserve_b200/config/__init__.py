from .kunserve_config import (EngineConfig, BalloonConfig, DispatchConfig, BenchConfig,
                              KunServeConfig, add_cli_args, get_cli_args, parse_args,
                              load_config_from_yaml, apply_yaml)
from .runtime import (LlamaArch, ARCHS, resolve_arch, CacheConfig, ParallelConfig,
                      SchedConfig, ModelConfig)
