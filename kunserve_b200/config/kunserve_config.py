"""Command-line and YAML configuration.

The flag names, defaults and the four YAML sections (``engine_config``,
``balloon_config``, ``dispatch_config``, ``bench_config``) are the reference's
public interface (``kunserve/kunserve_config.py:9-398``) and are kept so that
existing launch scripts and YAML files work unchanged.  Three reference bugs
are fixed here: ``zigzag_chunk_limit`` is read from its own key
(reference :349-350), ``dispatch_strategy`` under ``bench_config`` fills
``server_dispatch_strategy`` from the key that was tested (:364-365), and
``duplicate_server`` is a real field (:368-369).  ``--qps`` is a float.
Unlike the reference, YAML is optional (``-c`` may be omitted) and values are
validated.
"""
import argparse
import dataclasses
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

import yaml

BALLOON_MODES = ("recompute", "reshard", "livereshard", "exchange")
DISPATCH_STRATEGIES = ("round-robin", "memory", "load")
ARRIVAL_DISTS = ("poisson", "uniform", "gamma", "real")


def _from_ns(cls, ns):
    names = [f.name for f in dataclasses.fields(cls)]
    return cls(**{n: getattr(ns, n) for n in names if hasattr(ns, n)})


@dataclass
class EngineConfig:
    nservers: int = 1
    ngroups: int = 1
    group_size: int = 1
    pp: int = 1
    tp: int = 1
    block_size: int = 256
    use_tensor_cores: bool = False
    schedule_policy: str = "prefill-first"
    preempt_method: str = "recompute"
    max_batch_size: int = 256
    max_batch_tokens: int = 131072
    gpu_util: float = 0.9
    dtype: str = "bf16"
    enable_chunked_prefill: bool = False
    chunked_prefill_size: Optional[int] = None
    chunked_prefill_budget: int = 4096

    @classmethod
    def from_cli_args(cls, ns) -> "EngineConfig":
        return _from_ns(cls, ns)

    @staticmethod
    def add_cli_args(p: argparse.ArgumentParser) -> argparse.ArgumentParser:
        p.add_argument("--nservers", type=int, default=1)
        p.add_argument("--group-size", type=int, default=1,
                       help="instances per balloon group (they share parameters under overload)")
        p.add_argument("--ngroups", type=int, default=1, help="number of balloon groups per server")
        p.add_argument("--pp", type=int, default=1)
        p.add_argument("--tp", type=int, default=1)
        p.add_argument("--block-size", type=int, default=256)
        p.add_argument("--use-tensor-cores", action="store_true", default=False)
        p.add_argument("--schedule-policy", type=str, default="prefill-first")
        p.add_argument("--preempt-method", type=str, default="recompute", choices=["recompute", "swap"])
        p.add_argument("--max-batch-size", type=int, default=256)
        p.add_argument("--max-batch-tokens", type=int, default=131072)
        p.add_argument("--gpu-util", type=float, default=0.9)
        p.add_argument("--dtype", type=str, default="bf16", choices=["bf16", "fp16", "fp32"])
        p.add_argument("--enable-chunked-prefill", action="store_true", default=False)
        p.add_argument("--chunked-prefill-size", type=int, default=None)
        p.add_argument("--chunked-prefill-budget", type=int, default=4096)
        return p

    def validate(self) -> None:
        for name in ("nservers", "ngroups", "group_size", "pp", "tp", "block_size",
                     "max_batch_size", "max_batch_tokens", "chunked_prefill_budget"):
            if getattr(self, name) is not None and getattr(self, name) <= 0:
                raise ValueError(f"engine_config.{name} must be positive")
        if not 0.0 < self.gpu_util <= 1.0:
            raise ValueError("engine_config.gpu_util must be in (0, 1]")
        if self.preempt_method not in ("recompute", "swap"):
            raise ValueError(f"unknown preempt_method {self.preempt_method!r}")


@dataclass
class BalloonConfig:
    enable_balloon: bool = False
    balloon_mode: str = "exchange"
    balloon_ratio: float = 1.0
    exchange_batch_size: int = 8
    restore_batch_size: int = 8
    max_balloon_memory_ratio: float = 0.5
    max_restore_memory_ratio: float = 0.8
    restore_memory_threshold: float = 0.5
    # cross-group transfer of running requests between unfused instances
    enable_transfer: bool = False

    @classmethod
    def from_cli_args(cls, ns) -> "BalloonConfig":
        return _from_ns(cls, ns)

    @staticmethod
    def add_cli_args(p: argparse.ArgumentParser) -> argparse.ArgumentParser:
        p.add_argument("--enable-balloon", action="store_true", default=False)
        p.add_argument("--balloon-mode", type=str, default="exchange")
        p.add_argument("--balloon-ratio", type=float, default=1.0)
        p.add_argument("--exchange-batch-size", type=int, default=8,
                       help="requests whose KV blocks are exchanged together")
        p.add_argument("--max-balloon-memory-ratio", type=float, default=0.5)
        p.add_argument("--max-restore-memory-ratio", type=float, default=0.8)
        p.add_argument("--restore-memory-threshold", type=float, default=0.5)
        p.add_argument("--restore-batch-size", type=int, default=8)
        p.add_argument("--enable-transfer", action="store_true", default=False,
                       help="move running requests (with their KV) from an overloaded instance to one of "
                            "another group")
        return p

    @property
    def effective_mode(self) -> str:
        """``exchange`` (the reference's CLI default) is its bulk reshard."""
        return "reshard" if self.balloon_mode == "exchange" else self.balloon_mode

    def validate(self) -> None:
        if self.balloon_mode not in BALLOON_MODES:
            raise ValueError(f"unknown balloon_mode {self.balloon_mode!r}")
        if self.exchange_batch_size <= 0 or self.restore_batch_size <= 0:
            raise ValueError("exchange/restore batch sizes must be positive")


@dataclass
class DispatchConfig:
    dispatch_strategy: str = "round-robin"

    @classmethod
    def from_cli_args(cls, ns) -> "DispatchConfig":
        return _from_ns(cls, ns)

    @staticmethod
    def add_cli_args(p: argparse.ArgumentParser) -> argparse.ArgumentParser:
        p.add_argument("--dispatch-strategy", type=str, default="round-robin")
        return p

    def validate(self) -> None:
        if self.dispatch_strategy not in DISPATCH_STRATEGIES:
            raise ValueError(f"unknown dispatch_strategy {self.dispatch_strategy!r}")


@dataclass
class BenchConfig:
    model: str = ""
    dataset: Optional[str] = None
    dataset_offset: int = 0
    nlimit: int = 1000
    ngroups: Optional[int] = None
    max_model_len: int = 16384
    qps: float = 1.0
    cv: float = 0.1
    dist: str = "poisson"
    trace: Optional[str] = None
    trace_offset: int = 0
    trace_repeat_start: Optional[int] = None
    trace_repeat_end: Optional[int] = None
    trace_repeat_times: Optional[int] = None
    trace_repeat_interval: Optional[int] = None
    seed: float = 42
    dataset_scale_factor: float = 1.0
    time_scale_factor: float = 1.0
    enable_look_ahead: bool = False
    enable_restore: bool = False
    enable_packing: bool = False
    long_threshold: float = 0.5
    enable_decode_balance: bool = False
    enable_prefill_balance: bool = False
    enable_reorder: bool = False
    zigzag_chunk_limit: int = 16
    log_path: str = "logs"
    log_name: str = "replica"
    num_gpu_blocks: Optional[int] = None
    shuffle_dataset: bool = False
    server_dispatch_strategy: Optional[str] = None
    enable_migration: bool = False
    duplicate_server: bool = False

    @classmethod
    def from_cli_args(cls, ns) -> "BenchConfig":
        return _from_ns(cls, ns)

    @staticmethod
    def add_cli_args(p: argparse.ArgumentParser) -> argparse.ArgumentParser:
        p.add_argument("--model", type=str, default="")
        p.add_argument("--dataset", type=str)
        p.add_argument("--dataset-offset", type=int, default=0)
        p.add_argument("--nlimit", type=int, default=1000, help="number of requests to send")
        p.add_argument("--qps", type=float, default=1.0)
        p.add_argument("--cv", type=float, default=0.1)
        p.add_argument("--dist", type=str, default="poisson", choices=list(ARRIVAL_DISTS))
        p.add_argument("--max-model-len", type=int, default=16384)
        p.add_argument("--trace", type=str)
        p.add_argument("--trace-offset", type=int, default=0)
        p.add_argument("--trace-repeat-start", type=int, default=None)
        p.add_argument("--trace-repeat-end", type=int, default=None)
        p.add_argument("--trace-repeat-times", type=int, default=None)
        p.add_argument("--trace-repeat-interval", type=int, default=None)
        p.add_argument("--dataset-scale-factor", type=float, default=1.0)
        p.add_argument("--time-scale-factor", type=float, default=1.0)
        p.add_argument("--seed", type=float, default=42)
        p.add_argument("--log-path", type=str, default="logs")
        p.add_argument("--log-name", type=str, default="replica")
        p.add_argument("--enable-decode-balance", action="store_true", default=False)
        p.add_argument("--enable-prefill-balance", action="store_true", default=False)
        p.add_argument("--enable-look-ahead", action="store_true", default=False)
        p.add_argument("--enable-packing", action="store_true", default=False)
        p.add_argument("--long-threshold", type=float, default=0.5)
        p.add_argument("--enable-reorder", action="store_true", default=False)
        p.add_argument("--zigzag-chunk-limit", type=int, default=16)
        p.add_argument("--enable-restore", action="store_true", default=False)
        p.add_argument("--num-gpu-blocks", type=int, default=None)
        p.add_argument("--shuffle-dataset", action="store_true", default=False)
        p.add_argument("--server-dispatch-strategy", type=str, default=None)
        p.add_argument("--enable-migration", action="store_true", default=False)
        p.add_argument("--duplicate-server", action="store_true", default=False)
        return p

    def validate(self) -> None:
        if self.dist not in ARRIVAL_DISTS:
            raise ValueError(f"unknown dist {self.dist!r}")
        if self.qps <= 0:
            raise ValueError("bench_config.qps must be positive")


@dataclass
class KunServeConfig:
    engine_config: EngineConfig = field(default_factory=EngineConfig)
    balloon_config: BalloonConfig = field(default_factory=BalloonConfig)
    dispatch_config: DispatchConfig = field(default_factory=DispatchConfig)
    bench_config: BenchConfig = field(default_factory=BenchConfig)

    def validate(self) -> "KunServeConfig":
        self.engine_config.validate()
        self.balloon_config.validate()
        self.dispatch_config.validate()
        self.bench_config.validate()
        return self

    def to_dict(self) -> Dict[str, Dict[str, Any]]:
        return {k: dataclasses.asdict(getattr(self, k)) for k in
                ("engine_config", "balloon_config", "dispatch_config", "bench_config")}


# YAML keys that are copied as-is into each section.  A key present in the
# file overrides the command line.
_ENGINE_KEYS = [f.name for f in dataclasses.fields(EngineConfig)]
_BALLOON_KEYS = [f.name for f in dataclasses.fields(BalloonConfig)]
_BENCH_KEYS = [f.name for f in dataclasses.fields(BenchConfig)]


def apply_yaml(cfg: KunServeConfig, data: Dict[str, Any]) -> KunServeConfig:
    eng = data.get("engine_config") or {}
    for k in _ENGINE_KEYS:
        if k in eng:
            setattr(cfg.engine_config, k, eng[k])
    bal = data.get("balloon_config") or {}
    for k in _BALLOON_KEYS:
        if k in bal:
            setattr(cfg.balloon_config, k, bal[k])
    if "balloon_mode" in bal:
        # a balloon section with a mode turns the mechanism on, as in the reference
        cfg.balloon_config.enable_balloon = bool(bal.get("enable_balloon", True))
    dis = data.get("dispatch_config") or {}
    if "dispatch_strategy" in dis:
        cfg.dispatch_config.dispatch_strategy = dis["dispatch_strategy"]
    bench = data.get("bench_config") or {}
    for k in _BENCH_KEYS:
        if k in bench:
            setattr(cfg.bench_config, k, bench[k])
    if "dispatch_strategy" in bench and "server_dispatch_strategy" not in bench:
        cfg.bench_config.server_dispatch_strategy = bench["dispatch_strategy"]
    return cfg


def load_config_from_yaml(cfg: KunServeConfig, fname: str) -> KunServeConfig:
    with open(fname, "r", encoding="utf-8") as f:
        data = yaml.safe_load(f) or {}
    return apply_yaml(cfg, data)


def add_cli_args(parser: argparse.ArgumentParser) -> argparse.ArgumentParser:
    EngineConfig.add_cli_args(parser)
    BalloonConfig.add_cli_args(parser)
    DispatchConfig.add_cli_args(parser)
    BenchConfig.add_cli_args(parser)
    parser.add_argument("--config", "-c", type=str, default=None)
    return parser


def get_cli_args(ns: argparse.Namespace) -> KunServeConfig:
    cfg = KunServeConfig(
        engine_config=EngineConfig.from_cli_args(ns),
        balloon_config=BalloonConfig.from_cli_args(ns),
        dispatch_config=DispatchConfig.from_cli_args(ns),
        bench_config=BenchConfig.from_cli_args(ns),
    )
    if getattr(ns, "config", None):
        load_config_from_yaml(cfg, ns.config)
    return cfg.validate()


def parse_args(argv=None) -> KunServeConfig:
    parser = add_cli_args(argparse.ArgumentParser("kunserve_b200"))
    return get_cli_args(parser.parse_args(argv))
