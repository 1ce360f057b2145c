from .logger import init_logger
from .misc import GB, MB, Stage, EngineState, Event, cdiv, set_random_seed, get_gpu_memory, instance_name
from .metrics import RequestMetrics, SLO, calculate_metrics, goodput, percentiles, summarize
