"""Building a serving job: workers (one per device or CPU rank), instances,
balloon groups and the front end.

Parity: ``kunserve/setup.py`` (``connect_to_ray_cluster`` :10-36,
``setup_kunserve`` :38-73) and the worker/communicator set-up of
``flash_backend.py:323-376``.  Workers are process actors (or Ray actors when
``KUNSERVE_USE_RAY=1``); a single-device job keeps its worker in-process.
Each worker process joins one ``torch.distributed`` job (NCCL on GPU, gloo on
CPU) and builds the five communicators of ``parallel/topology.py``.
"""
import os
import socket
from typing import List, Optional

import torch

from .config.kunserve_config import KunServeConfig
from .config.runtime import CacheConfig, ModelConfig, ParallelConfig, SchedConfig
from .engine.instance import InstanceEngine
from .engine.worker import Worker
from .parallel.topology import Topology
from .runtime.actors import LocalActor, ProcessActor, make_actor, ray_available
from .utils.logger import init_logger

logger = init_logger(__name__)


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def connect_to_ray_cluster(address: Optional[str] = None) -> bool:
    """Join a Ray cluster when Ray is installed and enabled; otherwise the
    built-in process actors are used and this is a no-op."""
    if not ray_available():
        return False
    import ray

    if not ray.is_initialized():
        ray.init(address=address or "auto", namespace="kunserve", ignore_reinit_error=True)
    return True


def make_worker_process(rank: int, world: int, rendezvous, topo: Topology, mc: ModelConfig, cc: CacheConfig,
                        pc: ParallelConfig, backend: str, device: str, seed: int, timeout_s: float = 120.0):
    """Runs inside a worker process: joins the job and builds the Worker.
    ``rendezvous`` is a file path (workers on this node) or a TCP port."""
    from .parallel.comm import Communicator, init_default_group

    if device.startswith("cuda"):
        torch.cuda.set_device(torch.device(device))
    dist_backend = "nccl" if device.startswith("cuda") else "gloo"
    if isinstance(rendezvous, str):
        init_default_group(dist_backend, rank, world, timeout_s=timeout_s, init_file=rendezvous)
    else:
        init_default_group(dist_backend, rank, world, timeout_s=timeout_s, master_port=rendezvous)
    comm = Communicator(topo, rank, dist_backend)
    return Worker(rank, mc, cc, pc, backend=backend, device=device, comm=comm, seed=seed)


def build_instances(cfg: KunServeConfig, mc: ModelConfig, cc: CacheConfig, sc: SchedConfig,
                    server_id: int = 0, backend: str = "auto", actor_kind: str = "auto",
                    devices: Optional[List[str]] = None, seed: int = 0, tokenizer=None,
                    output_callback=None) -> List[List[InstanceEngine]]:
    ec = cfg.engine_config
    topo = Topology(1, ec.ngroups, ec.group_size, ec.pp, ec.tp)
    world = topo.world_size
    if devices is None:
        n = torch.cuda.device_count()
        devices = [f"cuda:{r % n}" for r in range(world)] if n else ["cpu"] * world
    if actor_kind == "auto":
        actor_kind = "ray" if ray_available() else ("local" if world == 1 else "process")
    # worker processes of one node meet through a fresh file (a TCP port
    # picked here could be taken by someone else before rank 0 binds it);
    # Ray actors may live on other nodes and use a port
    import tempfile
    import uuid
    rendezvous = (free_port() if actor_kind == "ray"
                  else os.path.join(tempfile.gettempdir(), f"kus-rdzv-{os.getpid()}-{uuid.uuid4().hex[:12]}"))
    handles = {}
    for rank in range(world):
        pc = rank_parallel_config(topo, rank)
        if actor_kind == "local":
            handles[rank] = LocalActor(Worker(rank, mc, cc, pc, backend=backend, device=devices[rank], seed=seed))
        elif actor_kind == "process":
            env = {"KUNSERVE_WORKER_RANK": str(rank)}
            # every rank must be spawned before any can finish joining the job
            handles[rank] = ProcessActor(make_worker_process, rank, world, rendezvous, topo, mc, cc, pc, backend,
                                         devices[rank], seed, env=env, wait_ready=False)
        else:
            handles[rank] = make_actor("ray", make_worker_process, rank, world, rendezvous, topo, mc, cc, pc,
                                       backend, devices[rank], seed, num_gpus=1 if devices[rank] != "cpu" else 0)
    if actor_kind == "process":
        for h in handles.values():
            h.wait_ready()
    return instances_from_handles(cfg, mc, cc, sc, topo, handles, server_id, tokenizer, output_callback)


def rank_parallel_config(topo: Topology, rank: int) -> ParallelConfig:
    """The parallel coordinates of one global rank."""
    _, g, i, st, t = topo.coords(rank)
    return ParallelConfig(tensor_parallel_size=topo.tp, tensor_parallel_rank=t, pipeline_parallel_size=topo.pp,
                          pipeline_parallel_rank=st, group_parallel_size=topo.group_size * topo.pp,
                          group_parallel_rank=i * topo.pp + st, replica_size=topo.group_size, replica_rank=i,
                          global_rank=rank, global_size=topo.world_size)


def instances_from_handles(cfg: KunServeConfig, mc: ModelConfig, cc: CacheConfig, sc: SchedConfig, topo: Topology,
                           handles, server_id: int = 0, tokenizer=None,
                           output_callback=None) -> List[List[InstanceEngine]]:
    """Instance engines (grouped by balloon group) over worker handles
    indexed by global rank."""
    ec = cfg.engine_config
    groups = []
    for g in range(ec.ngroups):
        insts = []
        for i in range(ec.group_size):
            workers = [[handles[topo.rank_of(0, g, i, st, t)] for t in range(ec.tp)] for st in range(ec.pp)]
            pc = ParallelConfig(tensor_parallel_size=ec.tp, pipeline_parallel_size=ec.pp,
                                replica_size=ec.group_size, replica_rank=i)
            inst = InstanceEngine(server_id, g * ec.group_size + i, mc, pc, cc, sc, cfg.balloon_config,
                                  cfg.bench_config, workers, tokenizer=tokenizer, output_callback=output_callback)
            insts.append(inst)
        groups.append(insts)
    return groups


class LaunchedRank:
    """One rank of a job that an external launcher started: its worker and the
    socket it serves the worker on."""

    def __init__(self, worker, listener, ports, authkey):
        self.worker, self.listener, self.ports, self.authkey = worker, listener, ports, authkey

    def serve(self) -> None:
        """Serve this rank's worker to the front end until it lets go."""
        from .runtime.actors import serve_connection
        serve_connection(self.worker, self.listener)


def join_launched_job(cfg: KunServeConfig, mc: ModelConfig, cc: CacheConfig, rank: int, device: str,
                      seed: int = 0, backend: str = "native") -> LaunchedRank:
    """A rank of a serving job whose processes an external launcher started
    (``torchrun``: one rank per GPU, the default ``torch.distributed`` group
    already joined).  Builds the five communicators and this rank's
    ``Worker``, opens a local socket for it and shares every rank's port; the
    front end (a separate process, so that scheduling never competes with a
    worker's step for the interpreter) then reaches all workers with
    ``connect_launched_job``.  Call ``serve()`` afterwards."""
    import secrets
    from multiprocessing.connection import Listener

    import torch.distributed as dist

    from .parallel.comm import Communicator

    ec = cfg.engine_config
    topo = Topology(1, ec.ngroups, ec.group_size, ec.pp, ec.tp)
    world = dist.get_world_size()
    if topo.world_size != world:
        raise ValueError(f"the job has {world} ranks but the topology needs {topo.world_size}")
    comm = Communicator(topo, rank, "nccl" if device.startswith("cuda") else "gloo")
    worker = Worker(rank, mc, cc, rank_parallel_config(topo, rank), backend=backend, device=device, comm=comm,
                    seed=seed)
    key = [secrets.token_bytes(16) if rank == 0 else None]
    dist.broadcast_object_list(key, src=0)
    listener = Listener(("127.0.0.1", 0), authkey=key[0])
    ports = [None] * world
    dist.all_gather_object(ports, listener.address[1])
    return LaunchedRank(worker, listener, ports, key[0])


def connect_launched_job(cfg: KunServeConfig, mc: ModelConfig, cc: CacheConfig, sc: SchedConfig, ports, authkey,
                         server_id: int = 0, tokenizer=None, output_callback=None):
    """Front end of a launched job: ``ConnActor`` handles on every rank's
    worker and the instance engines over them.  Returns ``(instance groups,
    handles by rank)``."""
    from .runtime.actors import ConnActor

    ec = cfg.engine_config
    topo = Topology(1, ec.ngroups, ec.group_size, ec.pp, ec.tp)
    handles = {r: ConnActor(("127.0.0.1", p), authkey) for r, p in enumerate(ports)}
    groups = instances_from_handles(cfg, mc, cc, sc, topo, handles, server_id, tokenizer, output_callback)
    return groups, handles


async def setup_kunserve(cfg: KunServeConfig, model_config: Optional[ModelConfig] = None, **kw):
    """Create ``nservers`` front ends (``AsyncLLM``) and initialise them."""
    from .llm import AsyncLLM

    servers = []
    for s in range(cfg.engine_config.nservers):
        llm = await AsyncLLM.create(cfg, model_config=model_config, server_id=s, **kw)
        servers.append(llm)
    return servers
