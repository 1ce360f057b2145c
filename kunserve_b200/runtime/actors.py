"""Actor runtime with a Ray-like ``handle.method.remote(*args)`` surface.

The reference runs every layer as a Ray actor (``kunserve/setup.py:38-73``,
``flash_backend.py:1278-1295``).  Ray is optional here: when it is importable
and ``KUNSERVE_USE_RAY=1`` the same calls go to Ray actors; otherwise one of
three built-in kinds is used:

* ``local``   — the object lives in the caller's process; calls run inline
  and return an already-completed future (lowest latency, used for a single
  GPU worker driven by its own engine);
* ``thread``  — calls run in order on one dedicated thread;
* ``process`` — the object is built in a child process (``spawn``), calls and
  results travel over a pipe; one process per GPU or per CPU rank;
* ``conn``    — the object lives in a process that an external launcher
  started (a ``torchrun`` rank): that process serves it on a local socket
  (``serve_connection``) and the front end holds a ``ConnActor``.

Every future can be awaited (``asyncio.wrap_future``) or waited with
``get(futures, timeout=...)``.  A child process that dies fails all of its
pending futures with ``ActorDiedError`` instead of hanging the caller.
"""
import asyncio
import concurrent.futures as cf
import multiprocessing as mp
import os
import queue
import threading
import traceback
from typing import Any, Callable, Dict, List, Optional, Sequence


class ActorDiedError(RuntimeError):
    pass


class RemoteError(RuntimeError):
    def __init__(self, msg: str, remote_tb: str = ""):
        super().__init__(f"{msg}\n--- remote traceback ---\n{remote_tb}")
        self.remote_tb = remote_tb


def _done_future(fn, args, kwargs) -> cf.Future:
    f: cf.Future = cf.Future()
    try:
        f.set_result(fn(*args, **kwargs))
    except BaseException as e:  # noqa: BLE001 - forwarded to the caller
        f.set_exception(e)
    return f


class _Method:
    def __init__(self, actor, name: str):
        self._actor, self._name = actor, name

    def remote(self, *args, **kwargs) -> cf.Future:
        return self._actor._submit(self._name, args, kwargs)

    def __call__(self, *args, **kwargs):
        raise TypeError(f"call {self._name}.remote(...) on an actor handle")


class ActorHandle:
    kind = "base"

    def __getattr__(self, name: str) -> _Method:
        if name.startswith("__"):
            raise AttributeError(name)
        return _Method(self, name)

    def _submit(self, name, args, kwargs) -> cf.Future:
        raise NotImplementedError

    def kill(self) -> None:
        pass


class LocalActor(ActorHandle):
    kind = "local"

    def __init__(self, obj):
        object.__setattr__(self, "_obj", obj)

    def _submit(self, name, args, kwargs):
        return _done_future(getattr(self._obj, name), args, kwargs)

    @property
    def obj(self):
        return self._obj


class ThreadActor(ActorHandle):
    kind = "thread"

    def __init__(self, obj, name: str = "actor", init: Optional[Callable[[], None]] = None):
        """``init`` runs once on the actor's thread before any call (for
        example ``torch.cuda.set_device``: the current device is per thread)."""
        object.__setattr__(self, "_obj", obj)
        object.__setattr__(self, "_pool", cf.ThreadPoolExecutor(1, thread_name_prefix=name, initializer=init))

    def _submit(self, name, args, kwargs):
        return self._pool.submit(getattr(self._obj, name), *args, **kwargs)

    def kill(self):
        self._pool.shutdown(wait=False, cancel_futures=True)

    @property
    def obj(self):
        return self._obj


def _process_main(conn, factory, fargs, fkwargs, env):
    os.environ.update(env or {})
    try:
        obj = factory(*fargs, **fkwargs)
        conn.send(("__ready__", True, None))
    except BaseException as e:  # noqa: BLE001
        conn.send(("__ready__", False, (repr(e), traceback.format_exc())))
        return
    _serve_loop(obj, conn)


def _serve_loop(obj, conn) -> None:
    """Run ``(call_id, name, args, kwargs)`` messages against ``obj`` in
    order and answer ``(call_id, ok, result or (repr, traceback))`` until the
    peer sends ``None`` or goes away."""
    while True:
        try:
            msg = conn.recv()
        except (EOFError, OSError):
            return
        if msg is None:
            return
        call_id, name, args, kwargs = msg
        try:
            res = getattr(obj, name)(*args, **kwargs)
            conn.send((call_id, True, res))
        except BaseException as e:  # noqa: BLE001
            conn.send((call_id, False, (repr(e), traceback.format_exc())))


class _ConnectionActor(ActorHandle):
    """Calls over a ``multiprocessing`` connection: a reader thread resolves
    each call's future from the answers, and a closed connection fails every
    pending call with ``ActorDiedError``."""

    def _start(self, conn, proc=None, ready: bool = False) -> None:
        d = self.__dict__
        d["_conn"], d["_proc"] = conn, proc
        d["_pending"]: Dict[int, cf.Future] = {}
        d["_lock"] = threading.Lock()
        d["_next"] = 0
        d["_ready"] = cf.Future()
        if ready:
            d["_ready"].set_result(True)
        d["_dead"] = False
        t = threading.Thread(target=self._reader, daemon=True)
        d["_reader_thread"] = t
        t.start()

    def _died(self) -> "ActorDiedError":
        return ActorDiedError("actor connection closed")

    def _reader(self):
        while True:
            try:
                call_id, ok, payload = self._conn.recv()
            except (EOFError, OSError):
                break
            if call_id == "__ready__":
                if ok:
                    self._ready.set_result(True)
                else:
                    self._ready.set_exception(RemoteError(*payload))
                continue
            with self._lock:
                fut = self._pending.pop(call_id, None)
            if fut is None:
                continue
            if ok:
                fut.set_result(payload)
            else:
                fut.set_exception(RemoteError(*payload))
        self.__dict__["_dead"] = True
        err = self._died()
        if not self._ready.done():
            self._ready.set_exception(err)
        with self._lock:
            pend, self.__dict__["_pending"] = self._pending, {}
        for f in pend.values():
            if not f.done():
                f.set_exception(err)

    def _submit(self, name, args, kwargs):
        fut: cf.Future = cf.Future()
        if self._dead:
            fut.set_exception(ActorDiedError("actor is dead"))
            return fut
        with self._lock:
            cid = self._next
            self.__dict__["_next"] = cid + 1
            self._pending[cid] = fut
        try:
            self._conn.send((cid, name, args, kwargs))
        except (OSError, BrokenPipeError) as e:
            with self._lock:
                self._pending.pop(cid, None)
            fut.set_exception(ActorDiedError(str(e)))
        return fut


class ProcessActor(_ConnectionActor):
    kind = "process"

    def __init__(self, factory: Callable, *args, env: Optional[Dict[str, str]] = None,
                 ready_timeout: float = 600.0, wait_ready: bool = True, **kwargs):
        ctx = mp.get_context("spawn")
        parent, child = ctx.Pipe()
        proc = ctx.Process(target=_process_main, args=(child, factory, args, kwargs, env), daemon=True)
        proc.start()
        child.close()
        self._start(parent, proc)
        if wait_ready:
            self._ready.result(timeout=ready_timeout)

    def wait_ready(self, timeout: float = 600.0) -> None:
        """Block until the object was built in the child (raises its error)."""
        self._ready.result(timeout=timeout)

    def _died(self) -> ActorDiedError:
        return ActorDiedError(f"actor process {self._proc.pid} exited (code {self._proc.exitcode})")

    @property
    def pid(self) -> int:
        return self._proc.pid

    def is_alive(self) -> bool:
        return self._proc.is_alive() and not self._dead

    def kill(self, timeout: float = 10.0) -> None:
        try:
            self._conn.send(None)
        except (OSError, BrokenPipeError):
            pass
        self._proc.join(timeout)
        if self._proc.is_alive():
            self._proc.terminate()
            self._proc.join(timeout)


class ConnActor(_ConnectionActor):
    """Handle on an object served by another process of the same job (for
    example a ``torchrun`` rank hosting its GPU worker) over a local socket;
    see ``serve_connection``."""
    kind = "conn"

    def __init__(self, address, authkey: bytes, timeout: float = 60.0):
        import time as _time
        from multiprocessing.connection import Client

        deadline = _time.time() + timeout
        while True:
            try:
                conn = Client(address, authkey=authkey)
                break
            except ConnectionRefusedError:
                if _time.time() > deadline:
                    raise
                _time.sleep(0.05)
        self.__dict__["_address"] = address
        self._start(conn, ready=True)

    def _died(self) -> ActorDiedError:
        return ActorDiedError(f"served actor at {self._address} closed its connection")

    def kill(self, timeout: float = 10.0) -> None:
        """Ask the serving process to stop serving (it then returns from
        ``serve_connection``)."""
        try:
            self._conn.send(None)
        except (OSError, BrokenPipeError):
            pass
        self._reader_thread.join(timeout)


def serve_connection(obj, listener, accept_timeout: float = 900.0) -> None:
    """Serve ``obj`` to one ``ConnActor`` that connects to ``listener``
    (a ``multiprocessing.connection.Listener``) until it sends the stop
    message or disconnects.  Calls run in arrival order on this thread.
    Raises ``TimeoutError`` when nobody connects within ``accept_timeout``
    seconds (the front end died before it connected)."""
    connected = threading.Event()

    def give_up():
        if not connected.is_set():
            listener.close()

    timer = threading.Timer(accept_timeout, give_up)
    timer.daemon = True
    timer.start()
    try:
        conn = listener.accept()
    except OSError as e:
        raise TimeoutError(f"no front end connected within {accept_timeout:.0f} s") from e
    finally:
        connected.set()
        timer.cancel()
    try:
        _serve_loop(obj, conn)
    finally:
        conn.close()
        listener.close()


def ray_available() -> bool:
    if os.environ.get("KUNSERVE_USE_RAY", "0") != "1":
        return False
    try:
        import ray  # noqa: F401
        return True
    except ImportError:
        return False


def make_actor(kind: str, factory: Callable, *args, **kwargs) -> ActorHandle:
    if kind == "local":
        return LocalActor(factory(*args, **kwargs))
    if kind == "thread":
        return ThreadActor(factory(*args, **kwargs))
    if kind == "process":
        return ProcessActor(factory, *args, **kwargs)
    if kind == "ray":
        import ray

        num_gpus = kwargs.pop("num_gpus", 0)
        kwargs.pop("env", None)
        return ray.remote(num_gpus=num_gpus)(factory).remote(*args, **kwargs)
    raise ValueError(f"unknown actor kind {kind!r}")


def get(futures, timeout: Optional[float] = None):
    """Block for one future or a list of them (like ``ray.get``)."""
    if isinstance(futures, (list, tuple)):
        return [f.result(timeout=timeout) for f in futures]
    return futures.result(timeout=timeout)


def aw(fut: cf.Future) -> "asyncio.Future":
    """Await a remote call's future from asyncio code."""
    return asyncio.wrap_future(fut)
