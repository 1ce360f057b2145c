"""Sharing GPU memory between worker processes for in-kernel P2P copies.

A worker exports the physical allocations of its VMM arena (KV pool and
every decoder layer's weight segment) as POSIX file descriptors and serves
them on a Unix socket (``SCM_RIGHTS``); a group peer fetches them, maps each
into its own address space (``PeerMapping`` in the native library: cuMem
import + map + access for the peer's device) and hands the resulting
pointers to the copy kernel, which then pulls bytes over NVLink with plain
loads.  No TMA (and no multicast) ever reads peer memory.
"""
import os
import socket
import tempfile
import threading
import uuid
from typing import Dict, List, Tuple


class FdServer:
    """Serves a fixed list of fds to any number of clients (one message each)."""

    def __init__(self, fds: List[int]):
        self.fds = list(fds)
        self.path = os.path.join(tempfile.gettempdir(), f"kus-{os.getpid()}-{uuid.uuid4().hex[:8]}.sock")
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.bind(self.path)
        self.sock.listen(16)
        self._stop = False
        self.thread = threading.Thread(target=self._serve, daemon=True)
        self.thread.start()

    def _serve(self):
        while not self._stop:
            try:
                conn, _ = self.sock.accept()
            except OSError:
                return
            with conn:
                socket.send_fds(conn, [len(self.fds).to_bytes(4, "little")], self.fds)

    def close(self):
        self._stop = True
        try:
            self.sock.close()
        finally:
            if os.path.exists(self.path):
                os.unlink(self.path)
            for fd in self.fds:
                try:
                    os.close(fd)
                except OSError:
                    pass


def fetch_fds(path: str, timeout: float = 30.0) -> List[int]:
    s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    s.settimeout(timeout)
    s.connect(path)
    with s:
        msg, fds, _, _ = socket.recv_fds(s, 16, 1024)
    n = int.from_bytes(msg[:4], "little")
    if len(fds) != n:
        raise RuntimeError(f"expected {n} fds from {path}, got {len(fds)}")
    return fds


class PeerMemory:
    """One peer's KV pool and layer segments mapped into this process."""

    def __init__(self, native, device: int, fds: List[int], sizes: List[int]):
        self.maps = []
        try:
            for fd, size in zip(fds, sizes):
                self.maps.append(native.PeerMapping(device, fd, size))
        finally:
            for fd in fds:
                os.close(fd)
        self.kv = self.maps[0].ptr()
        self.layers = [m.ptr() for m in self.maps[1:]]
        # mapped extents: copies that read the peer are checked against them
        self.kv_bytes = int(sizes[0])
        self.layer_bytes = [int(x) for x in sizes[1:]]
