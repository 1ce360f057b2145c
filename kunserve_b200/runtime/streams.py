"""Per-request output streams (parity: ``AsyncStream``,
``kunserve/llm_engine.py:57-104``; the reference's PutQueue/RayQueue actor
hops, ``kunserve/ray_queue.py:13-119``, become a direct callback because
instances live in the front-end process).
"""
import asyncio
from typing import Dict, List, Optional

from ..request import RequestOutput


class AsyncStream:
    def __init__(self, request_id: int):
        self.request_id = request_id
        self._queue: asyncio.Queue = asyncio.Queue()
        self._finished = False

    def put(self, item: RequestOutput) -> None:
        if not self._finished:
            self._queue.put_nowait(item)

    def finish(self) -> None:
        if not self._finished:
            self._queue.put_nowait(StopAsyncIteration())
            self._finished = True

    @property
    def finished(self) -> bool:
        return self._finished

    def __aiter__(self):
        return self

    async def __anext__(self) -> RequestOutput:
        item = await self._queue.get()
        if isinstance(item, Exception):
            raise item
        return item


class StreamRouter:
    """Routes engine outputs to the streams of their requests (thread-safe:
    engines may call it from a worker thread)."""

    def __init__(self, loop: Optional[asyncio.AbstractEventLoop] = None):
        self.streams: Dict[int, AsyncStream] = {}
        self.loop = loop

    def register(self, rid: int) -> AsyncStream:
        s = AsyncStream(rid)
        self.streams[rid] = s
        return s

    def abort(self, rid: int, err: Optional[Exception] = None) -> None:
        s = self.streams.pop(rid, None)
        if s is not None:
            if err is not None:
                s._queue.put_nowait(err)
            s.finish()

    def __call__(self, outputs: List[RequestOutput]) -> None:
        def deliver():
            for o in outputs:
                s = self.streams.get(o.request_id)
                if s is None:
                    continue
                s.put(o)
                if o.finished:
                    s.finish()
                    self.streams.pop(o.request_id, None)
        try:
            running = asyncio.get_running_loop()
        except RuntimeError:
            running = None
        if self.loop is not None and running is not self.loop:
            self.loop.call_soon_threadsafe(deliver)
        else:
            deliver()
