"""Stream placement across GPUs: one engine process per GPU, streams
independent.  The reference serves every stream from one process on one
device (parakeet/engine/asr_engine.py:14-41, ``create_stream``); with one
engine per GPU, a router in front of them picks the engine for each new
stream.  Nothing crosses GPUs: a stream's pages, conv cache, feature history
and prediction state live on the GPU that serves it from its first chunk to
its release.

``StreamRouter`` sends each new stream to the engine with the fewest live
streams (ties to the lowest rank), optionally bounded by a per-engine
capacity (slots).  It is deterministic, so every rank can compute the same
placement from the same arrival sequence with no exchange."""
from __future__ import annotations

import heapq


class StreamRouter:
    def __init__(self, world_size: int, capacity: int | None = None):
        if world_size < 1:
            raise ValueError("world_size >= 1")
        self.world_size = world_size
        self.capacity = capacity
        self.load = [0] * world_size
        self._where: dict[int, int] = {}
        self._heap = [(0, r) for r in range(world_size)]     # (load, rank), lazily updated

    def place(self, stream_id: int) -> int | None:
        """The rank that serves ``stream_id`` (a new stream), or None when
        every engine is at capacity."""
        if stream_id in self._where:
            raise ValueError(f"stream {stream_id} is already placed")
        while self._heap:
            load, r = heapq.heappop(self._heap)
            if load != self.load[r]:
                continue                                      # stale entry
            if self.capacity is not None and load >= self.capacity:
                heapq.heappush(self._heap, (load, r))
                return None
            self.load[r] += 1
            heapq.heappush(self._heap, (self.load[r], r))
            self._where[stream_id] = r
            return r
        return None

    def release(self, stream_id: int) -> int:
        """Frees ``stream_id``'s place; returns the rank that served it."""
        r = self._where.pop(stream_id)
        self.load[r] -= 1
        heapq.heappush(self._heap, (self.load[r], r))
        return r

    def rank_of(self, stream_id: int) -> int | None:
        return self._where.get(stream_id)

    def streams_of(self, rank: int) -> list[int]:
        """Live streams on ``rank`` in placement order."""
        return [s for s, r in self._where.items() if r == rank]


__all__ = ["StreamRouter"]
