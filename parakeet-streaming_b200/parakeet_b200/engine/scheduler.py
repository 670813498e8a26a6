"""Scheduler with a paged state pool: drop-in for ``Scheduler``
(parakeet/engine/scheduler.py:20-201).

Admission queue (``add``/``admit_ready``/``release``/``active_sequences``) and
the slot free list keep the reference's behaviour: slots come from a FIFO
deque seeded with range(pool_size); acquire pops the left end, release
appends on the right, a full pool returns None.  What changes is the state
behind a slot: instead of a dense window per slot that ``pack_states`` and
``unpack_states`` copy in and out of a batch buffer every step
(scheduler.py:128-201), the K/V window lives in pages that the kernels read
in place, so ``pack_states`` only uploads the batch's slot ids and
``unpack_states`` has nothing to copy back.

Pages are reserved per slot at acquire time (``pages_per_stream`` each), so
with a pool capped below full demand a stream is admitted only when its
worst-case window fits: acquire returns None instead of failing mid-step.
"""
from __future__ import annotations

import threading
from collections import deque
from dataclasses import dataclass
from typing import Deque, Iterable

import torch

from ..modules.cache import PagedModelCache, StreamingState
from .sequence import Sequence, SequenceStatus


@dataclass
class StreamResult:
    stream_id: int
    text: str
    token_ids: list[int]
    is_final: bool


class SlotAllocator:
    """FIFO slot free list with per-slot page reservations (host only).

    Matches the reference's deque discipline (scheduler.py:84,93-104) and adds
    one check: a slot is handed out only if ``pages_per_slot`` more pages can
    be reserved within ``num_pages``."""

    def __init__(self, num_slots: int, pages_per_slot: int = 0, num_pages: int | None = None):
        self.free: Deque[int] = deque(range(num_slots))
        self.pages_per_slot = pages_per_slot
        self.num_pages = num_pages if num_pages is not None else num_slots * pages_per_slot
        self.reserved = 0
        self.held: set[int] = set()

    def acquire(self) -> int | None:
        if not self.free or self.reserved + self.pages_per_slot > self.num_pages:
            return None
        slot = self.free.popleft()
        self.reserved += self.pages_per_slot
        self.held.add(slot)
        return slot

    def release(self, slot: int) -> None:
        if slot not in self.held:
            raise ValueError(f"slot {slot} is not held")
        self.held.remove(slot)
        self.reserved -= self.pages_per_slot
        self.free.append(slot)


class Scheduler:
    def __init__(self, max_active: int = 64):
        self.max_active = max_active
        self.waiting: Deque[Sequence] = deque()
        self.active: Deque[Sequence] = deque()
        self._lock = threading.Lock()
        self._state_lock = threading.Lock()
        self._pool = None
        self._slots: SlotAllocator | None = None
        self._state_device: torch.device | None = None

    # ---------------------------------------------------------- admission queue
    def add(self, seq: Sequence) -> None:
        with self._lock:
            if len(self.active) < self.max_active:
                seq.status = SequenceStatus.RUNNING
                self.active.append(seq)
            else:
                seq.status = SequenceStatus.WAITING
                self.waiting.append(seq)

    def admit_ready(self) -> list[Sequence]:
        admitted = []
        with self._lock:
            while self.waiting and len(self.active) < self.max_active:
                seq = self.waiting.popleft()
                if seq.status == SequenceStatus.FINISHED:
                    continue
                seq.status = SequenceStatus.RUNNING
                self.active.append(seq)
                admitted.append(seq)
        return admitted

    def release(self, seq: Sequence) -> None:
        with self._lock:
            if seq in self.waiting:
                self.waiting.remove(seq)
            if seq in self.active:
                self.active.remove(seq)
            seq.status = SequenceStatus.FINISHED

    def active_sequences(self) -> Iterable[Sequence]:
        with self._lock:
            return list(self.active)

    # ---------------------------------------------------------- state pool
    @property
    def pool(self):
        return self._pool

    def init_state_pool(self, encoder, device, dtype, pool_size: int, *, num_pages=None,
                        page_size: int = 16, page_order=None) -> None:
        """Pool of ``pool_size`` slots; ``num_pages`` defaults to full demand
        (every slot's worst-case window)."""
        with self._state_lock:
            self._pool = encoder.make_pool(pool_size, device=device, dtype=dtype,
                                           num_pages=num_pages, page_size=page_size,
                                           page_order=page_order)
            self._slots = SlotAllocator(pool_size, self._pool.per_stream, self._pool.num_pages)
            self._state_device = torch.device(device)

    def acquire_state_slot(self) -> int | None:
        with self._state_lock:
            if self._slots is None:
                raise RuntimeError("State pool not initialized.")
            slot = self._slots.acquire()
        if slot is not None:
            self._pool.zero_conv_slot(slot)
        return slot

    def release_state_slot(self, slot: int) -> None:
        with self._state_lock:
            self._slots.release(slot)
            self._pool.release_slot(slot)

    def pack_states(self, seqs: Iterable[Sequence]) -> tuple[StreamingState, torch.Tensor]:
        if self._pool is None:
            raise RuntimeError("State pool not initialized.")
        ids = [seq.encoder_state for seq in seqs]
        if len(set(ids)) != len(ids):
            raise ValueError("a slot appears twice in one batch")
        slots = torch.tensor(ids, dtype=torch.int32).to(self._state_device)
        return StreamingState(PagedModelCache(self._pool, slots)), slots.long()

    def unpack_states(self, batch_state: StreamingState, slot_index: torch.Tensor) -> None:
        """Nothing to scatter: pages and the conv cache were updated in place
        and the step's counters by the encoder's end-of-step kernel."""
        return None


__all__ = ["Scheduler", "SlotAllocator", "StreamResult"]
