"""Scheduler with a paged state pool: drop-in for ``Scheduler``
(parakeet/engine/scheduler.py:20-201), driven by the reference's own
``ModelRunner`` and ``Sequence`` (parakeet/engine/model_runner.py:19-496,
parakeet/engine/sequence.py:16-179).

Two halves, as in the reference:

* **Admission** (``add`` / ``admit_ready`` / ``release`` /
  ``active_sequences``): at most ``max_active`` sequences run; the rest wait
  in arrival order and are admitted by ``admit_ready``.  Every sequence gets
  an arrival ticket; the running and the waiting sets are ticket-keyed
  dictionaries (insertion order = arrival order), so ``release`` finds a
  sequence in O(1) by identity instead of scanning two queues.  Statuses are
  written with the caller's own enum: ``seq.status`` already holds a member
  of the ``SequenceStatus`` class that created the sequence (WAITING at
  construction, sequence.py:33), and the new status is that class's member
  of the same name, so ``ModelRunner``'s comparisons against its own enum
  (model_runner.py:176,260,330) hold.
* **State pool** (``init_state_pool`` ... ``unpack_states``): slots come
  from a FIFO free list seeded with range(pool_size) (acquire takes the
  oldest free slot, release returns a slot to the back), so slot ids equal
  the reference's.  What changes is the state behind a slot: instead of a
  dense window per slot that ``pack_states`` and ``unpack_states`` copy in
  and out of a batch buffer every step (scheduler.py:128-201), the K/V window
  lives in pages that the kernels read in place, so ``pack_states`` only
  uploads the batch's slot ids and ``unpack_states`` has nothing to copy
  back.  Pages are reserved per slot at acquire time (``pages_per_stream``
  each), so with a pool capped below full demand a stream is admitted only
  when its worst-case window fits: acquire returns None instead of failing
  mid-step.
"""
from __future__ import annotations

import itertools
import threading
from collections import deque
from dataclasses import dataclass
from enum import Enum
from typing import Iterable

import torch

from ..modules.cache import PagedModelCache, StreamingState


@dataclass
class StreamResult:
    """Per-stream result record of the engine façade (scheduler.py:12-17)."""
    stream_id: int
    text: str
    token_ids: list[int]
    is_final: bool


class SequenceStatus(Enum):
    """Statuses for sequences that carry none of their own (the reference's
    ``Sequence`` always does: its own enum is used for those)."""
    WAITING = 1
    RUNNING = 2
    FINISHED = 3


def _set_status(seq, name: str) -> None:
    cur = getattr(seq, "status", None)
    cls = type(cur) if isinstance(cur, Enum) else SequenceStatus
    seq.status = cls[name]


def _is_finished(seq) -> bool:
    cur = getattr(seq, "status", None)
    return isinstance(cur, Enum) and cur.name == "FINISHED"


class SlotAllocator:
    """FIFO slot free list with per-slot page reservations (host only).

    The free-list discipline is the reference's (scheduler.py:84,93-104):
    slot ids must match.  One check is added: a slot is handed out only if
    ``pages_per_slot`` more pages can be reserved within ``num_pages``."""

    def __init__(self, num_slots: int, pages_per_slot: int = 0, num_pages: int | None = None):
        self.free = deque(range(num_slots))
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
        self._lock = threading.Lock()          # admission sets
        self._state_lock = threading.Lock()    # slot pool
        self._tickets = itertools.count()
        self._ticket_of: dict[int, int] = {}   # id(seq) -> arrival ticket
        self._running: dict[int, object] = {}  # ticket -> seq, admission order
        self._waiting: dict[int, object] = {}  # ticket -> seq, arrival order
        self._pool = None
        self._slots: SlotAllocator | None = None
        self._state_device: torch.device | None = None

    # ---------------------------------------------------------- admission
    def add(self, seq) -> None:
        with self._lock:
            t = next(self._tickets)
            self._ticket_of[id(seq)] = t
            room = len(self._running) < self.max_active
            (self._running if room else self._waiting)[t] = seq
            _set_status(seq, "RUNNING" if room else "WAITING")

    def admit_ready(self) -> list:
        """Moves waiting sequences to the running set in arrival order while
        there is room; sequences finished while waiting are dropped."""
        admitted = []
        with self._lock:
            for t in list(self._waiting):
                if len(self._running) >= self.max_active:
                    break
                seq = self._waiting.pop(t)
                if _is_finished(seq):
                    self._ticket_of.pop(id(seq), None)
                    continue
                self._running[t] = seq
                _set_status(seq, "RUNNING")
                admitted.append(seq)
        return admitted

    def release(self, seq) -> None:
        with self._lock:
            t = self._ticket_of.pop(id(seq), None)
            if t is not None:
                self._running.pop(t, None)
                self._waiting.pop(t, None)
            _set_status(seq, "FINISHED")

    def active_sequences(self) -> list:
        with self._lock:
            return list(self._running.values())

    @property
    def num_waiting(self) -> int:
        return len(self._waiting)

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

    def pack_states(self, seqs: Iterable) -> tuple[StreamingState, torch.Tensor]:
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


__all__ = ["Scheduler", "SequenceStatus", "SlotAllocator", "StreamResult"]
