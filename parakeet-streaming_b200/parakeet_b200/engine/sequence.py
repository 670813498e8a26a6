"""Per-stream encoder-side state: drop-in for the parts of ``Sequence``
(parakeet/engine/sequence.py:10-179) that the batched encoder step uses -
the slot id, the queue of subsampled frames waiting for a chunk, the queue
of encoder outputs, and the status used by the scheduler.  Audio buffering
and feature extraction are outside this package."""
from __future__ import annotations

import threading
from collections import deque
from enum import Enum, auto
from itertools import count

import torch


class SequenceStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Sequence:
    counter = count()

    def __init__(self, enc_hidden_dim: int, enc_chunk_size: int, encoder_state,
                 device: torch.device | str = "cpu", dtype=torch.float32):
        self.request_id = next(Sequence.counter)
        self.status = SequenceStatus.WAITING
        self.lock = threading.Lock()
        self.encoder_state = encoder_state
        self.enc_chunk_size = enc_chunk_size
        self.enc_buffer = torch.empty((1, 0, enc_hidden_dim), device=device, dtype=dtype)
        self.encoded_queue: deque[torch.Tensor] = deque()
        self.final = False
        self.in_flight = 0

    def push_encoded_frames(self, frames: torch.Tensor, final: bool = False) -> None:
        """Append subsampled frames [1, n, D] (the pre-encoder's output)."""
        if frames.numel():
            self.enc_buffer = torch.cat([self.enc_buffer, frames.to(self.enc_buffer)], dim=1)
        self.final = self.final or final

    def has_chunk_ready(self) -> bool:
        if self.enc_buffer is None:
            return False
        n = self.enc_buffer.size(1)
        return n >= self.enc_chunk_size or (self.final and n > 0)

    def pop_chunk(self):
        """Next chunk [1, T, D] and its length; a final partial chunk is zero
        padded to T and reported with length T, as sequence.py:125-147 does."""
        if not self.has_chunk_ready():
            return None, None
        T = self.enc_chunk_size
        take = min(T, self.enc_buffer.size(1))
        chunk = self.enc_buffer[:, :take]
        self.enc_buffer = self.enc_buffer[:, take:]
        if take < T:
            chunk = torch.cat([chunk, chunk.new_zeros(1, T - take, chunk.size(2))], dim=1)
        return chunk, T

    def enqueue_encoded(self, out: torch.Tensor) -> None:
        if out is not None and out.numel() > 0:
            self.encoded_queue.append(out)

    def has_encoded(self) -> bool:
        return bool(self.encoded_queue)

    def pop_encoded(self):
        return self.encoded_queue.popleft() if self.encoded_queue else None


__all__ = ["Sequence", "SequenceStatus"]
