from .decoding import BatchedGreedyDecoder
from .scheduler import Scheduler, SlotAllocator, StreamResult
from .sequence import Sequence, SequenceStatus

__all__ = ["BatchedGreedyDecoder", "Scheduler", "SlotAllocator", "StreamResult", "Sequence",
           "SequenceStatus"]
