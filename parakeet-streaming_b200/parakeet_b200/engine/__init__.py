from .scheduler import Scheduler, SlotAllocator, StreamResult
from .sequence import Sequence, SequenceStatus

__all__ = ["Scheduler", "SlotAllocator", "StreamResult", "Sequence", "SequenceStatus"]
