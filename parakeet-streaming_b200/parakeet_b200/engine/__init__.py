from .decoding import BatchedGreedyDecoder
from .pipeline import OverlappedStreamingRunner, StreamingPipeline
from .pre_encode import BatchedPreEncoder
from .scheduler import Scheduler, SlotAllocator, StreamResult
from .sequence import Sequence, SequenceStatus

__all__ = ["BatchedGreedyDecoder", "BatchedPreEncoder", "OverlappedStreamingRunner", "Scheduler", "SlotAllocator", "StreamResult", "Sequence",
           "SequenceStatus", "StreamingPipeline"]
