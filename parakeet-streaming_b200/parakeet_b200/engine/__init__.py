from .decoding import BatchedGreedyDecoder
from .pipeline import OverlappedStreamingRunner, StreamingPipeline
from .pre_encode import BatchedPreEncoder
from .router import StreamRouter
from .scheduler import Scheduler, SequenceStatus, SlotAllocator, StreamResult

__all__ = ["BatchedGreedyDecoder", "BatchedPreEncoder", "OverlappedStreamingRunner", "Scheduler",
           "SequenceStatus", "SlotAllocator", "StreamResult", "StreamRouter", "StreamingPipeline"]
