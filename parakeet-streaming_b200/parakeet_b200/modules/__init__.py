from .attention import ConformerAttention, PositionalEncoding
from .cache import ConvCacheRef, ModelCache, PagedModelCache, StreamingState
from .convolution import ConformerConvolution
from .decoder import Joiner, Predictor
from .subsample import ConvSubsampling
from .features import FeatureExtractor
from .encoder import ConformerEncoder, ConformerLayer
from .feedforward import ConformerFeedForward

__all__ = ["ConformerAttention", "PositionalEncoding", "ConvCacheRef", "ModelCache",
           "PagedModelCache", "StreamingState", "ConformerConvolution", "ConformerEncoder",
           "ConformerLayer", "ConformerFeedForward", "Joiner", "Predictor", "ConvSubsampling",
           "FeatureExtractor"]
