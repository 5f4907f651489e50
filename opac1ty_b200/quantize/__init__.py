"""Quantizer producing the fused path's inputs (API of opacc1ty/quantize/)."""

from .codebook import CodebookConfig, CodebookLearner
from .outlier import OutlierConfig, OutlierDetector
from .vq import QuantizeConfig, VectorQuantizer

__all__ = ["QuantizeConfig", "VectorQuantizer", "CodebookConfig", "CodebookLearner", "OutlierConfig",
           "OutlierDetector"]
