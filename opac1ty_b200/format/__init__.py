"""The .bf2 on-disk format (reference layout, opacc1ty/format/)."""

from .bf2 import BF2Reader, BF2Writer
from .header import HEADER_SIZE, MAGIC, VERSION, BF2Header, LayerFormat, LayerType

__all__ = ["BF2Header", "LayerFormat", "LayerType", "BF2Writer", "BF2Reader", "MAGIC", "VERSION", "HEADER_SIZE"]
